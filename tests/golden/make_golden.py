"""Generate golden vectors from the REFERENCE kernels (run on a B200 box).

Loads ``oracle/_ref/libctu_ref.so`` -- the reference's own ConvRot quantizers, W8A8
and W4A8 GEMMs and int32->bf16 epilogue (kernel/csrc/turing/{convrot_quant,w4a8,
bf16_epilogue}.cu of comfyui-turing-utils 0.31.0), compiled from the reference tree
by ``oracle/Makefile`` -- runs them on seeded inputs and writes compressed ``.npz``
fixtures.  The fixtures are committed under ``tests/golden/`` and pin the CPU oracle
(``oracle/convrot_oracle.py``) in the CPU test suite.

Usage (GPU box):  python tests/golden/make_golden.py --out gpurun_out/golden
"""

from __future__ import annotations

import argparse
import ctypes
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]


def load_ref():
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libctu_ref.so"))
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.ref_bf16_convrot_quantize.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, vp]
    lib.ref_bf16_gelu_convrot_quantize.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp]
    lib.ref_int8_linear.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]
    lib.ref_w4a8_linear.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]
    lib.ref_dequantize_int8_bf16.argtypes = [vp, vp, vp, i32, vp, i32, i32, i32, vp]
    lib.ref_codebook_w4a8_linear.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i32, vp, i32, i32, i32, i32, i32, i32, vp]
    lib.ref_swiglu_int8_convrot_quantize_scaled.argtypes = [vp, vp, vp, i32, i32, vp]
    for name in ("ref_bf16_convrot_quantize", "ref_bf16_gelu_convrot_quantize", "ref_int8_linear",
                 "ref_w4a8_linear", "ref_dequantize_int8_bf16", "ref_codebook_w4a8_linear",
                 "ref_swiglu_int8_convrot_quantize_scaled"):
        getattr(lib, name).restype = i32
    lib.ref_last_error.restype = ctypes.c_char_p
    return lib


def check(lib, rc):
    if rc != 0:
        raise RuntimeError(lib.ref_last_error().decode())


def p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def activations(rows, width, seed, outliers=True):
    """N(0,1) bf16 with 1% of channels scaled x30 (the BASELINE activation model)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((rows, width), generator=g, dtype=torch.float32)
    if outliers:
        idx = torch.randperm(width, generator=g)[: max(1, width // 100)]
        x[:, idx] *= 30.0
    return x.to(torch.bfloat16)


def special_rows(k):
    """Rows with zeros, tiny/subnormal, huge, inf and NaN values (bf16)."""
    g = torch.Generator().manual_seed(77)
    base = torch.randn((10, k), generator=g)
    rows = [
        torch.zeros(k),
        base[1] * 1e-38,                       # bf16 subnormal / tiny range
        base[2] * 1e-20,                       # tiny but normal
        base[3] * 1e36,                        # near overflow of the fp32 rotation
        torch.where(torch.arange(k) == 7, torch.tensor(3.0e38), base[4]),
        torch.where(torch.arange(k) == 3, torch.tensor(float("inf")), base[5]),
        torch.where(torch.arange(k) == 9, torch.tensor(float("nan")), base[6]),
        torch.where(torch.arange(k) % 2 == 0, torch.tensor(float("-inf")), torch.tensor(float("inf"))),
        torch.full((k,), 1.0),                 # constant row: one nonzero per group
        base[9].sign() * 2.0 ** torch.randint(-30, 30, (k,), generator=g).float(),
    ]
    return torch.stack(rows).to(torch.bfloat16)


def run_quant(lib, x, k, bits, mode, threads):
    rows = x.shape[0]
    xd = x.cuda().contiguous()
    codes = torch.empty((rows, k // 2 if bits == 4 else k), dtype=torch.int8, device="cuda")
    scales = torch.empty((rows, 1), dtype=torch.float32, device="cuda")
    if mode == "gelu":
        check(lib, lib.ref_bf16_gelu_convrot_quantize(p(xd), p(codes), p(scales), rows, k, bits, threads, stream()))
    else:
        check(lib, lib.ref_bf16_convrot_quantize(p(xd), p(codes), p(scales), rows, k, bits,
                                                 1 if mode == "swiglu" else 0, threads, stream()))
    torch.cuda.synchronize()
    return codes.cpu().numpy(), scales.cpu().numpy().reshape(-1)


def quant_cases():
    cases = []
    for mode, shapes in (
        ("plain", [(8, 256), (6, 1536), (4, 5120), (2, 13824)]),
        ("swiglu", [(4, 512), (2, 5120)]),
        ("gelu", [(4, 512), (2, 5120)]),
    ):
        for i, (rows, k) in enumerate(shapes):
            width = 2 * k if mode == "swiglu" else k
            cases.append((f"{mode}_m{rows}_k{k}", mode, activations(rows, width, 1000 + 17 * i + len(cases)), k))
    cases.append(("special_k512", "plain", special_rows(512), 512))
    cases.append(("special_swiglu_k256", "swiglu", torch.cat([special_rows(256), special_rows(256)], dim=1), 256))
    return cases


# Grouped-codebook W4A8 cases: (m, n, k, group_size, chunk_rows or 0 for the inline
# decode).  Inputs come from seeded generators (codebook_inputs), so the large inline
# case stores only its output.
CODEBOOK_CASES = [(33, 64, 256, 16, 64), (17, 72, 512, 4, 16), (9, 136, 768, 8, 136), (5, 64, 1024, 32, 32),
                  (65, 128, 256, 64, 128), (8200, 8, 64, 16, 0)]


def codebook_inputs(m, n, k, gs, seed):
    """Seeded codebook W4A8 operands (numpy), with e4m3 special bytes and tie values."""
    rng = np.random.default_rng(seed)
    a = rng.integers(-128, 128, size=(m, k), dtype=np.int8)
    codes = rng.integers(0, 16, size=(n, k), dtype=np.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8).view(np.int8)
    # e4m3fn bytes: mostly moderate scales (exponent 4..9), plus NaN, max, subnormals,
    # zeros and negative scales.
    scale = rng.integers(0x20, 0x50, size=(n, k // gs), dtype=np.uint8)
    special = np.array([0x7F, 0xFF, 0x7E, 0x01, 0x00, 0x80, 0xB8, 0x38], dtype=np.uint8)
    flat = scale.reshape(-1)
    flat[rng.choice(flat.size, size=min(flat.size, 8), replace=False)] = special[: min(flat.size, 8)]
    codebook = np.array([-8.0, -6.5, -4.0, -2.5, -1.5, -0.5, 0.0, 0.5, 1.5, 2.5, 3.25, 4.0, 6.0, 7.5, 64.0, 200.0],
                        dtype=np.float32)
    a_s = (rng.random(m, dtype=np.float32) * 0.02 + 0.001).astype(np.float32)
    c_s = (rng.random(n, dtype=np.float32) * 0.009 + 0.001).astype(np.float32)
    bias = (rng.standard_normal(n).astype(np.float32) * 0.02) if seed % 2 == 0 else None
    return a, packed, scale, codebook, a_s, c_s, bias


def extra_cases(lib, out):
    extras = {}
    for idx, (m, n, k, gs, chunk) in enumerate(CODEBOOK_CASES):
        a, packed, scale, codebook, a_s, c_s, bias = codebook_inputs(m, n, k, gs, 4500 + idx)
        dev = [None if t is None else torch.from_numpy(t).cuda() for t in (a, packed, scale, codebook, a_s, c_s, bias)]
        o = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        ws = torch.empty((chunk, k), dtype=torch.int8, device="cuda") if chunk else None
        check(lib, lib.ref_codebook_w4a8_linear(p(dev[0]), p(dev[1]), p(dev[4]), p(dev[2]), p(dev[5]), p(dev[3]),
                                                p(dev[6]), p(ws), chunk, p(o), m, n, k, gs, 0 if chunk else 1, 0,
                                                stream()))
        torch.cuda.synchronize()
        key = f"codebook_m{m}_n{n}_k{k}_g{gs}"
        extras[f"{key}__seed"] = np.array([4500 + idx], dtype=np.int64)
        extras[f"{key}__out"] = o.view(torch.int16).cpu().numpy().view(np.uint16)
    # SwiGLU shard quantized with caller-supplied row scales (special scales included).
    rows, k = 8, 512
    x = torch.cat([special_rows(256), special_rows(256)], dim=1)[:rows].repeat(1, 2)
    x[6:] = activations(2, 2 * k, 4600)
    scales = torch.tensor([0.05, 0.0, float("nan"), float("inf"), -0.02, 1e-40, 3e38, 0.013], dtype=torch.float32)
    codes = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    xd, sd = x.cuda().contiguous(), scales.cuda()
    check(lib, lib.ref_swiglu_int8_convrot_quantize_scaled(p(xd), p(sd), p(codes), rows, k, stream()))
    torch.cuda.synchronize()
    extras["scaled_swiglu__x"] = x.view(torch.int16).numpy().view(np.uint16)
    extras["scaled_swiglu__scales"] = scales.numpy()
    extras["scaled_swiglu__codes"] = codes.cpu().numpy()
    np.savez_compressed(out / "extras.npz", **extras)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--only", choices=["all", "extras"], default="all")
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    lib = load_ref()
    torch.cuda.init()
    extra_cases(lib, out)
    if args.only == "extras":
        print("golden vectors written to", out, file=sys.stderr)
        return

    # ConvRot rotate + quantize, int8 and int4; every block geometry must agree.
    quant = {}
    for name, mode, x, k in quant_cases():
        quant[f"{name}__x"] = x.view(torch.int16).numpy().view(np.uint16)
        for bits in (8, 4):
            results = [run_quant(lib, x, k, bits, mode, t) for t in (512, 768, 1024)]
            for codes, scales in results[1:]:
                assert np.array_equal(codes, results[0][0]), (name, bits)
                assert np.array_equal(scales.view(np.uint32), results[0][1].view(np.uint32)), (name, bits)
            quant[f"{name}__int{bits}_codes"] = results[0][0]
            quant[f"{name}__int{bits}_scales"] = results[0][1]
    np.savez_compressed(out / "convrot_quant.npz", **quant)

    # W8A8 / W4A8 GEMMs and the int32 epilogue.
    gemm = {}
    for idx, (m, n, k, with_bias) in enumerate([(33, 64, 256, True), (17, 72, 128, False),
                                                (130, 136, 512, True), (1, 16, 64, False)]):
        g = torch.Generator().manual_seed(4300 + idx)
        a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
        w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
        w4 = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
        a_s = torch.rand((m,), generator=g) * 0.02 + 0.001
        w_s = torch.rand((n,), generator=g) * 0.009 + 0.001
        bias = (torch.randn((n,), generator=g) * 0.02) if with_bias else None
        packed = ((w4[:, 0::2].to(torch.int32) & 0xF) | ((w4[:, 1::2].to(torch.int32) & 0xF) << 4)).to(torch.uint8).view(torch.int8)
        dev = [t.cuda() if t is not None else None for t in (a, w, packed, a_s, w_s, bias)]
        out8 = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        out4 = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        check(lib, lib.ref_int8_linear(p(dev[0]), p(dev[1]), p(dev[3]), p(dev[4]), p(dev[5]), p(out8), m, n, k, 0, stream()))
        check(lib, lib.ref_w4a8_linear(p(dev[0]), p(dev[2]), p(dev[3]), p(dev[4]), p(dev[5]), p(out4), m, n, k, 0, stream()))
        torch.cuda.synchronize()
        key = f"m{m}_n{n}_k{k}"
        gemm[f"{key}__a"] = a.numpy()
        gemm[f"{key}__w"] = w.numpy()
        gemm[f"{key}__w4_packed"] = packed.numpy()
        gemm[f"{key}__a_scale"] = a_s.numpy()
        gemm[f"{key}__w_scale"] = w_s.numpy()
        if bias is not None:
            gemm[f"{key}__bias"] = bias.numpy()
        gemm[f"{key}__int8_linear"] = out8.view(torch.int16).cpu().numpy().view(np.uint16)
        gemm[f"{key}__w4a8_linear"] = out4.view(torch.int16).cpu().numpy().view(np.uint16)

    # int32 accumulator -> bf16 (vector and scalar weight scale).
    g = torch.Generator().manual_seed(4400)
    acc = torch.randint(-(1 << 22), 1 << 22, (33, 64), generator=g, dtype=torch.int32)
    a_s = torch.rand((33,), generator=g) * 0.02
    w_s = torch.rand((64,), generator=g) * 0.02
    w_scalar = torch.tensor([0.0123])
    for tag, ws in (("vec", w_s), ("scalar", w_scalar)):
        o = torch.empty((33, 64), dtype=torch.bfloat16, device="cuda")
        accd, asd, wsd = acc.cuda(), a_s.cuda(), ws.cuda()
        check(lib, lib.ref_dequantize_int8_bf16(p(accd), p(asd), p(wsd), ws.numel(), p(o), 33, 64, 64, stream()))
        torch.cuda.synchronize()
        gemm[f"dequant_{tag}__out"] = o.view(torch.int16).cpu().numpy().view(np.uint16)
        gemm[f"dequant_{tag}__w_scale"] = ws.numpy()
    gemm["dequant__acc"] = acc.numpy()
    gemm["dequant__a_scale"] = a_s.numpy()
    np.savez_compressed(out / "gemm.npz", **gemm)
    print("golden vectors written to", out, file=sys.stderr)


if __name__ == "__main__":
    main()
