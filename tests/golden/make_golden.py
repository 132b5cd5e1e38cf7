"""Generate golden vectors from the REFERENCE kernels (run on a B200 box).

Loads ``oracle/_ref/libctu_ref.so`` -- the reference's own ConvRot quantizers, W8A8
and W4A8 GEMMs, int32->bf16 epilogue and norm + AdaLN kernels (kernel/csrc/turing/
{convrot_quant,w4a8,bf16_epilogue,segmented_rms_adaln}.cu of comfyui-turing-utils
0.31.0), compiled from the reference tree
by ``oracle/Makefile`` -- runs them on seeded inputs and writes compressed ``.npz``
fixtures.  The fixtures are committed under ``tests/golden/`` and pin the CPU oracle
(``oracle/convrot_oracle.py``) in the CPU test suite.

Usage (on a B200):  python tests/golden/make_golden.py --out <directory> [--only extras|norms|staged|gemm]
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
    f32 = ctypes.c_float
    lib.ref_segmented_rms_adaln.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32, i32, vp]
    lib.ref_layer_norm_adaln.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, f32, i32, vp]
    lib.ref_staged_convrot_quantize.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]
    lib.ref_swiglu_int8_convrot_quantize_scaled_f16.argtypes = [vp, vp, vp, i32, i32, vp]
    for name in ("ref_bf16_convrot_quantize", "ref_bf16_gelu_convrot_quantize", "ref_int8_linear",
                 "ref_w4a8_linear", "ref_dequantize_int8_bf16", "ref_codebook_w4a8_linear",
                 "ref_swiglu_int8_convrot_quantize_scaled", "ref_segmented_rms_adaln", "ref_layer_norm_adaln",
                 "ref_staged_convrot_quantize", "ref_swiglu_int8_convrot_quantize_scaled_f16"):
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


# ----------------------------------------------------------------------------- norms
NORM_TORCH = {0: torch.bfloat16, 1: torch.float16, 2: torch.float32}

# (name, dtype code, rows, hidden, param_rows, scale_stride, x_offset, segments, epsilon)
# segments: (start, stop, row) triples; rows outside every segment and rows mapped
# past param_rows fall back to parameter row 0 in the reference kernel.
RMS_CASES = [
    ("bf16_h1024", 0, 37, 1024, 3, 1024, 0, [(0, 5, 2), (5, 20, 0), (20, 37, 1)], 1e-5),
    ("bf16_h5376_minimax", 0, 9, 5376, 2, 5376, 0, [(0, 4, 1), (4, 9, 0)], 1e-6),
    ("bf16_h200_gap", 0, 12, 200, 2, 200, 0, [(0, 3, 1), (5, 9, 7), (9, 12, 1)], 1e-5),
    ("bf16_h1001_scalar", 0, 10, 1001, 2, 1001, 0, [(0, 10, 1)], 1e-5),
    ("bf16_h1024_stride1040", 0, 11, 1024, 3, 1040, 0, [(0, 4, 2), (4, 11, 1)], 1e-5),
    ("bf16_h1024_stride1036_scalar", 0, 11, 1024, 3, 1036, 0, [(0, 11, 2)], 1e-5),
    ("bf16_h1024_broadcast", 0, 8, 1024, 4, 0, 0, [(0, 8, 3)], 1e-5),
    ("bf16_h1024_misaligned", 0, 9, 1024, 2, 1024, 1, [(0, 9, 1)], 1e-5),
    ("bf16_h20480_tail", 0, 3, 20480, 1, 20480, 0, [(0, 3, 0)], 1e-5),
    ("fp16_h1024", 1, 13, 1024, 2, 1024, 0, [(0, 6, 1), (6, 13, 0)], 1e-5),
    ("fp16_h970_scalar", 1, 7, 970, 1, 970, 0, [(0, 7, 0)], 1e-5),
    ("fp32_h1024", 2, 13, 1024, 2, 1024, 0, [(0, 6, 1), (6, 13, 0)], 1e-5),
    ("fp32_h1002_scalar", 2, 7, 1002, 1, 1002, 0, [(0, 7, 0)], 1e-5),
    ("fp32_h9000_tail", 2, 3, 9000, 1, 9000, 0, [(0, 3, 0)], 1e-5),
]

# (name, dtype code, batch, sequence, hidden, modulation_steps, epsilon, input transform)
LN_CASES = [
    ("bf16_b2_s17_h1024", 0, 2, 17, 1024, 4, 1e-6, "plain"),
    ("bf16_offset100", 0, 2, 17, 1024, 4, 1e-6, "offset100"),
    ("bf16_offset1000", 0, 2, 17, 1024, 4, 1e-6, "offset1000"),
    ("bf16_small", 0, 1, 9, 1024, 1, 1e-6, "eighth"),
    ("bf16_h200", 0, 2, 5, 200, 5, 1e-5, "plain"),
    ("bf16_h5120_wan", 0, 1, 6, 5120, 1, 1e-6, "plain"),
    ("bf16_h1001_steps_gt_seq", 0, 1, 3, 1001, 5, 1e-5, "plain"),
    ("bf16_h20000_tail", 0, 1, 2, 20000, 2, 1e-6, "offset100"),
    ("bf16_h30000_wide", 0, 1, 3, 30000, 1, 1e-5, "plain"),
    ("fp16_b2_s7_h1024", 1, 2, 7, 1024, 3, 1e-5, "plain"),
    ("fp32_b2_s7_h1024", 2, 2, 7, 1024, 3, 1e-5, "offset1000"),
    ("fp32_h300", 2, 1, 4, 300, 2, 1e-5, "plain"),
]


def _norm_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def norm_special_rows(x: torch.Tensor) -> torch.Tensor:
    """Rows 0-3 of a norm input: zeros, a NaN, an infinity, values whose squares overflow."""
    x = x.clone()
    if x.shape[0] >= 4:
        x[0] = 0
        x[1, 3] = float("nan")
        x[2, 5] = float("inf")
        x[3] = x[3].sign() * (3.0e38 if x.dtype != torch.float16 else 6.0e4)
    return x


def norm_cases(lib, out):
    norms = {}
    for idx, (name, code, rows, hidden, prow, stride, off, segs, eps) in enumerate(RMS_CASES):
        dt = NORM_TORCH[code]
        g = torch.Generator().manual_seed(6000 + idx)
        x = (torch.randn((rows, hidden), generator=g) * 1.5).to(dt)
        if idx == 0:
            x = norm_special_rows(x)
        w = (torch.randn((hidden,), generator=g) * 0.5 + 1.0).to(dt)
        width = max(stride, hidden) if stride else hidden
        scale = (torch.randn((prow if stride else 1, width), generator=g) * 0.1).to(dt)
        shift = (torch.randn((prow if stride else 1, width), generator=g) * 0.1).to(dt)
        seg = torch.tensor(segs, dtype=torch.int32)
        xbuf = torch.zeros(rows * hidden + 8, dtype=dt, device="cuda")
        xbuf[off:off + rows * hidden] = x.flatten().cuda()
        xd = xbuf[off:off + rows * hidden]
        wd, sd, hd, segd = w.cuda(), scale.cuda(), shift.cuda(), seg.cuda()
        o = torch.empty((rows, hidden), dtype=dt, device="cuda")
        check(lib, lib.ref_segmented_rms_adaln(p(xd), p(wd), p(sd), p(hd), p(segd), p(o), rows, hidden, prow, stride,
                                               stride, len(segs), eps, code, stream()))
        torch.cuda.synchronize()
        key = f"rms_{name}"
        norms[f"{key}__meta"] = np.array([code, rows, hidden, prow, stride, off], dtype=np.int64)
        norms[f"{key}__eps"] = np.array([eps], dtype=np.float32)
        norms[f"{key}__x"] = _norm_np(x)
        norms[f"{key}__weight"] = _norm_np(w)
        norms[f"{key}__scale"] = _norm_np(scale)
        norms[f"{key}__shift"] = _norm_np(shift)
        norms[f"{key}__segments"] = seg.numpy()
        norms[f"{key}__out"] = _norm_np(o)
    for idx, (name, code, batch, seq, hidden, steps, eps, transform) in enumerate(LN_CASES):
        dt = NORM_TORCH[code]
        g = torch.Generator().manual_seed(6500 + idx)
        x = torch.randn((batch, seq, hidden), generator=g)
        x = {"plain": x, "offset100": x + 100.0, "offset1000": x + 1000.0, "eighth": x * 0.125}[transform].to(dt)
        if idx == 0:
            x = norm_special_rows(x.view(batch * seq, hidden)).view(batch, seq, hidden)
            x[1, 4] = 2.5  # a constant row: zero variance
        scale = (torch.randn((batch, steps, hidden), generator=g) * 0.1).to(dt)
        shift = (torch.randn((batch, steps, hidden), generator=g) * 0.1).to(dt)
        xd, sd, hd = x.cuda(), scale.cuda(), shift.cuda()
        o = torch.empty_like(xd)
        check(lib, lib.ref_layer_norm_adaln(p(xd), p(sd), p(hd), p(o), batch, seq, hidden, steps, eps, code, stream()))
        torch.cuda.synchronize()
        key = f"ln_{name}"
        norms[f"{key}__meta"] = np.array([code, batch, seq, hidden, steps], dtype=np.int64)
        norms[f"{key}__eps"] = np.array([eps], dtype=np.float32)
        norms[f"{key}__x"] = _norm_np(x)
        norms[f"{key}__scale"] = _norm_np(scale)
        norms[f"{key}__shift"] = _norm_np(shift)
        norms[f"{key}__out"] = _norm_np(o)
    np.savez_compressed(out / "norms.npz", **norms)


# The reference's staged quantizers (SwiGLU and GELU, int8 and int4) on special and
# random rows: (name, act, k, rows of special values, random rows).
STAGED_CASES = [("swiglu_k256", 1, 256), ("swiglu_k5120", 1, 5120), ("swiglu_k13824", 1, 13824),
                ("gelu_k256", 2, 256), ("gelu_k5120", 2, 5120), ("gelu_k13824", 2, 13824)]


def staged_cases(lib, out):
    staged = {}
    for fp16 in (False, True):
        for idx, (name, act, k) in enumerate(STAGED_CASES):
            if fp16 and k == 13824:
                continue
            width = 2 * k if act == 1 else k
            x = activations(24, width, 6900 + idx).float()
            special = special_rows(width).float()
            x[: special.shape[0]] = special[: x.shape[0]]
            if fp16:
                x[4:8] = x[4:8].clamp(-7e4, 7e4)  # values past 65504 become infinities in fp16
                x[11] = x[11] * 2.0e-6             # fp16 subnormal range
            x = x.to(torch.float16 if fp16 else torch.bfloat16)
            xd = x.cuda().contiguous()
            rows = x.shape[0]
            key = f"{'f16_' if fp16 else ''}{name}"
            staged[f"{key}__x"] = x.view(torch.int16).numpy().view(np.uint16)
            for bits in (8, 4):
                codes = torch.empty((rows, k // 2 if bits == 4 else k), dtype=torch.int8, device="cuda")
                scales = torch.empty((rows, 1), dtype=torch.float32, device="cuda")
                rotated = torch.empty((rows, k), dtype=x.dtype, device="cuda")
                partial = torch.empty((rows, k // 256), dtype=torch.float32, device="cuda")
                check(lib, lib.ref_staged_convrot_quantize(p(xd), p(codes), p(scales), p(rotated), p(partial), rows,
                                                           k, bits, act, 1 if fp16 else 0, stream()))
                torch.cuda.synchronize()
                staged[f"{key}__int{bits}_codes"] = codes.cpu().numpy()
                staged[f"{key}__int{bits}_scales"] = scales.cpu().numpy().reshape(-1)
    # fp16 SwiGLU shard with caller-supplied scales (special scales included).
    rows, k = 8, 512
    x = activations(rows, 2 * k, 6990).float().to(torch.float16)
    scales = torch.tensor([0.05, 0.0, float("nan"), float("inf"), -0.02, 1e-9, 7e4, 0.013], dtype=torch.float32)
    codes = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    check(lib, lib.ref_swiglu_int8_convrot_quantize_scaled_f16(p(x.cuda()), p(scales.cuda()), p(codes), rows, k,
                                                               stream()))
    torch.cuda.synchronize()
    staged["scaled_f16__x"] = x.view(torch.int16).numpy().view(np.uint16)
    staged["scaled_f16__scales"] = scales.numpy()
    staged["scaled_f16__codes"] = codes.cpu().numpy()
    np.savez_compressed(out / "staged.npz", **staged)


def gemm_cases(lib, out: Path) -> None:
    """W8A8 / W4A8 GEMMs (w4a8.cu:1000-1086, 1185-1219) and the int32 epilogue
    (bf16_epilogue.cu:146-217) -> gemm.npz."""
    gemm = {}
    for idx, (m, n, k, with_bias) in enumerate([(33, 64, 256, True), (17, 72, 128, False),
                                                (130, 136, 512, True), (1, 16, 64, False),
                                                (64, 128, 256, "cancel")]):
        g = torch.Generator().manual_seed(4300 + idx)
        a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
        w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
        w4 = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
        a_s = torch.rand((m,), generator=g) * 0.02 + 0.001
        w_s = torch.rand((n,), generator=g) * 0.009 + 0.001
        bias = (torch.randn((n,), generator=g) * 0.02) if with_bias else None
        if with_bias == "cancel":
            # Column j's bias cancels the separately rounded product of row j % m, so
            # that output is the product's rounding error under a fused multiply-add
            # and zero without one: the case pins the epilogue's contraction.
            acc = (a.to(torch.int64) @ w.to(torch.int64).t()).numpy().astype(np.float32)
            prod = (acc * a_s.numpy()[:, None]) * w_s.numpy()[None, :]
            bias = torch.from_numpy(-prod[np.arange(n) % m, np.arange(n)].astype(np.float32))
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--only", choices=["all", "extras", "norms", "staged", "gemm"], default="all")
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    lib = load_ref()
    torch.cuda.init()
    if args.only == "gemm":
        gemm_cases(lib, out)
        print("golden vectors written to", out, file=sys.stderr)
        return
    if args.only in ("all", "staged"):
        staged_cases(lib, out)
    if args.only == "staged":
        print("golden vectors written to", out, file=sys.stderr)
        return
    if args.only in ("all", "norms"):
        norm_cases(lib, out)
    if args.only == "norms":
        print("golden vectors written to", out, file=sys.stderr)
        return
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

    gemm_cases(lib, out)
    print("golden vectors written to", out, file=sys.stderr)


if __name__ == "__main__":
    main()
