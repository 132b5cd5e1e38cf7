"""Parity of the B200 CUDA path with the reference (golden vectors) and the CPU oracle.

All calls go through the drop-in ``_C`` module, i.e. through libctu_b200.so's C ABI.
Integer outputs (codes, int32 accumulators) and the bf16 GEMM outputs must be bit-exact.
The GEMM epilogue is the reference build's fma(acc * a_s, w_s, bias) (the golden case
m64_n128_k256 pins the contraction); the 1-ulp bound checked before equality only makes
a failure's report say how far off it is.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import convrot_oracle as oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def C():
    from comfyui_turing_utils_kernel import _C, _lib

    _lib.device_error(0, clear=True)
    yield _C
    assert _lib.device_error(0, clear=True) == 0, "a kernel recorded a bounded-wait timeout"


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def activations(rows, width, seed, outlier_scale=30.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((rows, width), generator=g)
    idx = torch.randperm(width, generator=g)[: max(1, width // 100)]
    x[:, idx] *= outlier_scale
    return x.to(torch.bfloat16)


def ulp_diff(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 units in the last place (sign-magnitude aware)."""
    def key(b):
        b = b.astype(np.int32)
        return np.where(b & 0x8000, -(b & 0x7FFF), b & 0x7FFF)
    return np.abs(key(a_bits) - key(b_bits))


# ----------------------------------------------------------------------------- quantizer
QUANT = np.load(GOLDEN / "convrot_quant.npz")
QUANT_NAMES = sorted({k.split("__")[0] for k in QUANT.files})


def _run_quant(C, x_bits, bits, mode):
    x = to_bf16_tensor(x_bits).cuda()
    if mode == "gelu":
        fn = C.turing_bf16_gelu_int8_convrot_quantize if bits == 8 else C.turing_bf16_gelu_int4_convrot_quantize
        codes, scales = fn(x, 256)
    else:
        fn = C.turing_bf16_int8_convrot_quantize if bits == 8 else C.turing_bf16_int4_convrot_quantize
        codes, scales = fn(x, 256, mode == "swiglu")
    torch.cuda.synchronize()
    return codes.cpu().numpy(), scales.cpu().numpy().reshape(-1)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("name", QUANT_NAMES)
def test_quantize_matches_reference_golden(C, name, bits):
    mode = "swiglu" if "swiglu" in name else ("gelu" if name.startswith("gelu") else "plain")
    codes, scales = _run_quant(C, QUANT[f"{name}__x"], bits, mode)
    assert np.array_equal(codes, QUANT[f"{name}__int{bits}_codes"])
    assert np.array_equal(scales.view(np.uint32), QUANT[f"{name}__int{bits}_scales"].view(np.uint32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,k", [(1, 256), (3, 512), (17, 1536), (33, 5120), (5, 13824), (130, 768),
                                    (7, 2560), (64, 1024), (2, 16384)])
def test_quantize_matches_oracle(C, rows, k, bits):
    x = activations(rows, k, seed=rows * 131 + k)
    xb = bf16_bits(x)
    codes, scales = _run_quant(C, xb, bits, "plain")
    ref_codes, ref_scales = oracle.convrot_quantize(xb, bits)
    assert np.array_equal(codes, ref_codes)
    assert np.array_equal(scales.view(np.uint32), ref_scales.view(np.uint32))


@pytest.mark.parametrize("bits", [8, 4])
def test_quantize_swiglu_matches_oracle_codes(C, bits):
    x = activations(9, 2 * 1280, seed=5)
    xb = bf16_bits(x)
    codes, scales = _run_quant(C, xb, bits, "swiglu")
    ref_codes, ref_scales = oracle.convrot_quantize(xb, bits, oracle.MODE_SWIGLU)
    # expf differs by at most one ulp between CUDA and glibc: codes may move by one
    # step in rare positions, scales by one ulp.
    diff = np.abs(scales.view(np.int32).astype(np.int64) - ref_scales.view(np.int32).astype(np.int64))
    assert diff.max() <= 1
    if bits == 8:
        assert np.abs(codes.astype(np.int32) - ref_codes.astype(np.int32)).max() <= 1
        assert (codes != ref_codes).mean() < 1e-3


def test_quantize_zero_and_edge_rows(C):
    # validate_compatible.py:146-155: zero rows -> codes 0, int4 scale floor 1e-10.
    z = np.zeros((3, 512), dtype=np.uint16)
    codes, scales = _run_quant(C, z, 4, "plain")
    assert not codes.any() and np.all(scales == np.float32(1e-10))
    codes, scales = _run_quant(C, z, 8, "plain")
    assert not codes.any() and np.all(scales == np.float32(1e-30))


def test_quantize_large_m_rows_sample(C):
    # Full Wan-14B row count; compare a deterministic sample of rows with the oracle.
    rows, k = 32760, 5120
    x = activations(rows, k, seed=11).cuda()
    codes, scales = C.turing_bf16_int8_convrot_quantize(x, 256, False)
    torch.cuda.synchronize()
    sample = torch.tensor([0, 1, 127, 128, 4095, 16383, 32639, 32759])
    xb = bf16_bits(x[sample.cuda()])
    ref_codes, ref_scales = oracle.convrot_quantize(xb, 8)
    assert np.array_equal(codes[sample.cuda()].cpu().numpy(), ref_codes)
    assert np.array_equal(scales[sample.cuda()].cpu().numpy().reshape(-1).view(np.uint32), ref_scales.view(np.uint32))


def test_quantize_rejects_bad_width(C):
    x = torch.zeros((2, 300), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="divisible by 256"):
        C.turing_bf16_int8_convrot_quantize(x, 256, False)
    with pytest.raises(RuntimeError, match="group_size=256"):
        C.turing_bf16_int8_convrot_quantize(torch.zeros((2, 512), dtype=torch.bfloat16, device="cuda"), 128, False)


# ----------------------------------------------------------------------------- GEMM
GEMM = np.load(GOLDEN / "gemm.npz")
GEMM_KEYS = sorted({k.split("__")[0] for k in GEMM.files if k.startswith("m")})


@pytest.mark.parametrize("key", GEMM_KEYS)
def test_int8_linear_matches_reference_golden(C, key):
    a = torch.from_numpy(GEMM[f"{key}__a"]).cuda()
    w = torch.from_numpy(GEMM[f"{key}__w"]).cuda()
    a_s = torch.from_numpy(GEMM[f"{key}__a_scale"]).cuda()
    w_s = torch.from_numpy(GEMM[f"{key}__w_scale"]).cuda()
    bias = torch.from_numpy(GEMM[f"{key}__bias"]).cuda() if f"{key}__bias" in GEMM.files else None
    out = C.turing_int8_linear(a, w, a_s, w_s, bias)
    torch.cuda.synchronize()
    got = bf16_bits(out)
    ref = GEMM[f"{key}__int8_linear"]
    assert ulp_diff(got, ref).max() <= 1
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("key", GEMM_KEYS)
def test_w4a8_linear_matches_reference_golden(C, key):
    a = torch.from_numpy(GEMM[f"{key}__a"]).cuda()
    w4 = torch.from_numpy(GEMM[f"{key}__w4_packed"]).cuda()
    a_s = torch.from_numpy(GEMM[f"{key}__a_scale"]).cuda()
    w_s = torch.from_numpy(GEMM[f"{key}__w_scale"]).cuda()
    bias = torch.from_numpy(GEMM[f"{key}__bias"]).cuda() if f"{key}__bias" in GEMM.files else None
    out = C.turing_w4a8_linear(a, w4, a_s, w_s, bias)
    torch.cuda.synchronize()
    got, ref = bf16_bits(out), GEMM[f"{key}__w4a8_linear"]
    assert ulp_diff(got, ref).max() <= 1
    assert np.array_equal(got, ref)


# kernel/scripts/validate_compatible.py:158-201 edge cases (N and K tails, long M),
# plus full-width tiles; compared with the oracle (signed int4 unpack + exact GEMM).
@pytest.mark.parametrize("m,n,k", [(7, 13, 64), (3, 16, 12), (1, 8, 16), (17, 72, 80), (33, 128, 128),
                                   (129, 264, 256), (513, 520, 508), (513, 520, 64), (8193, 8, 16),
                                   (300, 512, 1536), (1024, 768, 5120)])
def test_w4a8_linear_matches_oracle(C, m, n, k):
    idx = [7, 3, 1, 17, 33, 129, 513, 5130, 8193, 300, 1024].index(m if (m, k) != (513, 64) else 5130)
    g = torch.Generator().manual_seed(4300 + idx)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 0.001
    w_s = torch.rand((n,), generator=g) * 0.03 + 0.001
    bias = torch.randn((n,), generator=g) * 0.1 if idx % 2 == 0 else None
    packed = oracle.pack_int4(w.numpy())
    out = C.turing_w4a8_linear(a.cuda(), torch.from_numpy(packed).cuda(), a_s.cuda(), w_s.cuda(),
                               None if bias is None else bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.w4a8_linear(a.numpy(), packed, a_s.numpy(), w_s.numpy(), None if bias is None else bias.numpy())
    got = bf16_bits(out)
    assert got.shape == (m, n)
    assert ulp_diff(got, ref).max() <= 1
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("m,n,k", [(1, 8, 16), (7, 16, 64), (33, 72, 128), (127, 264, 144), (129, 256, 512),
                                   (300, 520, 1040), (513, 1024, 5120), (256, 13824 // 54 * 2, 1536)])
def test_int8_gemm_s32_bit_exact(C, m, n, k):
    g = torch.Generator().manual_seed(m * 7 + n * 3 + k)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8)
    acc = C.int8_gemm_s32(a.cuda(), w.cuda())
    torch.cuda.synchronize()
    ref = oracle.int8_gemm_s32(a.numpy(), w.numpy())
    assert np.array_equal(acc.cpu().numpy(), ref)


@pytest.mark.parametrize("m,n,k,with_bias", [(1, 8, 16, True), (45, 136, 256, False), (200, 264, 1536, True),
                                             (1024, 768, 1536, True)])
def test_int8_linear_matches_oracle(C, m, n, k, with_bias):
    g = torch.Generator().manual_seed(m + n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 1e-3
    w_s = torch.rand((n,), generator=g) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.02 if with_bias else None
    out = C.turing_int8_linear(a.cuda(), w.cuda(), a_s.cuda(), w_s.cuda(), None if bias is None else bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.int8_linear(a.numpy(), w.numpy(), a_s.numpy(), w_s.numpy(), None if bias is None else bias.numpy())
    got = bf16_bits(out)
    assert ulp_diff(got, ref).max() <= 1
    assert np.array_equal(got, ref)


def test_int8_gemm_full_size_against_cublas(C):
    # Wan-14B QKV shape: the int32 accumulators must equal an independent exact
    # contraction (cuBLASLt int8 through torch._int_mm) everywhere.
    m, n, k = 32760, 5120, 5120
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8, device="cuda")
    w = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8, device="cuda")
    acc = C.int8_gemm_s32(a, w)
    ref = torch._int_mm(a, w.t())
    torch.cuda.synchronize()
    assert torch.equal(acc, ref)


def test_int8_linear_rejects_bad_shapes(C):
    a = torch.zeros((4, 24), dtype=torch.int8, device="cuda")
    w = torch.zeros((8, 24), dtype=torch.int8, device="cuda")
    s = torch.ones(4, device="cuda")
    with pytest.raises(RuntimeError, match="K%16=0"):
        C.turing_int8_linear(a, w, s, torch.ones(8, device="cuda"))


@pytest.mark.parametrize("tag", ["vec", "scalar"])
def test_dequantize_matches_reference_golden(C, tag):
    acc = torch.from_numpy(GEMM["dequant__acc"]).cuda()
    out = C.turing_dequantize_int8_bf16(acc, torch.from_numpy(GEMM["dequant__a_scale"]).cuda(),
                                        torch.from_numpy(GEMM[f"dequant_{tag}__w_scale"]).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(bf16_bits(out), GEMM[f"dequant_{tag}__out"])


def test_quantize_then_gemm_matches_oracle_end_to_end(C):
    m, k, n = 257, 1536, 512
    x = activations(m, k, seed=21)
    g = torch.Generator().manual_seed(22)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    w_s = torch.rand((n,), generator=g) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.02
    q, s = C.turing_bf16_int8_convrot_quantize(x.cuda(), 256, False)
    out = C.turing_int8_linear(q, w.cuda(), s, w_s.cuda(), bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.convrot_w8a8_linear(bf16_bits(x), w.numpy(), w_s.numpy(), bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)


def test_gemm_bounded_wait_reports_and_context_survives(C):
    # Failure detection without a GPU fault: the MMA issuer waits on a barrier that
    # nothing arrives on; the bounded wait expires, the kernel records flag 64 and
    # exits cleanly, and the context keeps working.
    import ctypes

    from comfyui_turing_utils_kernel import _lib

    a = torch.ones((128, 128), dtype=torch.int8, device="cuda")
    w = torch.ones((256, 128), dtype=torch.int8, device="cuda")
    acc = torch.empty((128, 256), dtype=torch.int32, device="cuda")
    _lib.device_error(0, clear=True)
    _lib.check(_lib.load().ctu_debug_gemm_injected_timeout(
        ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(acc.data_ptr()),
        128, 256, 128, 20_000_000, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    flags = _lib.device_error(0, clear=True)
    assert flags & 64
    acc2 = C.int8_gemm_s32(a, w)
    torch.cuda.synchronize()
    assert torch.all(acc2 == 128)
    assert _lib.device_error(0, clear=True) == 0


# ----------------------------------------------------------------------------- W4A4 and dispatch
@pytest.mark.parametrize("m,n,k", [(1, 8, 32), (33, 72, 256), (130, 264, 1536), (513, 520, 5120), (7, 13, 64)])
def test_w4a4_linear_matches_oracle(C, m, n, k):
    g = torch.Generator().manual_seed(m * 3 + n + k)
    a4 = torch.randint(-7, 8, (m, k), generator=g, dtype=torch.int8)
    w4 = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 1e-3
    w_s = torch.rand((n,), generator=g) * 0.03 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.05
    ap, wp = oracle.pack_int4(a4.numpy()), oracle.pack_int4(w4.numpy())
    out = C.int4_linear(torch.from_numpy(ap).cuda(), torch.from_numpy(wp).cuda(), a_s.cuda(), w_s.cuda(), bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.w4a4_linear(ap, wp, a_s.numpy(), w_s.numpy(), bias.numpy())
    got = bf16_bits(out)
    assert ulp_diff(got, ref).max() <= 1
    assert np.array_equal(got, ref)


def _dispatch():
    import comfyui_turing_utils_b200 as d

    return d


def test_dispatch_int8_linear_matches_oracle_3d(C):
    d = _dispatch()
    b, s, k, n = 2, 97, 1536, 264
    x = activations(b * s, k, seed=31)
    g = torch.Generator().manual_seed(32)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    w_s = torch.rand((n,), generator=g) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.02
    out = d.int8_linear(x.reshape(b, s, k).cuda(), w.cuda(), w_s.cuda(), bias.cuda(), convrot=True)
    torch.cuda.synchronize()
    assert out.shape == (b, s, n) and out.dtype == torch.bfloat16
    ref = oracle.convrot_w8a8_linear(bf16_bits(x), w.numpy(), w_s.numpy(), bias.numpy())
    assert np.array_equal(bf16_bits(out.reshape(b * s, n)), ref)
    # scalar weight scale is expanded like dispatch.py:629-648
    out1 = d.int8_linear(x.cuda(), w.cuda(), torch.tensor([0.004]).cuda(), None, convrot=True)
    ref1 = oracle.convrot_w8a8_linear(bf16_bits(x), w.numpy(), np.full((n,), 0.004, np.float32), None)
    assert np.array_equal(bf16_bits(out1), ref1)


@pytest.mark.parametrize("linear_dtype", ["int8", "int4"])
def test_dispatch_convrot_w4a4_linear(C, linear_dtype):
    d = _dispatch()
    m, k, n = 65, 1024, 136
    x = activations(m, k, seed=41)
    g = torch.Generator().manual_seed(42)
    w4 = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    wp = oracle.pack_int4(w4.numpy())
    w_s = torch.rand((n,), generator=g) * 0.03 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.05
    out = d.convrot_w4a4_linear(x.cuda(), torch.from_numpy(wp).cuda(), w_s.cuda(), bias.cuda(),
                                linear_dtype=linear_dtype)
    torch.cuda.synchronize()
    bits = 8 if linear_dtype == "int8" else 4
    codes, scales = oracle.convrot_quantize(bf16_bits(x), bits)
    if bits == 8:
        ref = oracle.w4a8_linear(codes, wp, scales, w_s.numpy(), bias.numpy())
    else:
        ref = oracle.w4a4_linear(codes, wp, scales, w_s.numpy(), bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)


def test_w8_output_slices_reassemble_the_linear(C):
    # fusions.py:56-85: a W8 linear evaluated as contiguous output-channel intervals
    # from one quantized activation equals the whole linear, for per-channel and
    # scalar weight scales.
    d = _dispatch()
    m, k, n = 300, 1536, 520
    x = activations(m, k, seed=51).cuda()
    g = torch.Generator().manual_seed(52)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).cuda()
    bias = (torch.randn((n,), generator=g) * 0.02).cuda()
    q, s = d.quantize_convrot_int8_activation(x)
    for w_s in ((torch.rand((n,), generator=g) * 0.009 + 1e-3).cuda(), torch.tensor([0.004]).cuda()):
        full = d.int8_linear_from_quantized(q, s, w, w_s, bias)
        cuts = [0, 8, 264, 448, n]
        parts = [d.convrot_w8_output_slice(q, s, w, w_s, bias, a, b, torch.bfloat16) for a, b in zip(cuts, cuts[1:])]
        torch.cuda.synchronize()
        assert torch.equal(torch.cat(parts, dim=1), full)


def test_linears_capture_into_a_cuda_graph(C):
    # The reference requires capture safety (no sync, no allocation inside capture,
    # w4a8.cu:308-312).  After a first call per shape (which resolves launch attributes
    # and the error word), quantize + GEMM for W8A8, widened W4A8 and codebook W4A8
    # capture into one graph whose replays equal the eager results.
    d = _dispatch()
    m, k, n = 600, 1536, 264
    x = activations(m, k, seed=61).cuda()
    g = torch.Generator().manual_seed(62)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).cuda()
    w4 = torch.from_numpy(oracle.pack_int4(torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8).numpy())).cuda()
    w_s = (torch.rand((n,), generator=g) * 0.009 + 1e-3).cuda()
    bias = (torch.randn((n,), generator=g) * 0.02).cuda()

    def run():
        q, s = C.turing_bf16_int8_convrot_quantize(x, 256, False)
        return (C.turing_int8_linear(q, w, s, w_s, bias), C.turing_w4a8_linear(q, w4, s, w_s, bias),
                d.int8_linear(x, w, w_s, bias, convrot=True))

    eager = run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run()  # warm the caching allocator on the capture stream
    torch.cuda.current_stream().wait_stream(side)
    with torch.cuda.graph(graph):
        captured = run()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, captured):
        assert torch.equal(a, b)


def test_dispatch_preflights_and_scaled_swiglu_helper(C):
    # dispatch.py:88-199 self-tests pass on the B200 ops; dispatch.py:450-465 quantizes
    # a SwiGLU channel shard with whole-row scales, which must reproduce the codes of
    # the unscaled op for the scales it computed.
    d = _dispatch()
    d.preflight_w4a8(torch.device("cuda", 0))
    d.preflight_codebook_w4a8(torch.device("cuda", 0))
    assert d.convrot_swiglu_channel_sharding_available()
    m, half = 37, 1024
    x = activations(m, 2 * half, seed=71).cuda()
    q_full, s_full = d.quantize_convrot_swiglu_activation(x)
    gate, up = x[:, :half], x[:, half:]
    shard = torch.cat([gate[:, 256:768], up[:, 256:768]], dim=1)
    q_shard = d.quantize_convrot_swiglu_with_scale(shard, s_full)
    torch.cuda.synchronize()
    assert torch.equal(q_shard, q_full[:, 256:768])
