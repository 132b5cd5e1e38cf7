"""Both integer GEMM kernels -- single CTA (128 x 256 tiles) and CTA pair (256 x 256
tiles, tcgen05.mma.cta_group::2) -- against the oracle, for every operand format.

By default the library picks the pair kernel for M > 128; ``ctu_debug_set_gemm_kernel``
forces one kernel so each is checked at the tile edges of the other's shapes too.
"""

import ctypes

import numpy as np
import pytest
import torch

import convrot_oracle as oracle

pytestmark = pytest.mark.gpu

KERNELS = {"single": 1, "pair": 2}


@pytest.fixture(scope="module")
def C():
    from comfyui_turing_utils_kernel import _C, _lib

    _lib.device_error(0, clear=True)
    yield _C
    assert _lib.device_error(0, clear=True) == 0, "a kernel recorded a bounded-wait timeout"


@pytest.fixture(params=list(KERNELS))
def kernel(request):
    from comfyui_turing_utils_kernel import _lib

    prev = _lib.load().ctu_debug_set_gemm_kernel(KERNELS[request.param])
    assert prev >= 0
    yield request.param
    _lib.load().ctu_debug_set_gemm_kernel(0)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


SHAPES = [(1, 8, 16), (7, 16, 64), (128, 256, 128), (129, 264, 256), (255, 512, 384), (256, 256, 128),
          (257, 520, 1040), (600, 136, 1536), (1000, 1032, 5120)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_s32_matches_oracle(C, kernel, m, n, k):
    g = torch.Generator().manual_seed(11 * m + 5 * n + k)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8)
    acc = C.int8_gemm_s32(a.cuda(), w.cuda())
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), oracle.int8_gemm_s32(a.numpy(), w.numpy()))


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_w8a8_linear_matches_oracle(C, kernel, m, n, k):
    g = torch.Generator().manual_seed(3 * m + n + 7 * k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 1e-3
    w_s = torch.rand((n,), generator=g) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.02 if m % 2 else None
    out = C.turing_int8_linear(a.cuda(), w.cuda(), a_s.cuda(), w_s.cuda(), None if bias is None else bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.int8_linear(a.numpy(), w.numpy(), a_s.numpy(), w_s.numpy(), None if bias is None else bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)


@pytest.mark.parametrize("m,n,k", [s for s in SHAPES if s[2] % 32 == 0])
def test_w4a8_linear_matches_oracle(C, kernel, m, n, k):
    g = torch.Generator().manual_seed(5 * m + 3 * n + k)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 1e-3
    w_s = torch.rand((n,), generator=g) * 0.03 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.1
    wp = oracle.pack_int4(w.numpy())
    out = C.turing_w4a8_linear(a.cuda(), torch.from_numpy(wp).cuda(), a_s.cuda(), w_s.cuda(), bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.w4a8_linear(a.numpy(), wp, a_s.numpy(), w_s.numpy(), bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)


@pytest.mark.parametrize("m,n,k", [s for s in SHAPES if s[2] % 32 == 0])
def test_w4a4_linear_matches_oracle(C, kernel, m, n, k):
    g = torch.Generator().manual_seed(7 * m + n + 3 * k)
    a = torch.randint(-7, 8, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 1e-3
    w_s = torch.rand((n,), generator=g) * 0.03 + 1e-3
    ap, wp = oracle.pack_int4(a.numpy()), oracle.pack_int4(w.numpy())
    out = C.int4_linear(torch.from_numpy(ap).cuda(), torch.from_numpy(wp).cuda(), a_s.cuda(), w_s.cuda(), None)
    torch.cuda.synchronize()
    ref = oracle.w4a4_linear(ap, wp, a_s.numpy(), w_s.numpy(), None)
    assert np.array_equal(bf16_bits(out), ref)


def test_pair_and_single_agree_at_full_size(C):
    # Wan-14B FFN-down shape: both kernels must produce identical int32 accumulators.
    from comfyui_turing_utils_kernel import _lib

    m, n, k = 32760, 5120, 13824
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8, device="cuda")
    w = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8, device="cuda")
    try:
        _lib.load().ctu_debug_set_gemm_kernel(2)
        pair = C.int8_gemm_s32(a, w)
        _lib.load().ctu_debug_set_gemm_kernel(1)
        single = C.int8_gemm_s32(a, w)
    finally:
        _lib.load().ctu_debug_set_gemm_kernel(0)
    ref = torch._int_mm(a, w.t())
    torch.cuda.synchronize()
    assert torch.equal(pair, ref)
    assert torch.equal(single, ref)


def test_bounded_wait_stops_both_ctas(C, kernel):
    # The leader's MMA issuer waits on a barrier nothing arrives on; the timeout must
    # stop both CTAs of every pair (the abort is forwarded to the peer) and leave the
    # context usable.
    from comfyui_turing_utils_kernel import _lib

    m, n, k = 512, 512, 1024
    a = torch.ones((m, k), dtype=torch.int8, device="cuda")
    w = torch.ones((n, k), dtype=torch.int8, device="cuda")
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    _lib.device_error(0, clear=True)
    _lib.check(_lib.load().ctu_debug_gemm_injected_timeout(
        ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(acc.data_ptr()),
        m, n, k, 20_000_000, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    flags = _lib.device_error(0, clear=True)
    assert flags & 64
    acc2 = C.int8_gemm_s32(a, w)
    torch.cuda.synchronize()
    assert torch.all(acc2 == k)
    assert _lib.device_error(0, clear=True) == 0


def test_int4_unpack_matches_oracle(C):
    from comfyui_turing_utils_kernel import _C as cabi

    g = torch.Generator().manual_seed(17)
    v = torch.randint(-8, 8, (67, 1536), generator=g, dtype=torch.int8)
    packed = oracle.pack_int4(v.numpy())
    wide = cabi._widen_s4(torch.from_numpy(packed).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(wide.cpu().numpy(), v.numpy())


@pytest.mark.parametrize("mode", ["w4a8", "w4a4"])
def test_fused_w4_kernels_at_long_sequences(C, kernel, mode):
    # The op layer widens int4 operands from W4_WIDEN_MIN_ROWS rows on; the fused kernels
    # (int4 widened in shared memory) stay reachable through the C ABI at any M.
    import ctypes

    from comfyui_turing_utils_kernel import _lib

    m, n, k = 1000, 520, 1536
    g = torch.Generator().manual_seed(23)
    a = torch.randint(-128 if mode == "w4a8" else -7, 128 if mode == "w4a8" else 8, (m, k), generator=g,
                      dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 1e-3
    w_s = torch.rand((n,), generator=g) * 0.03 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.05
    wp = oracle.pack_int4(w.numpy())
    act = a.numpy() if mode == "w4a8" else oracle.pack_int4(a.numpy())
    dev = [torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in (act, wp, a_s.numpy(), w_s.numpy(), bias.numpy())]
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    fn = _lib.load().ctu_w4a8_linear if mode == "w4a8" else _lib.load().ctu_w4a4_linear
    _lib.check(fn(p(dev[0]), p(dev[1]), p(dev[2]), p(dev[3]), n, p(dev[4]), p(out), m, n, k,
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    if mode == "w4a8":
        ref = oracle.w4a8_linear(a.numpy(), wp, a_s.numpy(), w_s.numpy(), bias.numpy())
    else:
        ref = oracle.w4a4_linear(act, wp, a_s.numpy(), w_s.numpy(), bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)


# ----------------------------------------------------------------------------- half-width tail tiles
@pytest.mark.parametrize("m,n,k", [(257, 520, 1040), (600, 136, 1536), (1000, 1032, 5120), (4095, 5120, 512)])
@pytest.mark.parametrize("split", [1, 3, 10**6])
def test_pair_gemm_split_tiles_match_oracle(C, m, n, k, split):
    """The CTA-pair W8A8 kernel with its last `split` tiles run as two 256 x 128 halves
    (10**6: every tile) gives the oracle's bytes -- N tails that end inside the first
    or second half, M tails inside a tile -- and so does its int32 output."""
    from comfyui_turing_utils_kernel import _lib

    g = torch.Generator().manual_seed(13 * m + 7 * n + k + split % 97)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 1e-3
    w_s = torch.rand((n,), generator=g) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.02
    lib = _lib.load()
    prev_kernel = lib.ctu_debug_set_gemm_kernel(2)
    prev_split = lib.ctu_debug_set_gemm_split(split)
    try:
        out = C.turing_int8_linear(a.cuda(), w.cuda(), a_s.cuda(), w_s.cuda(), bias.cuda())
        acc = C.int8_gemm_s32(a.cuda(), w.cuda())
        torch.cuda.synchronize()
    finally:
        lib.ctu_debug_set_gemm_split(prev_split)
        lib.ctu_debug_set_gemm_kernel(prev_kernel)
    ref = oracle.int8_linear(a.numpy(), w.numpy(), a_s.numpy(), w_s.numpy(), bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)
    assert np.array_equal(acc.cpu().numpy(), oracle.int8_gemm_s32(a.numpy(), w.numpy()))


def test_pair_gemm_shard_shapes_split_automatically(C):
    """Row shards of the configs[1] linears at 2 and 8 GPUs (16380 and 4095 rows): the
    automatic tail split gives the same output as running every tile whole."""
    from comfyui_turing_utils_kernel import _lib

    lib = _lib.load()
    for m, n, k in ((4095, 5120, 5120), (16380, 5120, 5120), (4095, 5120, 13824)):
        g = torch.Generator(device="cuda").manual_seed(m + n + k)
        a = torch.randint(-127, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
        w = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
        a_s = torch.rand((m,), generator=g, device="cuda") * 0.02 + 1e-3
        w_s = torch.rand((n,), generator=g, device="cuda") * 0.009 + 1e-3
        bias = torch.randn((n,), generator=g, device="cuda") * 0.02
        auto = C.turing_int8_linear(a, w, a_s, w_s, bias)
        prev = lib.ctu_debug_set_gemm_split(0)
        try:
            whole = C.turing_int8_linear(a, w, a_s, w_s, bias)
        finally:
            lib.ctu_debug_set_gemm_split(prev)
        torch.cuda.synchronize()
        assert torch.equal(auto.view(torch.int16), whole.view(torch.int16)), (m, n, k)
