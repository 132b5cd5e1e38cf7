"""The fused ConvRot W8A8 linear (ctu_convrot_int8_linear): quantizer warps inside the
CTA-pair GEMM publish finished 128-row blocks that the GEMM then loads (forced on here
wherever it applies; by default it runs where it measured faster).  Its codes, scales
and bf16 outputs must equal, bit for bit, the reference path the plugin composes
(dispatch.py:748-800: turing_bf16_int8_convrot_quantize, then turing_int8_linear) and the
oracle -- at every groups-per-team variant (K up to 5120), ragged M and N, rows with NaN,
infinities and large magnitudes, half-tile splits, and the full Wan-14B shapes.
"""

import numpy as np
import pytest
import torch

import convrot_oracle as oracle
from test_gpu_quant_variants import activations, bf16_bits, large_rows, special_rows, to_bf16_tensor

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from comfyui_turing_utils_kernel import _C, _lib

    _lib.device_error(0, clear=True)
    yield _C
    assert _lib.device_error(0, clear=True) == 0, "a kernel recorded a bounded-wait timeout"


@pytest.fixture(params=["fused", "separate"])
def path(request):
    from comfyui_turing_utils_kernel import _lib

    prev = _lib.load().ctu_debug_set_fused_linear(1 if request.param == "separate" else 2)
    assert prev >= 0
    yield request.param
    _lib.load().ctu_debug_set_fused_linear(0)


def weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    w_s = torch.rand((n,), generator=g) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.02
    return w, w_s, bias


def two_ops(C, x, w, w_s, bias):
    codes, scales = C.turing_bf16_int8_convrot_quantize(x, 256)
    out = C.turing_int8_linear(codes, w, scales, w_s, bias)
    return out, codes, scales


# (m, n, k): k covers every groups-per-team variant of the fused kernel (1..5 groups per
# team, partially filled teams at 9 and 19 groups), m straddles 128-row blocks and
# 256-row pair tiles, n straddles 256- and 128-column tiles.
SHAPES = [(129, 256, 256), (300, 264, 1280), (513, 392, 2304), (256, 520, 3072), (1000, 1032, 4096),
          (257, 136, 4864), (777, 5120, 5120), (4095, 5120, 5120)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_matches_two_ops_and_oracle(C, path, m, n, k):
    x = activations(m, k, seed=m + 3 * k).cuda()
    w, w_s, bias = (t.cuda() for t in weights(n, k, seed=n + k))
    bias = bias if m % 2 else None
    out, codes, scales = C.convrot_int8_linear(x, w, w_s, bias, return_quantized=True)
    ref_out, ref_codes, ref_scales = two_ops(C, x, w, w_s, bias)
    torch.cuda.synchronize()
    assert torch.equal(codes, ref_codes)
    assert torch.equal(scales.view(torch.int32), ref_scales.view(torch.int32))
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
    if m * k <= 1000 * 4096:
        xb = bf16_bits(x)
        oc, os_ = oracle.convrot_quantize(xb, 8)
        assert np.array_equal(codes.cpu().numpy(), oc)
        ref = oracle.int8_linear(oc, w.cpu().numpy(), os_, w_s.cpu().numpy(),
                                 None if bias is None else bias.cpu().numpy())
        assert np.array_equal(bf16_bits(out), ref)


@pytest.fixture()
def fused():
    from comfyui_turing_utils_kernel import _lib

    prev = _lib.load().ctu_debug_set_fused_linear(2)
    yield
    _lib.load().ctu_debug_set_fused_linear(prev)


@pytest.mark.parametrize("rows_fn", [special_rows, large_rows], ids=["special", "large"])
def test_special_and_large_rows(C, fused, rows_fn):
    m, n, k = 300, 264, 5120
    xb = rows_fn(m, k, seed=17)
    x = to_bf16_tensor(xb).cuda()
    w, w_s, bias = (t.cuda() for t in weights(n, k, seed=5))
    out, codes, scales = C.convrot_int8_linear(x, w, w_s, bias, return_quantized=True)
    ref_out, ref_codes, ref_scales = two_ops(C, x, w, w_s, bias)
    torch.cuda.synchronize()
    oc, os_ = oracle.convrot_quantize(xb, 8)
    assert np.array_equal(codes.cpu().numpy(), oc)
    assert np.array_equal(scales.cpu().numpy().reshape(-1).view(np.uint32), os_.view(np.uint32))
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))


@pytest.mark.parametrize("split", [0, 3, 20])
def test_half_tile_splits(C, fused, split):
    from comfyui_turing_utils_kernel import _lib

    m, n, k = 1100, 1280, 5120
    x = activations(m, k, seed=split + 1).cuda()
    w, w_s, bias = (t.cuda() for t in weights(n, k, seed=split + 2))
    ref_out, _, _ = two_ops(C, x, w, w_s, bias)
    prev = _lib.load().ctu_debug_set_gemm_split(split)
    try:
        out = C.convrot_int8_linear(x, w, w_s, bias)
    finally:
        _lib.load().ctu_debug_set_gemm_split(prev)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))


def test_repeated_calls_and_changing_rows(C, fused):
    # The progress counters are cleared on the stream before every launch.
    n, k = 520, 5120
    w, w_s, bias = (t.cuda() for t in weights(n, k, seed=9))
    for m in (4095, 129, 1000, 4095, 257):
        x = activations(m, k, seed=m).cuda()
        out = C.convrot_int8_linear(x, w, w_s, bias)
        ref_out, _, _ = two_ops(C, x, w, w_s, bias)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16)), m


def test_graph_replay(C, fused):
    m, n, k = 2048, 1024, 5120
    x = activations(m, k, seed=3).cuda()
    w, w_s, bias = (t.cuda() for t in weights(n, k, seed=4))
    ref_out, _, _ = two_ops(C, x, w, w_s, bias)
    C.convrot_int8_linear(x, w, w_s, bias)  # allocations and tensor maps before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = C.convrot_int8_linear(x, w, w_s, bias)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
    del graph


def test_rejects_bad_inputs(C):
    w = torch.zeros((8, 256), dtype=torch.int8, device="cuda")
    s = torch.ones(8, device="cuda")
    with pytest.raises(RuntimeError):  # width not a multiple of 256
        C.convrot_int8_linear(torch.zeros((4, 128), dtype=torch.bfloat16, device="cuda"), w[:, :128].contiguous(), s)
    with pytest.raises(RuntimeError):  # fp16 rows
        C.convrot_int8_linear(torch.zeros((4, 256), dtype=torch.float16, device="cuda"), w, s)
    with pytest.raises(RuntimeError):  # N not a multiple of 8
        C.convrot_int8_linear(torch.zeros((4, 256), dtype=torch.bfloat16, device="cuda"), w[:6].contiguous(), s[:6])


@pytest.mark.parametrize("k,n", [(5120, 5120), (5120, 13824)], ids=["qkvo", "ffn_up"])
def test_full_size_wan14b(C, path, k, n):
    m = 32760
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(n)
    x = torch.randn((m, k), generator=g, device=dev)
    x[:, torch.randperm(k, generator=g, device=dev)[: k // 100]] *= 30.0
    x = x.to(torch.bfloat16)
    w = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
    w_s = torch.rand((n,), generator=g, device=dev) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g, device=dev) * 0.02
    out, codes, scales = C.convrot_int8_linear(x, w, w_s, bias, return_quantized=True)
    ref_out, ref_codes, ref_scales = two_ops(C, x, w, w_s, bias)
    torch.cuda.synchronize()
    assert torch.equal(codes, ref_codes)
    assert torch.equal(scales.view(torch.int32), ref_scales.view(torch.int32))
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
