"""Per-group (128 along K) formats: the per-token-per-group int4 ConvRot quantizer, the
asymmetric uint4 W4A8 linear (fp16 scale + uint4 zero point per group) and the W4A4
linear with per-token-per-group activation scales, against the oracle, bit for bit.

The reference runs these through comfy-kitchen (dispatch.py:876-936), whose source is not
available: parity is against this build's oracle definition (unpinned), while the int32
group partials inside it are exact arithmetic.
"""

import numpy as np
import pytest
import torch

import convrot_oracle as oracle
from test_gpu_quant_variants import activations, bf16_bits, large_rows, special_rows, tiny_rows, to_bf16_tensor

pytestmark = pytest.mark.gpu

SHAPES = [(1, 8, 128), (7, 16, 256), (129, 200, 384), (255, 192, 512), (256, 384, 1024), (257, 392, 1280),
          (600, 136, 1536), (1000, 1032, 5120)]


@pytest.fixture(scope="module")
def K():
    import comfyui_turing_utils_kernel as K
    from comfyui_turing_utils_kernel import _lib

    _lib.device_error(0, clear=True)
    yield K
    assert _lib.device_error(0, clear=True) == 0, "a kernel recorded a bounded-wait timeout"


@pytest.fixture(params=["single", "pair"])
def tiling(request):
    """The per-group GEMM's tiling, forced through the GEMM-kernel test hook: 128 x 128
    tiles on single CTAs (1) or 256 x 128 tiles on CTA pairs (2)."""
    from comfyui_turing_utils_kernel import _lib

    prev = _lib.load().ctu_debug_set_gemm_kernel(1 if request.param == "single" else 2)
    yield request.param
    _lib.load().ctu_debug_set_gemm_kernel(prev)


def quantize(K, xb, block=256):
    codes, scales = K.turing_bf16_int4_g128_convrot_quantize(to_bf16_tensor(xb).cuda(), block)
    torch.cuda.synchronize()
    return codes.cpu().numpy(), scales.cpu().numpy()


def check_quant(K, xb, block=256):
    codes, scales = quantize(K, xb, block)
    ref_codes, ref_scales = oracle.convrot_quantize_int4_g128(xb, block)
    assert np.array_equal(codes, ref_codes)
    assert np.array_equal(scales.view(np.uint32), ref_scales.view(np.uint32))


# block: the rotation block -- 256 (the reference's rotation) or 128 (this build's block-128
# rotation, the block the benchmark's configs name).
@pytest.mark.parametrize("block", [256, 128])
@pytest.mark.parametrize("rows,k", [(1, 256), (7, 512), (33, 1280), (129, 5120), (64, 13824), (5, 16384),
                                    (3, 32768), (130, 768)])
def test_group_quantizer_matches_oracle(K, rows, k, block):
    check_quant(K, bf16_bits(activations(rows, k, seed=rows * 17 + k)), block)


@pytest.mark.parametrize("block", [256, 128])
@pytest.mark.parametrize("rows,k", [(12, 512), (18, 5120), (7, 13824)])
def test_group_quantizer_special_values(K, rows, k, block):
    check_quant(K, special_rows(rows, k, seed=rows + k + 5), block)


@pytest.mark.parametrize("block", [256, 128])
@pytest.mark.parametrize("rows,k", [(14, 512), (14, 5120), (7, 13824)])
def test_group_quantizer_large_magnitudes(K, rows, k, block):
    check_quant(K, large_rows(rows, k, seed=rows * 5 + k), block)


@pytest.mark.parametrize("block", [256, 128])
@pytest.mark.parametrize("rows,k", [(16, 512), (16, 5120), (8, 13824)])
def test_group_quantizer_scale_floor_rows(K, rows, k, block):
    # Per-group scales meet their 1e-10 floor in the tiny rows' groups.
    check_quant(K, tiny_rows(rows, k, seed=rows * 7 + k), block)


def test_group_quantizer_rejects_bad_widths(K):
    for width in (128, 300):
        with pytest.raises(RuntimeError):
            K.turing_bf16_int4_g128_convrot_quantize(torch.zeros((4, width), dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(RuntimeError):  # rotation blocks other than 256 and 128
        K.turing_bf16_int4_g128_convrot_quantize(torch.zeros((4, 512), dtype=torch.bfloat16, device="cuda"), 64)
    with pytest.raises(TypeError):  # the op layer's dtype check, as for the other bf16 quantizers
        K.turing_bf16_int4_g128_convrot_quantize(torch.zeros((4, 256), dtype=torch.float16, device="cuda"))


def weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int32).to(torch.uint8)
    zeros = torch.randint(0, 16, (n, k // 128), generator=g, dtype=torch.int32).to(torch.uint8)
    scales = (torch.rand((n, k // 128), generator=g) * 0.009 + 1e-3).to(torch.float16)
    bias = torch.randn((n,), generator=g) * 0.02
    return packed, zeros, scales, bias


def int8_activations(m, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int32).to(torch.int8)
    a_scale = torch.rand((m,), generator=g) * 0.01 + 1e-3
    return a, a_scale


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("with_bias", [True, False])
def test_asym_w4a8_matches_oracle(K, tiling, m, n, k, with_bias):
    a, a_scale = int8_activations(m, k, seed=m + n + k)
    packed, zeros, scales, bias = weights(n, k, seed=3 * n + k)
    bias = bias if with_bias else None
    out = K.turing_asym_w4a8_g128_linear(a.cuda(), packed.cuda(), a_scale.cuda(), scales.cuda(), zeros.cuda(),
                                         None if bias is None else bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.asym_w4a8_g128_linear(a.numpy(), packed.numpy(), a_scale.numpy(), scales.numpy(), zeros.numpy(),
                                       None if bias is None else bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("with_bias", [True, False])
def test_w4a4_matches_oracle(K, tiling, m, n, k, with_bias):
    g = torch.Generator().manual_seed(m * 7 + k)
    a_packed = torch.randint(-128, 128, (m, k // 2), generator=g, dtype=torch.int32).to(torch.int8)
    w_packed = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int32).to(torch.int8)
    a_scale = torch.rand((m, k // 128), generator=g) * 0.2 + 1e-3
    _, _, w_scale, bias = weights(n, k, seed=5 * n + k)
    bias = bias if with_bias else None
    out = K.turing_w4a4_g128_linear(a_packed.cuda(), w_packed.cuda(), a_scale.cuda(), w_scale.cuda(),
                                    None if bias is None else bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.w4a4_g128_linear(a_packed.numpy(), w_packed.numpy(), a_scale.numpy(), w_scale.numpy(),
                                  None if bias is None else bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)


def test_w4a4_end_to_end_from_bf16_rows(K, tiling):
    m, n, k = 300, 264, 5120
    xb = bf16_bits(activations(m, k, seed=11))
    codes, scales = K.turing_bf16_int4_g128_convrot_quantize(to_bf16_tensor(xb).cuda())
    _, _, w_scale, bias = weights(n, k, seed=12)
    w_packed = torch.randint(-128, 128, (n, k // 2), generator=torch.Generator().manual_seed(13),
                             dtype=torch.int32).to(torch.int8)
    out = K.turing_w4a4_g128_linear(codes, w_packed.cuda(), scales, w_scale.cuda(), bias.cuda())
    torch.cuda.synchronize()
    ref_codes, ref_scales = oracle.convrot_quantize_int4_g128(xb)
    ref = oracle.w4a4_g128_linear(ref_codes, w_packed.numpy(), ref_scales, w_scale.numpy(), bias.numpy())
    assert np.array_equal(bf16_bits(out), ref)


def test_grouped_linears_reject_bad_shapes(K):
    a = torch.zeros((4, 192), dtype=torch.int8, device="cuda")
    w = torch.zeros((8, 96), dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):  # K = 192 is not a multiple of 128
        K.turing_asym_w4a8_g128_linear(a, w, torch.ones(4, device="cuda"), torch.ones((8, 1), device="cuda"),
                                       torch.zeros((8, 1), dtype=torch.uint8, device="cuda"))
    a = torch.zeros((4, 128), dtype=torch.int8, device="cuda")
    w = torch.zeros((12, 64), dtype=torch.int8, device="cuda")
    with pytest.raises(RuntimeError):  # N = 12 is not a multiple of 8
        K.turing_w4a4_g128_linear(a[:, :64].contiguous(), w, torch.ones((4, 1), device="cuda"),
                                  torch.ones((12, 1), device="cuda"))


@pytest.mark.parametrize("k,n", [(5120, 5120), (13824, 5120)], ids=["k5120", "k13824"])
def test_full_size_grouped_linears_on_sampled_rows(K, tiling, k, n):
    # Wan-14B shapes (M = 32760); rows are independent, so the oracle checks a sample of
    # rows spread over every tile position, bit for bit.
    m = 32760
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(k)
    x = (torch.randn((m, k), generator=g, device=dev))
    idx = torch.randperm(k, generator=g, device=dev)[: k // 100]
    x[:, idx] *= 30.0
    x = x.to(torch.bfloat16)
    q8, s8 = K.turing_bf16_int8_convrot_quantize(x, 256)
    q4, s4 = K.turing_bf16_int4_g128_convrot_quantize(x, 256)
    packed, zeros, w_scale, bias = (t.to(dev) for t in weights(n, k, seed=n + k))
    w4 = torch.randint(-128, 128, (n, k // 2), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
    out8 = K.turing_asym_w4a8_g128_linear(q8, packed, s8, w_scale, zeros, bias)
    out4 = K.turing_w4a4_g128_linear(q4, w4, s4, w_scale, bias)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.arange(0, 8), np.arange(m - 8, m),
                                     np.random.default_rng(k).choice(m, 48, replace=False)]))
    rt = torch.from_numpy(rows).to(dev)
    ref8 = oracle.asym_w4a8_g128_linear(q8[rt].cpu().numpy(), packed.cpu().numpy(), s8[rt].cpu().numpy(),
                                        w_scale.cpu().numpy(), zeros.cpu().numpy(), bias.cpu().numpy())
    assert np.array_equal(bf16_bits(out8[rt]), ref8)
    ref4 = oracle.w4a4_g128_linear(q4[rt].cpu().numpy(), w4.cpu().numpy(), s4[rt].cpu().numpy(),
                                   w_scale.cpu().numpy(), bias.cpu().numpy())
    assert np.array_equal(bf16_bits(out4[rt]), ref4)
    # The quantizer on the same sampled rows.
    xs = bf16_bits(x[rt])
    ref_codes, ref_scales = oracle.convrot_quantize_int4_g128(xs)
    assert np.array_equal(q4[rt].cpu().numpy(), ref_codes)
    assert np.array_equal(s4[rt].cpu().numpy().view(np.uint32), ref_scales.view(np.uint32))
