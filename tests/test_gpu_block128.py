"""Rotation block 128 (ctu_convrot_quantize_b128): the benchmark's configs name block 128,
the reference's ops take block 256 only, so the block-128 rotation -- (1/sqrt 2) H2 (x) M (x)
M (x) M, the reference's radix-4 stages at strides 1, 4, 16 then a radix-2 stage at stride 64
-- is this build's definition (parity unpinned).  The GPU codes and scales must equal the
oracle's bit for bit on every width of the warp-row and multi-group kernels, on rows with
NaN, infinities, subnormals and large magnitudes, and at full size on sampled rows.
"""

import numpy as np
import pytest
import torch

import convrot_oracle as oracle
from test_gpu_quant_variants import activations, bf16_bits, large_rows, special_rows, tiny_rows, to_bf16_tensor

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    import comfyui_turing_utils_kernel as K
    from comfyui_turing_utils_kernel import _lib

    _lib.device_error(0, clear=True)
    yield K
    assert _lib.device_error(0, clear=True) == 0, "a kernel recorded a bounded-wait timeout"


def check(K, xb):
    codes, scales = K.turing_bf16_int8_convrot_quantize_b128(to_bf16_tensor(xb).cuda())
    torch.cuda.synchronize()
    ref_codes, ref_scales = oracle.convrot_quantize_b128(xb)
    assert np.array_equal(codes.cpu().numpy(), ref_codes)
    assert np.array_equal(scales.cpu().numpy().reshape(-1).view(np.uint32), ref_scales.view(np.uint32))


# Widths of every warp-row variant (1..6 groups a team, partial teams) and of the
# multi-group kernel (one and two groups a team).
@pytest.mark.parametrize("rows,k", [(1, 256), (7, 768), (33, 1280), (17, 2304), (64, 3072), (5, 4096),
                                    (129, 5120), (9, 6144), (4, 6400), (12, 13824), (3, 16384), (2, 32768)])
def test_matches_oracle(K, rows, k):
    check(K, bf16_bits(activations(rows, k, seed=rows * 7 + k)))


@pytest.mark.parametrize("rows,k", [(12, 512), (18, 5120), (7, 13824)])
def test_special_values(K, rows, k):
    check(K, special_rows(rows, k, seed=rows + k + 1))


@pytest.mark.parametrize("rows,k", [(14, 512), (14, 5120), (7, 13824)])
def test_large_magnitudes(K, rows, k):
    check(K, large_rows(rows, k, seed=rows * 3 + k + 1))


@pytest.mark.parametrize("rows,k", [(16, 512), (16, 5120), (8, 13824)])
def test_scale_floor_rows(K, rows, k):
    check(K, tiny_rows(rows, k, seed=rows * 5 + k + 1))


def test_differs_from_block_256(K):
    xb = bf16_bits(activations(8, 5120, seed=3))
    c128, _ = K.turing_bf16_int8_convrot_quantize_b128(to_bf16_tensor(xb).cuda())
    c256, _ = K.turing_bf16_int8_convrot_quantize(to_bf16_tensor(xb).cuda(), 256)
    torch.cuda.synchronize()
    assert not torch.equal(c128, c256)


def test_rejects_bad_inputs(K):
    with pytest.raises(RuntimeError):
        K.turing_bf16_int8_convrot_quantize_b128(torch.zeros((4, 384), dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(RuntimeError):  # wider than the kernels take
        K.turing_bf16_int8_convrot_quantize_b128(torch.zeros((1, 33024), dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("k", [5120, 13824])
def test_full_size_on_sampled_rows(K, k):
    m = 32760
    g = torch.Generator(device="cuda").manual_seed(k + 1)
    x = torch.randn((m, k), generator=g, device="cuda")
    x[:, torch.randperm(k, generator=g, device="cuda")[: k // 100]] *= 30.0
    x = x.to(torch.bfloat16)
    codes, scales = K.turing_bf16_int8_convrot_quantize_b128(x)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.arange(0, 8), np.arange(m - 8, m),
                                     np.random.default_rng(k).choice(m, 48, replace=False)]))
    rt = torch.from_numpy(rows).cuda()
    ref_codes, ref_scales = oracle.convrot_quantize_b128(bf16_bits(x[rt]))
    assert np.array_equal(codes[rt].cpu().numpy(), ref_codes)
    assert np.array_equal(scales[rt].cpu().numpy().reshape(-1).view(np.uint32), ref_scales.view(np.uint32))
