"""Grouped-codebook W4A8 (``turing_utils::codebook_w4a8_linear``) on B200: the int8
weight decode and the whole linear, bit-exact against the oracle and against the
reference's own kernels (tests/golden/extras.npz, written by make_golden.py)."""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import convrot_oracle as oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden  # noqa: E402  (seeded input generators shared with the fixture script)


@pytest.fixture(scope="module")
def C():
    from comfyui_turing_utils_kernel import _C, _lib

    _lib.device_error(0, clear=True)
    yield _C
    assert _lib.device_error(0, clear=True) == 0, "a kernel recorded a bounded-wait timeout"


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _cuda(*ts):
    return [None if t is None else torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in ts]


@pytest.mark.parametrize("n,k,gs", [(8, 64, 4), (64, 256, 16), (72, 512, 8), (136, 768, 32), (40, 1024, 64),
                                    (520, 5120, 16)])
def test_decode_matches_oracle(C, n, k, gs):
    _, packed, scale, codebook, _, _, _ = make_golden.codebook_inputs(1, n, k, gs, seed=n + k + gs)
    w, s, cb = _cuda(packed, scale, codebook)
    got = C.codebook_decode_s8(w, s, cb, gs)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), oracle.codebook_decode(packed, scale, codebook, gs))


def test_decode_every_scale_byte_and_code(C):
    # All 256 e4m3fn bytes (NaN, subnormals, +-448, zeros) against all 16 codes.
    n, k, gs = 256, 64, 4
    codes = np.tile(np.arange(16, dtype=np.uint8), (n, k // 16))
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8).view(np.int8)
    scale = np.repeat(np.arange(256, dtype=np.uint8)[:, None], k // gs, axis=1)
    codebook = np.array([-1e30, -130.0, -2.5, -1.5, -0.5, -0.0, 0.0, 0.25, 0.5, 1.5, 2.5, 3.5, 100.0, 126.5, 127.5,
                         np.inf], dtype=np.float32)
    w, s, cb = _cuda(packed, scale, codebook)
    got = C.codebook_decode_s8(w, s, cb, gs)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), oracle.codebook_decode(packed, scale, codebook, gs))


@pytest.mark.parametrize("m,n,k,gs,chunk", [(33, 64, 256, 16, 64), (17, 72, 512, 4, 16), (9, 136, 768, 8, 0),
                                             (300, 520, 1536, 16, 0), (300, 520, 1536, 16, 264),
                                             (1000, 1032, 5120, 32, 0), (129, 256, 1024, 64, 128)])
def test_linear_matches_oracle(C, m, n, k, gs, chunk):
    a, packed, scale, codebook, a_s, c_s, bias = make_golden.codebook_inputs(m, n, k, gs, seed=m * 3 + n + k)
    dev = _cuda(a, packed, a_s, scale, c_s, codebook, bias)
    out = C.turing_codebook_w4a8_linear(*dev[:6], dev[6], group_size=gs, chunk_rows=chunk)
    torch.cuda.synchronize()
    ref = oracle.codebook_w4a8_linear(a, packed, a_s, scale, c_s, codebook, bias, gs)
    assert np.array_equal(bf16_bits(out), ref)


EXTRAS = GOLDEN / "extras.npz"


@pytest.mark.skipif(not EXTRAS.exists(), reason="reference fixtures not generated")
@pytest.mark.parametrize("case", range(len(make_golden.CODEBOOK_CASES)))
def test_linear_matches_reference_golden(C, case):
    m, n, k, gs, chunk = make_golden.CODEBOOK_CASES[case]
    ref = np.load(EXTRAS)[f"codebook_m{m}_n{n}_k{k}_g{gs}__out"]
    a, packed, scale, codebook, a_s, c_s, bias = make_golden.codebook_inputs(m, n, k, gs, 4500 + case)
    dev = _cuda(a, packed, a_s, scale, c_s, codebook, bias)
    out = C.turing_codebook_w4a8_linear(*dev[:6], dev[6], group_size=gs, chunk_rows=chunk if chunk else -1)
    torch.cuda.synchronize()
    assert np.array_equal(bf16_bits(out), ref)


def test_chunk_policy_errors(C):
    a, packed, scale, codebook, a_s, c_s, _ = make_golden.codebook_inputs(16, 64, 256, 16, seed=1)
    dev = _cuda(a, packed, a_s, scale, c_s, codebook)
    with pytest.raises(RuntimeError, match="group_size=16 and M>8192"):
        C.turing_codebook_w4a8_linear(*dev, chunk_rows=-1)
    with pytest.raises(RuntimeError, match="divisible by 8"):
        C.turing_codebook_w4a8_linear(*dev, chunk_rows=12)
    with pytest.raises(RuntimeError, match="group_size"):
        C.turing_codebook_w4a8_linear(*dev, group_size=12)


def test_dispatch_codebook_linear_end_to_end(C):
    # dispatch.py:803-869: bf16 activations quantized with ConvRot, then the codebook GEMM.
    import comfyui_turing_utils_b200 as d

    m, n, k, gs = 97, 136, 1536, 16
    _, packed, scale, codebook, _, c_s, bias = make_golden.codebook_inputs(m, n, k, gs, seed=7)
    g = torch.Generator().manual_seed(8)
    x = torch.randn((m, k), generator=g).to(torch.bfloat16)
    w, s_rel, s_c, cb, b = _cuda(packed, scale, c_s, codebook, bias)
    out = d.codebook_w4a8_linear(x.cuda().reshape(1, m, k), w, s_rel.view(torch.float8_e4m3fn), s_c, codebook=cb,
                                 bias=b, group_size=gs)
    torch.cuda.synchronize()
    codes, a_s = oracle.convrot_quantize(bf16_bits(x), 8)
    ref = oracle.codebook_w4a8_linear(codes, packed, a_s, scale, c_s, codebook, bias, gs)
    assert out.shape == (1, m, n)
    assert np.array_equal(bf16_bits(out.reshape(m, n)), ref)
