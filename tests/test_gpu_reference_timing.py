"""The B200 ConvRot linear against the reference's own CUDA kernels on the same GPU.

oracle/_ref/libctu_ref.so is the reference's kernel/csrc/turing/convrot_quant.cu and
w4a8.cu built for sm_100a (the CUTLASS 2.x SM75 mma.sync path recompiled).  On one
configs[1] linear (Wan-2.1-14B, M = 32760 tokens, K = N = 5120) both implementations run
back to back on the same inputs, timed with CUDA events after warm-up: the quantizer
(the reference at its best block size of the three it chooses between,
bindings.cpp:109-150) and the W8A8 GEMM with its dequant + bias epilogue
(w4a8.cu:1185-1219).  The outputs must be bit-identical and the B200 kernels faster.
"""

import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libctu_ref.so"


def _timed(fn, reps):
    for _ in range(3):
        fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference kernels not built (make -C oracle ref)")
def test_convrot_linear_against_reference_kernels_timing(capsys):
    import comfyui_turing_utils_kernel as K

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import make_golden as mg

    lib = mg.load_ref()
    m, k, n = 32760, 5120, 5120
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
    ws = torch.rand((n,), generator=g, device="cuda") * 1e-3 + 1e-4
    bias = torch.randn((n,), generator=g, device="cuda")
    p = mg.p

    # Quantizer: rotate + per-token int8.
    codes, scales = K.turing_bf16_int8_convrot_quantize(x, 256)
    ours_q = _timed(lambda: K.turing_bf16_int8_convrot_quantize(x, 256), 20)
    ref_codes = torch.empty_like(codes)
    ref_scales = torch.empty_like(scales)
    ref_q = {}
    for threads in (512, 768, 1024):
        ref_q[threads] = _timed(lambda: mg.check(lib, lib.ref_bf16_convrot_quantize(
            p(x), p(ref_codes), p(ref_scales), m, k, 8, 0, threads, mg.stream())), 20)
        assert torch.equal(codes, ref_codes) and torch.equal(scales.view(torch.int32), ref_scales.view(torch.int32))

    # W8A8 GEMM + dequant + bias epilogue.
    a_scale = scales.view(-1)
    out = K.turing_int8_linear(codes, w, a_scale, ws, bias)
    ours_g = _timed(lambda: K.turing_int8_linear(codes, w, a_scale, ws, bias), 10)
    ref_out = torch.empty_like(out)
    ref_g = _timed(lambda: mg.check(lib, lib.ref_int8_linear(p(codes), p(w), p(a_scale), p(ws), p(bias), p(ref_out),
                                                              m, n, k, 0, mg.stream())), 5)
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))

    tops = lambda ms: 2.0 * m * n * k / (ms * 1e-3) / 1e12  # noqa: E731
    best_ref_q = min(ref_q.values())
    with capsys.disabled():
        print(f"\n[configs[1] linear M={m} K={k} N={n}] quantizer {ours_q * 1e3:.1f} us vs reference "
              f"{best_ref_q * 1e3:.1f} us (512/768/1024 threads: "
              + "/".join(f"{v * 1e3:.0f}" for v in ref_q.values())
              + f" us); int8 GEMM {ours_g * 1e3:.1f} us ({tops(ours_g):.0f} TOPS) vs reference "
              f"{ref_g * 1e3:.1f} us ({tops(ref_g):.0f} TOPS); linear {(ours_q + ours_g) * 1e3:.1f} us vs "
              f"{(best_ref_q + ref_g) * 1e3:.1f} us")
    assert ours_q < best_ref_q
    assert ours_g < ref_g
