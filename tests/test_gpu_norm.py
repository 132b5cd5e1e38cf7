"""Affine RMSNorm + segmented AdaLN and LayerNorm + AdaLN on B200.

* Bit-exact against the reference's own kernels (kernel/csrc/turing/
  segmented_rms_adaln.cu, run by tests/golden/make_golden.py into norms.npz), through
  the C ABI with the fixture's exact pointers and strides (misaligned input, strided
  and broadcast modulation tables, per-element order) and through the op layer.
* Against the CPU oracle on larger seeded inputs.  The oracle replaces the device
  rsqrtf with a correctly rounded 1/sqrt, so a rare output may differ by the rounding
  of one step (bf16/fp16) or a few fp32 ulps.
* The op layer's argument contract (ops.py:388-451, bindings.cpp:767-880).
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import convrot_oracle as oracle

pytestmark = pytest.mark.gpu

NORMS = Path(__file__).resolve().parent / "golden" / "norms.npz"
TORCH_TYPES = {0: torch.bfloat16, 1: torch.float16, 2: torch.float32}


@pytest.fixture(scope="module")
def K():
    import comfyui_turing_utils_kernel as k
    from comfyui_turing_utils_kernel import _lib

    _lib.device_error(0, clear=True)
    yield k
    assert _lib.device_error(0, clear=True) == 0


def _fixture():
    return np.load(NORMS)


def _names(prefix):
    with np.load(NORMS) as z:
        return sorted({key.split("__")[0] for key in z.files if key.startswith(prefix)})


def to_dev(arr: np.ndarray, code: int) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if code != 2:
        t = t.view(torch.int16).view(TORCH_TYPES[code])
    return t.cuda()


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)


def nan_mask(a: np.ndarray, code: int) -> np.ndarray:
    if code == 2:
        return np.isnan(a)
    mag = a.astype(np.uint32) & 0x7FFF
    return mag > (0x7F80 if code == 0 else 0x7C00)


def assert_same(got: np.ndarray, want: np.ndarray, code: int) -> None:
    gm, wm = nan_mask(got, code), nan_mask(want, code)
    assert np.array_equal(gm, wm), "NaN positions differ"
    g = got.view(np.uint32) if code == 2 else got
    w = want.view(np.uint32) if code == 2 else want
    bad = np.flatnonzero((g != w) & ~gm)
    assert bad.size == 0, f"{bad.size} outputs differ, first at flat index {bad[:5]}"


def as_float(a: np.ndarray, code: int) -> np.ndarray:
    if code == 2:
        return a.astype(np.float64)
    t = torch.from_numpy(np.ascontiguousarray(a)).view(torch.int16).view(TORCH_TYPES[code])
    return t.float().numpy().astype(np.float64)


def assert_close_to_oracle(got: np.ndarray, want: np.ndarray, code: int, atol: float) -> None:
    gm, wm = nan_mask(got, code), nan_mask(want, code)
    assert np.array_equal(gm, wm)
    gf, wf = as_float(got, code)[~gm], as_float(want, code)[~wm]
    diff = np.abs(gf - wf)
    assert np.all(diff <= atol + 1e-6 * np.abs(wf)), float(diff.max())
    if code != 2:
        assert np.mean(got[~gm] == want[~wm]) >= 0.999


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("name", _names("rms_") if NORMS.exists() else [])
def test_rms_matches_reference_kernel_bit_exact(K, name):
    from comfyui_turing_utils_kernel import _lib

    z = _fixture()
    code, rows, hidden, prow, stride, off = (int(v) for v in z[f"{name}__meta"])
    eps = float(z[f"{name}__eps"][0])
    x = to_dev(z[f"{name}__x"], code).reshape(-1)
    xbuf = torch.zeros(rows * hidden + 8, dtype=TORCH_TYPES[code], device="cuda")
    xbuf[off:off + rows * hidden] = x
    xd = xbuf[off:off + rows * hidden]
    w, sc, sh = (to_dev(z[f"{name}__{k}"], code) for k in ("weight", "scale", "shift"))
    seg = torch.from_numpy(z[f"{name}__segments"]).cuda()
    out = torch.empty((rows, hidden), dtype=TORCH_TYPES[code], device="cuda")
    _lib.check(_lib.load().ctu_segmented_rms_adaln(
        _p(xd), _p(w), _p(sc), stride, _p(sh), stride, _p(seg), seg.shape[0], _p(out), rows, hidden, prow, eps, code,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert_same(to_np(out), z[f"{name}__out"], code)

    if off == 0 and stride == hidden:
        # The op layer (its own allocation and checks) gives the same bits.
        y = K.turing_segmented_rms_adaln(xd.view(rows, hidden), w, sc, sh, seg, eps)
        torch.cuda.synchronize()
        assert_same(to_np(y), z[f"{name}__out"], code)


@pytest.mark.parametrize("name", _names("ln_") if NORMS.exists() else [])
def test_layer_norm_matches_reference_kernel_bit_exact(K, name):
    z = _fixture()
    code, batch, seq, hidden, steps = (int(v) for v in z[f"{name}__meta"])
    eps = float(z[f"{name}__eps"][0])
    x, sc, sh = (to_dev(z[f"{name}__{k}"], code) for k in ("x", "scale", "shift"))
    y = K.turing_layer_norm_adaln(x.view(batch, seq, hidden), sc.view(batch, steps, hidden),
                                  sh.view(batch, steps, hidden), eps)
    torch.cuda.synchronize()
    assert_same(to_np(y), z[f"{name}__out"], code)


@pytest.mark.parametrize("code,rows,hidden", [(0, 2048, 5376), (0, 300, 5120), (1, 257, 3072), (2, 129, 2048),
                                              (0, 64, 1000)])
def test_rms_matches_oracle(K, code, rows, hidden):
    dt = TORCH_TYPES[code]
    g = torch.Generator().manual_seed(rows + hidden + code)
    x = (torch.randn((rows, hidden), generator=g) * 2.0).to(dt)
    w = (torch.randn((hidden,), generator=g) * 0.3 + 1.0).to(dt)
    sc = (torch.randn((3, hidden), generator=g) * 0.1).to(dt)
    sh = (torch.randn((3, hidden), generator=g) * 0.1).to(dt)
    third = rows // 3
    segs = np.array([[0, third, 2], [third, 2 * third, 0], [2 * third, rows, 1]], dtype=np.int32)
    y = K.turing_segmented_rms_adaln(x.cuda(), w.cuda(), sc.cuda(), sh.cuda(), torch.from_numpy(segs).cuda(), 1e-6)
    torch.cuda.synchronize()
    width = 4 if code == 2 else 8
    want = oracle.segmented_rms_adaln(to_np(x), to_np(w), to_np(sc), to_np(sh), segs, 1e-6, code,
                                      vectorized=hidden % width == 0)
    assert_close_to_oracle(to_np(y), want, code, atol={0: 2**-6, 1: 2**-9, 2: 1e-6}[code])


@pytest.mark.parametrize("code,batch,seq,hidden,steps,offset",
                         [(0, 1, 2048, 5120, 1, 0.0), (0, 2, 300, 1536, 21, 100.0), (1, 2, 129, 2048, 4, 0.0),
                          (2, 1, 100, 3000, 3, 1000.0), (0, 1, 3, 30000, 1, 0.0), (2, 1, 5, 13000, 2, 10.0)])
def test_layer_norm_matches_oracle(K, code, batch, seq, hidden, steps, offset):
    dt = TORCH_TYPES[code]
    g = torch.Generator().manual_seed(batch * seq + hidden + code)
    x = (torch.randn((batch, seq, hidden), generator=g) + offset).to(dt)
    sc = (torch.randn((batch, steps, hidden), generator=g) * 0.1).to(dt)
    sh = (torch.randn((batch, steps, hidden), generator=g) * 0.1).to(dt)
    y = K.turing_layer_norm_adaln(x.cuda(), sc.cuda(), sh.cuda(), 1e-6)
    torch.cuda.synchronize()
    want = oracle.layer_norm_adaln(to_np(x), to_np(sc), to_np(sh), 1e-6, code)
    assert_close_to_oracle(to_np(y), want, code, atol={0: 2**-5, 1: 2**-8, 2: 1e-5}[code])


def test_rms_matches_torch_formula_like_the_reference_validation(K):
    # kernel/scripts/validate_compatible.py:295-325: the segmented norm against an fp32
    # torch restatement with rtol 0.01 / atol 0.02 for every storage type.
    rows, hidden = 19, 512
    segs = torch.tensor(((0, 1, 2), (1, 7, 0), (7, rows, 1)), dtype=torch.int32, device="cuda")
    row_ids = torch.tensor([2] + [0] * 6 + [1] * (rows - 7), device="cuda")
    for dt in (torch.float16, torch.bfloat16, torch.float32):
        x = torch.randn((rows, hidden), device="cuda", dtype=dt)
        w = torch.randn((hidden,), device="cuda", dtype=dt)
        sc = torch.randn((3, hidden), device="cuda", dtype=dt) * 0.1
        sh = torch.randn((3, hidden), device="cuda", dtype=dt) * 0.1
        y = K.turing_segmented_rms_adaln(x, w, sc, sh, segs, 1.0e-5)
        norm = x.float() * torch.rsqrt(x.float().square().mean(dim=-1, keepdim=True) + 1.0e-5)
        ref = norm * w.float() * (1.0 + sc.float()[row_ids]) + sh.float()[row_ids]
        torch.testing.assert_close(y.float(), ref, rtol=0.01, atol=0.02)


def test_norm_ops_reject_bad_arguments(K):
    x = torch.randn((4, 256), device="cuda", dtype=torch.bfloat16)
    w = torch.ones(256, device="cuda", dtype=torch.bfloat16)
    sc = torch.zeros((1, 256), device="cuda", dtype=torch.bfloat16)
    seg = torch.tensor([[0, 4, 0]], dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="int32"):
        K.turing_segmented_rms_adaln(x, w, sc, sc, seg.long())
    with pytest.raises(ValueError, match="2D"):
        K.turing_segmented_rms_adaln(x.view(2, 2, 256), w, sc, sc, seg)
    with pytest.raises(RuntimeError, match="weight length"):
        K.turing_segmented_rms_adaln(x, w[:128], sc, sc, seg)
    with pytest.raises(RuntimeError, match="epsilon"):
        K.turing_segmented_rms_adaln(x, w, sc, sc, seg, 0.0)
    with pytest.raises(RuntimeError, match="at least one row"):
        K.turing_segmented_rms_adaln(x, w, sc, sc, seg[:0])
    with pytest.raises(TypeError, match="3D"):
        K.turing_layer_norm_adaln(x, sc, sc)
    with pytest.raises(RuntimeError, match="batch and hidden"):
        K.turing_layer_norm_adaln(x.view(1, 4, 256), torch.zeros((2, 1, 256), device="cuda", dtype=x.dtype),
                                  torch.zeros((2, 1, 256), device="cuda", dtype=x.dtype))


REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libctu_ref.so"


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference kernels not built (make -C oracle ref)")
def test_norm_kernels_against_reference_kernels_timing(K, capsys):
    # The reference's own norm kernels (oracle/_ref, built for sm_100a) and the B200 ones on
    # the same bf16 rows, timed with CUDA events back to back after warm-up: both B200
    # kernels must be faster (measured: 1.5x RMS, 2.4x LayerNorm), results bit-identical.
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import make_golden as mg

    lib = mg.load_ref()
    m, h = 32760, 5376
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((m, h), generator=g, device="cuda").to(torch.bfloat16)
    w = torch.ones(h, dtype=torch.bfloat16, device="cuda")
    s = (torch.randn((1, h), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    seg = torch.tensor([[0, m, 0]], dtype=torch.int32, device="cuda")
    out = torch.empty_like(x)

    def timed(fn, reps=20):
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

    p = mg.p
    ours_rms = timed(lambda: K.turing_segmented_rms_adaln(x, w, s, s, seg, 1e-6))
    ref_rms = timed(lambda: mg.check(lib, lib.ref_segmented_rms_adaln(p(x), p(w), p(s), p(s), p(seg), p(out), m, h, 1,
                                                                       h, h, 1, 1e-6, 0, mg.stream())))
    assert torch.equal(K.turing_segmented_rms_adaln(x, w, s, s, seg, 1e-6).view(torch.int16), out.view(torch.int16))
    x3, s3, o3 = x.view(1, m, h), s.view(1, 1, h), out.view(1, m, h)
    ours_ln = timed(lambda: K.turing_layer_norm_adaln(x3, s3, s3, 1e-6))
    ref_ln = timed(lambda: mg.check(lib, lib.ref_layer_norm_adaln(p(x3), p(s3), p(s3), p(o3), 1, m, h, 1, 1e-6, 0,
                                                                   mg.stream())))
    assert torch.equal(K.turing_layer_norm_adaln(x3, s3, s3, 1e-6).view(torch.int16), o3.view(torch.int16))
    with capsys.disabled():
        print(f"\n[norm timing M={m} K={h} bf16] RMS+AdaLN {ours_rms * 1e3:.1f} us vs reference {ref_rms * 1e3:.1f} us; "
              f"LayerNorm+AdaLN {ours_ln * 1e3:.1f} us vs reference {ref_ln * 1e3:.1f} us")
    assert ours_rms < ref_rms
    assert ours_ln < ref_ln


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("code,batch,seq,hidden,steps", [
    (0, 2, 3000, 5120, 1), (0, 1, 4096, 1001, 3), (1, 3, 700, 3072, 2), (2, 1, 2500, 4096, 5),
    (0, 1, 5000, 24, 1), (0, 1, 300, 20000, 2), (0, 1, 200, 30000, 1), (2, 2, 400, 12288, 1),
    (0, 1, 120, 140000, 1),  # warp totals above 16384: the warp trees divide the IEEE way too
])
def test_layer_norm_many_rows_bit_exact_against_reference_kernel(K, code, batch, seq, hidden, steps):
    # Thousands of rows, so that every persistent CTA takes several rows (and the one-row
    # -ahead copies), with rows that leave the fast division range: zeros, a constant row,
    # NaN / infinity, and values near 1e-30 whose deltas fall below 2^-96.
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import make_golden as mg

    lib = mg.load_ref()
    dt = TORCH_TYPES[code]
    g = torch.Generator(device="cuda").manual_seed(hidden + seq + code)
    x = torch.randn((batch * seq, hidden), generator=g, device="cuda") * 3.0
    x[5] = 0.0
    x[17] = 1.5
    x[40, hidden // 2] = float("nan")
    x[41, 0] = float("inf")
    x[90] = x[90] * (1e-4 if code == 1 else 1e-30)  # fp16 cannot hold 1e-30
    x = x.to(dt).view(batch, seq, hidden)
    sc = (torch.randn((batch, steps, hidden), generator=g, device="cuda") * 0.1).to(dt)
    sh = (torch.randn((batch, steps, hidden), generator=g, device="cuda") * 0.1).to(dt)
    want = torch.empty_like(x)
    mg.check(lib, lib.ref_layer_norm_adaln(mg.p(x), mg.p(sc), mg.p(sh), mg.p(want), batch, seq, hidden, steps, 1e-6,
                                           code, mg.stream()))
    got = K.turing_layer_norm_adaln(x, sc, sh, 1e-6)
    torch.cuda.synchronize()
    assert_same(to_np(got), to_np(want), code)


def test_plugin_wrapper_builds_the_segment_table_and_runs_the_kernel(K):
    # fusions.py:241-269: the norm module's weight / eps, a validated segment table.
    from types import SimpleNamespace

    import comfyui_turing_utils_b200 as d

    rows, hidden = 19, 1024
    g = torch.Generator().manual_seed(97)
    x = torch.randn((rows, hidden), generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn((hidden,), generator=g) * 0.2 + 1).to(torch.bfloat16).cuda()
    sc = (torch.randn((3, hidden), generator=g) * 0.1).to(torch.bfloat16).cuda()
    sh = (torch.randn((3, hidden), generator=g) * 0.1).to(torch.bfloat16).cuda()
    segs = [(0, 1, 2), (1, 7, 0), (7, rows, 1)]
    y = d.segmented_rms_adaln(SimpleNamespace(weight=w, bias=None, eps=1e-6), x, sh, sc, segs)
    table = d.segment_table(segs, rows, 3, x.device)
    assert table is d.segment_table(segs, rows, 3, x.device)  # cached per segmentation and device
    ref = K.turing_segmented_rms_adaln(x, w, sc, sh, torch.tensor(segs, dtype=torch.int32, device="cuda"), 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    unit = d.segmented_rms_adaln(SimpleNamespace(weight=None, bias=None, eps=1e-6), x, sh, sc, segs)
    ref1 = K.turing_segmented_rms_adaln(x, torch.ones_like(w), sc, sh, table, 1e-6)
    assert torch.equal(unit, ref1)


def test_norms_and_fused_activation_quantizers_capture_into_a_cuda_graph(K):
    # No allocation and no synchronization inside the calls: after one eager call per
    # shape (which also fills the activation tables), norm + quantize chains capture.
    rows, hidden = 300, 5120
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((rows, hidden), generator=g, device="cuda").to(torch.bfloat16)
    xs = torch.randn((rows, 2 * hidden), generator=g, device="cuda").to(torch.bfloat16)
    w = torch.ones(hidden, dtype=torch.bfloat16, device="cuda")
    s = (torch.randn((2, hidden), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    seg = torch.tensor([[0, 100, 1], [100, rows, 0]], dtype=torch.int32, device="cuda")

    def run():
        h = K.turing_segmented_rms_adaln(x, w, s, s, seg, 1e-6)
        ln = K.turing_layer_norm_adaln(x.view(1, rows, hidden), s[:1].view(1, 1, hidden), s[1:].view(1, 1, hidden),
                                       1e-6)
        return (h, ln, *K.turing_bf16_int8_convrot_quantize(h, 256),
                *K.turing_bf16_gelu_int8_convrot_quantize(ln.view(rows, hidden), 256),
                *K.turing_bf16_int8_convrot_quantize(xs, 256, swiglu=True))

    eager = run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run()
    torch.cuda.current_stream().wait_stream(side)
    with torch.cuda.graph(graph):
        captured = run()
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, captured):
        assert torch.equal(a, b)
