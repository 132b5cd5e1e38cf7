"""Benchmark of the ConvRot W8A8 linear at Wan-2.1-14B shapes.

One step = the configs[1] sweep: six ConvRot W8A8 linears on M = 32760 tokens,
(K, N) in {(5120, 5120) x 4 (Q, K, V, O), (5120, 13824) (FFN up), (13824, 5120)
(FFN down)}; each linear is the fused rotate+quantize kernel followed by the
tcgen05 GEMM with the dequant+bias epilogue, and each has its own input, so no
activation is re-read from L2 within a step.  Metric: int8 tera-ops per second
(2*M*N*K per linear) summed over all GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--eager]
                    [--scaling strong|weak] [--workload configs1|configs4]

N > 1 is launched by torchrun, one process per GPU.  Default (--scaling strong): the
32760 token rows are sharded over the ranks, ceil(M/N) rows each, weights replicated;
rows are independent through rotation, quantization and the GEMM, so no collective
runs on the data path, and the step time is the maximum over ranks.  --scaling weak
gives every rank its own full 32760-row workload instead.  Each timed step is replayed
as one CUDA graph captured after the warm-up (--eager launches every op from the host).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "comfyui-turing-utils_b200"))

M_TOKENS = 32760
SHAPES = [(5120, 5120)] * 4 + [(5120, 13824), (13824, 5120)]  # (K, N)
METRIC = "ConvRot W8A8 linear TOPS at Wan-14B shapes (configs[1] sweep)"
UNIT = "TOPS"
# one Wan-1.3B FFN-up linear (M, K, N).
CFG0 = (1024, 1536, 8960)
# Token rows of each configs[1] linear that the CPU baseline times in full.
CPU_ROWS = 1024


def ops_per_step(m: int) -> float:
    return float(sum(2 * m * n * k for k, n in SHAPES))


def shard_rows(m_total: int, world: int, rank: int):
    """Row range [start, start + rows) of `rank` when m_total token rows are split
    into ceil(m_total / world) rows per rank (the last ranks may hold fewer, or none)."""
    per = -(-m_total // world)
    start = min(rank * per, m_total)
    return start, max(0, min(per, m_total - start))


def padded_shard(local, per: int):
    """`local` ([rows, cols], rows <= per) with zero rows appended up to `per` rows: the
    all-gather exchanges equal-sized shards, so a short last shard is padded."""
    import torch

    rows = local.shape[0]
    if rows == per:
        return local
    return torch.nn.functional.pad(local, (0, 0, 0, per - rows))


def gather_rows(local, per: int, full, async_op: bool = False):
    """All-gather every rank's row shard, padded to `per` rows, into `full`
    ([per * world, cols], in rank order).  With the rows split by shard_rows, rows
    [0, m_total) of `full` are the whole sequence in order; the rest is padding."""
    import torch.distributed as dist

    return dist.all_gather_into_tensor(full, padded_shard(local, per), async_op=async_op)


def synth_activation(m, k, generator):
    """bf16 [m, k] N(0,1) with 1 % of the channels scaled x30 (the BASELINE outliers)."""
    import torch

    x = torch.randn((m, k), generator=generator, dtype=torch.float32)
    idx = torch.randperm(k, generator=generator)[: k // 100]
    x[:, idx] *= 30.0
    return x.to(torch.bfloat16)


def synth_weight(n, k, seed):
    """int8 [n, k] U[-127, 127], fp32 per-channel scale U(1e-3, 1e-2), fp32 bias N(0, 0.02)."""
    import torch

    gw = torch.Generator(device="cpu").manual_seed(seed)
    w = torch.randint(-127, 128, (n, k), generator=gw, dtype=torch.int8)
    w_s = torch.rand((n,), generator=gw) * 0.009 + 1e-3
    b = torch.randn((n,), generator=gw) * 0.02
    return w, w_s, b


def synth_inputs(m, device, seed=0):
    """Seeded synthetic inputs with the BASELINE distributions (random weights): one
    activation per linear of the sweep (xs[i] for SHAPES[i]) and its weights."""
    g = torch_generator(seed)
    xs = [synth_activation(m, k, g).to(device) for k, _ in SHAPES]
    layers = []
    for i, (k, n) in enumerate(SHAPES):
        w, w_s, b = synth_weight(n, k, 1000 + i)
        layers.append((k, n, w.to(device), w_s.to(device), b.to(device)))
    return xs, layers


def torch_generator(seed):
    import torch

    return torch.Generator(device="cpu").manual_seed(seed)


def max_over_ranks(values, world: int, device=None):
    """Element-wise maximum of per-rank timings (every rank calls it, same order)."""
    import torch

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        finally:
            os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU arm
def _cpu_oracle(threads: int):
    import torch

    sys.path.insert(0, str(ROOT / "oracle"))
    import convrot_oracle as oracle

    torch.set_num_threads(threads)
    # The OpenMP runtime may already hold a launcher's OMP_NUM_THREADS=1: set the count
    # explicitly so the reported cores are the threads used.
    if oracle.set_threads(threads) != threads:
        raise RuntimeError("could not set the oracle's OpenMP thread count")
    return oracle


def cpu_sample_time(rows: int, threads: int):
    """Time the CPU oracle port (rotate+quantize in C/OpenMP, torch int32 GEMM on CPU,
    C epilogue) on `rows` tokens of every configs[1] linear.  Returns seconds."""
    import numpy as np
    import torch

    oracle = _cpu_oracle(threads)
    xs, layers = synth_inputs(rows, "cpu", seed=0)
    xbits = [x.view(torch.int16).numpy().view(np.uint16) for x in xs]
    t0 = time.perf_counter()
    for xb, (k, n, w, w_s, b) in zip(xbits, layers):
        codes, scales = oracle.convrot_quantize(xb, 8)
        oracle.int8_linear(codes, w.numpy(), scales, w_s.numpy(), b.numpy())
    return time.perf_counter() - t0


def cpu_cfg0_time(threads: int):
    """The whole configs[0] linear (M=1024, K=1536, N=8960) on the CPU oracle port."""
    import numpy as np
    import torch

    oracle = _cpu_oracle(threads)
    m, k, n = CFG0
    x = synth_activation(m, k, torch_generator(7))
    w, w_s, b = synth_weight(n, k, 2000)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    t0 = time.perf_counter()
    codes, scales = oracle.convrot_quantize(xb, 8)
    oracle.int8_linear(codes, w.numpy(), scales, w_s.numpy(), b.numpy())
    return time.perf_counter() - t0


def run_reference_arm(args, rank: int) -> None:
    """`--impl reference`: the reference has no CPU path of its own for this op, so the
    arm times the oracle's CPU restatement of its arithmetic (kind "port") on CPU_ROWS
    token rows of every configs[1] linear per step."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    rows = CPU_ROWS
    for _ in range(max(args.warmup, 1)):
        cpu_sample_time(rows, threads)
    times = [cpu_sample_time(rows, threads) for _ in range(args.steps)]
    t = statistics.median(times)
    value = ops_per_step(rows) / t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "configs[1] Wan-14B W8A8 sweep (six linears), a slice of the M=32760 tokens on CPU",
                   "m": M_TOKENS, "rows_per_step": rows, "shapes_kn": SHAPES},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{rows} token rows of each of the 6 configs[1] linears per step (rows are "
                                   f"independent, so TOPS on the slice is the rate on the whole M; "
                                   f"ms_per_step is the slice's own time)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def run_b200(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    import comfyui_turing_utils_kernel as kops
    from comfyui_turing_utils_kernel import _lib

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.scaling == "strong":
        m_total = args.m
        _, m = shard_rows(m_total, world, rank)
    else:
        m = args.m
        m_total = args.m * world
    # Seeded per rank: rank r's rows are its own slice of the token sequence.
    xs, layers = synth_inputs(m, dev, seed=rank)
    stream = torch.cuda.current_stream(dev)

    quant_ev, gemm_ev = [], []

    def step(record=False):
        outs = []
        for x, (k, n, w, w_s, b) in zip(xs, layers):
            if m == 0:
                continue
            if record:
                e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
                e0.record(stream)
            q, s = kops.turing_bf16_int8_convrot_quantize(x, 256)
            if record:
                e1.record(stream)
            outs.append(kops.turing_int8_linear(q, w, s, w_s, b))
            if record:
                e2.record(stream)
                quant_ev.append((e0, e1, 2 * m * k + 4 * m + m * k))
                gemm_ev.append((e1, e2, 2 * m * n * k))
        return outs

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    _lib.device_error(local_rank, clear=True)

    # By default the step (its 6 quantizations and 6 GEMMs) is captured once, after the
    # warm-up has done every first-call setup, and replayed: the same kernels on the same
    # inputs, without the per-op host work between launches (which at small row shards
    # would leave the GPU idle between kernels).  The per-kernel durations for the roofline
    # come from eager steps with events, taken first.
    graph = None
    if args.graph and m > 0:
        for _ in range(min(args.steps, 5)):
            step(record=True)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            graph_outs = step()  # noqa: F841  (kept alive with the graph's memory pool)
        graph.replay()
        torch.cuda.synchronize(dev)

    # ---------------------------------------------------------------- device-resident timing
    barrier()
    torch.cuda.synchronize(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step(record=True)
        stop.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    elapsed_ms = start.elapsed_time(stop)
    flags = _lib.device_error(local_rank, clear=True)
    if flags:
        raise RuntimeError(f"kernel bounded-wait flags {flags:#x} during the timed region")

    gemm_ms = sum(a.elapsed_time(b) for a, b, _ in gemm_ev)
    quant_ms = sum(a.elapsed_time(b) for a, b, _ in quant_ev)
    gemm_tops = sum(o for _, _, o in gemm_ev) / (gemm_ms * 1e-3) / 1e12 if gemm_ms else float("nan")
    quant_gbs = sum(o for _, _, o in quant_ev) / (quant_ms * 1e-3) / 1e9 if quant_ms else float("nan")
    x_rep = {k: x for x, (k, _) in zip(xs, SHAPES)}  # one input per width for the variants

    def timed(fn, reps):
        for _ in range(3):
            fn()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        t0.record(stream)
        for _ in range(reps):
            fn()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        return t0.elapsed_time(t1) / reps

    # ---------------------------------------------------------------- variants at the same shapes
    variants = {}
    if not args.skip_variants and m > 0:
        from comfyui_turing_utils_kernel import _C as cabi

        packed = [(k, n, (w[:, 0::2].to(torch.int32) & 7 | ((w[:, 1::2].to(torch.int32) & 7) << 4)).to(torch.int8),
                   w_s, b) for k, n, w, w_s, b in layers]

        # The same W8A8 sweep through the one-call linear (ctu_convrot_int8_linear): where it
        # measured faster (N <= 8192, M >= 16384: the four Q/K/V/O linears of a full-M step)
        # one kernel quantizes rows while its tensor cores work on finished ones.
        def one_call_step():
            for x, (k, n, w, w_s, b) in zip(xs, layers):
                kops.turing_convrot_int8_linear(x, w, w_s, b)

        ms = timed(one_call_step, max(5, min(args.steps, 30)))
        variants["convrot_int8_linear"] = {
            "value": world * ops_per_step(m) / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms,
            "format": "configs[1] W8A8 through turing_utils::convrot_int8_linear: the fused quantizer + CTA-pair "
                      "GEMM kernel for N <= 8192 at M >= 16384, quantizer then GEMM otherwise"}

        # configs[0]-[3] name rotation block 128: the same sweep with the block-128 quantizer
        # (this build's definition of that rotation; parity unpinned) and the W8A8 GEMM.
        def block128_step():
            for x, (k, n, w, w_s, b) in zip(xs, layers):
                q, s = kops.turing_bf16_int8_convrot_quantize_b128(x)
                kops.turing_int8_linear(q, w, s, w_s, b)

        ms = timed(block128_step, max(5, min(args.steps, 30)))
        variants["rotation_block_128"] = {
            "value": world * ops_per_step(m) / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms,
            "format": "configs[1] W8A8 with rotation block 128: (1/sqrt 2) H2 x M x M x M per 128 columns (the "
                      "reference's radix-4 stages at strides 1, 4, 16, then radix-2 at stride 64); parity "
                      "unpinned: the reference's ops take block 256 only"}

        def w4_step(act_bits):
            for x, (k, n, wp, w_s, b) in zip(xs, packed):
                q, s = (kops.turing_bf16_int8_convrot_quantize if act_bits == 8
                        else kops.turing_bf16_int4_convrot_quantize)(x, 256)
                if act_bits == 8:
                    kops.turing_w4a8_linear(q, wp, s, w_s, b)
                else:
                    cabi.int4_linear(q, wp, s, w_s, b)

        for name, bits in (("w4a8", 8), ("w4a4", 4)):
            ms = timed(lambda: w4_step(bits), max(5, min(args.steps, 50)))
            variants[name] = {"value": world * ops_per_step(m) / (ms * 1e-3) / 1e12, "unit": UNIT,
                              "ms_per_step": ms,
                              "format": "signed int4 weights, per-channel scale" +
                                        (", int8 activations" if bits == 8 else ", int4 ConvRot activations") +
                                        "; int4 operands widened to int8 ahead of the W8A8 GEMM (M >= 512)"}

        # the per-group-128 formats, with the rotation block those
        # configs name (128).  Asymmetric uint4 W4A8 (values U[0, 15], fp16 scale and uint4
        # zero point per 128 columns) on per-token int8 ConvRot activations; W4A4 (symmetric
        # int4 weights with fp16 per-group scales) on per-token-per-group int4 ConvRot
        # activations.  Each step quantizes and runs all six linears, so the per-call weight
        # widening is inside the timed work.
        gg = torch.Generator(device=dev).manual_seed(91)
        grouped = []
        for k, n, w, _, b in layers:
            u4 = torch.randint(0, 256, (n, k // 2), generator=gg, dtype=torch.int32, device=dev).to(torch.uint8)
            zp = torch.randint(0, 16, (n, k // 128), generator=gg, dtype=torch.int32, device=dev).to(torch.uint8)
            gsc = (torch.rand((n, k // 128), generator=gg, device=dev) * 0.009 + 1e-3).to(torch.float16)
            s4 = (w[:, 0::2].to(torch.int32) % 15 - 7) & 0xF | (((w[:, 1::2].to(torch.int32) % 15 - 7) & 0xF) << 4)
            grouped.append((u4, zp, gsc, s4.to(torch.int8), b))

        def asym_w4a8_step():
            for x, (u4, zp, gsc, _, b) in zip(xs, grouped):
                q, s = kops.turing_bf16_int8_convrot_quantize_b128(x)
                kops.turing_asym_w4a8_g128_linear(q, u4, s, gsc, zp, b)

        def w4a4_g128_step():
            for x, (_, _, gsc, s4, b) in zip(xs, grouped):
                q, s = kops.turing_bf16_int4_g128_convrot_quantize(x, 128)
                kops.turing_w4a4_g128_linear(q, s4, s, gsc, b)

        for name, fn, fmt in (
                ("asym_w4a8_g128", asym_w4a8_step,
                 "configs[2]: asymmetric uint4 weights, fp16 scale + uint4 zero point per 128 columns, per-token "
                 "int8 ConvRot activations (rotation block 128); weights widened to (nibble - zero) int8, then the per-group GEMM "
                 "(single-CTA 128 x 128 tiles; parity unpinned: no reference kernel)"),
                ("w4a4_g128", w4a4_g128_step,
                 "configs[3]: symmetric int4 weights with fp16 per-group-128 scales, int4 ConvRot activations with "
                 "per-token-per-group-128 scales (rotation block 128); both operands sign-extended, then the per-group GEMM "
                 "(single-CTA 128 x 128 tiles; parity unpinned: no reference kernel)")):
            ms = timed(fn, max(5, min(args.steps, 20)))
            variants[name] = {"value": world * ops_per_step(m) / (ms * 1e-3) / 1e12, "unit": UNIT,
                              "ms_per_step": ms, "format": fmt}
        del grouped

        # Grouped-codebook W4A8 (group 16, e4m3 scales, 16-entry codebook): decode to int8,
        # then the W8A8 pair GEMM, per linear.
        gc = torch.Generator(device=dev).manual_seed(77)
        book = torch.arange(-8, 8, dtype=torch.float32, device=dev)
        cb_layers = []
        for k, n, _, w_s, b in layers:
            codes = torch.randint(0, 256, (n, k // 2), generator=gc, dtype=torch.int32, device=dev).to(torch.uint8)
            scales = torch.randint(0x40, 0x58, (n, k // 16), generator=gc, dtype=torch.int32, device=dev).to(torch.uint8)
            cb_layers.append((k, codes.view(torch.int8), scales, w_s, b))

        def codebook_step():
            for x, (k, codes, scales, w_s, b) in zip(xs, cb_layers):
                q, s = kops.turing_bf16_int8_convrot_quantize(x, 256)
                kops.turing_codebook_w4a8_linear(q, codes, s, scales, w_s, book, b, 16)

        ms = timed(codebook_step, max(5, min(args.steps, 30)))
        variants["codebook_w4a8"] = {"value": world * ops_per_step(m) / (ms * 1e-3) / 1e12, "unit": UNIT,
                                     "ms_per_step": ms,
                                     "format": "4-bit codes, e4m3 group-16 scales, 16-entry codebook, int8 "
                                               "activations; decoded to int8 ahead of the W8A8 GEMM"}

        # the Wan-1.3B FFN-up linear, timed whole (quantize + GEMM).
        c0m, c0k, c0n = CFG0
        x0 = synth_activation(c0m, c0k, torch_generator(7)).to(dev)
        w0, ws0, b0 = (t.to(dev) for t in synth_weight(c0n, c0k, 2000))
        def cfg0_linear():
            q0, s0 = kops.turing_bf16_int8_convrot_quantize(x0, 256)
            return kops.turing_int8_linear(q0, w0, s0, ws0, b0)

        ms = timed(cfg0_linear, 50)
        variants["cfg0"] = {"value": 2.0 * c0m * c0n * c0k / (ms * 1e-3) / 1e12, "unit": UNIT, "us": ms * 1e3,
                            "shape_mkn": list(CFG0),
                            "note": "configs[0] (Wan-1.3B FFN up) on one GPU: rotate+quantize + W8A8 GEMM; "
                                    "inputs 3 MB fit in L2"}
        del x0, w0

        # Fused-activation quantizers at the model's widths (GB/s of algorithmic bytes).
        x_swiglu = torch.cat([x_rep[5120], x_rep[5120]], dim=1)
        quant_cases = {
            "swiglu_int8_k5120": (lambda: kops.turing_bf16_int8_convrot_quantize(x_swiglu, 256, swiglu=True),
                                  m * (2 * 10240 + 5120 + 4)),
            "gelu_int8_k13824": (lambda: kops.turing_bf16_gelu_int8_convrot_quantize(x_rep[13824], 256),
                                 m * (2 * 13824 + 13824 + 4)),
            "plain_int4_k5120": (lambda: kops.turing_bf16_int4_convrot_quantize(x_rep[5120], 256),
                                 m * (2 * 5120 + 2560 + 4)),
        }
        qv = {}
        for name, (fn, nbytes) in quant_cases.items():
            ms = timed(fn, 20)
            qv[name] = {"value": nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "us": ms * 1e3}
        variants["quantizers"] = qv
        del x_swiglu

        # Norm + AdaLN ops in front of the linears (MiniMax width 5376, Wan width 5120):
        # one bf16 read and one bf16 write per element (GB/s of algorithmic bytes).
        xn = torch.randn((m, 5376), generator=gc, device=dev).to(torch.bfloat16)
        wn = torch.ones(5376, dtype=torch.bfloat16, device=dev)
        sn = (torch.randn((1, 5376), generator=gc, device=dev) * 0.02).to(torch.bfloat16)
        seg = torch.tensor([[0, m, 0]], dtype=torch.int32, device=dev)
        s3 = (torch.randn((1, 1, 5120), generator=gc, device=dev) * 0.02).to(torch.bfloat16)
        x3 = x_rep[5120].view(1, m, 5120)
        nv = {}
        for name, fn, nbytes in (
                ("segmented_rms_adaln_bf16_k5376", lambda: kops.turing_segmented_rms_adaln(xn, wn, sn, sn, seg, 1e-6),
                 m * 5376 * 4),
                ("layer_norm_adaln_bf16_k5120", lambda: kops.turing_layer_norm_adaln(x3, s3, s3, 1e-6), m * 5120 * 4)):
            ms = timed(fn, 20)
            nv[name] = {"value": nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "us": ms * 1e3}
        variants["norms"] = nv
        del xn
        if _lib.device_error(local_rank, clear=True):
            raise RuntimeError("kernel bounded-wait flags raised during the variants")

    # ---------------------------------------------------------------- end-to-end (host buffers)
    # Every step copies each linear's activation from pinned host memory and reads every
    # output back.  The copies run on their own streams (PCIe is full duplex): a linear
    # starts when its input has landed, and its output streams back while later linears
    # compute and the next step's inputs stream in.
    e2e_ms, h2d, d2h = float("nan"), 0, 0
    if not args.skip_e2e and m > 0:
        host_x = [x.cpu().pin_memory() for x in xs]
        host_out = [torch.empty((m, n), dtype=torch.bfloat16).pin_memory() for _, n, _, _, _ in layers]
        h2d = sum(x.numel() * x.element_size() for x in host_x)
        d2h = sum(o.numel() * o.element_size() for o in host_out)
        dev_x = [torch.empty_like(x) for x in xs]
        s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        consumed = [torch.cuda.Event() for _ in dev_x]
        for ev in consumed:
            ev.record(stream)

        def e2e_step():
            ready = []
            for i in range(len(dev_x)):  # inputs in use order
                s_h2d.wait_event(consumed[i])  # the previous step's reader is done
                with torch.cuda.stream(s_h2d):
                    dev_x[i].copy_(host_x[i], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(s_h2d)
                    ready.append(ev)
            for i, (k, n, w, w_s, b) in enumerate(layers):
                stream.wait_event(ready[i])
                q, s = kops.turing_bf16_int8_convrot_quantize(dev_x[i], 256)
                consumed[i].record(stream)
                out = kops.turing_int8_linear(q, w, s, w_s, b)
                done = torch.cuda.Event()
                done.record(stream)
                s_d2h.wait_event(done)
                out.record_stream(s_d2h)
                with torch.cuda.stream(s_d2h):
                    host_out[i].copy_(out, non_blocking=True)

        e2e_steps = max(1, min(args.steps, 5))
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        s_h2d.wait_stream(stream)
        s_d2h.wait_stream(stream)
        for _ in range(e2e_steps):
            e2e_step()
        stream.wait_stream(s_h2d)
        stream.wait_stream(s_d2h)
        e_stop.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = e_start.elapsed_time(e_stop) / e2e_steps
    elif not args.skip_e2e:
        barrier()
        barrier()
        e2e_ms = 0.0

    # ---------------------------------------------------------------- reduce over ranks (max time)
    elapsed_ms, e2e_ms, h2d_all, d2h_all = max_over_ranks([elapsed_ms, e2e_ms, h2d, d2h], world, dev)
    ms_per_step = elapsed_ms / args.steps
    value = ops_per_step(m_total) / (ms_per_step * 1e-3) / 1e12
    e2e_value = None if args.skip_e2e else ops_per_step(m_total) / (e2e_ms * 1e-3) / 1e12

    if rank != 0:
        return
    peaks = {}
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    if peaks_path.exists():
        peaks = json.loads(peaks_path.read_text())
    # The GEMM launches last 0.5-1.9 ms each, so the burst figure is the comparable one.
    # MEASURED_PEAKS.json has no int8 entry: int8 dense = 2x bf16 dense on B200 (4.5 vs
    # 2.25 POPS nominal) is assumed.
    bf16_burst = peaks.get("bf16_tflops")
    if bf16_burst:
        peak = 2.0 * bf16_burst
        peak_src = ("2x measured burst cuBLAS bf16 (MEASURED_PEAKS.json bf16_tflops); int8 dense = 2x bf16 "
                    "dense assumed (no measured int8 figure); nominal int8 dense 4500 TOPS")
    else:
        peak, peak_src = 2.0 * 1590.0, "2x fallback burst bf16 1.59 PFLOP/s (int8 = 2x bf16 assumed)"
    hbm = peaks.get("hbm_gbs", 6650.0)
    for entry in variants.get("norms", {}).values():
        entry["frac"] = entry["value"] / hbm
        entry["peak"] = hbm
    frac = gemm_tops / peak
    if frac > 1.0:
        raise RuntimeError(f"GEMM roofline fraction {frac:.3f} > 1 against {peak:.0f} TOPS: the denominator "
                           "or the timing is wrong")

    cpu = None
    if world == 1 and not args.skip_cpu:
        threads = os.cpu_count() or 1
        rows = CPU_ROWS
        cpu_sample_time(rows, threads)
        tcpu = statistics.median(cpu_sample_time(rows, threads) for _ in range(3))
        cpu = {"value": ops_per_step(rows) / tcpu / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{rows} token rows of each of the six configs[1] linears ({tcpu:.2f} s), oracle "
                         f"C/OpenMP rotate+quantize + torch CPU int32 GEMM + C epilogue; rows are independent, "
                         f"so TOPS on the slice is the rate on the whole M"}
        if "cfg0" in variants:
            cpu_cfg0_time(threads)
            t0 = statistics.median(cpu_cfg0_time(threads) for _ in range(3))
            c0m, c0k, c0n = CFG0
            variants["cfg0"]["cpu_baseline"] = {
                "value": 2.0 * c0m * c0n * c0k / t0 / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"the whole configs[0] linear ({t0 * 1e3:.1f} ms)"}

    per_gpu = value / world
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": "configs[1]: ConvRot W8A8 linear sweep at Wan-2.1-14B shapes (six linears, each "
                               "with its own input)",
                   "m_total": m_total, "m_per_gpu": shard_rows(m_total, world, 0)[1] if args.scaling == "strong"
                   else args.m,
                   "shapes_kn": SHAPES, "rotation_block": 256,
                   "l2": "no L2 flush: every linear reads its own input and weights once per step; the "
                         "per-step working set (%.2f GB per GPU) is far larger than L2 (126 MB)" % (
                             sum(2 * m * k + k * n + 2 * m * n + m * k for k, n in SHAPES) / 1e9),
                   "parallelism": (f"token rows sharded over {world} rank(s), weights replicated, no collective"
                                   if args.scaling == "strong" else f"{world} independent full-M rank(s)"),
                   "launch": "each timed step replayed as one CUDA graph" if graph is not None else "eager"},
        "roofline": {"bound": "tensor", "achieved": gemm_tops, "peak": peak, "unit": UNIT,
                     "frac": frac, "traffic": args.gemm_traffic,
                     "kernel": "ctu::gemm::int8_gemm_pair_kernel<0> (CTA pair, tcgen05 cta_group::2)",
                     "traffic_note": "dram bytes of one 5120x5120 launch (ncu at M=16384, scaled to M=32760); "
                                     "algorithmic 529 MB",
                     "peak_source": peak_src,
                     "linear_frac": per_gpu / peak,
                     "linear_frac_note": "whole linear (quantize + GEMM) per GPU: value / n_gpus / peak"},
        "quantizer_roofline": {"bound": "hbm", "achieved": quant_gbs, "peak": hbm, "unit": "GB/s",
                               "frac": quant_gbs / hbm, "traffic": args.quant_traffic,
                               "kernel": "ctu::rot::convrot_quant_w8_kernel<0,8,5> (warp-row, K=5120 x5) and "
                                         "convrot_quant_g8_kernel<0,8,2,0> (multi-group, K=13824)",
                               "traffic_note": "dram bytes of one K=5120 launch (ncu at M=16384, scaled to "
                                               "M=32760); algorithmic 503 MB",
                               "peak_source": "measured copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"},
        "clocks": clocks.summary(),
        "e2e": None if args.skip_e2e else {
            "value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d_all), "d2h_bytes_per_step": int(d2h_all),
            "bytes_note": "per rank (the largest shard); every rank copies its own rows",
            "path": "pinned host activations -> turing_utils ops -> pinned host outputs; copies on their own "
                    "streams, overlapped with compute (PCIe full duplex)"},
        "gpu_launches": 2 * len(SHAPES) * args.steps if m > 0 else 0,
        "variants_same_shapes": variants or None,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- configs[4]
C4_BLOCKS = 40
C4_TEXT = 512
C4_DIM, C4_FFN = 5120, 13824


def c4_ops(m_local: int) -> float:
    """int8 ops of one configs[4] forward on m_local token rows: per block self Q/K/V/O,
    cross Q/O (m_local rows), cross K/V (512 text rows) and FFN up/down."""
    d, f = C4_DIM, C4_FFN
    per_block = 2 * m_local * d * d * 6 + 2 * C4_TEXT * d * d * 2 + 2 * m_local * d * f * 2
    return float(C4_BLOCKS * per_block)


def run_configs4(args, rank: int, world: int, local_rank: int) -> None:
    """every quantized linear of a 40-block Wan-2.1-14B-shaped DiT forward on
    one 32760-token sequence, token rows sharded across the ranks (strong scaling).  The
    only exchange is NCCL's all-gather of the self-attention K and V projections (the
    attention consumer needs the whole sequence): K's gather overlaps V's GEMM and both
    complete before the O projection.  Attention and norms are not part of the workload
    (they stay in bf16 torch in the reference); their outputs are stood in for by fixed
    synthetic activations of the same shapes, so values do not drift across 40 blocks."""
    import torch
    import torch.distributed as dist

    import comfyui_turing_utils_kernel as kops
    from comfyui_turing_utils_kernel import _lib

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    m_total = args.m
    per = -(-m_total // world)
    _, m_local = shard_rows(m_total, world, rank)
    d, f = C4_DIM, C4_FFN
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    def act(rows, cols):
        x = torch.randn((rows, cols), generator=g, device=dev)
        idx = torch.randperm(cols, device=dev, generator=g)[: cols // 100]
        x[:, idx] *= 30.0
        return x.to(torch.bfloat16)

    gw = torch.Generator(device=dev).manual_seed(4321)  # the same weights on every rank

    def weight(n, k):
        return (torch.randint(-127, 128, (n, k), generator=gw, dtype=torch.int8, device=dev),
                torch.rand((n,), generator=gw, device=dev) * 0.009 + 1e-3,
                torch.randn((n,), generator=gw, device=dev) * 0.02)

    blocks = [{name: weight(n, k) for name, n, k in (("q", d, d), ("k", d, d), ("v", d, d), ("o", d, d),
                                                     ("cq", d, d), ("ck", d, d), ("cv", d, d), ("co", d, d),
                                                     ("up", f, d), ("down", d, f))} for _ in range(C4_BLOCKS)]
    x_self, attn, x_cross, cross_attn, ffn_in = (act(m_local, d) for _ in range(5))
    ffn_hidden = act(m_local, f)
    text = act(C4_TEXT, d)
    k_full = torch.empty((per * world, d), dtype=torch.bfloat16, device=dev)
    v_full = torch.empty_like(k_full)

    def linear(q, s, w):
        return kops.turing_int8_linear(q, w[0], s, w[1], w[2])

    def forward():
        for blk in blocks:
            q8, s8 = kops.turing_bf16_int8_convrot_quantize(x_self, 256)  # shared by Q, K, V
            linear(q8, s8, blk["q"])
            k = linear(q8, s8, blk["k"])
            works = []
            if world > 1:
                works.append(gather_rows(k, per, k_full, async_op=True))
            v = linear(q8, s8, blk["v"])
            if world > 1:
                works.append(gather_rows(v, per, v_full, async_op=True))
                for w in works:
                    w.wait()  # the attention consumer needs the whole sequence
            linear(*kops.turing_bf16_int8_convrot_quantize(attn, 256), blk["o"])
            linear(*kops.turing_bf16_int8_convrot_quantize(x_cross, 256), blk["cq"])
            t8, ts = kops.turing_bf16_int8_convrot_quantize(text, 256)
            linear(t8, ts, blk["ck"])
            linear(t8, ts, blk["cv"])
            linear(*kops.turing_bf16_int8_convrot_quantize(cross_attn, 256), blk["co"])
            linear(*kops.turing_bf16_int8_convrot_quantize(ffn_in, 256), blk["up"])
            linear(*kops.turing_bf16_gelu_int8_convrot_quantize(ffn_hidden, 256), blk["down"])

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        forward()
    torch.cuda.synchronize(dev)
    graph = None
    if args.graph:
        # One CUDA graph per forward: 680 kernel launches and 80 collectives replayed
        # without host work.  Captured after the eager warm-up (communicators, launch
        # attributes and the error word exist), released before the process group.
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            forward()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            forward()
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize(dev)
    run = graph.replay if graph is not None else forward
    _lib.device_error(local_rank, clear=True)
    barrier()
    torch.cuda.synchronize(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        start.record()
        for _ in range(args.steps):
            run()
        stop.record()
        torch.cuda.synchronize(dev)
    del graph
    torch.cuda.synchronize(dev)
    barrier()
    if _lib.device_error(local_rank, clear=True):
        raise RuntimeError("kernel bounded-wait flags raised during the configs[4] run")
    (elapsed_ms,) = max_over_ranks([start.elapsed_time(stop)], world, dev)
    ms = elapsed_ms / args.steps
    ops_all = torch.tensor([c4_ops(m_local)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ops_all)
    ops = float(ops_all.item())
    if rank != 0:
        return
    line = {
        "metric": "configs[4] Wan-14B DiT forward: all ConvRot W8A8 linears, tokens/s", "value": m_total / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "tops": ops / (ms * 1e-3) / 1e12,
        "config": {"workload": "configs[4]: 40 blocks x (self Q/K/V/O, cross Q/O, cross K/V on 512 text rows, "
                               "FFN up/down with fused tanh-GELU), random-init W8A8 weights",
                   "tokens": m_total, "tokens_per_rank": per, "blocks": C4_BLOCKS,
                   "collective": "NCCL all-gather of self-attention K and V (bf16) per block" if world > 1 else None,
                   "launch": "one CUDA graph per forward" if args.graph else "eager",
                   "parallelism": f"token rows sharded over {world} rank(s)"},
        "clocks": clocks.summary(),
        "gpu_launches": C4_BLOCKS * 17 * args.steps,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--eager", action="store_true",
                    help="launch every op from the host in the timed region instead of replaying each timed step "
                         "(configs1) or forward (configs4) as one CUDA graph")
    ap.add_argument("--graph", action="store_true", help=argparse.SUPPRESS)  # the default; kept for old command lines
    ap.add_argument("--workload", choices=["configs1", "configs4"], default="configs1",
                    help="configs1: the metric's linear sweep; configs4: a whole DiT forward's linears on one "
                         "sequence sharded over the ranks (strong scaling, K/V all-gather)")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="configs1: strong = the M tokens sharded over the ranks (default); weak = every rank "
                         "runs its own M tokens")
    ap.add_argument("--m", type=int, default=M_TOKENS,
                    help="tokens: the whole sequence (strong scaling, configs4) or per GPU (weak scaling)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling runs: no host round trip")
    ap.add_argument("--skip-variants", action="store_true", help="skip the W4A8/W4A4 timings")
    # profiles/int8_gemm_pair_k5120_n5120_m16384.md: dram read+write of one 5120x5120 launch
    # at M=16384 (243.0 MB), scaled to M=32760 by rows processed.
    ap.add_argument("--gemm-traffic", type=float, default=(111.05e6 + 131.98e6) * 32760 / 16384,
                    help="ncu dram bytes per GEMM launch (profiles/), reported as roofline.traffic")
    # profiles/convrot_quant_w8_int8_k5120_m16384.md: dram read+write of one K=5120
    # launch at M=16384, scaled to M=32760.
    ap.add_argument("--quant-traffic", type=float, default=(167.85e6 + 49.64e6) * 32760 / 16384,
                    help="ncu dram bytes per quantizer launch (profiles/), reported as quantizer_roofline.traffic")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    args.graph = not args.eager

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "configs4":
            run_configs4(args, rank, world, local_rank)
        else:
            run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
