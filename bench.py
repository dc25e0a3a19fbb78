"""Benchmark of Kansai's int8 quantized-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

Default workload ("config 5", the north star's
sharded matmul): a stack of 4 int8 Linear layers [16384 -> 16384], weights
~ N(0, 0.01) quantized per output channel and column-sharded (Shard(1) of the
reference's [in, out] weight) within groups of tp ranks (tp = N up to 4
GPUs, 4 at 8: two row groups), activations fp32 [8192, 16384] ~ N(0, 1)
row-sharded and quantized per tensor with the absmax all-reduced over every
rank.  One step = one forward of the stack over the 8192-token batch: each
rank quantizes its input rows, the int8 codes reach the other ranks of its
group in row chunks (copy-engine pulls from IPC-shared buffers by default,
or NCCL all-gathers) while each layer's GEMM consumes the chunks already
present, and between layers the GEMM epilogues' absmax is all-reduced and
each rank quantizes its output columns for the next exchange.  Total work is
fixed as N grows ("strong" scaling); N = 1 runs the same stack on one GPU
with no exchange.  Inputs are larger than L2 (weights 1 GiB of int8 codes,
input 512 MiB fp32).

At N = 1 the line also carries, under "kernels", config 2 (one per-channel
Linear [4096 -> 4096] over 2048 tokens: activation quantize + int8 GEMM) and
each HBM-bound kernel of the path against the measured HBM peak.

Timing: W warm-up steps, then K steps between barrier + synchronize on both
sides, CUDA events on the launching stream, max over ranks.

--impl reference: the reference's own CPU implementation of the same
workload: its only quantized Linear, qlinear (quantize.py:115-122:
dequantize the int8 weight in Python every call, then the compiled
reference core's Tensor::matmul + add, oracle/_ref), four layers.  A full
step would take tens of minutes, so each step times a bounded sample -- the
Python dequantize of 1/64 of one layer's weight and the matmul of one row per
host thread against the full weight -- and scales it to the workload (4
layers x 64 slices, 8192 / threads rows).  Under torchrun only rank 0 runs it.

Other workloads (--workload): linear (config 2 as its own line), transformer
(config 3), sweep (config 4), mlp (config 1).
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "int8 GEMM TOPS & quantized-linear tokens/s vs int8 roofline at 1/2/4/8 B200"
FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS = 6650.0, 1590.0

STACK_M, STACK_D, STACK_L = 8192, 16384, 4
STACK_WORKLOAD = ("config5: 4 x int8 Linear [16384 -> 16384], weights per-channel int8 column-sharded over the "
                  "ranks, activations [8192, 16384] row-sharded, quantized per tensor, int8 all-gather between "
                  "layers, fp32 out")
M_TOK, K_IN, N_OUT = 2048, 4096, 4096
NSETS = 4
LINEAR_WORKLOAD = ("config2: per-channel int8 quantized Linear [4096 -> 4096], 2048 tokens/step/GPU, "
                   "per-tensor activation quant, fused rescale, fp32 out")
WORKLOAD = STACK_WORKLOAD


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel entries (N = 1)")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="replay the stack's forward from a CUDA graph (auto: when capture succeeds)")
    ap.add_argument("--exchange", choices=["peer", "collective", "fused", "ce"], default=None,
                    help="stack: pipelined NCCL all-gathers (collective, default), pipelined copy-engine pulls "
                         "(ce), copy-engine pulls feeding the gated GEMM (peer) or the all-gather inside the GEMM "
                         "launch (fused)")
    ap.add_argument("--workload", choices=["stack", "linear", "transformer", "sweep", "mlp", "kernels", "gemm",
                                           "attention", "dequantize", "quantize_cols"],
                    default="stack",
                    help="stack: config 5 (default); linear: config 2; transformer: config 3; sweep: config 4; "
                         "mlp: config 1; kernels: the per-kernel entries alone; gemm: one GEMM shape (--shape); "
                         "attention / dequantize / quantize_cols: that kernel alone at its bench shape "
                         "(profiling targets)")
    ap.add_argument("--shape", default="8192,16384,16384", help="gemm workload: M,N,K")
    ap.add_argument("--tp", type=int, default=None,
                    help="stack: column-sharding group size (default: the stack's, N up to 4, else 4)")
    return ap.parse_args()


_T0 = time.time()


def _stage(name):
    """Progress line on stderr (stdout carries only the JSON line)."""
    print(f"[bench rank {os.environ.get('RANK', '0')} +{time.time() - _T0:7.1f}s] {name}", file=sys.stderr,
          flush=True)


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of
    the named kernel from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", f"{name}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (read-only) while
    the timed region runs."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml"}


# --------------------------------------------------------- reference (CPU)

def _parallel(fns):
    out = [None] * len(fns)

    def work(i):
        out[i] = fns[i]()
    ts = [threading.Thread(target=work, args=(i,)) for i in range(len(fns))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    return out


class ReferenceStackSample:
    """Config 5 on the reference's CPU path, sampled: per layer the reference
    runs qlinear = Python dequantize of the whole weight (quantize.py:76-77,
    from_flat) + Tensor::matmul + add (compiled reference core).  One sample
    step times the dequantize of 1/64 of a layer's codes and the matmul of one
    row per host thread against the full [16384, 16384] weight (made inside
    the reference core by its own randn; the naive loop's time does not depend
    on the values), and scales both to the full step."""

    SLICES = 64

    def __init__(self):
        from oracle.refpkg import load_reference_core
        self.core = core = load_reference_core()
        self.threads = os.cpu_count() or 1
        D = STACK_D
        self.w = core.randn([D, D], 0.01, False, 5)
        rs = np.random.RandomState(9)
        self.q_slice = rs.randint(-127, 128, D * D // self.SLICES).tolist()
        self.scale = 4 * 0.01 / 127.0
        self.parts = [core.randn([1, D], 1.0, False, 100 + i) for i in range(self.threads)]
        self.bias = core.zeros([D])

    def step(self):
        """Seconds of one full config-5 step, extrapolated from one sample."""
        t0 = time.perf_counter()
        flat = [v * self.scale for v in self.q_slice]                 # quantize.py:76
        self.core.from_flat(flat, [STACK_D // self.SLICES, STACK_D])  # quantize.py:77
        t1 = time.perf_counter()
        _parallel([lambda x=x: x.matmul(self.w).add(self.bias) for x in self.parts])
        t2 = time.perf_counter()
        per_layer = (t1 - t0) * self.SLICES + (t2 - t1) * (STACK_M / self.threads)
        return STACK_L * per_layer, t2 - t0

    def describe(self):
        return (f"reference qlinear chain, 4 layers [16384 -> 16384] x 8192 rows, sampled per step: Python "
                f"dequantize + from_flat of 1/{self.SLICES} of a layer's weight (x {self.SLICES}) and Tensor::matmul"
                f" + add of 1 row on each of {self.threads} threads against the full weight "
                f"(x {STACK_M // self.threads}), times 4 layers")


class ReferenceLinear:
    """Config 2 on the reference's CPU path, the full 2048-row batch per call:
    qlinear (quantize.py:115-122) = one Python dequantize of the per-tensor
    int8 weight (16.8 M codes) + from_flat, then Tensor::matmul + add, the
    rows split over the host threads as the reference's Shard(0) DeviceMesh
    dispatch does (distributed.py:73-102)."""

    def __init__(self):
        from oracle import cpu as ocpu
        from oracle.refpkg import load_reference_core
        self.core = core = load_reference_core()
        self.threads = os.cpu_count() or 1
        rs = np.random.RandomState(7)
        w = (rs.standard_normal((K_IN, N_OUT)) * 0.02).astype(np.float32)
        q, self.scale = ocpu.quantize_tensor(w)            # the reference's per-tensor scheme
        self.q = q.ravel().tolist()
        x = rs.standard_normal((M_TOK, K_IN)).astype(np.float32)
        self.parts = [core.from_flat(p.ravel().tolist(), [p.shape[0], K_IN]) for p in np.array_split(x, self.threads)]
        self.bias = core.from_flat([0.0] * N_OUT, [N_OUT])

    def step(self):
        t0 = time.perf_counter()
        w = self.core.from_flat([v * self.scale for v in self.q], [K_IN, N_OUT])
        _parallel([lambda x=x: x.matmul(w).add(self.bias) for x in self.parts])
        dt = time.perf_counter() - t0
        return dt, dt

    def describe(self):
        return (f"reference qlinear on the full 2048-row config-2 batch per call: one Python dequantize of the "
                f"4096 x 4096 weight (quantize.py:121) + Tensor::matmul + add, rows split over {self.threads} threads")


def time_reference(kind, steps, warmup, budget_s=None):
    """(tokens/s, seconds per step, threads, sample text, steps timed, wall
    seconds spent) of the reference arm for the workload `kind`."""
    ref = ReferenceStackSample() if kind == "stack" else ReferenceLinear()
    tokens = STACK_M if kind == "stack" else M_TOK
    spent = 0.0
    for _ in range(max(warmup, 1)):
        spent += ref.step()[1]
    per = spent / max(warmup, 1)
    if budget_s is not None:
        steps = max(1, min(steps, int(budget_s / max(per, 1e-6))))
    est = []
    for _ in range(steps):
        full, wall = ref.step()
        est.append(full)
        spent += wall
    dt = sum(est) / len(est)
    return tokens / dt, dt, ref.threads, ref.describe(), steps, spent


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    kind = "stack" if args.workload == "stack" else "linear"
    try:
        value, dt, threads, sample, timed, _ = time_reference(kind, args.steps, min(args.warmup, 1), budget_s=120.0)
    except Exception as e:  # the compiled reference core is missing
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU path could not run: {e}"}))
        return
    workload = STACK_WORKLOAD if kind == "stack" else LINEAR_WORKLOAD
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": timed, "steps_requested": args.steps, "warmup": min(args.warmup, 1), "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "strong" if kind == "stack" else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload, "global_batch": STACK_M if kind == "stack" else M_TOK,
                       "parallelism": "host threads",
                       "reference_path": "the reference's only quantized Linear: int8 weight dequantized to fp32 "
                                         "every call (quantize.py:115-122), fp32 Tensor::matmul + add"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def port_stack_sample():
    """The C restatement (oracle/kz_oracle.c) of the W8A8 stack on all host
    threads, sampled: the per-tensor quantize of 64 activation rows, the
    int8 GEMM of those rows against one layer's codes and the epilogue; the
    full step scales the GEMM and epilogue by 8192 / 64 rows and 4 layers and
    adds the quantize of the full activation tensor per layer."""
    from oracle import cpu as ocpu
    rs = np.random.RandomState(11)
    rows = 64
    x = rs.standard_normal((rows, STACK_D)).astype(np.float32)
    wq = rs.randint(-127, 128, (STACK_D, STACK_D), dtype=np.int8)
    ws = np.full(STACK_D, 1e-4)
    t0 = time.perf_counter()
    xq, xs = ocpu.quantize_tensor(x)
    t1 = time.perf_counter()
    acc = ocpu.gemm_i8(xq, wq)
    ocpu.epilogue(acc, xs, ws)
    t2 = time.perf_counter()
    per_layer = (t1 - t0) * (STACK_M / rows) + (t2 - t1) * (STACK_M / rows)
    step = STACK_L * per_layer
    return {"value": STACK_M / step, "unit": "tokens/s", "cores": ocpu.default_threads(), "kind": "port",
            "sample": f"oracle/kz_oracle.c W8A8 layer (per-tensor quantize, int8 GEMM, epilogue) on {rows} of 8192 "
                      f"rows, all host threads, scaled to 8192 rows x 4 layers",
            "ms_per_step": step * 1e3}


def cpu_baseline(kind):
    try:
        value, dt, threads, sample, timed, spent = time_reference(kind, steps=3, warmup=1)
        out = {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
               "sample": f"{sample}; {timed} timed samples", "ms_per_step": dt * 1e3}
    except Exception as e:
        out = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}
    if kind == "stack":
        try:
            out["port"] = port_stack_sample()
        except Exception as e:
            out["port"] = {"value": None, "sample": f"unavailable: {e}"}
    return out


# ---------------------------------------------------------------- helpers

def _events(dev):
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _graph_of(fn, reps, dev):
    """A CUDA graph of `reps` calls of fn (warmed up eagerly first)."""
    import torch
    fn()
    torch.cuda.synchronize()
    st = torch.cuda.Stream(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for _ in range(reps):
            fn()
    torch.cuda.synchronize()
    return g


def _time_graph(g, reps_per_graph, steps, warmup, local_rank, dev):
    """Replays g until `steps` calls ran; returns (ms per call, calls, clocks)."""
    import torch
    for _ in range(max(1, -(-warmup // reps_per_graph))):
        g.replay()
    torch.cuda.synchronize()
    n = max(1, -(-steps // reps_per_graph))
    stream = torch.cuda.current_stream(dev)
    start, end = _events(dev)
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for _ in range(n):
            g.replay()
        end.record(stream)
        torch.cuda.synchronize()
    return start.elapsed_time(end) / (n * reps_per_graph), n * reps_per_graph, clk.summary()


KERNEL_CLOCKS = []  # (kernel entry, NVML clock summary) of each _kernel_us timing


def _kernel_us(fn, dev, reps=16, replays=8, name=None):
    """Average device time (us) of one call of fn: a CUDA graph of `reps`
    calls replayed `replays` times back to back, CUDA events around the
    replays only.  The replays repeat until they span at least 20 ms so the
    NVML sampler sees the clock under this kernel's load; its summary is
    kept in KERNEL_CLOCKS under `name`."""
    import torch
    g = _graph_of(fn, reps, dev)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    a, b = _events(dev)
    stream = torch.cuda.current_stream(dev)
    a.record(stream)
    g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    per_replay = max(a.elapsed_time(b), 1e-3)
    replays = max(replays, min(int(20.0 / per_replay) + 1, 4000))
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        a.record(stream)
        for _ in range(replays):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize()
    del g
    if name:
        KERNEL_CLOCKS.append((name, clk.summary()))
    return a.elapsed_time(b) / (reps * replays) * 1e3


def _sh(dev):
    import torch
    return torch.cuda.current_stream(dev).cuda_stream


def _ok(st):
    from kansaiml_b200 import _lib
    if st:
        raise RuntimeError(_lib.last_error())


# ------------------------------------------------------- config 2 (linear)

def measure_linear(args, rank, world, local_rank, dev, steps, with_e2e):
    """Config 2: one per-channel int8 Linear [4096 -> 4096] over 2048 tokens
    per step and per rank.  Four rotating (X, W, Y) sets (336 MB > L2); steps
    run from CUDA graphs of 8 steps (activation quantize + GEMM, PDL between
    them).  Returns the measurements as a dict."""
    import torch
    import torch.distributed as dist

    import kansaiml_b200 as kz
    from kansaiml_b200 import _lib
    from kansaiml_b200 import quantize as kq

    lib = _lib.load()
    rs = np.random.RandomState(1000 + rank)
    layers = []
    for _ in range(NSETS):
        w = torch.from_numpy((rs.standard_normal((K_IN, N_OUT)) * 0.02).astype(np.float32)).to(dev)

        class _Lin:
            pass
        lin = _Lin()
        lin.weight, lin.bias = kz.Tensor(w), None
        layers.append(kq.QLinear(lin, per_channel=True))
        del w
    xs = [torch.from_numpy(rs.standard_normal((M_TOK, K_IN)).astype(np.float32)).to(dev) for _ in range(NSETS)]
    ys = [torch.empty((M_TOK, N_OUT), dtype=torch.float32, device=dev) for _ in range(NSETS)]
    xq = torch.empty((M_TOK, K_IN), dtype=torch.int8, device=dev)
    s64 = torch.empty(1, dtype=torch.float64, device=dev)
    s32 = torch.empty(1, dtype=torch.float32, device=dev)
    partials = torch.zeros(_lib.KZ_PARTIALS_WORDS, dtype=torch.int32, device=dev)
    n_el = M_TOK * K_IN
    B = [(L.qweight.kmajor().data_ptr(), L.qweight.scale_f32.data_ptr()) for L in layers]
    X = [x.data_ptr() for x in xs]
    Y = [y.data_ptr() for y in ys]
    XQ, S64, S32, PP = xq.data_ptr(), s64.data_ptr(), s32.data_ptr(), partials.data_ptr()

    def quantize_only(i):
        _ok(lib.kz_quantize_tensor_f32(X[i % NSETS], n_el, XQ, S64, S32, PP, _sh(dev)))

    def gemm_only(i):
        j = i % NSETS
        _ok(lib.kz_gemm_i8(XQ, B[j][0], M_TOK, N_OUT, K_IN, K_IN, S32, 0, B[j][1], 1, None, 0, Y[j], None, N_OUT,
                           None, _sh(dev)))

    def step(i):
        quantize_only(i)
        gemm_only(i)

    step(0)
    torch.cuda.synchronize()
    if kq.device_status() != 0:
        raise RuntimeError("device status set after the first step")
    S = 8
    cap_stream = torch.cuda.Stream(dev)

    def capture(idx, fn=step):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=cap_stream):
            for i in idx:
                fn(i)
        return gr

    K = steps
    chunk_graph = capture(range(S))
    tail_graph = capture(range(K % S)) if K % S else None
    quant_graph = capture(range(S), quantize_only)
    gemm_graph = capture(range(S), gemm_only)
    torch.cuda.synchronize()
    for _ in range(max(1, -(-args.warmup // S))):
        chunk_graph.replay()
    if tail_graph is not None:
        tail_graph.replay()
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = _events(dev)
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for _ in range(K // S):
            chunk_graph.replay()
        if tail_graph is not None:
            tail_graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    reps = max(1, K // S)

    def kernel_ms(gr):
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize()
        a, b = _events(dev)
        a.record(stream)
        for _ in range(reps):
            gr.replay()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / (reps * S)
    quant_avg = kernel_ms(quant_graph)
    gemm_avg = kernel_ms(gemm_graph)
    del chunk_graph, tail_graph, quant_graph, gemm_graph
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / K
    hbm_gbs, bf16, _, peak_src = peaks()
    int8_peak = 2.0 * bf16
    ops = 2.0 * M_TOK * N_OUT * K_IN
    tops = ops / (gemm_avg / 1e3) / 1e12
    out = {"workload": LINEAR_WORKLOAD, "tokens_per_s": M_TOK * world / (ms_per_step / 1e3),
           "ms_per_step": ms_per_step, "steps": K, "clocks": clk.summary(),
           "launch": f"CUDA graphs of {S} steps (2 libkz kernels per step) replayed back to back",
           "l2": f"inputs larger than L2: {NSETS} rotating (X, W, Y) sets, "
                 f"{NSETS * (M_TOK * K_IN * 4 + K_IN * N_OUT + M_TOK * N_OUT * 4) / 1e6:.0f} MB",
           "gemm": {"kernel": "gemm_i8_kernel", "bound": "tensor", "avg_us": gemm_avg * 1e3, "achieved": tops,
                    "peak": int8_peak, "unit": "TOP/s", "frac": tops / int8_peak,
                    "traffic": profile_traffic("gemm_i8_config2"),
                    "peak_source": f"2 x bf16_tflops ({bf16:.1f}, {peak_src}) -- int8 dense = 2x bf16 dense on B200",
                    "algorithmic": f"2*M*N*K = {ops:.3e} op per launch",
                    "timing": f"CUDA events around {reps} replays of a graph of {S} launches of this kernel alone"},
           "quantize_activations": _hbm_entry("quantize_resident_kernel", quant_avg * 1e3, 9.0 * n_el, hbm_gbs,
                                              "9 B/element algorithmic (absmax 4 + quantize 4 + 1, per pass)",
                                              dram_bytes=5.0 * n_el)}
    if not with_e2e:
        return out
    # e2e through the public API with host buffers (pinned), three buffers in flight
    NB = 3
    x_host = [torch.from_numpy(rs.standard_normal((M_TOK, K_IN)).astype(np.float32)).pin_memory() for _ in range(NB)]
    y_host = [torch.empty((M_TOK, N_OUT), dtype=torch.float32).pin_memory() for _ in range(NB)]
    x_dev = [torch.empty((M_TOK, K_IN), dtype=torch.float32, device=dev) for _ in range(NB)]
    layer = layers[0]

    def forward(xd):
        return layer(kz.Tensor(xd)).data

    e2e_ms = _e2e_loop(forward, x_host, y_host, x_dev, args.e2e_steps, world, dev)
    out["e2e"] = {"value": M_TOK * world / (e2e_ms / args.e2e_steps / 1e3), "unit": "tokens/s",
                  "h2d_bytes_per_step": M_TOK * K_IN * 4, "d2h_bytes_per_step": M_TOK * N_OUT * 4}
    return out


def _hbm_entry(kernel, avg_us, alg_bytes, hbm_gbs, algorithmic, dram_bytes=None):
    gbs = alg_bytes / (avg_us / 1e6) / 1e9
    e = {"kernel": kernel, "bound": "hbm", "avg_us": avg_us, "achieved_gbs": gbs, "peak_gbs": hbm_gbs,
         "frac": gbs / hbm_gbs, "algorithmic": algorithmic}
    if dram_bytes is not None:
        d = dram_bytes / (avg_us / 1e6) / 1e9
        e["dram_bytes_per_launch"] = dram_bytes
        e["achieved_gbs_dram"] = d
        e["frac_dram"] = d / hbm_gbs
    return e


def _e2e_loop(forward, x_host, y_host, x_dev, steps, world, dev):
    """Every step copies its pinned host input to the device (copy stream),
    runs `forward` on the compute stream and copies the result back to pinned
    host memory (another copy stream); NB buffers in flight, so uploads,
    forwards and downloads of neighbouring steps overlap while every step
    still moves its own bytes.  Returns device ms for `steps` steps, max over
    ranks."""
    import torch
    import torch.distributed as dist
    NB = len(x_host)
    stream = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(NB)]
    ev_fwd = [torch.cuda.Event() for _ in range(NB)]
    ev_out = [torch.cuda.Event() for _ in range(NB)]
    for e in ev_fwd + ev_out:
        e.record(stream)

    def e2e_step(i):
        b = i % NB
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_fwd[b])            # the forward that read x_dev[b] NB steps ago is done
            x_dev[b].copy_(x_host[b], non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[b])              # y of NB steps ago has been read back
        y = forward(x_dev[b])
        ev_fwd[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_fwd[b])
            y_host[b].copy_(y, non_blocking=True)
            y.record_stream(s_out)
            ev_out[b].record(s_out)

    for i in range(NB):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = _events(dev)
    e0.record(stream)
    for i in range(steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def _copies_only_ms(x_host, y_host, x_dev, y_dev, steps, world, dev):
    """The e2e loop's host copies alone (the same pinned buffers, streams and
    sizes, no forward): device ms for `steps` steps, max over ranks.  When it
    is close to the e2e time, the host links, not the GPU, bound the e2e."""
    import torch
    import torch.distributed as dist
    NB = len(x_host)
    stream = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = _events(dev)
    e0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(steps):
        b = i % NB
        with torch.cuda.stream(s_in):
            x_dev[b].copy_(x_host[b], non_blocking=True)
        with torch.cuda.stream(s_out):
            y_host[b].copy_(y_dev, non_blocking=True)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


class _GpuLocalCpus:
    """Binds the calling thread to the CPUs NVML reports as local to the GPU
    (nvmlDeviceGetCpuAffinity, read-only) for the duration of the block, so
    pinned host buffers allocated inside it land on the GPU's NUMA node and
    the launching thread runs there; restores the previous affinity after."""

    def __init__(self, local_rank):
        self.local_rank, self.prev, self.cpus, self.note = local_rank, None, None, "not bound"

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.local_rank)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
            cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
            self.prev = os.sched_getaffinity(0)
            cpus &= self.prev
            if cpus:
                os.sched_setaffinity(0, cpus)
                self.cpus = sorted(cpus)
                self.note = f"{len(cpus)} GPU-local CPUs ({self.cpus[0]}..{self.cpus[-1]})"
        except Exception as e:  # no NVML, or no affinity information: leave the thread as it is
            self.note = f"not bound ({type(e).__name__})"
        return self

    def __exit__(self, *a):
        if self.prev is not None:
            try:
                os.sched_setaffinity(0, self.prev)
            except OSError:
                pass


# ----------------------------------------------- per-kernel HBM rooflines

def measure_kernels(args, rank, world, local_rank, dev):
    """N = 1: config 2 (quantize + GEMM step), the int8 GEMM at 8192^3, the
    reference-semantics W8A32 qlinear at config 2's shape, and each HBM-bound
    kernel of the path on rotating inputs larger than L2."""
    import torch
    from kansaiml_b200 import _lib
    lib = _lib.load()
    hbm_gbs, bf16, _, peak_src = peaks()
    int8_peak = 2.0 * bf16
    out = {}
    out["config2_linear"] = measure_linear(args, rank, world, local_rank, dev, steps=max(8, 4 * args.steps),
                                           with_e2e=False)
    torch.cuda.empty_cache()
    i = [0]

    def nxt(n):
        i[0] += 1
        return i[0] % n

    # int8 GEMM 8192^3, per-row x per-column scale epilogue (config 4's headline size)
    n = 8192
    g = torch.Generator(device=dev)
    g.manual_seed(8192)
    sets = [(torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=g),
             torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=g),
             torch.rand(n, device=dev, generator=g) * 9e-3 + 1e-3, torch.rand(n, device=dev, generator=g) * 9e-3 + 1e-3,
             torch.empty((n, n), dtype=torch.float32, device=dev)) for _ in range(2)]

    def gemm8k():
        a, b, rs_, cs_, y = sets[nxt(2)]
        _ok(lib.kz_gemm_i8(a.data_ptr(), b.data_ptr(), n, n, n, n, rs_.data_ptr(), 1, cs_.data_ptr(), 1, None, 0,
                           y.data_ptr(), None, n, None, _sh(dev)))
    us = _kernel_us(gemm8k, dev, reps=4, replays=6, name="gemm_8192_cubed")
    tops = 2.0 * n ** 3 / (us / 1e6) / 1e12
    out["gemm_8192_cubed"] = {"kernel": "gemm_i8_kernel", "bound": "tensor", "avg_us": us, "achieved": tops,
                              "peak": int8_peak, "unit": "TOP/s", "frac": tops / int8_peak,
                              "algorithmic": "2*8192^3 op per launch, fp32 epilogue (per-row x per-column scales)"}
    del sets
    torch.cuda.empty_cache()
    # W8A32 qlinear (the reference's own semantics) at config 2's shape
    xw = [torch.randn((M_TOK, K_IN), device=dev) for _ in range(2)]
    qw = torch.randint(-127, 128, (K_IN, N_OUT), dtype=torch.int8, device=dev)
    yw = torch.empty((M_TOK, N_OUT), device=dev)

    def w8a32():
        _ok(lib.kz_qlinear_w8a32_f32(xw[nxt(2)].data_ptr(), M_TOK, K_IN, qw.data_ptr(), 0.02 / 127, None, N_OUT, 0,
                                     yw.data_ptr(), _sh(dev)))
    us = _kernel_us(w8a32, dev, reps=2, replays=3, name="w8a32_qlinear_config2")
    flops = 2.0 * M_TOK * N_OUT * K_IN
    props = torch.cuda.get_device_properties(dev)
    fp32_peak = props.multi_processor_count * 128 * 2 * 1.965e9 / 1e12
    tf = flops / (us / 1e6) / 1e12
    out["w8a32_qlinear_config2"] = {
        "kernel": "qlinear_w8a32_kernel", "bound": "fp32 SIMT (k-ordered)", "avg_us": us, "achieved": tf,
        "unit": "TFLOP/s", "peak": fp32_peak / 2, "frac": tf / (fp32_peak / 2),
        "peak_source": f"{props.multi_processor_count} SMs x 128 fp32 lanes x 1.965 GHz = {fp32_peak:.1f} TFLOP/s "
                       "of FMA; the reference's loop rounds each product and sum separately (no FMA), so 2 "
                       "instructions per multiply-add: half that",
        "algorithmic": f"2*M*N*K = {flops:.3e} flop per call, per-tensor int8 weight, fp32 activations"}
    del xw, qw, yw
    # config 3's attention core (batch 32, context 256, 4 heads of 64, causal), reference operation order
    Ba, Sa, Da, Ha = 32, 256, 256, 4
    qkvs = [torch.randn((Ba, Sa, 3 * Da), device=dev) for _ in range(4)]
    att_out = torch.empty((Ba, Sa, Da), device=dev)
    att_parts = torch.zeros(_lib.KZ_PARTIALS_WORDS, dtype=torch.int32, device=dev)

    def attn():
        t = qkvs[nxt(4)]
        _ok(lib.kz_attention_f32(t.data_ptr(), t.data_ptr() + 4 * Da, t.data_ptr() + 8 * Da, Ba, Ha, Sa, Sa, Da // Ha,
                                 3 * Da, 3 * Da, 3 * Da, None, 0, 0, 0, 1, 0.125, att_out.data_ptr(), Da,
                                 att_parts.data_ptr(), _sh(dev)))
    us = _kernel_us(attn, dev, reps=8, replays=4, name="attention_config3")
    att_ops = Ba * Ha * (Sa * (Sa + 1) // 2) * 4.0 * (Da // Ha)
    out["attention_config3"] = {
        "kernel": "attention_ref_kernel<64>", "bound": "fp32 SIMT (ordered, no FMA)", "avg_us": us,
        "achieved": att_ops / (us / 1e6) / 1e12, "unit": "Top/s", "peak": fp32_peak / 2,
        "frac": att_ops / (us / 1e6) / 1e12 / (fp32_peak / 2),
        "peak_source": "fp32 instruction issue: SMs x 128 lanes x 1.965 GHz (each product and each sum its own "
                       "instruction, as the reference's loops round them)",
        "algorithmic": f"{att_ops:.3e} op per call: per (batch, head) S(S+1)/2 causal (query, key) pairs x d_k "
                       "x (mul + add) for q.k^T and again for w.v"}
    del qkvs, att_out
    # dequantize, 8.4 M codes (config 2's activation size), 4 rotating sets
    nd = M_TOK * K_IN
    qs = [torch.randint(-127, 128, (nd,), dtype=torch.int8, device=dev) for _ in range(NSETS)]
    ds = [torch.empty(nd, device=dev) for _ in range(NSETS)]

    def deq():
        j = nxt(NSETS)
        _ok(lib.kz_dequantize_i8_f32(qs[j].data_ptr(), nd, 0.01, ds[j].data_ptr(), _sh(dev)))
    out["dequantize"] = _hbm_entry("dequantize_kernel", _kernel_us(deq, dev, name="dequantize"), 5.0 * nd, hbm_gbs,
                                   "5 B/element (1 B code in, 4 B fp32 out)", dram_bytes=5.0 * nd)
    del qs, ds
    # per-channel weight quantize, config 2's 4096 x 4096 weight (absmax_cols4 + quantize_cols4)
    ws = [torch.randn((K_IN, N_OUT), device=dev) * 0.02 for _ in range(NSETS)]
    qT = torch.empty((N_OUT, K_IN), dtype=torch.int8, device=dev)
    s64 = torch.empty(N_OUT, dtype=torch.float64, device=dev)
    s32 = torch.empty(N_OUT, device=dev)
    wsb = torch.empty(lib.kz_quantize_cols_workspace_bytes(K_IN, N_OUT), dtype=torch.uint8, device=dev)

    def qcols():
        _ok(lib.kz_quantize_cols_f32(ws[nxt(NSETS)].data_ptr(), K_IN, N_OUT, qT.data_ptr(), s64.data_ptr(),
                                     s32.data_ptr(), wsb.data_ptr(), wsb.numel(), _sh(dev)))
    ne = K_IN * N_OUT
    out["quantize_cols"] = _hbm_entry("quantize_cols_strip_kernel", _kernel_us(qcols, dev, name="quantize_cols"),
                                      9.0 * ne, hbm_gbs,
                                      "9 B/element counted as absmax (4) + quantize (4 + 1), the accounting of a "
                                      "two-pass form; this single pass moves 5 B/element (frac_dram)",
                                      dram_bytes=5.0 * ne)
    del ws, qT, wsb
    # LayerNorm -> absmax partials (config 3's 8192 x 256 activations)
    Ml, Dl = 8192, 256
    lx = [torch.randn((Ml, Dl), device=dev) for _ in range(16)]
    ly = [torch.empty((Ml, Dl), device=dev) for _ in range(16)]
    gm, bt = torch.ones(Dl, device=dev), torch.zeros(Dl, device=dev)
    lp = torch.zeros(_lib.KZ_PARTIALS_WORDS, dtype=torch.int32, device=dev)

    def lnorm():
        j = nxt(16)
        _ok(lib.kz_layernorm_partials_f32(lx[j].data_ptr(), Ml, Dl, gm.data_ptr(), bt.data_ptr(), 1e-5,
                                          ly[j].data_ptr(), lp.data_ptr(), _sh(dev)))
    out["layernorm"] = _hbm_entry("layernorm_partials_kernel", _kernel_us(lnorm, dev, name="layernorm"), 8.0 * Ml * Dl, hbm_gbs,
                                  "8 B/element (4 in, 4 out); 16 rotating 8 MB sets (128 MB, about L2)")
    del lx, ly
    torch.cuda.empty_cache()
    for name, clk in KERNEL_CLOCKS:  # the SM clock each kernel's replays ran at
        if name in out:
            out[name]["clocks"] = clk
    return out


# ------------------------------------------------- config 5: sharded stack

def run_stack(args, rank, world, local_rank, dev):
    import torch
    import torch.distributed as dist

    from kansaiml_b200 import _lib
    from kansaiml_b200.distributed import DeviceMesh, ShardedQLinearStack
    from kansaiml_b200.quantize import device_status

    mesh = DeviceMesh.spmd() if world > 1 else None

    def weight(l):
        g = torch.Generator(device=dev)
        g.manual_seed(5000 + l)
        return torch.randn((STACK_D, STACK_D), generator=g, device=dev) * 0.01

    _stage("stack: quantizing weights")
    stack = ShardedQLinearStack([weight] * STACK_L, mesh, exchange=args.exchange, tp=args.tp)
    M = STACK_M
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    x_full = torch.randn((M, STACK_D), generator=g, device=dev)
    pipelined = stack.exchange in ("collective", "ce")
    x_local = stack.local_input(x_full) if (pipelined and world > 1) else x_full
    if pipelined:
        del x_full
    torch.cuda.empty_cache()
    C = stack.chunks(M) if pipelined else 1
    if pipelined and world > 1:
        # leave SMs for the NCCL all-gather that overlaps each GEMM chunk
        # (KZ_BENCH_SM_TARGET overrides the GEMMs' SM budget; 0 = every SM)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        target = int(os.environ.get("KZ_BENCH_SM_TARGET", max(2, sms - 16)))
        _ok(_lib.load().kz_set_sm_count_target(target))

    def fwd():
        if pipelined:
            return stack.forward_local(x_local, M)
        return stack(x_local)

    _stage("stack: eager warm-up")
    for _ in range(max(args.warmup, 3)):
        fwd()
    torch.cuda.synchronize()
    if device_status() != 0:
        raise RuntimeError("device status set during warm-up")
    _stage("stack: graph capture")
    graph, graph_note = None, "eager launches"
    if args.graph != "off" and pipelined:
        try:
            st = torch.cuda.Stream(dev)
            st.wait_stream(torch.cuda.current_stream(dev))
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_, stream=st):
                fwd()
            torch.cuda.synchronize()
            g_.replay()
            torch.cuda.synchronize()
            graph, graph_note = g_, "one CUDA graph per step (the whole forward, NCCL collectives included)"
            del g_
        except Exception as e:  # capture unsupported: eager launches
            if args.graph == "on":
                raise
            graph_note = f"eager launches (graph capture failed: {type(e).__name__})"
            g_ = None   # release a partial capture (it may hold NCCL work)
            torch.cuda.synchronize()
    # the same decision on every rank
    if world > 1:
        flag = torch.tensor([1 if graph is not None else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 0 and graph is not None:
            graph.reset()
            graph, graph_note = None, "eager launches (graph capture failed on another rank)"

    def step():
        if graph is not None:
            graph.replay()
        else:
            fwd()

    _stage(f"stack: warm-up steps ({graph_note})")
    for _ in range(max(args.warmup, 3)):
        step()
    K = args.steps
    _stage("stack: timed region")
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = _events(dev)
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for _ in range(K):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / K
    status = device_status()
    _stage("stack: checksum / parity")
    # A checksum of the whole output (the int32 bit patterns of every rank's
    # column shard, summed): sharding changes no arithmetic, so it is the same
    # number at every N when the sharded forward is bit-identical to N = 1.
    y_chk = fwd().data
    chk = y_chk.view(torch.int32).to(torch.int64).sum().reshape(1)
    if world > 1:
        dist.all_reduce(chk)
    checksum = f"{int(chk.item()) & 0xFFFFFFFFFFFFFFFF:016x}"
    del y_chk
    # N > 1: rank 0 also runs the unsharded stack on one GPU over the same
    # input and weights, and the line records whether the two outputs match
    parity = None
    if world > 1:
        if rank == 0:
            one = ShardedQLinearStack([weight] * STACK_L, None)
            g1 = torch.Generator(device=dev)
            g1.manual_seed(77)
            x1 = torch.randn((M, STACK_D), generator=g1, device=dev)
            y1 = one.forward_local(x1, M).data
            chk1 = int(y1.view(torch.int32).to(torch.int64).sum().item()) & 0xFFFFFFFFFFFFFFFF
            parity = {"one_gpu_checksum": f"{chk1:016x}", "equal": f"{chk1:016x}" == checksum}
            del one, x1, y1
            torch.cuda.empty_cache()
        dist.barrier()

    _stage("stack: per-phase pass")
    # per-phase device times of one eager forward (events on the compute stream)
    phases = None
    if pipelined:
        stack.timing = True
        for _ in range(2):
            fwd()
            phases = stack.phase_times()
        stack.timing = False
        if world > 1:
            keys = sorted(phases)
            t = torch.tensor([phases[k] for k in keys], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            phases = {k: float(v) for k, v in zip(keys, t.tolist())}

    _stage("stack: GEMM alone")
    # the dominant kernel alone: the forward's GEMM launches (same shapes) back to back
    n_loc = STACK_D // stack.tp
    mc = (M // stack.dp) // C
    qt0 = stack.layers[0][0]
    a_chunk = torch.randint(-127, 128, (mc, STACK_D), dtype=torch.int8, device=dev)
    ys = [torch.empty((mc, n_loc), dtype=torch.float32, device=dev) for _ in range(2)]
    a_s = torch.full((1,), 1e-3, device=dev)
    lib = _lib.load()
    j = [0]

    def gemm_launch():
        j[0] += 1
        qt = stack.layers[j[0] % STACK_L][0]
        _ok(lib.kz_gemm_i8(a_chunk.data_ptr(), qt.kmajor().data_ptr(), mc, n_loc, STACK_D, STACK_D, a_s.data_ptr(),
                           0, qt.scale_f32.data_ptr(), 1, None, 0, ys[j[0] % 2].data_ptr(), None, n_loc, None,
                           _sh(dev)))
    gemm_us = _kernel_us(gemm_launch, dev, reps=4 * C, replays=4, name="stack_gemm")
    del a_chunk, ys, qt0
    hbm_gbs, bf16, bf16_sus, peak_src = peaks()
    int8_peak = 2.0 * bf16
    gemm_ops = 2.0 * mc * n_loc * STACK_D
    gemm_tops = gemm_ops / (gemm_us / 1e6) / 1e12
    # the same GEMMs inside the step (per-phase pass: sustained load, power-capped
    # clocks), against the sustained int8 peak
    in_step = None
    if phases and phases.get("gemm"):
        t_in = phases["gemm"] / (STACK_L * C)
        a_in = gemm_ops / (t_in / 1e3) / 1e12
        in_step = {"avg_launch_us": t_in * 1e3, "achieved": a_in, "peak": 2.0 * bf16_sus,
                   "frac": a_in / (2.0 * bf16_sus),
                   "peak_source": f"2 x bf16_tflops_sustained ({bf16_sus:.1f}, {peak_src})",
                   "timing": "CUDA events around each GEMM launch of one eager forward (phases_ms.gemm / launches)"}
    # ours per step: input absmax + quantize, C GEMMs per layer, C quantizes per layer boundary
    launches_per_step = (2 + STACK_L * C + (STACK_L - 1) * C) if pipelined else (1 + 2 * STACK_L - 1)

    # e2e: host input rows in, this rank's fp32 output columns out, through the stack's public forward
    NB = 3
    rows = stack.input_rows(M) if pipelined else [(0, M)]
    m_loc = sum(b - a for a, b in rows)
    rs = np.random.RandomState(2000 + rank)
    del x_local
    torch.cuda.empty_cache()

    def forward_host_rows(xd):
        return (stack.forward_local(xd, M) if pipelined else stack(xd)).data

    _stage("stack: e2e")
    with _GpuLocalCpus(local_rank) as numa:
        x_host = [torch.from_numpy(rs.standard_normal((m_loc, STACK_D)).astype(np.float32)).pin_memory()
                  for _ in range(NB)]
        y_host = [torch.empty((M // stack.dp, n_loc), dtype=torch.float32).pin_memory() for _ in range(NB)]
        x_dev = [torch.empty((m_loc, STACK_D), dtype=torch.float32, device=dev) for _ in range(NB)]
        e2e_ms = _e2e_loop(forward_host_rows, x_host, y_host, x_dev, args.e2e_steps, world, dev)
        y_dev = torch.empty(y_host[0].shape, dtype=torch.float32, device=dev)
        copy_ms = _copies_only_ms(x_host, y_host, x_dev, y_dev, args.e2e_steps, world, dev)
    in_b, out_b = m_loc * STACK_D * 4, (M // stack.dp) * n_loc * 4
    e2e = {"value": M / (e2e_ms / args.e2e_steps / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": in_b * world, "d2h_bytes_per_step": out_b * world,
           "ms_per_step": e2e_ms / args.e2e_steps,
           "note": "bytes summed over ranks: each rank uploads its input rows and downloads its output columns",
           "host_copies_only": {
               "ms_per_step": copy_ms / args.e2e_steps,
               "h2d_gbs_per_rank": in_b / (copy_ms / args.e2e_steps / 1e3) / 1e9,
               "d2h_gbs_per_rank": out_b / (copy_ms / args.e2e_steps / 1e3) / 1e9,
               "note": "the same pinned copies, streams and sizes with no forward, all ranks at once (max over "
                       "ranks): the floor the host links put under the e2e step"},
           "host_threads": numa.note}
    del x_host, y_host, x_dev, y_dev
    torch.cuda.empty_cache()

    kernels = None
    if world == 1 and not args.no_kernels:
        _stage("kernels")
        kernels = measure_kernels(args, rank, world, local_rank, dev)
    if graph is not None:
        # a graph holding NCCL collectives must be released before the process
        # group is destroyed, or the destroy waits for it forever
        graph.reset()
        graph = None
    if world > 1:
        stack.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline("stack")
    ops = 2.0 * M * STACK_D * STACK_D * STACK_L
    line = {
        "metric": METRIC, "value": M / (ms_per_step / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": STACK_WORKLOAD, "global_batch": M, "seq_len": None,
                   "parallelism": ("single GPU" if world == 1 else
                                   f"dp{stack.dp} x tp{stack.tp} (weights column-sharded within groups of "
                                   f"{stack.tp}, activations row-sharded within and across them)"),
                   "exchange": stack.exchange, "row_chunks": C, "launch": graph_note,
                   "l2": "inputs larger than L2 (weights 1 GiB int8 codes in total, input 512 MiB fp32)"},
        "tops": ops / (ms_per_step / 1e3) / 1e12,
        "gpu_launches": launches_per_step * K,
        "roofline": {"kernel": "gemm_i8_kernel", "bound": "tensor", "achieved": gemm_tops, "peak": int8_peak,
                     "unit": "TOP/s", "frac": gemm_tops / int8_peak,
                     "traffic": profile_traffic(f"gemm_i8_{mc}x{n_loc}x{STACK_D}"),
                     "avg_launch_us": gemm_us,
                     "shape": f"M={mc} N={n_loc} K={STACK_D} (one row chunk of one layer on one rank)",
                     "algorithmic": f"2*M*N*K = {gemm_ops:.3e} op per launch",
                     "peak_source": f"2 x bf16_tflops ({bf16:.1f}, {peak_src}) -- int8 dense = 2x bf16 dense on B200",
                     "timing": f"CUDA events around replays (at least 20 ms) of a graph of the step's {4 * C} "
                               "GEMM launches (same shapes and weights) alone, right after the timed region",
                     "clocks": dict(KERNEL_CLOCKS).get("stack_gemm"),
                     "in_step": in_step},
        "phases_ms": phases,
        "output_checksum": checksum,
        "output_checksum_note": "sum of the int32 bit patterns of the full fp32 output over all ranks; equal at "
                                "every N when the sharded forward is bit-identical to the one-GPU forward",
        "parity_vs_one_gpu": parity,
        "device_status": status,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
    }
    if kernels is not None:
        line["kernels"] = kernels
    print(json.dumps(line))


# ----------------------------------------------------------- other lines

def run_linear(args, rank, world, local_rank, dev):
    """Config 2 as its own line: N > 1 runs it data-parallel (each rank its
    own 2048-token batch, weights replicated, no collective: "weak")."""
    import torch.distributed as dist
    r = measure_linear(args, rank, world, local_rank, dev, steps=args.steps, with_e2e=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None if (world > 1 or args.no_cpu_baseline) else cpu_baseline("linear")
    line = {"metric": METRIC, "value": r["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": r["steps"],
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": LINEAR_WORKLOAD, "launch": r["launch"], "global_batch": M_TOK * world,
                       "seq_len": None, "parallelism": f"dp{world} (row-sharded activations)", "l2": r["l2"]},
            "gpu_launches": 2 * r["steps"], "roofline": r["gemm"],
            "kernels": {"quantize_activations": r["quantize_activations"]},
            "e2e": r["e2e"], "cpu_baseline": cpu, "clocks": r["clocks"]}
    print(json.dumps(line))


def run_transformer(args, rank, world, local_rank, dev):
    """int8 2-layer decoder (d_model 256, 4 heads, FFN 1024
    GELU, vocab 65, context 256, batch 32 = 8192 tokens), per-channel int8
    weights, per-tensor int8 activations, fp32 LayerNorm / attention / softmax.
    One step = one forward of the batch, captured in a CUDA graph."""
    from kansaiml_b200 import workloads

    model = workloads.Decoder(seed=3, device=dev)
    ids = workloads.config3_ids(seed=4, device=dev)
    reps = 4
    g = _graph_of(lambda: model(ids), reps, dev)
    ms, steps, clocks = _time_graph(g, reps, args.steps, max(args.warmup, 3), local_rank, dev)
    if rank != 0:
        return
    tokens = ids.numel()
    ops = 2 * 2 * tokens * (4 * 256 * 256 + 2 * 256 * 1024) + 2 * tokens * 256 * 65
    line = {
        "metric": METRIC, "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "config3: int8 2-layer decoder d256 h4 ff1024 vocab65 ctx256, batch 32",
                   "global_batch": tokens, "seq_len": 256, "parallelism": "single GPU",
                   "launch": f"CUDA graphs of {reps} forwards replayed back to back",
                   "attention": "kz_attention_f32: the reference's operation order, fp32, no FMA"},
        "int8_ops_per_step": ops, "int8_tops": ops / (ms / 1e3) / 1e12,
        "clocks": clocks,
    }
    print(json.dumps(line))


SWEEP_N = (1024, 2048, 4096, 8192, 16384)


def run_sweep(args, rank, world, local_rank, dev):
    """square int8 GEMMs M = N = K in SWEEP_N, operands
    ~ U{-127..127}, per-row x per-column fp32 scales ~ U[1e-3, 1e-2] fused into
    the epilogue (fp32 out), and the int32-output form.  Sets of operands
    rotate so that each size's working set exceeds L2."""
    import torch
    from kansaiml_b200 import _lib

    lib = _lib.load()
    hbm_gbs, bf16, _, peak_src = peaks()
    peak = 2.0 * bf16
    rows, clocks = [], None
    for n in SWEEP_N:
        nsets = max(1, -(-(256 << 20) // (6 * n * n)))
        g = torch.Generator(device=dev)
        g.manual_seed(n)
        sets = []
        for _ in range(nsets):
            a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
            b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
            rs = torch.rand(n, device=dev, generator=g) * 9e-3 + 1e-3
            cs = torch.rand(n, device=dev, generator=g) * 9e-3 + 1e-3
            sets.append((a, b, rs, cs, torch.empty((n, n), dtype=torch.float32, device=dev)))
        res = {"n": n, "sets": nsets}
        for form in ("fp32_epilogue", "int32"):
            def call():
                for a, b, rs, cs, y in sets:
                    if form == "int32":
                        st = lib.kz_gemm_i8(a.data_ptr(), b.data_ptr(), n, n, n, n, None, 0, None, 0, None, 0, None,
                                            y.data_ptr(), n, None, _sh(dev))
                    else:
                        st = lib.kz_gemm_i8(a.data_ptr(), b.data_ptr(), n, n, n, n, rs.data_ptr(), 1, cs.data_ptr(), 1,
                                            None, 0, y.data_ptr(), None, n, None, _sh(dev))
                    _ok(st)
            reps = max(1, 16 // nsets) if n <= 4096 else 1
            gr = _graph_of(call, reps, dev)
            steps = max(4, min(args.steps, int(2e13 / (2.0 * n ** 3))))
            ms, done, clocks = _time_graph(gr, reps * nsets, steps, max(args.warmup, 3), local_rank, dev)
            tops = 2.0 * n ** 3 / (ms / 1e3) / 1e12
            res[form] = {"us": ms * 1e3, "tops": tops, "frac": tops / peak, "launches": done}
            del gr
        rows.append(res)
        del sets
        torch.cuda.empty_cache()
    head = next(r for r in rows if r["n"] == 8192)
    line = {
        "metric": METRIC, "value": head["fp32_epilogue"]["tops"], "unit": "TOP/s", "n_gpus": 1,
        "steps": head["fp32_epilogue"]["launches"], "warmup": max(args.warmup, 3),
        "ms_per_step": head["fp32_epilogue"]["us"] / 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "config4: square int8 GEMM sweep, per-row x per-column fp32 scale epilogue; "
                               "value = M=N=K=8192", "global_batch": None, "seq_len": None,
                   "parallelism": "single GPU", "l2": "operand sets rotate so each size's working set exceeds L2"},
        "sweep": rows,
        "roofline": {"kernel": "gemm_i8_kernel", "bound": "tensor", "peak": peak, "unit": "TOP/s",
                     "peak_source": f"2 x bf16_tflops ({bf16:.1f}, {peak_src})"},
        "clocks": clocks,
    }
    print(json.dumps(line))


def run_mlp(args, rank, world, local_rank, dev):
    """int8 MLP 784 -> 256 -> 10 (ReLU), batch 64, per-tensor
    weights and fp32 activations: the reference's own semantics
    (qlinear = x @ dequantize(W) + b), bit-identical outputs.  One step = one
    forward, captured in a CUDA graph."""
    import kansaiml_b200 as kz
    from kansaiml_b200 import nn
    from kansaiml_b200.quantize import QLinear

    l1, l2 = nn.Linear(784, 256, seed=1, device=dev), nn.Linear(256, 10, seed=2, device=dev)
    model = nn.Sequential(QLinear(l1), nn.ReLU(), QLinear(l2))
    x = kz.from_numpy(np.random.RandomState(0).uniform(0, 1, (64, 784)).astype(np.float32), device=dev)
    reps = 16
    g = _graph_of(lambda: model(x), reps, dev)
    ms, steps, clocks = _time_graph(g, reps, args.steps, max(args.warmup, 3), local_rank, dev)
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": 64 / (ms / 1e3), "unit": "rows/s", "n_gpus": 1, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (W8A32, reference semantics)", "data": "synthetic",
        "config": {"workload": "config1: int8 MLP 784-256-10 ReLU, batch 64, per-tensor weights, fp32 activations",
                   "global_batch": 64, "seq_len": None, "parallelism": "single GPU",
                   "launch": f"CUDA graphs of {reps} forwards"},
        "us_per_forward": ms * 1e3,
        "clocks": clocks,
    }
    print(json.dumps(line))


def run_kernels(args, rank, world, local_rank, dev):
    """The per-kernel entries of the default line on their own (N = 1)."""
    k = measure_kernels(args, rank, world, local_rank, dev)
    if rank == 0:
        print(json.dumps({"metric": METRIC, "workload": "per-kernel entries (N = 1)", "kernels": k}))


def run_gemm(args, rank, world, local_rank, dev):
    """A few launches of the int8 GEMM at one shape (--shape M,N,K), fp32
    epilogue with per-row x per-column scales and absmax partials, as the
    sharded stack launches it: a profiling target."""
    import torch
    from kansaiml_b200 import _lib
    lib = _lib.load()
    M, N, K = (int(v) for v in args.shape.split(","))
    g = torch.Generator(device=dev)
    g.manual_seed(M + N + K)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
    rs_ = torch.full((1,), 1e-3, device=dev)
    cs_ = torch.rand(N, device=dev, generator=g) * 9e-3 + 1e-3
    y = torch.empty((M, N), dtype=torch.float32, device=dev)
    parts = torch.zeros(_lib.KZ_PARTIALS_WORDS, dtype=torch.int32, device=dev)

    def call():
        _ok(lib.kz_gemm_i8(a.data_ptr(), b.data_ptr(), M, N, K, K, rs_.data_ptr(), 0, cs_.data_ptr(), 1, None, 0,
                           y.data_ptr(), None, N, parts.data_ptr(), _sh(dev)))
    for _ in range(max(args.warmup, 1)):
        call()
    torch.cuda.synchronize()
    start, end = _events(dev)
    start.record(torch.cuda.current_stream(dev))
    for _ in range(args.steps):
        call()
    end.record(torch.cuda.current_stream(dev))
    torch.cuda.synchronize()
    us = start.elapsed_time(end) / args.steps * 1e3
    if rank == 0:
        print(json.dumps({"metric": METRIC, "workload": f"int8 GEMM M={M} N={N} K={K}", "avg_us": us,
                          "tops": 2.0 * M * N * K / (us / 1e6) / 1e12, "launches": args.steps + max(args.warmup, 1)}))


def run_attention(args, rank, world, local_rank, dev):
    """Config 3's attention core alone (batch 32, 4 heads, 256 queries and
    keys, d_k 64, causal, q|k|v read from one [32, 256, 768] projection
    output): W + K launches, CUDA events around the K; a profiling target."""
    import torch
    from kansaiml_b200 import _lib
    lib = _lib.load()
    B, S, D, H = 32, 256, 256, 4
    g = torch.Generator(device=dev)
    g.manual_seed(256)
    qkv = torch.randn((B, S, 3 * D), generator=g, device=dev)
    out = torch.empty((B, S, D), device=dev)
    parts = torch.zeros(_lib.KZ_PARTIALS_WORDS, dtype=torch.int32, device=dev)

    def call():
        _ok(lib.kz_attention_f32(qkv.data_ptr(), qkv.data_ptr() + 4 * D, qkv.data_ptr() + 8 * D, B, H, S, S, D // H,
                                 3 * D, 3 * D, 3 * D, None, 0, 0, 0, 1, 0.125, out.data_ptr(), D, parts.data_ptr(),
                                 _sh(dev)))
    _time_launches(args, rank, dev, call, "attention core, config 3 (32 x 4 heads x 256, d_k 64, causal)",
                   {"op": B * H * (S * (S + 1) // 2) * 4.0 * (D // H)})


def run_dequantize(args, rank, world, local_rank, dev):
    """kz_dequantize_i8_f32 on config 2's 2048 x 4096 activation codes, scale
    0.01: W + K launches, CUDA events around the K; a profiling target."""
    import torch
    from kansaiml_b200 import _lib
    lib = _lib.load()
    n = M_TOK * K_IN
    g = torch.Generator(device=dev)
    g.manual_seed(n)
    q = torch.randint(-127, 128, (n,), dtype=torch.int8, device=dev, generator=g)
    out = torch.empty(n, device=dev)

    def call():
        _ok(lib.kz_dequantize_i8_f32(q.data_ptr(), n, 0.01, out.data_ptr(), _sh(dev)))
    _time_launches(args, rank, dev, call, "dequantize, 2048 x 4096 codes", {"bytes": 5.0 * n})


def run_quantize_cols(args, rank, world, local_rank, dev):
    """kz_quantize_cols_f32 on config 2's 4096 x 4096 weight (per-channel
    int8, K-major codes): W + K launches, CUDA events around the K; a
    profiling target."""
    import torch
    from kansaiml_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device=dev)
    g.manual_seed(K_IN)
    w = torch.randn((K_IN, N_OUT), generator=g, device=dev) * 0.02
    qT = torch.empty((N_OUT, K_IN), dtype=torch.int8, device=dev)
    s64 = torch.empty(N_OUT, dtype=torch.float64, device=dev)
    s32 = torch.empty(N_OUT, device=dev)
    ws = torch.empty(lib.kz_quantize_cols_workspace_bytes(K_IN, N_OUT), dtype=torch.uint8, device=dev)

    def call():
        _ok(lib.kz_quantize_cols_f32(w.data_ptr(), K_IN, N_OUT, qT.data_ptr(), s64.data_ptr(), s32.data_ptr(),
                                     ws.data_ptr(), ws.numel(), _sh(dev)))
    _time_launches(args, rank, dev, call, "per-channel weight quantize, 4096 x 4096", {"bytes": 5.0 * K_IN * N_OUT})


def _time_launches(args, rank, dev, call, name, work):
    import torch
    for _ in range(max(args.warmup, 1)):
        call()
    torch.cuda.synchronize()
    start, end = _events(dev)
    start.record(torch.cuda.current_stream(dev))
    for _ in range(args.steps):
        call()
    end.record(torch.cuda.current_stream(dev))
    torch.cuda.synchronize()
    us = start.elapsed_time(end) / args.steps * 1e3
    if rank == 0:
        line = {"metric": METRIC, "workload": name, "avg_us": us, "launches": args.steps + max(args.warmup, 1)}
        if "op" in work:
            line["top_s"] = work["op"] / (us / 1e6) / 1e12
        if "bytes" in work:
            line["gb_s"] = work["bytes"] / (us / 1e6) / 1e9
        print(json.dumps(line))


# ------------------------------------------------------------------- main

def main():
    args = parse()
    if os.environ.get("KZ_BENCH_TRACEBACK_S"):
        # diagnosis of a stalled run: every rank prints its threads' stacks periodically
        import faulthandler
        faulthandler.dump_traceback_later(int(os.environ["KZ_BENCH_TRACEBACK_S"]), repeat=True)
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    rank, world, local_rank = dist_env()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        # The communicator's set-up prints a version banner on stdout (file
        # descriptor 1); stdout carries only rank 0's JSON line, so fd 1
        # points at stderr while the group and its communicator come up.
        sys.stdout.flush()
        saved_fd = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved_fd, 1)
            os.close(saved_fd)
    {"stack": run_stack, "linear": run_linear, "transformer": run_transformer, "sweep": run_sweep,
     "mlp": run_mlp, "kernels": run_kernels, "gemm": run_gemm, "attention": run_attention,
     "dequantize": run_dequantize, "quantize_cols": run_quantize_cols}[args.workload](args, rank, world, local_rank,
                                                                                     dev)


if __name__ == "__main__":
    main()
