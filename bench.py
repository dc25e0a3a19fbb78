"""Benchmark of Kansai's int8 quantized-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ("config 2"): one per-channel int8
quantized Linear, fp32 weight [4096, 4096] ~ N(0, 0.02) quantized once per
output channel, fp32 activations [2048, 4096] ~ N(0, 1).  One step = one
forward of that layer over one batch of 2048 tokens: per-tensor activation
absmax + quantize (one HBM-bound cooperative launch), then the tcgen05 int8
GEMM with the per-row x per-channel rescale fused into its epilogue, fp32
output.  Weight
quantization is the layer's one-time construction (QLinear.__init__), as in
the reference (quantize.py:139-141), and is not in the step.

Inputs exceed L2: 4 rotating sets of (X fp32, weight codes, Y fp32) = 336 MB,
so every step reads cold data.  Timing: W warm-up steps, then K steps (CUDA
graphs of 8 steps replayed back to back) between barrier + synchronize on
both sides, CUDA events on the launching stream, max over ranks.  N > 1 (torchrun): activations row-sharded, weights replicated:
every rank runs its own 2048-token batch, no collective on the data path
("weak" scaling).

--impl reference: the reference's own CPU implementation of this layer,
qlinear (quantize.py:115-122) = dequantize the weight in Python, then the
reference's C++ Tensor::matmul + add (oracle/_ref, compiled from the
reference's sources), on a bounded row sample, rows spread over all host
threads as the reference's Shard(0) DeviceMesh dispatch does
(distributed.py:73-102).  Under torchrun only rank 0 runs it.
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

M_TOK, K_IN, N_OUT = 2048, 4096, 4096
NSETS = 4
METRIC = "int8 GEMM TOPS & quantized-linear tokens/s vs int8 roofline at 1/2/4/8 B200"
WORKLOAD = ("config2: per-channel int8 quantized Linear [4096 -> 4096], 2048 tokens/step/GPU, "
            "per-tensor activation quant, fused rescale, fp32 out")
FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS = 6650.0, 1590.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--exchange", choices=["peer", "collective", "fused"], default=None,
                    help="stack workload, N > 1: plain NCCL all-gather (collective, default) or the copy-engine "
                         "all-gather overlapped with the gated GEMM (peer)")
    ap.add_argument("--workload", choices=["linear", "stack", "transformer", "sweep", "mlp"], default="linear",
                    help="linear: config 2 (default); stack: config 5, column-sharded 4-layer stack; "
                         "transformer: config 3 decoder; sweep: config 4 square GEMMs; mlp: config 1")
    return ap.parse_args()


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

def reference_sample_step(core, q_list, scale, shape, x_parts, bias_t, threads):
    """One qlinear call of the reference (quantize.py:115-122) on the row sample:
    dequantize in Python (quantize.py:76-77), then the compiled reference core's
    Tensor::matmul + add per row part on its own thread (GIL released)."""
    flat = [v * scale for v in q_list]
    w = core.from_flat(flat, shape)
    out = [None] * len(x_parts)

    def work(i):
        out[i] = x_parts[i].matmul(w).add(bias_t)

    ts = [threading.Thread(target=work, args=(i,)) for i in range(len(x_parts))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    return out


def reference_setup(rows_per_thread=8):
    from oracle import cpu as ocpu
    from oracle.refpkg import load_reference_core
    core = load_reference_core()
    threads = os.cpu_count() or 1
    rs = np.random.RandomState(7)
    w = (rs.standard_normal((K_IN, N_OUT)) * 0.02).astype(np.float32)
    q, scale = ocpu.quantize_tensor(w)           # the reference's per-tensor scheme
    rows = rows_per_thread * threads
    x = rs.standard_normal((rows, K_IN)).astype(np.float32)
    parts = [core.from_flat(p.ravel().tolist(), [p.shape[0], K_IN]) for p in np.array_split(x, threads)]
    bias = core.from_flat([0.0] * N_OUT, [N_OUT])
    return core, q.ravel().tolist(), float(scale), [K_IN, N_OUT], parts, bias, threads, rows


def time_reference(steps, warmup, budget_s=None):
    """Times `steps` reference qlinear calls (after `warmup`); with a budget,
    runs as many of the requested steps as fit in it.  Returns
    (tokens/s, seconds per step, threads, rows per step, steps timed)."""
    core, ql, scale, shape, parts, bias, threads, rows = reference_setup()
    t_w = time.perf_counter()
    for _ in range(max(warmup, 1)):
        reference_sample_step(core, ql, scale, shape, parts, bias, threads)
    est = (time.perf_counter() - t_w) / max(warmup, 1)
    if budget_s is not None:
        steps = max(1, min(steps, int(budget_s / max(est, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(steps):
        reference_sample_step(core, ql, scale, shape, parts, bias, threads)
    dt = (time.perf_counter() - t0) / steps
    return rows / dt, dt, threads, rows, steps


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    try:
        value, dt, threads, rows, timed = time_reference(args.steps, min(args.warmup, 1), budget_s=120.0)
    except Exception as e:  # the compiled reference core is missing
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU path could not run: {e}"}))
        return
    sample = (f"reference qlinear on {rows} of 2048 rows of config 2 (weight dequantized in Python every call, "
              f"quantize.py:121, then Tensor::matmul + add split over {threads} threads)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": timed, "steps_requested": args.steps, "warmup": min(args.warmup, 1), "ms_per_step": dt * 1e3,
            "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": M_TOK, "parallelism": "host threads",
                       "reference_path": "the reference's only qlinear: per-tensor int8 weight dequantized to fp32 "
                                         "every call (quantize.py:115-122), fp32 Tensor::matmul + add"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def cpu_baseline():
    try:
        value, dt, threads, rows, _ = time_reference(steps=3, warmup=1)
        return {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                "sample": f"reference qlinear (quantize.py:115-122; dequantize in Python each call, compiled "
                          f"reference Tensor::matmul + add) on {rows} rows of config 2, 3 timed calls, "
                          f"{threads} threads"}
    except Exception as e:
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}


# ---------------------------------------------------------------- our path

def main():
    args = parse()
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
    if args.workload != "linear":
        {"stack": run_stack, "transformer": run_transformer, "sweep": run_sweep, "mlp": run_mlp}[args.workload](
            args, rank, world, local_rank, dev)
        return

    import kansaiml_b200 as kz
    from kansaiml_b200 import _lib
    from kansaiml_b200 import quantize as kq

    lib = _lib.load()
    rs = np.random.RandomState(1000 + rank)
    # one-time layer construction: NSETS independent weights, quantized per channel
    layers = []
    for i in range(NSETS):
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
        """The activation absmax + quantize of set i % NSETS (one cooperative launch)."""
        sh = torch.cuda.current_stream(dev).cuda_stream
        if lib.kz_quantize_tensor_f32(X[i % NSETS], n_el, XQ, S64, S32, PP, sh):
            raise RuntimeError(_lib.last_error())

    def gemm_only(i):
        """The int8 GEMM with fused rescale of set i % NSETS."""
        j = i % NSETS
        sh = torch.cuda.current_stream(dev).cuda_stream
        if lib.kz_gemm_i8(XQ, B[j][0], M_TOK, N_OUT, K_IN, K_IN, S32, 0, B[j][1], 1, None, 0, Y[j], None, N_OUT,
                          None, sh):
            raise RuntimeError(_lib.last_error())

    def step(i):
        """One forward of the layer on rotating set i % NSETS: activation absmax +
        quantize (one cooperative launch), int8 GEMM with fused rescale."""
        quantize_only(i)
        gemm_only(i)

    # first step eagerly (sets up per-device state), then check the device status
    step(0)
    torch.cuda.synchronize()
    if kq.device_status() != 0:
        raise RuntimeError("device status set after the first step")

    # Timed steps run from CUDA graphs of S consecutive steps (2 kernel nodes
    # each, no event nodes), replayed back to back, as a model captures its
    # layers.  A second pass times each kernel alone: graphs of S launches of
    # just that kernel over the same rotating sets, replayed back to back with
    # CUDA events only around the replays (event nodes between the two kernels
    # of a step would break their programmatic dependent launch and add the
    # gaps to both), for the per-kernel and roofline figures.
    S = 8
    cap_stream = torch.cuda.Stream(dev)

    def capture(idx, fn=step):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=cap_stream):
            for i in idx:
                fn(i)
        return gr

    K = args.steps
    chunk_graph = capture(range(S))
    tail_graph = capture(range(K % S)) if K % S else None
    quant_graph = capture(range(S), quantize_only)
    gemm_graph = capture(range(S), gemm_only)
    torch.cuda.synchronize()

    # warm-up: at least W steps, through the same graphs the timed region replays
    for _ in range(max(1, -(-args.warmup // S))):
        chunk_graph.replay()
    if tail_graph is not None:
        tail_graph.replay()
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    # per-kernel device times: as many launches of each kernel alone as the timed region made
    reps = max(1, K // S)

    def kernel_ms(gr):
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            gr.replay()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / (reps * S)
    quant_avg = kernel_ms(quant_graph)
    gemm_avg = kernel_ms(gemm_graph)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / K
    tokens = M_TOK * world
    value = tokens / (ms_per_step / 1e3)
    ops = 2.0 * M_TOK * N_OUT * K_IN
    hbm_gbs, bf16, bf16_sus, peak_src = peaks()
    int8_peak = 2.0 * bf16   # B200 int8 dense rate is 2x its bf16 dense rate
    tops = ops / (gemm_avg / 1e3) / 1e12
    # algorithmic bytes: absmax pass 4 B/element + quantize pass 4 + 1 B/element,
    # counted per pass although the single launch reads x from HBM once
    quant_bytes = 9.0 * n_el

    # ------------------------------------------------------------ e2e
    # Through the public API with host buffers: every step copies its pinned
    # host X to the device, runs QLinear, and copies its fp32 Y back to pinned
    # host memory.  Copies run on their own streams over NB buffers, so step
    # i's upload, earlier steps' forwards and downloads overlap (PCIe carries
    # both directions at once); every step still moves its own bytes.
    NB = 3
    x_host = [torch.from_numpy(rs.standard_normal((M_TOK, K_IN)).astype(np.float32)).pin_memory() for _ in range(NB)]
    y_host = [torch.empty((M_TOK, N_OUT), dtype=torch.float32).pin_memory() for _ in range(NB)]
    x_dev = [torch.empty((M_TOK, K_IN), dtype=torch.float32, device=dev) for _ in range(NB)]
    y_dev = [None] * NB
    layer = layers[0]
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
        stream.wait_event(ev_out[b])              # y_dev[b] of NB steps ago has been read back
        y_dev[b] = layer(kz.Tensor(x_dev[b])).data
        ev_fwd[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_fwd[b])
            y_host[b].copy_(y_dev[b], non_blocking=True)
            y_dev[b].record_stream(s_out)
            ev_out[b].record(s_out)

    for i in range(3):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.e2e_steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = tokens / (e2e_ms / args.e2e_steps / 1e3)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()
    traffic = profile_traffic("gemm_i8_config2")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD,
                   "launch": f"CUDA graphs of {S} steps (2 libkz kernels per step) replayed back to back",
                   "global_batch": tokens, "seq_len": None, "parallelism": f"dp{world} (row-sharded activations)",
                   "l2": f"inputs larger than L2: {NSETS} rotating (X, W, Y) sets, "
                         f"{NSETS * (M_TOK * K_IN * 4 + K_IN * N_OUT + M_TOK * N_OUT * 4) / 1e6:.0f} MB"},
        "tops": ops * world / (ms_per_step / 1e3) / 1e12,
        "gpu_launches": 2 * K,
        "roofline": {"kernel": "gemm_i8_kernel", "bound": "tensor", "achieved": tops, "peak": int8_peak,
                     "unit": "TOP/s", "frac": tops / int8_peak, "traffic": traffic,
                     "peak_source": f"2 x bf16_tflops ({bf16:.1f}, {peak_src}) -- int8 dense = 2x bf16 dense on B200",
                     "avg_launch_us": gemm_avg * 1e3,
                     "timing": f"CUDA events around {reps} back-to-back replays of a graph of {S} launches of "
                               "this kernel alone over the same rotating sets, right after the timed region",
                     "algorithmic": f"2*M*N*K = {ops:.3e} op per launch"},
        "kernels": {"quantize_activations": {"avg_us": quant_avg * 1e3, "bound": "hbm",
                                             "achieved_gbs": quant_bytes / (quant_avg / 1e3) / 1e9,
                                             "peak_gbs": hbm_gbs, "frac": quant_bytes / (quant_avg / 1e3) / 1e9 / hbm_gbs,
                                             "algorithmic": "9 B/element (absmax 4 + quantize 4+1, per pass; the launch reads x from HBM once, "
                                                             "5 B/element of DRAM traffic)"}},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": M_TOK * K_IN * 4,
                "d2h_bytes_per_step": M_TOK * N_OUT * 4},
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
    }
    print(json.dumps(line))


# ------------------------------------------------- config 5: sharded stack

STACK_M, STACK_D, STACK_L = 8192, 16384, 4


def run_stack(args, rank, world, local_rank, dev):
    """4 int8 Linear layers [16384 -> 16384], weights
    ~ N(0, 0.01) quantized per output channel and column-sharded over the
    ranks, activations fp32 [8192, 16384] ~ N(0, 1) quantized per tensor and
    all-gathered (int8, NCCL over NVLink) between layers.  One step = one
    forward of the stack over the 8192-token batch; total work fixed as N grows
    ("strong" scaling).  Output: each rank's fp32 column shard."""
    import torch
    import torch.distributed as dist

    from kansaiml_b200.distributed import DeviceMesh, ShardedQLinearStack

    mesh = DeviceMesh.spmd() if world > 1 else None

    def weight(l):
        g = torch.Generator(device=dev)
        g.manual_seed(5000 + l)
        return torch.randn((STACK_D, STACK_D), generator=g, device=dev) * 0.01

    stack = ShardedQLinearStack([weight] * STACK_L, mesh, exchange=args.exchange)
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    x = torch.randn((STACK_M, STACK_D), generator=g, device=dev)
    torch.cuda.synchronize()
    for _ in range(max(args.warmup, 3)):
        stack(x)
    K = args.steps
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for _ in range(K):
            stack(x)
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        stack.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    ms_per_step = ms / K
    ops = 2.0 * STACK_M * STACK_D * STACK_D * STACK_L
    tops = ops / (ms_per_step / 1e3) / 1e12
    hbm_gbs, bf16, _, peak_src = peaks()
    line = {
        "metric": METRIC, "value": STACK_M / (ms_per_step / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "config5: 4 x int8 Linear [16384 -> 16384] column-sharded, 8192 tokens, per-tensor "
                               "activation quant + NCCL all-gather between layers",
                   "global_batch": STACK_M, "seq_len": None, "parallelism": f"tp{world} (column-sharded weights)",
                   "exchange": stack.exchange,
                   "l2": "inputs larger than L2 (weights 1 GiB int8 in total, activations 512 MiB fp32)"},
        "tops": tops,
        "roofline": {"kernel": "whole stack", "bound": "tensor", "achieved": tops, "peak": 2.0 * bf16 * world,
                     "unit": "TOP/s", "frac": tops / (2.0 * bf16 * world), "traffic": None,
                     "peak_source": f"{world} x 2 x bf16_tflops ({bf16:.1f}, {peak_src})"},
        "gpu_launches": (1 + 2 * STACK_L - 1) * K,
        "clocks": clk.summary(),
    }
    print(json.dumps(line))



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
    """Replays g until `steps` calls ran; returns (ms per call, clocks)."""
    import torch
    for _ in range(max(1, -(-warmup // reps_per_graph))):
        g.replay()
    torch.cuda.synchronize()
    n = max(1, -(-steps // reps_per_graph))
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for _ in range(n):
            g.replay()
        end.record(stream)
        torch.cuda.synchronize()
    return start.elapsed_time(end) / (n * reps_per_graph), n * reps_per_graph, clk.summary()


def run_transformer(args, rank, world, local_rank, dev):
    """int8 2-layer decoder (d_model 256, 4 heads, FFN 1024
    GELU, vocab 65, context 256, batch 32 = 8192 tokens), per-channel int8
    weights, per-tensor int8 activations, fp32 LayerNorm / attention / softmax.
    One step = one forward of the batch, captured in a CUDA graph."""
    import torch
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
                   "launch": f"CUDA graphs of {reps} forwards replayed back to back"},
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
                sh = torch.cuda.current_stream(dev).cuda_stream
                for a, b, rs, cs, y in sets:
                    if form == "int32":
                        st = lib.kz_gemm_i8(a.data_ptr(), b.data_ptr(), n, n, n, n, None, 0, None, 0, None, 0, None,
                                            y.data_ptr(), n, None, sh)
                    else:
                        st = lib.kz_gemm_i8(a.data_ptr(), b.data_ptr(), n, n, n, n, rs.data_ptr(), 1, cs.data_ptr(), 1,
                                            None, 0, y.data_ptr(), None, n, None, sh)
                    if st:
                        raise RuntimeError(_lib.last_error())
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
    import torch
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


if __name__ == "__main__":
    main()
