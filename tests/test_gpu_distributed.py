"""GPU parity of the sharded int8 stack and of DTensor
dispatch.  Sharding changes no arithmetic, so every configuration must equal
the oracle's unsharded chain bit for bit:

    a0 = quantize_tensor(x); for each layer: acc = a @ Wq^T (int32),
    y = epilogue(acc, s_a, s_w) (fp32); (a, s_a) = quantize_tensor(y)

The multi-GPU cases run only where two GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import cpu as ocpu

pytestmark = pytest.mark.gpu

DIMS = [1024, 1024, 2048, 1024]   # in -> ... -> out
M = 384


def make_weights():
    rs = np.random.RandomState(55)
    return [(rs.standard_normal((DIMS[i], DIMS[i + 1])) * 0.01).astype(np.float32) for i in range(len(DIMS) - 1)]


def make_x(m=M):
    return np.random.RandomState(56).standard_normal((m, DIMS[0])).astype(np.float32)


def oracle_chain(x, weights):
    a, s_a = ocpu.quantize_tensor(x)
    y = None
    for i, w in enumerate(weights):
        wq, ws = ocpu.quantize_cols(w)
        acc = ocpu.gemm_i8(a, wq)
        y = ocpu.epilogue(acc, s_a, ws)
        if i < len(weights) - 1:
            a, s_a = ocpu.quantize_tensor(y)
    return y


@pytest.fixture(scope="module")
def expected():
    return oracle_chain(make_x(), make_weights())


def test_stack_single_gpu_bit_exact(cuda_device, expected):
    from kansaiml_b200.distributed import ShardedQLinearStack
    stack = ShardedQLinearStack([torch.from_numpy(w).cuda() for w in make_weights()])
    y = stack(torch.from_numpy(make_x()).cuda()).numpy()
    assert y.tobytes() == expected.tobytes()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spmd_worker(rank, world, port, q, exchange, tp=None):
    try:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        from kansaiml_b200.distributed import DeviceMesh, ShardedQLinearStack
        mesh = DeviceMesh.spmd()
        stack = ShardedQLinearStack([torch.from_numpy(w).cuda() for w in make_weights()], mesh, exchange=exchange,
                                    tp=tp)
        assert stack.exchange == (exchange if stack.tp > 1 else "collective")
        x = torch.from_numpy(make_x()).cuda()
        y = stack(x, return_local=False).numpy()
        y2 = stack(x, return_local=False).numpy()   # buffers, flags and tokens reused
        q.put((rank, y if y.tobytes() == y2.tobytes() else "second forward differs"))
        from kansaiml_b200.quantize import device_status
        assert device_status() == 0
        stack.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["collective", "peer", "fused", "ce"])
def test_stack_two_gpus_spmd_bit_exact(expected, exchange):
    """Two ranks over NCCL: the plain all-gather; the all-gather overlapped
    with the next GEMM (peer buffers + copy engines + the gated GEMM); and the
    all-gather inside the GEMM launch (copy CTAs TMA-load this rank's block
    from local memory and push it to the peers with 16-byte stores)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_spmd_worker, args=(r, 2, port, q, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, y = q.get(timeout=300)
        res[r] = y
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert isinstance(res[r], np.ndarray), res[r]
        assert res[r].tobytes() == expected.tobytes()


@pytest.mark.parametrize("world,tp,exchange", [(2, 1, "collective"), (4, 2, "ce"), (4, 2, "collective")])
def test_stack_row_groups_spmd_bit_exact(expected, world, tp, exchange):
    """Row groups x column shards: world / tp groups of tp ranks, each group
    on its own rows (tp = 1 is pure data parallelism), the absmax all-reduced
    over every rank: the gathered output equals the oracle's unsharded chain
    bit for bit.  Needs `world` GPUs."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_spmd_worker, args=(r, world, port, q, exchange, tp)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, y = q.get(timeout=300)
        res[r] = y
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert isinstance(res[r], np.ndarray), res[r]
        assert res[r].tobytes() == expected.tobytes()


M_PIPE = 2048   # four row chunks of 512 on two ranks


def _pipelined_worker(rank, world, port, q, exchange="collective"):
    try:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        from kansaiml_b200 import _lib
        from kansaiml_b200 import distributed as kd
        mesh = kd.DeviceMesh.spmd()
        stack = kd.ShardedQLinearStack([torch.from_numpy(w).cuda() for w in make_weights()], mesh, exchange=exchange)
        assert stack.chunks(M_PIPE) == 4
        x = torch.from_numpy(make_x(M_PIPE)).cuda()
        full = stack(x, return_local=False).numpy()
        # the same forward replayed from a CUDA graph (NCCL all-gathers and
        # all-reduces captured), with the GEMMs' SM budget cut for the overlap
        assert _lib.load().kz_set_sm_count_target(100) == 0
        xl = stack.local_input(x)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            out = stack.forward_local(xl, M_PIPE)
        g.replay()
        g.replay()
        torch.cuda.synchronize()
        lo, hi = kd.column_shard_bounds(DIMS[-1], rank, world)
        graphed = out.data.cpu().numpy()
        ok = graphed.tobytes() == np.ascontiguousarray(full[:, lo:hi]).tobytes()
        # per-phase timing path
        stack.timing = True
        stack.forward_local(xl, M_PIPE)
        phases = stack.phase_times()
        stack.timing = False
        ok = ok and set(phases) >= {"gemm", "input_quantize", "quantize", "allreduce_max"}
        # dtensor_grad over NCCL: Replicate -> all-reduce sum in the
        # reference's double order, Shard(0) -> concatenation
        local = torch.full((3, 2), float(rank + 1), device="cuda") / 3
        rep, sh = kd.dtensor_grad(lambda t: (t, t * 2), [kd.Replicate(), kd.Shard(0)],
                                  kd.DTensor(mesh, kd.Shard(0), [kz_tensor(local)]))
        want_rep = np.float32(sum(np.float64(np.float32((r + 1) / 3)) for r in range(world)))
        ok = ok and np.all(rep.numpy() == want_rep)
        ok = ok and sh.shape == [3 * world, 2]
        from kansaiml_b200.quantize import device_status
        assert device_status() == 0
        g.reset()
        del g
        stack.close()
        q.put((rank, full if ok else "graph replay, phases or dtensor_grad differ"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def kz_tensor(t):
    from kansaiml_b200.tensor import Tensor
    return Tensor(t)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["collective", "ce"])
def test_stack_pipelined_two_gpus_graph_and_grad(exchange):
    """Two ranks, 2048 rows in four row chunks: the pipelined forward (input
    rows quantized per rank and exchanged chunk by chunk, every layer's codes
    exchanged chunk by chunk under the next GEMM -- by NCCL all-gathers, or by
    copy-engine pulls from IPC-shared buffers) equals the oracle's unsharded
    chain bit for bit, also when replayed from a CUDA graph that captured its
    collectives and copies; dtensor_grad's NCCL reductions match the
    reference's double-precision sum."""
    expected_pipe = oracle_chain(make_x(M_PIPE), make_weights())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pipelined_worker, args=(r, 2, port, q, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, y = q.get(timeout=300)
        res[r] = y
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert isinstance(res[r], np.ndarray), res[r]
        assert res[r].tobytes() == expected_pipe.tobytes()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_dtensor_single_process_two_gpus():
    """The reference's threaded mesh, on two GPUs: batch Shard(0), weight
    replicated, per-channel W8A8 qlinear on each device, gathered result equal
    to one device's."""
    import kansaiml_b200 as kz
    from kansaiml_b200 import distributed as kd
    from kansaiml_b200.quantize import QTensor, qlinear
    w = make_weights()[0]
    x = make_x()
    mesh = kd.DeviceMesh(["cuda:0", "cuda:1"])
    xd = kd.DTensor.from_tensor(kz.from_numpy(x, device="cuda:0"), mesh, kd.Shard(0))
    wq = {i: QTensor.from_tensor(kz.from_numpy(w, device=f"cuda:{i}"), per_channel=True) for i in range(2)}

    def fwd(xs):
        return qlinear(xs, wq[xs.device.index])
    out = kd.dtensor_run(fwd, kd.Shard(0), xd).to_tensor().numpy()
    whole = qlinear(kz.from_numpy(x, device="cuda:0"), wq[0]).numpy()
    # per-tensor activation scales differ per shard (each shard is its own
    # tensor, as in the reference's dtensor_run); compare each half to its own run
    for i, (lo, hi) in enumerate([(0, M // 2), (M // 2, M)]):
        part = qlinear(kz.from_numpy(x[lo:hi], device="cuda:0"), wq[0]).numpy()
        assert out[lo:hi].tobytes() == part.tobytes()
    assert out.shape == whole.shape
