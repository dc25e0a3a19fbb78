"""Host-side logic of kansaiml_b200.distributed on CPU: the reference's
split/concat and chunking rules (pinned to the reference's own _chunk_sizes
outputs), mesh validation, threaded dispatch, and the collectives of the
sharded stack on world_size-2 gloo process groups.  No GPU compute."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import kansaiml_b200 as kz
from conftest import golden
from kansaiml_b200 import distributed as kd


def test_chunk_sizes_match_reference():
    g = golden("chunk_cases.npz")
    flat, lens = g["flat"].tolist(), g["lens"].tolist()
    off = 0
    for (total, n), ln in zip(g["pairs"].tolist(), lens):
        assert kd._chunk_sizes(total, n) == flat[off:off + ln]
        off += ln


def test_split_concat_roundtrip_uneven_and_dim1():
    """tests/test_distributed.py:32-51 restated."""
    vals = np.random.RandomState(0).uniform(-1, 1, 7 * 4).astype(np.float32)
    t = kz.from_flat(vals, [7, 4], device="cpu")
    pieces = kd._split_tensor(t, 0, 3)
    assert [p.shape for p in pieces] == [[3, 4], [2, 4], [2, 4]]
    assert kd._concat_tensors(pieces, 0).tolist() == vals.tolist()
    vals2 = np.random.RandomState(1).uniform(-1, 1, 3 * 8).astype(np.float32)
    t2 = kz.from_flat(vals2, [3, 8], device="cpu")
    pieces2 = kd._split_tensor(t2, 1, 4)
    assert [p.shape for p in pieces2] == [[3, 2]] * 4
    assert kd._concat_tensors(pieces2, 1).tolist() == vals2.tolist()


def test_mesh_rejects_unknown_device():
    with pytest.raises(ValueError, match="unknown device"):
        kd.DeviceMesh(["cpu", "tpu"])
    with pytest.raises(ValueError, match="unknown device"):
        kd.DeviceMesh(["metal"])


def test_dtensor_cpu_mesh_shard_and_replicate():
    mesh = kd.DeviceMesh(["cpu", "cpu"])
    x = kz.from_flat(np.arange(8 * 3, dtype=np.float32), [8, 3], device="cpu")
    dt = kd.DTensor.from_tensor(x, mesh, kd.Shard(0))
    assert [s.shape for s in dt.shards] == [[4, 3], [4, 3]]
    out = kd.dtensor_run(lambda s: s.mul(2.0), kd.Shard(0), dt)
    assert out.to_tensor().tolist() == (np.arange(24, dtype=np.float32) * 2).tolist()
    rep = kd.DTensor.from_tensor(x, mesh, kd.Replicate())
    assert rep.to_tensor().tolist() == x.tolist()
    with pytest.raises(ValueError):
        kd.DTensor(mesh, kd.Shard(0), [x])


def test_run_parallel_reraises_worker_error():
    def bad():
        raise KeyError("boom")
    with pytest.raises(KeyError):
        kd._run_parallel([lambda: 1, bad])


def test_column_shard_bounds():
    assert [kd.column_shard_bounds(16384, r, 8) for r in (0, 7)] == [(0, 2048), (14336, 16384)]
    assert [kd.column_shard_bounds(10, r, 4) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        # absmax partials: per-rank maxima combine by integer MAX (float bit order)
        p = torch.zeros(1024, dtype=torch.int32)
        vals = np.asarray([0.5 + rank, 3.0 - rank, 1e-3 * (rank + 1)], np.float32).view(np.int32)
        p[0] = 3
        p[1:4] = torch.from_numpy(vals.copy())
        p[-1] = 7 + rank                      # barrier generation word: left untouched
        kd.allreduce_partials_max(p)
        got = p[1:4].numpy().view(np.float32).tolist()
        # all-gather of column shards into rank-major blocks
        local = torch.full((3, 2), float(rank + 1))
        blocked = kd.allgather_blocked(local)
        # SPMD DTensor round trip on a 6 x 4 tensor sharded along dim 1
        mesh = kd.DeviceMesh.spmd()
        x = kz.from_flat(np.arange(24, dtype=np.float32), [6, 4], device="cpu")
        dt = kd.DTensor.from_tensor(x, mesh, kd.Shard(1))
        back = dt.to_tensor().tolist()
        q.put((rank, got, int(p[-1]), blocked.shape, blocked[:, 0, 0].tolist(), dt.local.shape, back))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def test_gloo_collectives_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        item = q.get(timeout=120)
        res[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert len(res[r]) > 1, res[r]
        got, gen, shape, firsts, local_shape, back = res[r]
        assert np.allclose(got, [1.5, 3.0, 2e-3])
        assert gen == 7 + r
        assert tuple(shape) == (2, 3, 2) and firsts == [1.0, 2.0]
        assert local_shape == [6, 2]
        assert back == np.arange(24, dtype=np.float32).tolist()


def _sum_cases():
    rs = np.random.RandomState(17)
    # values whose fp32 sum depends on the order and precision of the adds
    return [(rs.standard_normal(257) * 10.0 ** rs.uniform(-3, 3, 257)).astype(np.float32) for _ in range(3)]


def test_all_reduce_sum_matches_reference():
    """_all_reduce_sum (distributed.py:268-287): double adds in device order,
    one narrowing to fp32; pinned against the reference's own function where
    its checkout is available, else against the formula."""
    from oracle import refpkg
    parts = _sum_cases()
    ours = kd._all_reduce_sum([kz.from_numpy(p, device="cpu") for p in parts]).numpy()
    expect = np.asarray([float(a) + float(b) + float(c) for a, b, c in zip(*parts)], np.float64).astype(np.float32)
    assert ours.tobytes() == expect.tobytes()
    if refpkg.reference_available():
        ref = refpkg.import_reference_kansai()
        import sys
        import kansai_reference.distributed as rdist
        core = sys.modules["kansai_reference._core"]
        r = rdist._all_reduce_sum([core.from_flat(p.tolist(), [p.size], False) for p in parts])
        assert np.asarray(r.tolist(), np.float32).tobytes() == ours.tobytes()
        assert ref is not None


def test_dtensor_grad_threaded_cpu_mesh():
    """Replicate() gradients all-reduce by sum, Shard(0) gradients concatenate."""
    mesh = kd.DeviceMesh(["cpu", "cpu", "cpu"])
    x = kz.from_flat(np.arange(7 * 4, dtype=np.float32) / 7, [7, 4], device="cpu")
    dt = kd.DTensor.from_tensor(x, mesh, kd.Shard(0))

    def grad_fn(shard):
        t = shard.data
        return kz.Tensor(t.sum(0)), kz.Tensor(t * 2)

    gw, gx = kd.dtensor_grad(grad_fn, [kd.Replicate(), kd.Shard(0)], dt)
    pieces = [p.data.sum(0).numpy() for p in kd._split_tensor(x, 0, 3)]
    expect = (pieces[0].astype(np.float64) + pieces[1] + pieces[2]).astype(np.float32)
    assert gw.numpy().tobytes() == expect.tobytes()
    assert gx.numpy().tobytes() == (x.numpy() * 2).tobytes()
    with pytest.raises(ValueError):
        kd.dtensor_grad(lambda s: (s,), [kd.Replicate(), kd.Shard(0)], dt)


def _gloo_grad_worker(rank, world, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        mesh = kd.DeviceMesh.spmd()
        parts = _sum_cases()
        x = kz.from_flat(np.arange(6 * 4, dtype=np.float32), [6, 4], device="cpu")
        dt = kd.DTensor.from_tensor(x, mesh, kd.Shard(0))

        def grad_fn(shard):
            return kz.from_numpy(parts[rank], device="cpu"), kz.Tensor(shard.data + 1)

        gw, gx = kd.dtensor_grad(grad_fn, [kd.Replicate(), kd.Shard(0)], dt)
        q.put((rank, gw.numpy().tobytes(), gx.numpy().tobytes()))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), None))


def test_dtensor_grad_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_grad_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, gw, gx = q.get(timeout=120)
        res[r] = (gw, gx)
    for p in procs:
        p.join(timeout=60)
    parts = _sum_cases()
    expect = (parts[0].astype(np.float64) + parts[1]).astype(np.float32).tobytes()
    for r in range(2):
        assert res[r][1] is not None, res[r][0]
        assert res[r][0] == expect
        assert res[r][1] == (np.arange(24, dtype=np.float32) + 1).tobytes()


def test_gather_row_chunks():
    """The overlapped all-gather's row chunks: multiples of 128 rows that
    divide M, at most 8 of them, and the smallest such chunk."""
    from kansaiml_b200.distributed import _row_chunk
    for M in [128, 256, 384, 640, 896, 1024, 1152, 1664, 8192, 128 * 13, 128 * 97]:
        rows = _row_chunk(M)
        assert rows % 128 == 0 and M % rows == 0 and M // rows <= 8, M
        smaller = [r for r in range(128, rows, 128) if M % r == 0 and M // r <= 8]
        assert not smaller, (M, rows, smaller)
    assert _row_chunk(8192) == 1024 and _row_chunk(128 * 13) == 128 * 13


# ------------------------------------------------- properties (hypothesis)

from hypothesis import given, settings, strategies as st  # noqa: E402


@settings(max_examples=300, deadline=None)
@given(total=st.integers(0, 10 ** 6), n=st.integers(1, 64))
def test_chunk_sizes_properties(total, n):
    """The reference's split (distributed.py:157-159): n pieces that sum to
    total, as equal as possible, the larger ones first."""
    from kansaiml_b200.distributed import _chunk_sizes
    sizes = _chunk_sizes(total, n)
    assert len(sizes) == n and sum(sizes) == total
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


@settings(max_examples=300, deadline=None)
@given(total=st.integers(0, 10 ** 6), world=st.integers(1, 64))
def test_column_shard_bounds_tile_the_columns(total, world):
    """Shard(1) column ranges of all ranks are contiguous, disjoint and cover
    [0, total) in rank order."""
    from kansaiml_b200.distributed import _chunk_sizes, column_shard_bounds
    stop = 0
    for rank, size in enumerate(_chunk_sizes(total, world)):
        start, end = column_shard_bounds(total, rank, world)
        assert start == stop and end - start == size
        stop = end
    assert stop == total


@settings(max_examples=300, deadline=None)
@given(m128=st.integers(1, 4096))
def test_gather_row_chunk_properties(m128):
    from kansaiml_b200.distributed import _row_chunk
    M = 128 * m128
    rows = _row_chunk(M)
    assert rows % 128 == 0 and M % rows == 0 and M // rows <= 8
    assert all(M % r or M // r > 8 for r in range(128, rows, 128))


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 40), st.sampled_from([1, 2, 4, 8]))
def test_pipeline_input_rows_tile_the_batch_in_gather_order(m_blocks, world):
    """Every row of the batch belongs to exactly one rank, each rank owns the
    same count, and concatenating chunk c's blocks in rank order (what the
    all-gather of chunk c produces) walks rows c * M / C .. in natural order."""
    from kansaiml_b200.distributed import pipeline_chunks, pipeline_input_rows
    M = 64 * m_blocks * world
    C = pipeline_chunks(M, world)
    assert C >= 1 and M % (C * world) == 0
    per_rank = [pipeline_input_rows(M, world, r) for r in range(world)]
    assert all(len(p) == C for p in per_rank)
    order = []
    for c in range(C):
        for r in range(world):
            a, b = per_rank[r][c]
            order.extend(range(a, b))
    assert order == list(range(M))
    assert len({sum(b - a for a, b in p) for p in per_rank}) == 1


def test_pipeline_chunks_rejects_uneven_batches():
    from kansaiml_b200.distributed import pipeline_chunks, pipeline_input_rows
    assert pipeline_chunks(8192, 8) == 4 and pipeline_chunks(8192, 1) == 1
    assert pipeline_chunks(384, 2) == 1 or 384 // pipeline_chunks(384, 2) >= 256
    assert pipeline_chunks(1001, 2) == 0
    with pytest.raises(ValueError):
        pipeline_input_rows(1001, 2, 0)


# ----------------------- the pipelined sharded stack's data movement on gloo

PIPE_DIMS, PIPE_M = [256, 512, 256, 256], 1024   # four row chunks on two ranks


def _pipe_weights():
    rs = np.random.RandomState(81)
    return [(rs.standard_normal((PIPE_DIMS[i], PIPE_DIMS[i + 1])) * 0.05).astype(np.float32)
            for i in range(len(PIPE_DIMS) - 1)]


def _pipe_x():
    return np.random.RandomState(82).standard_normal((PIPE_M, PIPE_DIMS[0])).astype(np.float32)


def _install_cpu_kernels():
    """The stack's four device primitives, restated on the CPU through the
    oracle with the same contracts (absmax partials words, per-tensor
    quantize from partials, blocked-A int8 GEMM with fused epilogue and output
    absmax), so the pipelined forward's chunking, row ownership and gather
    layouts run on gloo ranks without a GPU."""
    from oracle import cpu as ocpu

    def put_absmax(partials, value):
        partials[0] = 1
        partials[1] = int(np.asarray([value], np.float32).view(np.int32)[0])

    def absmax_from(partials):
        n = int(partials[0])
        return float(partials[1:1 + n].numpy().view(np.float32).max()) if n else 0.0

    def quantize_cols_cpu(w):
        qT, s = ocpu.quantize_cols(w.numpy())
        return torch.from_numpy(qT), torch.from_numpy(s), torch.from_numpy(s.astype(np.float32))

    def absmax_cpu(x, partials=None):
        put_absmax(partials, np.abs(x.numpy()).max())
        return partials

    def quantize_partials_cpu(x, partials, q=None, s64=None, s32=None):
        codes, scale = ocpu.quantize_with_absmax(x.numpy(), absmax_from(partials))
        q = torch.empty(x.shape, dtype=torch.int8) if q is None else q
        s64 = torch.empty(1, dtype=torch.float64) if s64 is None else s64
        s32 = torch.empty(1, dtype=torch.float32) if s32 is None else s32
        q.copy_(torch.from_numpy(codes))
        s64.fill_(scale)
        s32.fill_(float(np.float32(scale)))
        return q, s64, s32

    def gemm_cpu(a, b, row_scale=None, col_scale=None, a_kblock=None, m=None, out=None, partials=None, **_):
        N, K = b.shape
        kb = a_kblock or K
        a2 = a.reshape(K // kb, m, kb).permute(1, 0, 2).reshape(m, K).numpy()
        y = ocpu.epilogue(ocpu.gemm_i8(a2, b.numpy()), row_scale.numpy()[0], col_scale.numpy())
        out.copy_(torch.from_numpy(y))
        if partials is not None:
            put_absmax(partials, np.abs(y).max())
        return out, None

    kd.quantize_cols_device = quantize_cols_cpu
    kd.absmax_partials_device = absmax_cpu
    kd.quantize_partials_device = quantize_partials_cpu
    kd.gemm_i8_device = gemm_cpu


def _pipe_worker(rank, world, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        _install_cpu_kernels()
        mesh = kd.DeviceMesh.spmd() if world > 1 else None
        stack = kd.ShardedQLinearStack([torch.from_numpy(w) for w in _pipe_weights()], mesh)
        assert stack.chunks(PIPE_M) == (4 if world > 1 else 1)
        y = stack(torch.from_numpy(_pipe_x()), return_local=False).numpy()
        q.put((rank, y))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def test_pipelined_stack_world2_gloo_matches_oracle_chain():
    """Two gloo ranks run the pipelined forward (input rows quantized per rank
    and all-gathered in four row chunks, each layer's codes all-gathered in
    chunks into [C][G][M/C][N/G] blocks) over CPU restatements of the device
    primitives: the gathered output equals the oracle's unsharded chain."""
    from oracle import cpu as ocpu
    a, s_a = ocpu.quantize_tensor(_pipe_x())
    want = None
    for i, w in enumerate(_pipe_weights()):
        wq, ws = ocpu.quantize_cols(w)
        want = ocpu.epilogue(ocpu.gemm_i8(a, wq), s_a, ws)
        if i < len(PIPE_DIMS) - 2:
            a, s_a = ocpu.quantize_tensor(want)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pipe_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, y = q.get(timeout=240)
        res[r] = y
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r], np.ndarray), res[r]
        assert res[r].tobytes() == want.tobytes()


def _pipe2d_worker(rank, world, port, q, tp):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        _install_cpu_kernels()
        stack = kd.ShardedQLinearStack([torch.from_numpy(w) for w in _pipe_weights()], kd.DeviceMesh.spmd(), tp=tp)
        assert (stack.tp, stack.dp, stack.g, stack.d) == (tp, world // tp, rank % tp, rank // tp)
        rows = stack.input_rows(PIPE_M)
        y = stack(torch.from_numpy(_pipe_x()), return_local=False).numpy()
        q.put((rank, (y, rows)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world,tp", [(4, 2), (2, 1)])
def test_pipelined_stack_row_groups_gloo_matches_oracle_chain(world, tp):
    """gloo ranks as row groups of column shards -- four ranks as two groups
    of two (tp=2), and two ranks as two groups of one (tp=1: each rank holds
    whole weights and half the rows, the one exchange the absmax): each group
    runs the pipelined forward on its rows, the absmax is all-reduced over all
    ranks, and the gathered output equals the oracle's unsharded chain; the
    ranks' input rows tile the batch."""
    from oracle import cpu as ocpu
    a, s_a = ocpu.quantize_tensor(_pipe_x())
    want = None
    for i, w in enumerate(_pipe_weights()):
        wq, ws = ocpu.quantize_cols(w)
        want = ocpu.epilogue(ocpu.gemm_i8(a, wq), s_a, ws)
        if i < len(PIPE_DIMS) - 2:
            a, s_a = ocpu.quantize_tensor(want)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pipe2d_worker, args=(r, world, port, q, tp)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, v = q.get(timeout=300)
        res[r] = v
    for p in procs:
        p.join(timeout=60)
    covered = []
    for r in range(world):
        assert isinstance(res[r], tuple), res[r]
        y, rows = res[r]
        assert y.tobytes() == want.tobytes()
        covered += [i for a0, b0 in rows for i in range(a0, b0)]
    assert sorted(covered) == list(range(PIPE_M))
