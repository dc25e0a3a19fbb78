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
