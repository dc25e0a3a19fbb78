"""DeviceMesh / DTensor for the int8 path on B200s (python/kansai/distributed.py).

Same names and placement semantics as the reference: ``DeviceMesh``,
``Shard(dim)`` / ``Replicate()``, ``DTensor.from_tensor`` / ``to_tensor``,
``_chunk_sizes`` (remainder to the first pieces, distributed.py:157-159),
``_split_tensor`` / ``_concat_tensors`` (distributed.py:162-182), ``_run_parallel``
(one thread per device, errors re-raised, distributed.py:73-102) and
``dtensor_run`` (distributed.py:219-267).  The reference's mesh entries name
in-process backends ("cpu", "metal") over host memory; here they are GPUs.

Two ways to drive a mesh:

* **one process, several GPUs**: ``DeviceMesh(["cuda:0", "cuda:1"])`` -- the
  reference's model.  ``DTensor.from_tensor`` splits and places each piece on
  its device, ``dtensor_run(fn, placement, *dts)`` runs ``fn`` per device on its
  own thread (libkz and torch release the GIL), ``to_tensor`` concatenates.
  ``dtensor_run`` takes a callable: the reference's KIR graphs (kir.py) are not
  part of this path.
* **one process per GPU** (torchrun): ``DeviceMesh.spmd()`` -- each rank holds
  its own shard; collectives run on NCCL over NVLink.

``ShardedQLinearStack`` is BASELINE config 5: a stack of int8 Linear layers
whose weights are column-sharded over the mesh (``Shard(1)`` of the reference's
[in, out] weight), activations row-sharded, quantized per tensor and
all-gathered between layers.  The default forward (``forward_local``,
``exchange="collective"``) is pipelined over C row chunks: each rank quantizes
its own input rows (global absmax by an integer MAX all-reduce), and every
layer's int8 activations travel as C async NCCL all-gathers while the next
layer's GEMM runs chunk by chunk, each chunk waiting (a stream dependency, no
spinning) only for its own all-gather.  Between layers the GEMM epilogues'
absmax partials are combined and MAX-all-reduced once (the per-tensor scale
needs the whole layer), each rank quantizes its output columns, and the codes
land in the rank-major layout [G][M/C][N/G] per chunk, which the next GEMM
reads directly (a_kblock = N/G).  Sharding changes no arithmetic: the result
equals the unsharded stack bit for bit.

Two earlier exchanges stay as options: ``exchange="peer"`` (IPC-exported
gather buffers pulled by the copy engines in row chunks while the gated GEMM
waits, bounded, on each chunk's token) and ``exchange="fused"`` (the
all-gather inside the GEMM launch: its first CTAs push this rank's block to
every peer with 16-byte stores and raise the peers' flags).  Both are
bit-exact; on B200s they lost to NCCL past two GPUs (one copy-engine stream
moved ~470 GB/s per GPU; the copy CTAs slowed the computing ones).
"""
import ctypes
from concurrent.futures import ThreadPoolExecutor, wait

import torch
import torch.distributed as dist

from . import _lib
from .quantize import (QTensor, absmax_partials_device, gemm_i8_device, new_partials, quantize_cols_device,
                       quantize_partials_device, quantize_tensor_device)
from .tensor import ptr, stream_handle
from .tensor import Tensor, as_tensor, cat


# ------------------------------------------------------------ host helpers

def _run_parallel(work_fns):
    """Contract of distributed.py:73-102: every callable runs concurrently on
    its own thread (libkz and torch release the GIL), the results come back
    in input order, and if any callable raised, the earliest one's exception
    is raised here once all of them have finished."""
    if not work_fns:
        return []
    with ThreadPoolExecutor(max_workers=len(work_fns)) as pool:
        futures = [pool.submit(fn) for fn in work_fns]
        wait(futures)
    failed = next((f.exception() for f in futures if f.exception() is not None), None)
    if failed is not None:
        raise failed
    return [f.result() for f in futures]


def _chunk_sizes(total, n):
    """distributed.py:157-159: as equal as possible, remainder to the first pieces."""
    base, remainder = divmod(total, n)
    return [base + 1 if i < remainder else base for i in range(n)]


def _split_tensor(tensor, dim, n):
    """distributed.py:162-176: n contiguous pieces along dim, sized by
    _chunk_sizes (torch.split at those sizes, each piece copied out as
    Tensor.slice does)."""
    t = as_tensor(tensor).data
    return [Tensor(p.contiguous()) for p in torch.split(t, _chunk_sizes(t.shape[dim], n), dim)]


def _concat_tensors(tensors, dim):
    return cat(tensors, dim)


def _parse_device(d):
    if d == "cpu":
        return torch.device("cpu")
    if d == "cuda":
        return torch.device("cuda", 0)
    if isinstance(d, str) and d.startswith("cuda:") and d[5:].isdigit():
        return torch.device(d)
    return None


class DeviceMesh:
    """A 1-D list of devices, one shard each (distributed.py:105-129).

    Entries are "cuda:N" (or "cpu" for data-only use).  In SPMD mode (one
    process per GPU, ``DeviceMesh.spmd()``) ``devices`` lists every rank's GPU
    and ``rank`` / ``group`` identify this process."""

    _VALID_DEVICES = ("cuda:N", "cpu")

    def __init__(self, devices):
        devices = list(devices)
        parsed = []
        for d in devices:
            dev = _parse_device(d)
            if dev is None:
                raise ValueError(f"unknown device {d!r} -- kansaiml_b200 meshes take {self._VALID_DEVICES}")
            if dev.type == "cuda" and (not torch.cuda.is_available() or dev.index >= torch.cuda.device_count()):
                raise RuntimeError(f"DeviceMesh includes {d!r} but that CUDA device is not available")
            parsed.append(dev)
        self.devices = devices
        self.torch_devices = parsed
        self.rank = None
        self.group = None

    @classmethod
    def spmd(cls, group=None):
        """The mesh of an initialised torch.distributed job: one GPU per rank."""
        if not dist.is_initialized():
            raise RuntimeError("DeviceMesh.spmd() needs torch.distributed to be initialised")
        world = dist.get_world_size(group)
        obj = cls.__new__(cls)
        obj.devices = [f"rank{r}" for r in range(world)]
        obj.torch_devices = None
        obj.rank = dist.get_rank(group)
        obj.group = group
        return obj

    @property
    def is_spmd(self):
        return self.rank is not None

    def __len__(self):
        return len(self.devices)

    def __repr__(self):
        return f"DeviceMesh({self.devices})"


class Shard:
    """Split along `dim` into len(mesh) pieces, remainder to the first pieces."""

    def __init__(self, dim):
        self.dim = dim

    def __repr__(self):
        return f"Shard({self.dim})"

    def __eq__(self, other):
        return isinstance(other, Shard) and self.dim == other.dim


class Replicate:
    def __repr__(self):
        return "Replicate()"

    def __eq__(self, other):
        return isinstance(other, Replicate)


class DTensor:
    """A tensor sharded or replicated across a DeviceMesh (distributed.py:185-216).

    ``shards[i]`` is mesh device i's piece, resident on that device.  In SPMD
    mode ``shards`` holds only this rank's piece (``local``)."""

    def __init__(self, mesh, placement, shards):
        expected = 1 if mesh.is_spmd else len(mesh)
        if len(shards) != expected:
            raise ValueError(f"DTensor needs one shard per mesh device ({expected}), got {len(shards)}")
        self.mesh = mesh
        self.placement = placement
        self.shards = list(shards)

    @property
    def local(self):
        """This rank's shard (SPMD mode) or the first device's."""
        return self.shards[0]

    @staticmethod
    def from_tensor(tensor, mesh, placement):
        tensor = as_tensor(tensor)
        if isinstance(placement, Replicate):
            pieces = [tensor] * (1 if mesh.is_spmd else len(mesh))
        elif isinstance(placement, Shard):
            pieces = _split_tensor(tensor, placement.dim, len(mesh))
            if mesh.is_spmd:
                pieces = [pieces[mesh.rank]]
        else:
            raise TypeError(f"unknown placement {placement!r}")
        if not mesh.is_spmd:
            pieces = [p.to(dev) for p, dev in zip(pieces, mesh.torch_devices)]
        else:
            here = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
            pieces = [p.to(here) for p in pieces]
        return DTensor(mesh, placement, pieces)

    def to_tensor(self):
        """Replicate -> shard 0; Shard(d) -> concatenation (an all-gather in SPMD mode)."""
        if isinstance(self.placement, Replicate):
            return self.shards[0]
        if not isinstance(self.placement, Shard):
            raise TypeError(f"unknown placement {self.placement!r}")
        if not self.mesh.is_spmd:
            first = self.shards[0].device
            return _concat_tensors([s.to(first) for s in self.shards], self.placement.dim)
        local = self.shards[0].data.contiguous()
        sizes = [torch.tensor(list(local.shape), device=local.device)]
        world = len(self.mesh)
        all_sizes = [torch.empty_like(sizes[0]) for _ in range(world)]
        dist.all_gather(all_sizes, sizes[0], group=self.mesh.group)
        parts = [torch.empty(s.tolist(), dtype=local.dtype, device=local.device) for s in all_sizes]
        dist.all_gather(parts, local, group=self.mesh.group)
        return Tensor(torch.cat(parts, self.placement.dim))

    def __repr__(self):
        return f"DTensor(mesh={self.mesh}, placement={self.placement}, shard_shapes={[s.shape for s in self.shards]})"


def dtensor_run(fn, output_placement, *dtensor_args):
    """distributed.py:219-267 with a callable: ``fn(*shards)`` runs once per
    mesh device, on its own thread, with that device current."""
    if callable(fn) is False:
        raise TypeError("dtensor_run takes a callable (kansaiml_b200 has no KIR graphs)")
    if not dtensor_args:
        raise ValueError("dtensor_run needs at least one DTensor argument")
    mesh = dtensor_args[0].mesh
    for dt in dtensor_args:
        if dt.mesh is not mesh:
            raise ValueError("all DTensor arguments must share the same DeviceMesh")
    if mesh.is_spmd:
        return DTensor(mesh, output_placement, [fn(*[dt.shards[0] for dt in dtensor_args])])

    def make(i, dev):
        shard_inputs = [dt.shards[i] for dt in dtensor_args]

        def work():
            if dev.type == "cuda":
                with torch.cuda.device(dev):
                    out = fn(*shard_inputs)
                    torch.cuda.current_stream(dev).synchronize()
                    return out
            return fn(*shard_inputs)
        return work

    results = _run_parallel([make(i, dev) for i, dev in enumerate(mesh.torch_devices)])
    return DTensor(mesh, output_placement, results)


def _all_reduce_sum(tensors):
    """distributed.py:268-287: element-wise sum of same-shape tensors.  The
    reference adds the fp32 values as Python floats (double) in device order
    and narrows the total to fp32 once; the same here, on the first tensor's
    device."""
    first = as_tensor(tensors[0])
    dev = first.data.device
    total = first.data.to(torch.float64)
    for t in tensors[1:]:
        total = total + as_tensor(t).data.to(dev, torch.float64)
    return Tensor(total.to(torch.float32))


def _all_reduce_sum_spmd(local, group=None):
    """_all_reduce_sum across the ranks of an SPMD mesh: every rank's fp32
    values are all-gathered (NCCL over NVLink, or gloo) and summed in double
    in rank order, so every rank holds the reference's exact result."""
    x = as_tensor(local).data.contiguous()
    world = dist.get_world_size(group)
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x, group=group)
    return _all_reduce_sum([Tensor(p) for p in parts])


def dtensor_grad(grad_fn, wrt_placements, *dtensor_args):
    """distributed.py:290-391 with a callable in place of the KIR graph:
    ``grad_fn(*shards)`` returns this device's local gradients (one per
    entry of wrt_placements), run per mesh device like dtensor_run; each
    entry is combined by its placement -- Replicate(): all-reduce sum
    (_all_reduce_sum), Shard(dim): concatenation along dim (an all-gather).
    Returns one Tensor per entry."""
    if not callable(grad_fn):
        raise TypeError("dtensor_grad takes a callable (kansaiml_b200 has no KIR graphs)")
    if not dtensor_args:
        raise ValueError("dtensor_grad needs at least one DTensor argument")
    mesh = dtensor_args[0].mesh
    for dt in dtensor_args:
        if dt.mesh is not mesh:
            raise ValueError("all DTensor arguments must share the same DeviceMesh")

    def as_tuple(out):
        return tuple(out) if isinstance(out, (tuple, list)) else (out,)

    per_device = [as_tuple(o) for o in dtensor_run(grad_fn, Replicate(), *dtensor_args).shards]
    for out in per_device:
        if len(out) != len(wrt_placements):
            raise ValueError("grad_fn must return one gradient per entry of wrt_placements")
    results = []
    for j, placement in enumerate(wrt_placements):
        local_j = [out[j] for out in per_device]
        if isinstance(placement, Replicate):
            if mesh.is_spmd:
                results.append(_all_reduce_sum_spmd(local_j[0], mesh.group))
            else:
                results.append(_all_reduce_sum(local_j))
        elif isinstance(placement, Shard):
            results.append(DTensor(mesh, placement, [as_tensor(t) for t in local_j]).to_tensor())
        else:
            raise TypeError(f"unknown placement {placement!r}")
    return results


# --------------------------------------------------------- collectives

def allreduce_partials_max(partials, group=None):
    """Element-wise MAX of absmax partials across ranks, in place.  The
    grid-barrier word and the reserved word at the end of the buffer are left
    out."""
    words = partials[: _lib.KZ_PARTIALS_WORDS - 2]
    dist.all_reduce(words, op=dist.ReduceOp.MAX, group=group)
    return partials


def allgather_blocked(local, group=None, out=None):
    """All-gather equally shaped shards into rank-major blocks [G, *local.shape]:
    the layout the int8 GEMM consumes directly as K blocks."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), local.contiguous(), group=group)
    return out


def _all_gather_async(out, local, group=None):
    """Async all-gather of equally shaped shards into out[G, *local.shape]
    (rank-major); returns the work handle, whose wait() makes the current
    stream wait for it (NCCL) or blocks until done (gloo)."""
    if dist.get_backend(group) == "nccl":
        return dist.all_gather_into_tensor(out, local, group=group, async_op=True)
    return dist.all_gather(list(out.unbind(0)), local, group=group, async_op=True)


def column_shard_bounds(total, rank, world):
    """[start, stop) of this rank's columns under Shard(1) (remainder first)."""
    sizes = _chunk_sizes(total, world)
    start = sum(sizes[:rank])
    return start, start + sizes[rank]


# -------------------------------------------------- config 5: sharded stack

def _row_chunk(M):
    """Rows per chunk of a gathered block: the smallest multiple of 128 that
    divides M (M % 128 == 0) and leaves at most 8 chunks, so the first GEMM
    tiles can start after about an eighth of each block has arrived."""
    m128 = M // 128
    d = next(v for v in range(-(-m128 // 8), m128 + 1) if m128 % v == 0)
    return d * 128


class _PeerGather:
    """Two [G][M][Kb] int8 gather buffers per rank (one per layer parity),
    exported to the other ranks through CUDA IPC.  Rank g writes block g of its
    own buffer; ``pull`` copies the other ranks' blocks into the local one on a
    side stream (copy engines), in row chunks of ``rows`` rows -- chunk 0 of
    every block first, then chunk 1, ... (the order the GEMM's first tiles need
    them) -- publishing ``token`` in flags[parity, h * chunks + c] after each."""

    def __init__(self, M, kb, world, rank, group, device):
        self.lib = _lib.load()
        self.world, self.rank, self.group, self.device = world, rank, group, device
        self.block = M * kb
        self.kb = kb
        self.rows = _row_chunk(M)
        self.chunks = M // self.rows
        # two gather buffers (one per layer parity) and, for the fused GEMM, one
        # flags buffer per parity (ready flags the peers write, then counters)
        self.flag_words = 2 * world * self.chunks
        sizes = [world * self.block, world * self.block, 4 * self.flag_words, 4 * self.flag_words]
        own, handles = [], []
        for nbytes in sizes:
            p, h = ctypes.c_void_p(), ctypes.create_string_buffer(_lib.KZ_IPC_HANDLE_BYTES)
            _lib.check(self.lib.kz_peer_alloc(nbytes, ctypes.byref(p), h), "kz_peer_alloc")
            own.append(p.value)
            handles.append(h.raw)
        self.own, self.xflags = own[:2], own[2:]
        gathered = [None] * world
        dist.all_gather_object(gathered, handles, group=group)
        self.peer, self.peer_xflags = [], []
        for r in range(world):
            if r == rank:
                self.peer.append(list(self.own))
                self.peer_xflags.append(list(self.xflags))
                continue
            ptrs = []
            for i in range(len(sizes)):
                p = ctypes.c_void_p()
                _lib.check(self.lib.kz_peer_open(gathered[r][i], ctypes.byref(p)), "kz_peer_open")
                ptrs.append(p.value)
            self.peer.append(ptrs[:2])
            self.peer_xflags.append(ptrs[2:])
        # per parity: world * chunks ready flags, then as many arrival counters
        self.flags = torch.zeros((2, 2 * world * self.chunks), dtype=torch.int32, device=device)
        self.side = torch.cuda.Stream(device)
        self.one = torch.zeros(1, dtype=torch.int32, device=device)
        self.token = 0

    def own_block(self, parity):
        return self.own[parity] + self.rank * self.block

    def fused(self, parity):
        """After every rank finished with the buffers of this parity: barrier,
        then the arguments of kz_gemm_i8_allgather (local buffer, the peers'
        buffers and flags, local flags, token)."""
        dist.all_reduce(self.one, group=self.group)
        self.token = self.token % 65535 + 1
        peer_a = (ctypes.c_void_p * self.world)(*[
            self.peer[h][parity] if h != self.rank else 0 for h in range(self.world)])
        peer_f = (ctypes.c_void_p * self.world)(*[
            self.peer_xflags[h][parity] if h != self.rank else 0 for h in range(self.world)])
        return self.own[parity], peer_a, peer_f, self.xflags[parity], self.token

    def pull(self, parity):
        """After every rank wrote its block: barrier, then copy the other
        ranks' blocks in ring order.  Returns (A pointer, flags, token)."""
        stream = torch.cuda.current_stream(self.device)
        dist.all_reduce(self.one, group=self.group)     # every rank's block is written
        self.token = self.token % 65535 + 1
        ready = torch.cuda.Event()
        ready.record(stream)
        side = self.side
        side.wait_event(ready)
        flags = self.flags[parity]
        M = self.block // self.kb
        for c in range(self.chunks):
            r0 = c * self.rows
            nbytes = (min(M, r0 + self.rows) - r0) * self.kb
            for j in range(1, self.world):
                h = (self.rank + j) % self.world
                off = h * self.block + r0 * self.kb
                _lib.check(self.lib.kz_copy_and_flag(self.own[parity] + off, self.peer[h][parity] + off, nbytes,
                                                     flags.data_ptr() + 4 * (h * self.chunks + c), self.token,
                                                     side.cuda_stream), "kz_copy_and_flag")
        return self.own[parity], flags, self.token

    def close(self):
        """Unmap the peers' buffers and free this rank's (collective)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for r in range(self.world):
            if r != self.rank:
                for p in self.peer[r] + self.peer_xflags[r]:
                    _lib.check(self.lib.kz_peer_close(ctypes.c_void_p(p)), "kz_peer_close")
        dist.barrier(group=self.group)
        for p in self.own + self.xflags:
            _lib.check(self.lib.kz_peer_free(ctypes.c_void_p(p)), "kz_peer_free")
        self.own, self.xflags, self.peer, self.peer_xflags = [], [], [], []


def pipeline_chunks(M, world):
    """Row chunks C of the sharded stack's pipelined exchange for an M-row
    batch: 1 on one GPU; otherwise the first of 4, 2, 1 that splits M into C x
    world equal row blocks with chunks of at least 256 rows; 0 when none
    does (the stack then takes its unpipelined forward)."""
    if world == 1:
        return 1
    for c in (4, 2, 1):
        if M % (c * world) == 0 and (c == 1 or M // c >= 256):
            return c
    return 0


def pipeline_input_rows(M, world, rank):
    """Rank `rank`'s rows of an [M, K] input in the pipelined layout, as
    [(start, stop)]: in each of the C row chunks (M / C rows) the rank owns
    the rank-th block of M / (C x world) rows, so the all-gather of chunk c
    lands the quantized input's rows in natural order."""
    C = pipeline_chunks(M, world)
    if C == 0:
        raise ValueError(f"{M} rows do not split into equal blocks over {world} ranks")
    mc = M // C
    mp = mc // world
    return [(c * mc + rank * mp, c * mc + (rank + 1) * mp) for c in range(C)]


class _CopyEngineGather:
    """Two gather buffers per rank (one per exchange parity), exported to the
    other ranks through CUDA IPC, each holding C x G blocks: block (c, g) is
    rank g's share of row chunk c.  A rank writes its own blocks (its quantize
    writes there directly); ``pull`` copies every other rank's blocks into the
    local buffer with the copy engines -- one stream per peer, so the peers'
    copies run side by side, chunk 0 first -- and returns, per chunk, the
    events its copies complete, for the GEMM of that chunk to wait on.  The
    copy engines use no SM, so the GEMM of chunk c runs on every SM it asked
    for while chunk c + 1 arrives."""

    def __init__(self, nbytes, world, rank, group, device):
        self.lib = _lib.load()
        self.world, self.rank, self.group, self.device = world, rank, group, device
        self.own, handles = [], []
        for _ in range(2):
            p, h = ctypes.c_void_p(), ctypes.create_string_buffer(_lib.KZ_IPC_HANDLE_BYTES)
            _lib.check(self.lib.kz_peer_alloc(nbytes, ctypes.byref(p), h), "kz_peer_alloc")
            self.own.append(p.value)
            handles.append(h.raw)
        self.nbytes = nbytes
        gathered = [None] * world
        dist.all_gather_object(gathered, handles, group=group)
        self.peer = {}
        for r in range(world):
            if r != rank:
                ptrs = []
                for i in range(2):
                    p = ctypes.c_void_p()
                    _lib.check(self.lib.kz_peer_open(gathered[r][i], ctypes.byref(p)), "kz_peer_open")
                    ptrs.append(p.value)
                self.peer[r] = ptrs
        self.streams = {r: torch.cuda.Stream(device) for r in self.peer}
        # kz_copy_and_flag also writes a token; these words take it (nothing reads them)
        self.sink = torch.zeros(world, dtype=torch.int32, device=device)
        self.one = torch.zeros(1, dtype=torch.int32, device=device)

    def block(self, parity, c, g, blk):
        return self.own[parity] + (c * self.world + g) * blk

    def pull(self, parity, chunks, blk):
        """Once every rank's own blocks of `parity` are written (an NCCL
        one-word barrier), copy the peers' blocks in; returns [events of
        chunk c for c in range(chunks)]."""
        cur = torch.cuda.current_stream(self.device)
        dist.all_reduce(self.one, group=self.group)
        ready = torch.cuda.Event()
        ready.record(cur)
        events = [[] for _ in range(chunks)]
        for h, st in self.streams.items():
            st.wait_event(ready)
            for c in range(chunks):
                off = (c * self.world + h) * blk
                _lib.check(self.lib.kz_copy_and_flag(self.own[parity] + off, self.peer[h][parity] + off, blk,
                                                     self.sink.data_ptr() + 4 * h, 1, st.cuda_stream),
                           "kz_copy_and_flag")
                e = torch.cuda.Event()
                e.record(st)
                events[c].append(e)
        return events

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for ptrs in self.peer.values():
            for p in ptrs:
                _lib.check(self.lib.kz_peer_close(ctypes.c_void_p(p)), "kz_peer_close")
        dist.barrier(group=self.group)
        for p in self.own:
            _lib.check(self.lib.kz_peer_free(ctypes.c_void_p(p)), "kz_peer_free")
        self.own, self.peer = [], {}


class _PhaseEvents:
    """CUDA events around the phases of a forward on the current stream
    (only when enabled).  ``finish()`` synchronises and returns
    {phase: milliseconds}, summed over the phase's intervals; a phase that
    waits for an all-gather measures the stall the stream actually saw."""

    def __init__(self, enabled, dev):
        self.enabled, self.dev = enabled, dev
        self.marks, self.open = [], None

    def begin(self, name):
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record(torch.cuda.current_stream(self.dev))
            self.open = (name, e)

    def end(self):
        if self.enabled and self.open is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(torch.cuda.current_stream(self.dev))
            self.marks.append((self.open[0], self.open[1], e))
            self.open = None

    def finish(self):
        if not self.enabled:
            return None
        torch.cuda.synchronize(self.dev)
        out = {}
        for name, a, b in self.marks:
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


class ShardedQLinearStack:
    """A stack of bias-free int8 Linear layers, weights column-sharded over the
    ranks of an SPMD mesh (or a single GPU when the mesh is None).

    weights: list of fp32 [K, N] tensors (the reference layout), or callables
    ``w(l)`` returning layer l's full weight on the current device.  Each rank
    keeps only its columns, quantized per output channel.  N / G must be a
    multiple of 128 between layers (the GEMM's K block).

    tp: the size of the column-sharding groups.  With tp = the mesh size (the
    default up to 4 ranks) every rank holds 1/tp of every weight and all
    ranks share the batch's rows; with tp < mesh size (the default at 8
    ranks: two groups of 4) consecutive groups of tp ranks each take
    1/(mesh size / tp) of the batch's rows -- the activations row-sharded
    across groups, the weights column-sharded within one -- so each rank
    exchanges 1/(mesh size / tp) as many activation bytes for the same GEMM
    work.  The per-tensor absmax is still all-reduced over every rank, so the
    output equals the unsharded stack's bit for bit either way."""

    def __init__(self, weights, mesh=None, exchange=None, tp=None):
        self.mesh = mesh
        self.world = len(mesh) if mesh is not None and mesh.is_spmd else 1
        self.rank = mesh.rank if mesh is not None and mesh.is_spmd else 0
        self.group = mesh.group if mesh is not None and mesh.is_spmd else None
        if tp is None:
            tp = 4 if self.world > 4 and self.world % 4 == 0 else self.world
        if tp < 1 or self.world % tp:
            raise ValueError(f"tp={tp} must divide the mesh size {self.world}")
        if tp < self.world and self.group is not None:
            raise ValueError("tp < mesh size needs the default process group")
        self.tp, self.dp = tp, self.world // tp
        self.g, self.d = self.rank % tp, self.rank // tp      # column shard, row group
        self.xgroup = self.group                              # the exchange group: this rank's tp ranks
        if tp < self.world:
            for d in range(self.dp):                          # every rank creates every group, in order
                grp = dist.new_group(list(range(d * tp, (d + 1) * tp)))
                if d == self.d:
                    self.xgroup = grp
        self.layers = []
        for i, w in enumerate(weights):
            full = w(i) if callable(w) else as_tensor(w).data
            K, N = full.shape
            if N % self.tp:
                raise ValueError(f"layer {i}: out_features {N} is not divisible by the group size {self.tp}")
            lo, hi = column_shard_bounds(N, self.g, self.tp)
            shard = full[:, lo:hi].contiguous()
            del full
            qT, s64, s32 = quantize_cols_device(shard)
            del shard
            qt = QTensor._from_device(qT, s64, s32, [K, hi - lo], "channel")
            qt._check_finite()
            self.layers.append((qt, K, N))
        for i in range(1, len(self.layers)):
            if self.layers[i][1] != self.layers[i - 1][2]:
                raise ValueError("consecutive layers' shapes do not chain")
        if self.tp > 1:
            n_loc = self.layers[0][2] // self.tp
            if n_loc % 128:
                raise ValueError("out_features / group size must be a multiple of 128")
        self.partials = None
        if exchange is None:
            # the copy-engine exchange where it can run (GPUs on NCCL): it beat
            # the NCCL all-gathers at 2 and 4 ranks per column-sharding group
            nccl = self.world > 1 and dist.get_backend(self.group) == "nccl"
            exchange = "ce" if nccl and self.tp > 1 else "collective"
        if exchange not in ("peer", "collective", "fused", "ce"):
            raise ValueError(f"unknown exchange {exchange!r}")
        if exchange != "collective" and self.world > 1 and dist.get_backend(self.group) != "nccl":
            raise ValueError(f'exchange="{exchange}" needs an NCCL mesh on GPUs')
        if tp < self.world and exchange not in ("collective", "ce"):
            raise ValueError(f'exchange="{exchange}" shards columns over the whole mesh (tp = mesh size)')
        self.exchange = exchange if self.tp > 1 else "collective"
        self.copy_ctas = 8
        self._peer = None
        self._bufs = {}
        self._ce = None
        self.timing = False        # record per-phase CUDA-event times in forward_local (phase_times)
        self._phases = None

    def close(self):
        """Release the peer exchange buffers (collective over the mesh)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None
        if self._ce is not None:
            self._ce.close()
            self._ce = None

    # ------------------------------------------------- pipelined forward

    def chunks(self, M):
        """Row chunks of the pipelined exchange (pipeline_chunks of this row
        group's M / dp rows over tp ranks); 0 when M does not split."""
        if M % self.dp:
            return 0
        return pipeline_chunks(M // self.dp, self.tp)

    def input_rows(self, M):
        """This rank's rows of an [M, K] input in the pipelined layout: the
        pipeline_input_rows of its column-shard index within its row group's
        M / dp rows."""
        if self.chunks(M) == 0:
            raise ValueError(f"{M} rows do not split into equal blocks over {self.world} ranks")
        base = self.d * (M // self.dp)
        return [(base + a, base + b) for a, b in pipeline_input_rows(M // self.dp, self.tp, self.g)]

    def local_input(self, x):
        """This rank's rows (input_rows) of a replicated [M, K] input, stacked."""
        xd = as_tensor(x).data
        return torch.cat([xd[a:b] for a, b in self.input_rows(xd.shape[0])]).contiguous()

    def _zeroed(self, key, shape, dtype, dev):
        buf = self._bufs.get(key)
        if buf is None or buf.device != dev or tuple(buf.shape) != tuple(shape):
            buf = torch.zeros(shape, dtype=dtype, device=dev)
            self._bufs[key] = buf
        return buf

    def forward_local(self, x_local, M):
        """The stack on this rank's input rows (local_input / input_rows
        layout, fp32 [M / world, K]).  Returns this rank's block of the last
        layer's fp32 output: its row group's M / dp rows x its N / tp columns.

        Pipelined over C row chunks: each layer's int8 activations travel as
        C NCCL all-gathers (async, on the process group's stream), and the
        next layer's GEMM runs chunk by chunk, each chunk waiting (stream
        order, no spinning) only for its own all-gather, so the all-gather of
        chunk c + 1 overlaps the GEMM of chunk c.  The per-tensor scale needs
        the whole layer's absmax first: the GEMM epilogues write absmax
        partials per chunk, combined and MAX-all-reduced once per layer."""
        xd = as_tensor(x_local).data
        dev = xd.device
        G, C = self.tp, self.chunks(M)
        M = M // self.dp              # this row group's rows
        mc = M // C
        mp = mc // G
        if xd.shape[0] != C * mp:
            raise ValueError(f"local input has {xd.shape[0]} rows, expected {C * mp}")
        if self.exchange == "ce" and G > 1:
            return self._forward_local_ce(xd.contiguous(), M)
        ev = _PhaseEvents(self.timing, dev)
        # layer-0 input: absmax of the local rows -> global absmax -> local codes
        ev.begin("input_quantize")
        parts = self._zeroed("in_parts", (_lib.KZ_PARTIALS_WORDS,), torch.int32, dev)
        absmax_partials_device(xd, parts)
        if self.world > 1:
            allreduce_partials_max(parts, self.group)
        codes, _, a_s32 = quantize_partials_device(xd, parts)
        ev.end()
        K0 = self.layers[0][1]
        works = [None] * C
        if G > 1:
            A = torch.empty((M, K0), dtype=torch.int8, device=dev)
            for c in range(C):
                works[c] = _all_gather_async(A[c * mc:(c + 1) * mc].view(G, mp, K0), codes[c * mp:(c + 1) * mp],
                                             self.xgroup)
        else:
            A = codes
        a_chunks = [(A[c * mc:(c + 1) * mc], K0) for c in range(C)]
        y = None
        for li, (qt, K, N) in enumerate(self.layers):
            n_loc = qt.shape[1]
            last = li == len(self.layers) - 1
            y = torch.empty((M, n_loc), dtype=torch.float32, device=dev)
            pb = None if last else self._zeroed(("chunk_parts", C), (C, _lib.KZ_PARTIALS_WORDS), torch.int32, dev)
            for c in range(C):
                if works[c] is not None:
                    ev.begin("wait_allgather")
                    works[c].wait()
                    ev.end()
                a, kb = a_chunks[c]
                ev.begin("gemm")
                gemm_i8_device(a, qt.kmajor(), row_scale=a_s32, col_scale=qt.scale_f32, a_kblock=kb, m=mc,
                               out=y[c * mc:(c + 1) * mc], partials=None if last else pb[c])
                ev.end()
            if last:
                break
            ev.begin("allreduce_max")
            lp = torch.amax(pb, 0) if C > 1 else pb[0]
            if self.world > 1:
                allreduce_partials_max(lp, self.group)
            ev.end()
            ev.begin("quantize")
            yq = torch.empty((M, n_loc), dtype=torch.int8, device=dev)
            s64 = torch.empty(1, dtype=torch.float64, device=dev)
            a_s32 = torch.empty(1, dtype=torch.float32, device=dev)
            gathered = torch.empty((C, G, mc, n_loc), dtype=torch.int8, device=dev) if G > 1 else None
            for c in range(C):
                rows = slice(c * mc, (c + 1) * mc)
                quantize_partials_device(y[rows], lp, q=yq[rows], s64=s64, s32=a_s32)
                if G > 1:
                    works[c] = _all_gather_async(gathered[c], yq[rows], self.xgroup)
            ev.end()
            a_chunks = [(gathered[c], n_loc) for c in range(C)] if G > 1 else [(yq, N)]
        self._phases = ev
        return Tensor(y)

    def phase_times(self):
        """{phase: ms} of the last forward_local run with ``timing`` on
        (synchronises the device), else None."""
        return self._phases.finish() if self._phases is not None else None

    def _forward_local_ce(self, xd, M):
        """forward_local with the copy-engine exchange (exchange="ce"): the
        same chunking, row ownership, scales and layouts, but each rank
        quantizes straight into its blocks of an IPC-exported gather buffer
        and the other ranks' blocks arrive by copy-engine pulls
        (_CopyEngineGather) instead of NCCL all-gathers; NCCL carries only the
        absmax all-reduces and a one-word barrier per exchange.  The absmax
        all-reduce of each exchange is also what keeps a buffer from being
        rewritten while a peer still reads it: every rank passes it only after
        its GEMMs of the previous layer, which waited for their pulls."""
        dev = xd.device
        G, C = self.tp, pipeline_chunks(M, self.tp)     # M: this row group's rows
        mc, mp = M // C, M // (C * G)
        blks = [mp * self.layers[0][1]] + [mc * qt.shape[1] for qt, _, _ in self.layers[:-1]]
        need = C * G * max(blks)
        if self._ce is None or self._ce.nbytes < need:
            self.close()
            self._ce = _CopyEngineGather(need, G, self.g, self.xgroup, dev)
        ce = self._ce
        sh = stream_handle(dev)
        cur = torch.cuda.current_stream(dev)
        ev = _PhaseEvents(self.timing, dev)
        # layer-0 input: global absmax, then this rank's rows straight into its blocks
        ev.begin("input_quantize")
        parts = self._zeroed("in_parts", (_lib.KZ_PARTIALS_WORDS,), torch.int32, dev)
        absmax_partials_device(xd, parts)
        allreduce_partials_max(parts, self.group)
        s64 = torch.empty(1, dtype=torch.float64, device=dev)
        a_s32 = torch.empty(1, dtype=torch.float32, device=dev)
        K0 = self.layers[0][1]
        blk, parity = blks[0], 0
        for c in range(C):
            _lib.call("kz_quantize_partials_f32", ptr(xd[c * mp:(c + 1) * mp]), mp * K0, ptr(parts),
                      ce.block(parity, c, self.g, blk), ptr(s64), ptr(a_s32), sh)
        events = ce.pull(parity, C, blk)
        ev.end()
        a_kblock = K0
        y = None
        for li, (qt, K, N) in enumerate(self.layers):
            n_loc = qt.shape[1]
            last = li == len(self.layers) - 1
            y = torch.empty((M, n_loc), dtype=torch.float32, device=dev)
            pb = None if last else self._zeroed(("chunk_parts", C), (C, _lib.KZ_PARTIALS_WORDS), torch.int32, dev)
            for c in range(C):
                ev.begin("wait_allgather")
                for e in events[c]:
                    cur.wait_event(e)
                ev.end()
                ev.begin("gemm")
                _lib.call("kz_gemm_i8", ce.own[parity] + c * G * blk, ptr(qt.kmajor()), mc, n_loc, K, a_kblock,
                          ptr(a_s32), 0, ptr(qt.scale_f32), 1, None, _lib.KZ_ACT_NONE, ptr(y[c * mc:(c + 1) * mc]),
                          None, n_loc, None if last else ptr(pb[c]), sh)
                ev.end()
            if last:
                break
            ev.begin("allreduce_max")
            lp = torch.amax(pb, 0) if C > 1 else pb[0]
            allreduce_partials_max(lp, self.group)
            ev.end()
            ev.begin("quantize")
            parity ^= 1
            blk = blks[li + 1]
            s64 = torch.empty(1, dtype=torch.float64, device=dev)
            a_s32 = torch.empty(1, dtype=torch.float32, device=dev)
            for c in range(C):
                _lib.call("kz_quantize_partials_f32", ptr(y[c * mc:(c + 1) * mc]), mc * n_loc, ptr(lp),
                          ce.block(parity, c, self.g, blk), ptr(s64), ptr(a_s32), sh)
            events = ce.pull(parity, C, blk)
            ev.end()
            a_kblock = n_loc
        self._phases = ev
        return Tensor(y)

    def forward(self, x, return_local=True):
        """x: fp32 [M, K] replicated on every rank.  Returns the last layer's
        fp32 output: this rank's column shard (return_local) or the full
        [M, N] (all-gathered).  With the collective exchange and M splitting
        into equal row blocks, each rank quantizes and all-gathers only its
        own rows of x (forward_local); otherwise every rank quantizes all of x."""
        xd = as_tensor(x).data.contiguous()
        M = xd.shape[0]
        if self.exchange in ("collective", "ce") and self.chunks(M) > 0:
            y = self.forward_local(self.local_input(xd) if self.world > 1 else xd, M).data
        elif self.tp < self.world:
            raise ValueError(f"{M} rows do not split into {self.dp} row groups of equal pipelined blocks")
        else:
            y = self._forward_replicated(xd)
        if return_local or self.world == 1:
            return Tensor(y)
        parts = allgather_blocked(y.contiguous(), self.group)     # [world, M / dp, N / tp], rank = d * tp + g
        n_loc = parts.shape[2]
        return Tensor(parts.view(self.dp, self.tp, M // self.dp, n_loc).permute(0, 2, 1, 3).reshape(M, -1))

    def _forward_replicated(self, xd):
        """Every rank quantizes the whole replicated input; one all-gather per
        layer boundary (or the peer / fused exchanges)."""
        dev = xd.device
        if self.partials is None or self.partials.device != dev:
            self.partials = new_partials(dev)
        M = xd.shape[0]
        a, _, a_s32 = quantize_tensor_device(xd)
        a_kblock = xd.shape[1]
        gate = None
        y = None
        for li, (qt, K, N) in enumerate(self.layers):
            n_loc = qt.shape[1]
            last = li == len(self.layers) - 1
            parts = None if last else self.partials
            if gate is None:
                y, _ = gemm_i8_device(a, qt.kmajor(), row_scale=a_s32, col_scale=qt.scale_f32, a_kblock=a_kblock, m=M,
                                      partials=parts)
            elif self.exchange == "fused":
                y = self._gemm_fused(gate, M, K, qt, a_s32, parts)
            else:
                y = self._gemm_gated(gate, M, K, a_kblock, qt, a_s32, parts)
            gate = None
            if last:
                break
            if self.world > 1:
                allreduce_partials_max(self.partials, self.group)
            if self.exchange in ("peer", "fused") and M % 128 == 0:
                if self._peer is None or self._peer.block != M * n_loc:
                    self.close()
                    self._peer = _PeerGather(M, n_loc, self.world, self.rank, self.group, dev)
                parity = li % 2
                s64 = torch.empty(1, dtype=torch.float64, device=dev)
                a_s32 = torch.empty(1, dtype=torch.float32, device=dev)
                _lib.call("kz_quantize_partials_f32", ptr(y), y.numel(), ptr(self.partials),
                          self._peer.own_block(parity), ptr(s64), ptr(a_s32), stream_handle(dev))
                gate = self._peer.pull(parity) if self.exchange == "peer" else self._peer.fused(parity)
                a_kblock = n_loc
                continue
            yq, _, a_s32 = quantize_partials_device(y, self.partials)
            if self.world > 1:
                a = allgather_blocked(yq, self.group)   # [G, M, n_loc]
                a_kblock = n_loc
            else:
                a = yq
                a_kblock = N
        return y

    def _gemm_fused(self, gate, M, K, qt, a_s32, partials):
        a_ptr, peer_a, peer_f, flags, token = gate
        N = qt.shape[1]
        dev = a_s32.device
        out = torch.empty((M, N), dtype=torch.float32, device=dev)
        _lib.call("kz_gemm_i8_allgather", a_ptr, peer_a, peer_f, self.world, self.rank, ptr(qt.kmajor()), M, N, K,
                  ptr(a_s32), 0, ptr(qt.scale_f32), 1, ptr(out), N, ptr(partials), flags, token, self._peer.rows,
                  self.copy_ctas, stream_handle(dev))
        return out

    def _gemm_gated(self, gate, M, K, a_kblock, qt, a_s32, partials):
        a_ptr, flags, token = gate
        N = qt.shape[1]
        dev = a_s32.device
        out = torch.empty((M, N), dtype=torch.float32, device=dev)
        _lib.call("kz_gemm_i8_gated", a_ptr, ptr(qt.kmajor()), M, N, K, a_kblock, ptr(a_s32), 0, ptr(qt.scale_f32), 1,
                  None, _lib.KZ_ACT_NONE, ptr(out), None, N, ptr(partials), ptr(flags), token, self.rank,
                  self._peer.rows, stream_handle(dev))
        return out

    __call__ = forward
