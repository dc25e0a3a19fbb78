"""KAN1 checkpoints with the reference's API (python/kansai/serialize.py),
extended to quantized models.

The file format is the reference's (serialize.py:17-30):

    bytes  0- 3   magic:      b"KAN1"
    bytes  4-11   header_len: uint64, little-endian
    bytes 12..    header:     UTF-8 JSON, {name: {dtype, shape, offset, nbytes}}
    remaining     data:       the tensors' raw little-endian bytes, concatenated

``save(module, path)`` / ``load(module, path)`` keep the reference's contract
(serialize.py:117-199): parameter values only, names from
``Module.named_parameters()``, the model is built first and filled in place,
every name, shape and byte range checked with the reference's messages.  A
float32 checkpoint written here loads in the reference and vice versa.

Extension for quantized models (no reference counterpart): a ``QLinear`` at
attribute path ``p`` is stored as ``p.qweight``
(dtype "int8", its codes in the reference's [in, out] layout, i.e. the order of
``QTensor.q``), ``p.qweight.scale`` (dtype "float64": shape [] for a per-tensor
weight, [out] for a per-channel one) and ``p.bias`` (float32, when present).
Tensors move between the device and the file as whole buffers (one copy each
way), not through per-element Python lists.
"""
import json
import struct

import numpy as np
import torch

from .nn import Module
from .quantize import QLinear, QTensor
from .tensor import Tensor

_MAGIC = b"KAN1"
_ITEMSIZE = {"float32": 4, "int8": 1, "float64": 8}


class _Scale:
    """Header entry for the scale(s) of a quantized weight."""
    __slots__ = ("qt",)

    def __init__(self, qt):
        self.qt = qt

    @property
    def shape(self):
        return [] if self.qt.granularity == "tensor" else [self.qt.shape[1]]


def _qlinear_entries(ql, prefix):
    yield f"{prefix}qweight", ql.qweight
    yield f"{prefix}qweight.scale", _Scale(ql.qweight)
    if ql.bias is not None:
        yield f"{prefix}bias", ql.bias


def _entries(module, prefix=""):
    """named_parameters() order and names, plus the int8 weights of quantized
    layers (QLinear attributes, alone or in lists)."""
    for key, value in vars(module).items():
        full = f"{prefix}{key}"
        if isinstance(value, Tensor) and value.requires_grad:
            yield full, value
        elif isinstance(value, QLinear):
            yield from _qlinear_entries(value, full + ".")
        elif isinstance(value, Module):
            yield from _entries(value, full + ".")
        elif isinstance(value, (list, tuple)):
            for i, item in enumerate(value):
                if isinstance(item, QLinear):
                    yield from _qlinear_entries(item, f"{full}.{i}.")
                elif isinstance(item, Module):
                    yield from _entries(item, f"{full}.{i}.")


def _dtype_of(value):
    if isinstance(value, QTensor):
        return "int8"
    if isinstance(value, _Scale):
        return "float64"
    return "float32"


def _to_bytes(value):
    if isinstance(value, QTensor):
        codes = value.codes
        if value.granularity == "channel":          # stored K-major [out, in] on the device
            codes = codes.t()
        return codes.contiguous().cpu().numpy().astype(np.int8).tobytes()
    if isinstance(value, _Scale):
        return value.qt.scale_f64.detach().cpu().numpy().astype("<f8").tobytes()
    return value.data.detach().contiguous().cpu().numpy().astype("<f4").tobytes()


def save(module, path: str) -> None:
    """serialize.py:117-140: every parameter (and quantized weight) of
    `module`, by name, in the KAN1 format."""
    header, blobs, offset = {}, [], 0
    for name, value in _entries(module):
        data = _to_bytes(value)
        header[name] = {"dtype": _dtype_of(value), "shape": list(value.shape), "offset": offset, "nbytes": len(data)}
        blobs.append(data)
        offset += len(data)
    header_bytes = json.dumps(header).encode("utf-8")
    with open(path, "wb") as f:
        f.write(_MAGIC)
        f.write(struct.pack("<Q", len(header_bytes)))
        f.write(header_bytes)
        for b in blobs:
            f.write(b)


def _set_by_path(root, path, value):
    """serialize.py:89-115: assign at a dotted attribute path."""
    parts = path.split(".")
    obj = root
    for part in parts[:-1]:
        obj = obj[int(part)] if isinstance(obj, (list, tuple)) else getattr(obj, part)
    setattr(obj, parts[-1], value)


def load(module, path: str) -> None:
    """serialize.py:143-199: fill `module` in place from `path`; names,
    shapes, dtypes and byte ranges must match exactly in both directions."""
    with open(path, "rb") as f:
        magic = f.read(4)
        if magic != _MAGIC:
            raise ValueError(f"{path}: not a Kansai checkpoint (expected magic {_MAGIC!r}, got {magic!r})")
        header_len = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(header_len).decode("utf-8"))
        blob = f.read()

    named = dict(_entries(module))
    missing = sorted(set(named) - set(header))
    unexpected = sorted(set(header) - set(named))
    if missing:
        raise ValueError(f"{path}: checkpoint is missing parameter(s) the model expects: {missing}")
    if unexpected:
        raise ValueError(f"{path}: checkpoint has parameter(s) the model doesn't expect: {unexpected}")

    arrays = {}
    for name, value in named.items():
        meta = header[name]
        dtype = _dtype_of(value)
        if meta.get("dtype", "float32") != dtype:
            raise ValueError(f"{path}: {name!r} dtype mismatch -- model has {dtype}, checkpoint has {meta.get('dtype')}")
        if list(value.shape) != meta["shape"]:
            raise ValueError(
                f"{path}: {name!r} shape mismatch -- model has {list(value.shape)}, "
                f"checkpoint has {meta['shape']}"
            )
        n = 1
        for d in meta["shape"]:
            n *= d
        expected_nbytes = n * _ITEMSIZE[dtype]
        if meta["nbytes"] != expected_nbytes:
            raise ValueError(
                f"{path}: {name!r} has an inconsistent header -- shape {meta['shape']} implies "
                f"{expected_nbytes} bytes but the header declares {meta['nbytes']}"
            )
        raw = blob[meta["offset"]:meta["offset"] + meta["nbytes"]]
        if len(raw) != meta["nbytes"]:
            raise ValueError(
                f"{path}: {name!r}'s declared byte range runs past the end of the file "
                f"(wanted {meta['nbytes']} bytes at offset {meta['offset']}, file has {len(raw)} there)"
            )
        np_dtype = {"float32": "<f4", "int8": np.int8, "float64": "<f8"}[dtype]
        arrays[name] = np.frombuffer(raw, dtype=np_dtype).reshape(meta["shape"])

    for name, value in named.items():
        if isinstance(value, _Scale):
            continue
        a = arrays[name]
        if isinstance(value, QTensor):
            dev = value.codes.device
            codes = torch.from_numpy(a.copy()).to(dev)
            if value.granularity == "channel":
                codes = codes.t().contiguous()
            s64 = torch.from_numpy(np.atleast_1d(arrays[name + ".scale"]).astype(np.float64)).to(dev)
            qt = QTensor._from_device(codes, s64, s64.to(torch.float32), list(value.shape), value.granularity)
            qt._check_finite()
            _set_by_path(module, name, qt)
        else:
            t = Tensor(torch.from_numpy(a.astype(np.float32)).to(value.data.device), value.requires_grad)
            _set_by_path(module, name, t)
