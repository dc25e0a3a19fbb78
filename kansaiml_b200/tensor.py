"""Device-resident fp32 tensor with the reference's `kansai._core.Tensor` surface.

The reference's Tensor (core/include/kansai/Tensor.hpp:30-256, bound at
python/bindings.cpp:20-122) is a host fp32 buffer.  Here a Tensor owns HBM
through a torch tensor -- torch is the device-memory and stream plumbing only.
The int8 quantized-linear path (quantize, int8 GEMM, dequantize, the W8A32
qlinear) runs in libkz (kansaiml_b200/_lib.py); the fp32 glue the models around
that path need (residual adds, LayerNorm, softmax attention in config 3,
split/concat for DTensor) runs on torch ops with TF32 disabled, i.e. outside
the hot path.

Names and meanings follow the reference: `shape` is a list, `tolist()` returns
the FLAT row-major list (Tensor::to_vector, core/src/Tensor.cpp:133-137),
`from_flat(values, shape)` raises on a length mismatch (Tensor.cpp:94-100),
`randn(shape, std, seed)` draws the same numbers as the reference
(std::mt19937 + std::normal_distribution<float>, Tensor.cpp:85-92).
"""
import ctypes

import numpy as np
import torch

from . import _lib

torch.backends.cuda.matmul.allow_tf32 = False
torch.backends.cudnn.allow_tf32 = False


def default_device():
    """cuda:<current device> when a GPU is present, else cpu (data only)."""
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _as_device(device):
    if device is None:
        return default_device()
    return torch.device(device)


def stream_handle(device):
    """The raw cudaStream_t of torch's current stream on `device`."""
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t, what):
    if t.device.type != "cuda":
        raise RuntimeError(f"{what}: kansaiml_b200 computes on the GPU only (tensor is on {t.device}); "
                           "there is no CPU fallback")


def ptr(t):
    return t.data_ptr() if t is not None else None


class Tensor:
    """fp32 tensor in device memory (or host memory for data-only use)."""

    __slots__ = ("_t", "requires_grad")

    def __init__(self, data, requires_grad=False):
        if not isinstance(data, torch.Tensor):
            raise TypeError("Tensor wraps a torch.Tensor; use from_flat/tensor/zeros/randn to build one")
        if data.dtype != torch.float32:
            data = data.to(torch.float32)
        self._t = data
        self.requires_grad = requires_grad

    # -------------------------------------------------------------- basics
    @property
    def shape(self):
        return list(self._t.shape)

    @property
    def device(self):
        return self._t.device

    @property
    def data(self):
        """The underlying torch tensor (device memory handle)."""
        return self._t

    def numel(self):
        return self._t.numel()

    def tolist(self):
        """Flat row-major list of Python floats (Tensor::to_vector)."""
        return self._t.detach().reshape(-1).cpu().tolist()

    def numpy(self):
        return self._t.detach().cpu().numpy()

    def to(self, device):
        return Tensor(self._t.to(device))

    def contiguous(self):
        return Tensor(self._t.contiguous())

    def __repr__(self):
        return f"Tensor(shape={self.shape}, device={self._t.device})"

    # ------------------------------------------------- fp32 glue (torch)
    @staticmethod
    def _other(o):
        return o._t if isinstance(o, Tensor) else o

    def add(self, other):
        return Tensor(self._t + self._other(other))

    def sub(self, other):
        return Tensor(self._t - self._other(other))

    def mul(self, other):
        return Tensor(self._t * self._other(other))

    def div(self, other):
        return Tensor(self._t / self._other(other))

    def matmul(self, other):
        return Tensor(torch.matmul(self._t, self._other(other)))

    def relu(self):
        # Ops.cpp:197-199: x > 0 ? x : 0 (maps -0.0 and NaN to +0.0)
        return Tensor(torch.where(self._t > 0, self._t, torch.zeros((), device=self._t.device)))

    def gelu(self):
        # Ops.cpp:250-256: x * 0.5 * (1 + erf(x / sqrt(2)))
        x = self._t
        return Tensor(x * (0.5 * (1.0 + torch.erf(x * 0.7071067811865476))))

    def sqrt(self):
        return Tensor(torch.sqrt(self._t))

    def exp(self):
        return Tensor(torch.exp(self._t))

    def tanh(self):
        return Tensor(torch.tanh(self._t))

    def sum(self, dim=None, keepdim=False):
        return Tensor(self._t.sum() if dim is None else self._t.sum(dim, keepdim=keepdim))

    def mean(self, dim=None, keepdim=False):
        return Tensor(self._t.mean() if dim is None else self._t.mean(dim, keepdim=keepdim))

    def max(self, dim, keepdim=False):
        return Tensor(self._t.amax(dim, keepdim=keepdim))

    def softmax(self, dim):
        return Tensor(torch.softmax(self._t, dim))

    def reshape(self, shape):
        return Tensor(self._t.reshape(list(shape)).contiguous())

    def transpose(self, dim0, dim1):
        return Tensor(self._t.transpose(dim0, dim1).contiguous())

    def slice(self, dim, start, stop):
        """Tensor::slice (core/src/Tensor.cpp:1022): a fresh contiguous copy."""
        if not 0 <= dim < self._t.dim():
            raise RuntimeError("slice: dim out of range")
        if not (0 <= start <= stop <= self._t.shape[dim]):
            raise RuntimeError("slice: start/stop out of range")
        return Tensor(self._t.narrow(dim, start, stop - start).contiguous())

    def detach(self):
        return Tensor(self._t)

    __add__ = add
    __sub__ = sub
    __mul__ = mul
    __truediv__ = div
    __matmul__ = matmul


# ---------------------------------------------------------------- factories

def from_numpy(a, device=None):
    return Tensor(torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(_as_device(device)))


def from_flat(data, shape, requires_grad=False, device=None):
    """Tensor::from_flat (core/src/Tensor.cpp:94-100)."""
    shape = [int(d) for d in shape]
    n = int(np.prod(shape)) if shape else 1
    arr = np.asarray(data, dtype=np.float32).reshape(-1)
    if arr.size != n:
        raise RuntimeError("from_flat: data length does not match shape")
    return Tensor(torch.from_numpy(arr.reshape(shape).copy()).to(_as_device(device)), requires_grad)


def zeros(shape, requires_grad=False, device=None):
    return Tensor(torch.zeros([int(d) for d in shape], dtype=torch.float32, device=_as_device(device)), requires_grad)


def ones(shape, requires_grad=False, device=None):
    return Tensor(torch.ones([int(d) for d in shape], dtype=torch.float32, device=_as_device(device)), requires_grad)


def randn_host(shape, std=1.0, seed=0):
    """numpy fp32 array with the reference's randn stream (Tensor.cpp:85-92)."""
    shape = [int(d) for d in shape]
    n = int(np.prod(shape)) if shape else 1
    out = np.empty(n, np.float32)
    _lib.check(_lib.load().kz_randn_host(out.ctypes.data_as(ctypes.c_void_p), n, float(std), int(seed)),
               "kz_randn_host")
    return out.reshape(shape)


def randn(shape, std=1.0, requires_grad=False, seed=0, device=None):
    """Tensor::randn: same values as the reference for the same seed."""
    return Tensor(torch.from_numpy(randn_host(shape, std, seed)).to(_as_device(device)), requires_grad)


def _flatten(nested):
    shape = []
    node = nested
    while isinstance(node, list):
        shape.append(len(node))
        node = node[0] if node else None
    flat = []

    def walk(x):
        if isinstance(x, list):
            for item in x:
                walk(item)
        else:
            flat.append(float(x))

    walk(nested)
    return flat, shape


def tensor(data, requires_grad=False, device=None):
    """kansai.tensor (python/kansai/__init__.py:27-30): from a nested list."""
    flat, shape = _flatten(data)
    return from_flat(flat, shape, requires_grad, device)


def cat(tensors, dim):
    """Tensor::cat (core/src/Tensor.cpp:1055)."""
    return Tensor(torch.cat([t._t for t in tensors], dim))


def as_tensor(x, device=None):
    """Accepts a Tensor, a torch/numpy array, or any object with the
    reference Tensor's `tolist()` + `shape` (e.g. a reference core.Tensor)."""
    if isinstance(x, Tensor):
        return x if device is None or x.device == torch.device(device) else x.to(device)
    if isinstance(x, torch.Tensor):
        return Tensor(x.to(_as_device(device) if device is not None else x.device).float())
    if isinstance(x, np.ndarray):
        return from_numpy(x, device)
    if hasattr(x, "tolist") and hasattr(x, "shape"):
        return from_flat(x.tolist(), list(x.shape), device=device)
    raise TypeError(f"cannot convert {type(x).__name__} to a kansaiml_b200 Tensor")
