"""kansaiml_b200: Kansai's int8 quantized-linear path, B200-native.

A drop-in for the reference's ``kansai`` API on that path: ``quantize``
(quantize_symmetric, dequantize, QTensor, qlinear, QLinear), ``tensor`` /
``from_flat`` / ``randn`` / ``zeros`` / ``ones``, ``nn`` (Linear, ReLU, GELU,
Sequential, TransformerBlock ...) and ``distributed`` (DeviceMesh, Shard,
Replicate, DTensor).  All compute on the path runs in libkz (include/kz.h),
hand-written sm_100a CUDA; there is no CPU fallback.
"""
from . import _lib
from .tensor import Tensor, cat, from_flat, from_numpy, ones, randn, tensor, zeros

__all__ = ["Tensor", "cat", "from_flat", "from_numpy", "ones", "randn", "tensor", "zeros", "quantize", "nn",
           "distributed", "build"]


def build():
    """Compile libkz.so in-tree (sm_100a)."""
    import os
    import subprocess
    here = os.path.dirname(os.path.abspath(__file__))
    subprocess.run(["make", "-s", "-C", os.path.join(here, "csrc")], check=True)


def __getattr__(name):
    if name in ("quantize", "nn", "distributed", "serialize", "workloads"):
        import importlib
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
