"""The reference's import path, ``kansai``, served by this repository's B200 backend.

A user's quantized model keeps its imports as they are -- ``from kansai.quantize
import QLinear``, ``from kansai import nn``, ``kansai.distributed.DTensor``,
``kansai.tensor([[...]])`` -- and runs on libkz.  Every name here is the
kansaiml_b200 object itself, and ``kansai.quantize`` / ``nn`` /
``distributed`` / ``serialize`` are the same module objects as
``kansaiml_b200.*``: one implementation, one set of per-device state.

The reference package's other top-level names on this path: ``where``
(python/kansai/__init__.py, composed from sub/mul/add as there) and
``no_grad``.  This backend is inference only -- no operation records a
gradient graph -- so ``no_grad`` has nothing to switch off and only keeps
``with kansai.no_grad():`` blocks working.
"""
import contextlib
import sys

from kansaiml_b200 import Tensor, cat, from_flat, from_numpy, ones, randn, tensor, zeros
from kansaiml_b200 import distributed, nn, quantize, serialize

for _name, _module in (("quantize", quantize), ("nn", nn), ("distributed", distributed), ("serialize", serialize)):
    sys.modules[f"{__name__}.{_name}"] = _module
del _name, _module


def where(cond, a, b):
    """Elementwise select, ``b + cond * (a - b)`` with cond in {0, 1}."""
    return b.add(cond.mul(a.sub(b)))


@contextlib.contextmanager
def no_grad():
    yield


__all__ = ["Tensor", "cat", "from_flat", "from_numpy", "ones", "randn", "tensor", "zeros", "where", "no_grad",
           "quantize", "nn", "distributed", "serialize"]
