"""TEST INFRASTRUCTURE ONLY: import the reference's own Python package.

``import_reference_kansai()`` loads ``python/kansai`` from the reference checkout,
unmodified, with its ``_core`` extension resolved from ``oracle/_ref`` (the
reference's C++ core compiled by ``make -C oracle ref``).  It is registered
as the package ``kansai_reference`` (its modules import each other relatively),
so the name ``kansai`` stays free for this repository's drop-in package and
both can be loaded in one process.  Nothing is copied:
the package's search path lists the reference directory first and the build
directory second.  Available only where the reference checkout exists; the GPU
box has only ``load_reference_core()``, the compiled core on its own.
"""
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_BUILD = os.path.join(HERE, "_ref")
REF_PACKAGE = "kansai_reference"
# $KZ_REFERENCE_ROOT, else a checkout named `reference` beside this repository
REF_ROOT = os.environ.get("KZ_REFERENCE_ROOT") or os.path.abspath(os.path.join(HERE, "..", "..", "reference"))


def reference_available() -> bool:
    return os.path.isdir(os.path.join(REF_ROOT, "python", "kansai")) and any(
        f.startswith("_core") for f in os.listdir(REF_BUILD)) if os.path.isdir(REF_BUILD) else False


def load_reference_core():
    """The reference's C++ core (Tensor, from_flat, matmul, ...) as a module."""
    name = next((f for f in os.listdir(REF_BUILD) if f.startswith("_core") and f.endswith(".so")), None)
    if name is None:
        raise ImportError("oracle/_ref has no compiled reference core; run `make -C oracle ref`")
    spec = importlib.util.spec_from_file_location("_core", os.path.join(REF_BUILD, name))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def import_reference_kansai():
    """The reference's ``kansai`` package (quantize, nn, distributed, optim ...)."""
    if REF_PACKAGE in sys.modules:
        return sys.modules[REF_PACKAGE]
    pkg_dir = os.path.join(REF_ROOT, "python", "kansai")
    if not os.path.isdir(pkg_dir):
        raise ImportError(f"reference checkout not found at {REF_ROOT}")
    spec = importlib.util.spec_from_file_location(
        REF_PACKAGE, os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir, REF_BUILD])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[REF_PACKAGE] = mod
    spec.loader.exec_module(mod)
    return mod
