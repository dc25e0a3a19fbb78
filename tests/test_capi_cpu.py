"""CPU checks of the drop-in boundary: libkz.so loads without a GPU, exports
every entry point include/kz.h declares (and the ctypes table binds each one),
and its host-only pieces behave as specified.  No kernel is launched here."""
import ctypes
import re

import numpy as np
import pytest

from kansaiml_b200 import _lib


def declared_symbols():
    text = open(_lib.INCLUDE_H).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kz_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/kz.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and include/kz.h disagree"


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.kz_version() >= 1
    assert isinstance(_lib.last_error(), str)


def test_randn_matches_reference_stream():
    """kz_randn_host reproduces Tensor::randn (std::mt19937 + normal_distribution):
    the reference Linear(784, 256, seed=1) weight hash is in the golden fixture."""
    import inputs
    from conftest import golden
    from kansaiml_b200.tensor import randn_host
    g = golden("mlp_config1.npz")
    w1 = randn_host([784, 256], std=1.0 / 28.0, seed=1)
    assert inputs.sha(w1) == str(g["w1_sha256"])
    np.testing.assert_array_equal(w1[0], g["w1_first_row"])


def test_host_argument_validation_without_gpu():
    """Shape checks fail before any device work."""
    lib = _lib.load()
    P = ctypes.c_void_p
    assert lib.kz_gemm_i8(None, None, -1, 1, 16, 16, None, 0, None, 0, None, 0, None, None, 1, None, None) == 1
    assert "negative" in _lib.last_error()
    assert lib.kz_gemm_i8(None, None, 4, 4, 16, 16, None, 0, None, 0, None, 0, None, None, 4, None, None) == 1
    assert "no output" in _lib.last_error()
    assert lib.kz_gemm_i8(P(16), P(16), 4, 4, 16, 16, None, 0, None, 0, None, 7, None, P(16), 4, None, None) == 1
    assert "activation" in _lib.last_error()
    assert lib.kz_gemm_i8(P(16), P(16), 4, 4, 1 << 20, 0, None, 0, None, 0, None, 0, None, P(16), 4, None, None) == 1
    assert lib.kz_absmax_f32(None, -5, None, None) == 1
    assert lib.kz_quantize_rows_f32(None, -1, 3, None, None, None, None) == 1
    assert lib.kz_qlinear_w8a32_f32(None, 1, 1, None, 1.0, None, 1, 9, None, None) == 1
    # empty work is a successful no-op
    assert lib.kz_dequantize_i8_f32(None, 0, 1.0, None, None) == 0
    assert lib.kz_qlinear_w8a32_f32(None, 0, 5, None, 1.0, None, 3, 0, None, None) == 0


def test_check_raises_with_message():
    lib = _lib.load()
    st = lib.kz_absmax_f32(None, -1, None, None)
    with pytest.raises(_lib.KzError, match="invalid argument"):
        _lib.check(st, "kz_absmax_f32")


def test_workspace_size_query():
    lib = _lib.load()
    assert lib.kz_quantize_cols_workspace_bytes(4096, 4096) >= 4 * 4096
    assert lib.kz_quantize_cols_workspace_bytes(0, 5) >= 4 * 5   # K == 0 clears one word per channel
    assert lib.kz_quantize_cols_workspace_bytes(16, 0) == 0


def test_dequantize_form_query():
    """The host picks the table-free dequantize only where the fp32 split
    form equals (float)((double)q * scale) for every byte: checked here
    against numpy for typical scales (split form) and for scales where it
    cannot hold (subnormal products, a negative scale's -0.0, overflow, NaN)."""
    import numpy as np
    lib = _lib.load()
    codes = np.arange(-128, 128).astype(np.float32)
    rs = np.random.RandomState(4)
    for s in [0.02 / 127, 1.0, 0.5, 1e-30] + list(rs.uniform(1e-5, 1.0, 200)):
        assert lib.kz_dequantize_uses_table(float(s)) == 0, s
        hi = np.float32(s)
        lo = np.float32(np.float64(s) - np.float64(hi))
        split = (codes.astype(np.float64) * np.float64(hi)       # exact: 24 x 24 bits
                 + (codes * lo).astype(np.float32).astype(np.float64)).astype(np.float32)
        exact = (codes.astype(np.float64) * s).astype(np.float32)
        # the double sum above is exact or off by far less than a float ulp here
        assert split.tobytes() == exact.tobytes(), s
    for s in (3e-39, 1e-42, -0.5, 1e39, float("nan")):
        assert lib.kz_dequantize_uses_table(s) == 1, s


def _f32_rn(v):
    """The fp32 nearest to the exact rational v (ties to even)."""
    import numpy as np
    from fractions import Fraction
    f = np.float32(float(v))
    best = None
    for c in (np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))):
        d = abs(Fraction(float(c)) - v)
        key = (d, int(np.asarray(c).view(np.uint32)) & 1)   # on a tie the even significand wins
        if best is None or key < best[0]:
            best = (key, c)
    return best[1]


def test_dequantize_split_predicate_against_exact_arithmetic():
    """The host's choice of the table-free dequantize is pinned to exact
    rational arithmetic: for random scales, the split form fma(q, s_hi,
    fl(q * s_lo)) -- evaluated here exactly and rounded once -- equals
    (float)((double)q * scale) for every byte value exactly when the library
    says so."""
    import numpy as np
    from fractions import Fraction
    lib = _lib.load()
    rs = np.random.RandomState(11)
    scales = list(rs.uniform(1e-6, 2.0, 150)) + list(10.0 ** rs.uniform(-30, 30, 50)) + [3e-39, 1e-42, -0.25]
    for s in scales:
        s = float(s)
        hi = np.float32(s)
        lo = np.float32(np.float64(s) - np.float64(hi))
        ok = bool(np.isfinite(hi) and np.isfinite(lo))
        for c in range(-128, 128):
            if not ok:
                break
            exact = np.float32(np.float64(c) * s)
            p = np.float32(np.float32(c) * lo)
            cand = _f32_rn(Fraction(c) * Fraction(float(hi)) + Fraction(float(p)))
            if np.asarray(exact).view(np.uint32) != np.asarray(cand).view(np.uint32):
                ok = False
        assert lib.kz_dequantize_uses_table(s) == (0 if ok else 1), s


def test_exchange_entry_points_validate_arguments_without_gpu():
    """The overlapped-exchange entry points reject bad arguments before any
    device work, with a message."""
    lib = _lib.load()
    P = ctypes.c_void_p
    one = P(16)
    # gated GEMM: ready flags are required
    assert lib.kz_gemm_i8_gated(one, one, 256, 256, 512, 256, one, 0, one, 1, None, 0, one, None, 256, None, None,
                                1, 0, 256, None) == 1
    assert "a_ready" in _lib.last_error()
    peers = (P * 2)(one, one)

    def allgather(**kw):
        args = dict(world=2, rank=0, M=512, N=256, K=512, flag_rows=128, copy_ctas=8)
        args.update(kw)
        return lib.kz_gemm_i8_allgather(one, peers, peers, args["world"], args["rank"], one, args["M"], args["N"],
                                        args["K"], one, 0, one, 1, one, args["N"], None, one, 1, args["flag_rows"],
                                        args["copy_ctas"], None)
    assert allgather(world=1) == 1 and "world" in _lib.last_error()
    assert allgather(world=9) == 1
    assert allgather(rank=2) == 1 and "rank" in _lib.last_error()
    assert allgather(copy_ctas=7) == 1 and "copy_ctas" in _lib.last_error()
    assert allgather(flag_rows=100) == 1 and "flag_rows" in _lib.last_error()
    assert allgather(flag_rows=384) == 1                     # does not divide M
    assert allgather(K=384) == 1                             # K / world not a multiple of 128
    # copy-engine transfer: flag required, token range
    assert lib.kz_copy_and_flag(one, one, 16, None, 1, None) == 1 and "flag" in _lib.last_error()
    assert lib.kz_copy_and_flag(one, one, 16, one, 70000, None) == 1 and "token" in _lib.last_error()
    assert lib.kz_copy_and_flag(None, one, 16, one, 1, None) == 1
    # peer buffers and LayerNorm
    assert lib.kz_peer_alloc(16, None, None) == 1
    assert lib.kz_peer_open(None, None) == 1
    assert lib.kz_layernorm_partials_f32(one, 4, 0, None, None, ctypes.c_float(1e-5), one, one, None) == 1
    assert lib.kz_layernorm_partials_f32(one, 4, 8, None, None, ctypes.c_float(1e-5), one, None, None) == 1
    # fused residual add + LayerNorm: the residual and the sum are required, the sum may not alias an input
    assert lib.kz_add_layernorm_partials_f32(one, None, 4, 8, None, None, ctypes.c_float(1e-5), P(32), one, one,
                                             None) == 1 and "res or sum_out" in _lib.last_error()
    assert lib.kz_add_layernorm_partials_f32(one, P(32), 4, 8, None, None, ctypes.c_float(1e-5), one, P(48), one,
                                             None) == 1 and "alias" in _lib.last_error()
