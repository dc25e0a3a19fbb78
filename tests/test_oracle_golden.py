"""Pin the C restatement (oracle/kz_oracle.c) to the reference's own outputs.

The fixtures were produced by the reference's unmodified Python running over
its own compiled C++ core (tests/golden/gen_golden.py).  Integer codes must be
bit-exact; scales must be the identical double; dequantized and fp32 matmul
outputs must be bit-identical fp32.
"""
import numpy as np
import pytest

import inputs
from conftest import golden
from oracle import cpu as ocpu
from oracle import refpkg


@pytest.fixture(scope="module")
def qcases():
    g = golden("quantize_cases.npz")
    cases = inputs.quantize_case_inputs()
    return g, cases


def test_quantize_inputs_match_fixture_hashes(qcases):
    g, cases = qcases
    for name, x in cases.items():
        assert inputs.sha(x) == str(g[f"{name}__x_sha256"]), name


def test_quantize_tensor_bit_exact_vs_reference(qcases):
    g, cases = qcases
    for name, x in cases.items():
        q, s = ocpu.quantize_tensor(x)
        assert s == float(g[f"{name}__scale"]), name
        np.testing.assert_array_equal(q, g[f"{name}__q"], err_msg=name)
        assert q.min() >= -127 and q.max() <= 127


def test_dequantize_bit_exact_vs_reference(qcases):
    g, cases = qcases
    for name in cases:
        if f"{name}__deq" not in g:
            continue
        deq = ocpu.dequantize(g[f"{name}__q"], float(g[f"{name}__scale"]))
        assert deq.tobytes() == g[f"{name}__deq"].astype(np.float32).tobytes(), name


def test_reference_properties_test_quantize_py(qcases):
    """tests/test_quantize.py:41-72 restated on the oracle."""
    g, cases = qcases
    x = cases["uniform1000"]
    q, s = ocpu.quantize_tensor(x)
    err = np.abs(x.astype(np.float64) - ocpu.dequantize(q, s).astype(np.float64)).max()
    assert err <= s / 2 + 1e-6
    q0, _ = ocpu.quantize_tensor(cases["zero_one"])
    assert q0[0] == 0
    assert int(g["randn256_seed1__nbytes"]) * 4 == 4 * 65536


def test_nonfinite_raises():
    for bad in (np.float32(np.nan), np.float32(np.inf), np.float32(-np.inf)):
        with pytest.raises(ValueError):
            ocpu.quantize_tensor(np.asarray([1.0, bad, 2.0], np.float32))


def test_percol_matches_reference_columnwise():
    g = golden("percol_cases.npz")
    w = inputs.percol_weight()
    assert inputs.sha(w) == str(g["w_sha256"])
    qT, s = ocpu.quantize_cols(w)
    np.testing.assert_array_equal(qT, g["qT"])
    np.testing.assert_array_equal(s, g["scales"])
    assert s[3] == 1.0 and not qT[3].any()


def test_qlinear_w8a32_bit_exact_vs_reference():
    g = golden("w8a32_cases.npz")
    for i in range(int(g["count"])):
        x, w, b = inputs.w8a32_inputs(i)
        assert inputs.sha(x) + inputs.sha(w) + inputs.sha(b) == str(g[f"c{i}__inputs_sha256"])
        q, s = ocpu.quantize_tensor(w)
        np.testing.assert_array_equal(q, g[f"c{i}__q"])
        assert s == float(g[f"c{i}__scale"])
        for act, key in ((0, "y"), (1, "y_relu")):
            y = ocpu.qlinear_w8a32(x, q, s, b, act=act)
            assert y.tobytes() == g[f"c{i}__{key}"].tobytes(), (i, key)
        # gelu: the same glibc erff and operation order as the reference's
        # gelu_fwd (Ops.cpp:250-256), so bit for bit as well
        y = ocpu.qlinear_w8a32(x, q, s, b, act=2)
        assert y.tobytes() == g[f"c{i}__y_gelu"].tobytes(), (i, "gelu")


def test_mlp_config1_vs_reference():
    g = golden("mlp_config1.npz")
    x, b1, b2 = inputs.mlp_config1_inputs()
    assert inputs.sha(x) == str(g["x_sha256"])
    h = ocpu.qlinear_w8a32(x, g["q1"], float(g["s1"]), b1, act=1)
    assert h.tobytes() == g["h"].tobytes()
    y = ocpu.qlinear_w8a32(h, g["q2"], float(g["s2"]), b2, act=0)
    assert y.tobytes() == g["y"].tobytes()


def test_xor_qlinear_vs_reference():
    g = golden("xor_qlinear.npz")
    q1, s1 = ocpu.quantize_tensor(g["w1"])
    q2, s2 = ocpu.quantize_tensor(g["w2"])
    h = ocpu.qlinear_w8a32(g["x"], q1, s1, g["b1"], act=1)
    y = ocpu.qlinear_w8a32(h, q2, s2, g["b2"], act=0)
    assert y.tobytes() == g["quant_preds"].tobytes()
    assert [round(float(v)) for v in y.ravel()] == [0, 1, 1, 0]


def test_layernorm_bit_exact_vs_reference():
    """The oracle's LayerNorm (kz_oracle.c) against the reference's own
    nn.LayerNorm (nn.py:323-331): with set and default parameters, of x and of
    the residual sum x.add(res), and the quantize_symmetric codes of the
    result -- all bit for bit."""
    g = golden("layernorm_cases.npz")
    for i in range(int(g["count"])):
        x, res, gamma, beta = inputs.layernorm_inputs(i)
        assert inputs.sha(x) + inputs.sha(res) + inputs.sha(gamma) + inputs.sha(beta) == str(g[f"c{i}__inputs_sha256"])
        y = ocpu.layernorm(x, gamma, beta, 1e-5)
        assert y.tobytes() == g[f"c{i}__y"].tobytes(), i
        assert ocpu.layernorm(x).tobytes() == g[f"c{i}__y_default"].tobytes(), i
        y_sum, total = ocpu.layernorm(x, gamma, beta, 1e-5, residual=res)
        assert total.tobytes() == g[f"c{i}__sum"].tobytes(), i
        assert y_sum.tobytes() == g[f"c{i}__y_sum"].tobytes(), i
        q, s = ocpu.quantize_tensor(y)
        assert s == float(g[f"c{i}__scale"]), i
        np.testing.assert_array_equal(q, g[f"c{i}__q"], err_msg=str(i))


def _attention_case(i, exp):
    B, Sq, Sk, D, H, kind = inputs.ATTENTION_CASES[i]
    q, k, v, mask = inputs.attention_inputs(i)
    if kind == "causal":
        return ocpu.attention(q, k, v, H, causal=True, exp=exp)
    return ocpu.attention(q, k, v, H, mask=mask, exp=exp)


def test_attention_bit_exact_vs_reference():
    """The oracle's attention core with the host's expf (the function the
    reference's std::exp calls) against the reference's own
    MultiHeadAttention.forward with identity projections: bit for bit, the
    causal mask given as the flag included (its keys' exponentials are 0)."""
    g = golden("attention_cases.npz")
    for i in range(int(g["count"])):
        q, k, v, mask = inputs.attention_inputs(i)
        assert inputs.sha(q) + inputs.sha(k) + inputs.sha(v) + (inputs.sha(mask) if mask is not None else "") == \
            str(g[f"c{i}__inputs_sha256"])
        assert _attention_case(i, "libm").tobytes() == g[f"c{i}__y"].tobytes(), i
        if inputs.ATTENTION_CASES[i][5] == "causal":   # the explicit mask gives the same bits
            H = inputs.ATTENTION_CASES[i][4]
            assert ocpu.attention(q, k, v, H, mask=mask, exp="libm").tobytes() == g[f"c{i}__y"].tobytes(), i


def test_attention_rounded_exp_vs_reference():
    """With the correctly rounded exp (the CUDA kernel's), the oracle differs
    from the reference only where the host's expf is not correctly rounded:
    a handful of outputs, by a few ulps."""
    g = golden("attention_cases.npz")
    diff = total = 0
    for i in range(int(g["count"])):
        y, ref = _attention_case(i, "rn"), g[f"c{i}__y"]
        bad = y.view(np.int32) != ref.view(np.int32)
        diff += int(bad.sum())
        total += y.size
        np.testing.assert_allclose(y, ref, rtol=2e-6, atol=1e-7, err_msg=str(i))
    assert diff <= total // 1000, (diff, total)


def test_attention_exp_modes_agree_where_expf_rounds_correctly():
    """The two exp modes of the oracle: the host's expf against the double
    exp narrowed to fp32 over the softmax's input range -- they differ only on
    inputs whose exponential lies within a hair of a rounding midpoint, a
    fraction of a percent."""
    x = -np.random.RandomState(5).uniform(0, 60, 100000).astype(np.float32)
    libm = ocpu.expf_host(x)
    rn = np.exp(x.astype(np.float64)).astype(np.float32)
    bad = libm.view(np.int32) != rn.view(np.int32)
    assert bad.sum() <= 200, int(bad.sum())
    assert np.all(np.abs(libm.view(np.int32).astype(np.int64) - rn.view(np.int32)) <= 1)
    # every disagreement sits next to a midpoint of the two neighbouring floats
    exact = np.exp(x[bad].astype(np.float64))
    lo = np.minimum(libm[bad], rn[bad]).astype(np.float64)
    hi = np.maximum(libm[bad], rn[bad]).astype(np.float64)
    assert np.all(np.abs((exact - lo) / (hi - lo) - 0.5) < 0.01)


def test_int8_gemm_and_epilogue_small():
    rs = np.random.RandomState(1)
    a = rs.randint(-127, 128, (33, 80)).astype(np.int8)
    b = rs.randint(-127, 128, (17, 80)).astype(np.int8)
    acc = ocpu.gemm_i8(a, b)
    np.testing.assert_array_equal(acc, a.astype(np.int64) @ b.astype(np.int64).T)
    rsc = rs.uniform(1e-3, 1e-2, 33)
    csc = rs.uniform(1e-3, 1e-2, 17)
    y = ocpu.epilogue(acc, rsc, csc)
    ref = (acc.astype(np.float32) * rsc.astype(np.float32)[:, None]).astype(np.float32) * csc.astype(np.float32)[None, :]
    assert y.tobytes() == ref.astype(np.float32).tobytes()


# ------------------------------------------- randomized restatement check

from hypothesis import given, settings, strategies as st  # noqa: E402


def _py_quantize(x):
    """quantize.py:66-69 verbatim in plain Python: fp32 values widened to
    float, max |v|, scale = max / 127.0 (1.0 for all zeros), codes
    max(-127, min(127, round(v / scale))) with Python's half-to-even round."""
    flat = [float(v) for v in np.asarray(x, np.float32).ravel()]
    max_abs = max((abs(v) for v in flat), default=0.0)
    scale = max_abs / 127.0 if max_abs > 0.0 else 1.0
    return [max(-127, min(127, round(v / scale))) for v in flat], scale


_BIG = float(np.float32(1e30))
_f32s = st.floats(min_value=-_BIG, max_value=_BIG, allow_nan=False, allow_infinity=False, width=32)


@settings(max_examples=400, deadline=None)
@given(st.lists(_f32s, min_size=1, max_size=64))
def test_oracle_quantize_matches_plain_python(values):
    x = np.asarray(values, np.float32)
    q, s = ocpu.quantize_tensor(x)
    q_py, s_py = _py_quantize(x)
    assert s == s_py
    assert q.tolist() == q_py


@settings(max_examples=300, deadline=None)
@given(st.integers(1, 127), st.lists(st.tuples(st.integers(-127, 127), st.sampled_from([-1, 0, 1])),
                                     min_size=1, max_size=32))
def test_oracle_quantize_near_ties(top, steps):
    """Values placed on and one ulp either side of (k + 1/2) * scale, where
    round-half-even decides: the oracle's codes equal Python's."""
    scale = top / 127.0
    vals = [np.float32(top)]
    for k, d in steps:
        v = np.float32((k + 0.5) * scale)
        if d:
            v = np.nextafter(v, np.float32(np.inf if d > 0 else -np.inf))
        vals.append(v)
    x = np.asarray(vals, np.float32)
    q, s = ocpu.quantize_tensor(x)
    q_py, s_py = _py_quantize(x)
    assert s == s_py
    assert q.tolist() == q_py


@settings(max_examples=200, deadline=None)
@given(st.integers(1, 12), st.integers(1, 12), st.integers(0, 2 ** 31 - 1))
def test_oracle_quantize_cols_is_per_column_quantize(K, N, seed):
    """Per-output-channel quantize = quantize.py:66-69 applied to each column
    of the [in, out] weight, codes stored K-major [N, K]."""
    rs = np.random.RandomState(seed)
    w = (rs.standard_normal((K, N)) * rs.uniform(1e-3, 1e3, N)).astype(np.float32)
    w[:, rs.rand(N) < 0.1] = 0.0                       # some all-zero channels (scale 1.0)
    qT, s = ocpu.quantize_cols(w)
    for n in range(N):
        q_py, s_py = _py_quantize(w[:, n])
        assert s[n] == s_py
        assert qT[n].tolist() == q_py


@settings(max_examples=200, deadline=None)
@given(st.integers(1, 8), st.integers(1, 8), st.booleans(), st.booleans(), st.integers(0, 2 ** 31 - 1))
def test_oracle_epilogue_is_fp32_arithmetic(M, N, per_row, with_bias, seed):
    """The W8A8 epilogue y = ((float)acc * row_scale) * col_scale (+ bias),
    each step one fp32 rounding, as numpy's float32 operations give it."""
    rs = np.random.RandomState(seed)
    acc = rs.randint(-2 ** 31 + 1, 2 ** 31 - 1, (M, N), dtype=np.int64).astype(np.int32)
    row = rs.uniform(1e-4, 1e-1, M if per_row else 1)
    col = rs.uniform(1e-4, 1e-1, N)
    bias = rs.standard_normal(N).astype(np.float32) if with_bias else None
    y = ocpu.epilogue(acc, row if per_row else row[0], col, bias)
    ref = (acc.astype(np.float32) * row.astype(np.float32).reshape(-1, 1)) * col.astype(np.float32)
    if with_bias:
        ref = ref + bias
    assert y.tobytes() == ref.astype(np.float32).tobytes()


@settings(max_examples=150, deadline=None)
@given(st.integers(1, 9), st.integers(1, 9), st.integers(1, 200), st.integers(0, 2 ** 31 - 1))
def test_oracle_gemm_i8_is_exact_integer_matmul(M, N, K, seed):
    rs = np.random.RandomState(seed)
    a = rs.randint(-128, 128, (M, K)).astype(np.int8)
    b = rs.randint(-128, 128, (N, K)).astype(np.int8)
    acc = ocpu.gemm_i8(a, b)
    assert np.array_equal(acc, (a.astype(np.int64) @ b.astype(np.int64).T).astype(np.int32))


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 4), st.integers(1, 4), st.integers(1, 40), st.booleans(), st.integers(0, 2 ** 31 - 1))
def test_oracle_qlinear_w8a32_is_the_k_ordered_loop(M, N, K, relu, seed):
    """quantize.py:115-122 on Linux: the weight dequantized to fp32
    (fl32(fl64(q) * scale)), then Ops.cpp's loop: every out[i, j] summed in
    k order with each product and each sum rounded to fp32, bias, ReLU."""
    rs = np.random.RandomState(seed)
    x = rs.standard_normal((M, K)).astype(np.float32)
    q = rs.randint(-127, 128, (K, N)).astype(np.int8)
    scale = float(rs.uniform(1e-3, 1e-1))
    bias = rs.standard_normal(N).astype(np.float32)
    y = ocpu.qlinear_w8a32(x, q, scale, bias, act=1 if relu else 0)
    w = (q.astype(np.float64) * scale).astype(np.float32)
    ref = np.empty((M, N), np.float32)
    for i in range(M):
        for j in range(N):
            acc = np.float32(0.0)
            for k in range(K):
                acc = np.float32(acc + np.float32(x[i, k] * w[k, j]))
            v = np.float32(acc + bias[j])
            ref[i, j] = (v if v > 0 else np.float32(0.0)) if relu else v   # x > 0 ? x : 0, as Ops.cpp
    assert y.tobytes() == ref.tobytes()


@pytest.mark.skipif(not refpkg.reference_available(), reason="reference checkout / compiled core not present")
def test_attention_oracle_vs_reference_random_shapes():
    """Beyond the fixtures: random shapes (1-3 batches, 1-4 heads, head widths
    8 / 16 / 32, query and key lengths 1-90), the reference's own
    MultiHeadAttention.forward with identity projections against the oracle
    with the host's expf -- bit for bit -- with and without a random additive
    mask."""
    kansai = refpkg.import_reference_kansai()
    from kansai_reference import nn
    core = kansai.core

    def from_np(x):
        return core.from_flat(np.asarray(x, np.float32).ravel().tolist(), list(x.shape))

    rs = np.random.RandomState(77)
    for case in range(12):
        B, H, dk = rs.randint(1, 4), rs.randint(1, 5), int(rs.choice([8, 16, 32]))
        Sq, Sk = rs.randint(1, 91), rs.randint(1, 91)
        D = H * dk
        q = (rs.standard_normal((B, Sq, D)) * 2).astype(np.float32)
        k = (rs.standard_normal((B, Sk, D)) * 2).astype(np.float32)
        v = rs.standard_normal((B, Sk, D)).astype(np.float32)
        mask = None
        if case % 2:
            mask = (rs.uniform(-5, 0, (B, 1, Sq, Sk)) * (rs.uniform(size=(B, 1, Sq, Sk)) < 0.5)).astype(np.float32)
        mha = nn.MultiHeadAttention(D, H)
        eye = from_np(np.eye(D, dtype=np.float32))
        mha.w_q = mha.w_k = mha.w_v = mha.w_o = eye
        y = mha.forward(from_np(q), from_np(k), from_np(v), mask=from_np(mask) if mask is not None else None)
        ref = np.asarray(y.tolist(), np.float32).reshape(B, Sq, D)
        assert ocpu.attention(q, k, v, H, mask=mask, exp="libm").tobytes() == ref.tobytes(), (case, B, H, dk, Sq, Sk)


@pytest.mark.skipif(not refpkg.reference_available(), reason="reference checkout / compiled core not present")
def test_layernorm_oracle_vs_reference_random_shapes():
    """Beyond the fixtures: the reference's own nn.LayerNorm at random row
    counts and widths (1-300), with random gamma / beta and the residual sum,
    against the oracle -- bit for bit."""
    kansai = refpkg.import_reference_kansai()
    from kansai_reference import nn
    core = kansai.core

    def from_np(x):
        return core.from_flat(np.asarray(x, np.float32).ravel().tolist(), list(x.shape))

    def to_np(t):
        return np.asarray(t.tolist(), np.float32).reshape(list(t.shape))

    rs = np.random.RandomState(91)
    for case in range(10):
        M, D = int(rs.randint(1, 40)), int(rs.randint(1, 301))
        x = (rs.standard_normal((M, D)) * rs.uniform(0.1, 10) + rs.uniform(-3, 3)).astype(np.float32)
        res = rs.standard_normal((M, D)).astype(np.float32)
        gamma = rs.uniform(0.5, 1.5, D).astype(np.float32)
        beta = (rs.standard_normal(D) * 0.1).astype(np.float32)
        ln = nn.LayerNorm(D)
        ln.weight, ln.bias = from_np(gamma), from_np(beta)
        total = from_np(x).add(from_np(res))
        ref = to_np(ln(total))
        y, tot = ocpu.layernorm(x, gamma, beta, 1e-5, residual=res)
        assert tot.tobytes() == to_np(total).tobytes(), case
        assert y.tobytes() == ref.tobytes(), (case, M, D)
