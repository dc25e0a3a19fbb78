"""Seeded inputs shared by gen_golden.py and the tests.

numpy's legacy RandomState streams are frozen across numpy versions, so these
regenerate bit-identically anywhere; the fixtures store a sha256 of each input
so drift would be caught rather than silently compared against.
"""
import hashlib
import random

import numpy as np


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def near_tie_values(seed, scale, count):
    """fp32 values whose quotient v / scale lies at or within 3 fp32 ulps of a
    half-integer -- where a fast fp32 estimate of the quotient must defer to
    the exact double division."""
    r = random.Random(seed)
    out = []
    for _ in range(count):
        k = r.randint(-126, 126)
        v = np.float32((k + 0.5) * scale)
        for d in range(-3, 4):
            w = v
            step = np.float32(np.inf) if d > 0 else np.float32(-np.inf)
            for _ in range(abs(d)):
                w = np.nextafter(w, step)
            out.append(w)
    return np.asarray(out, np.float32)


def quantize_case_inputs():
    """name -> fp32 input for the quantize_symmetric golden cases (cases whose
    input comes from the reference's own randn are produced in gen_golden.py)."""
    cases = {}
    r = random.Random(0)  # tests/test_quantize.py:41
    cases["uniform1000"] = np.asarray([r.uniform(-3.0, 3.0) for _ in range(1000)], np.float32)
    cases["zero_one"] = np.asarray([0.0, 1.0, -1.0], np.float32)  # tests/test_quantize.py:58
    cases["ties_unit"] = np.asarray([0.5, 1.5, 2.5, -2.5, 127.0, -0.5, 126.5, -126.5], np.float32)
    cases["ties_pow2"] = np.asarray([31.75, 0.125, 0.375, -0.625, 0.875, 30.875, -30.625, 0.0], np.float32)
    cases["all_zero"] = np.zeros(17, np.float32)
    cases["single_neg"] = np.asarray([-3.25], np.float32)
    rs = np.random.RandomState(11)
    for i, amax in enumerate([0.7, 3.0e-3, 1234.5678]):
        v = near_tie_values(100 + i, amax / 127.0, 300)
        v = np.concatenate([v, np.asarray([amax, -amax], np.float32)])
        v = np.clip(v, -np.float32(amax), np.float32(amax)).astype(np.float32)
        cases[f"near_ties_{i}"] = v[rs.permutation(v.size)]
    cases["subnormal"] = (np.random.RandomState(5).standard_normal(513) * 1e-41).astype(np.float32)
    cases["tiny_normal"] = (np.random.RandomState(6).standard_normal(257) * 1e-33).astype(np.float32)
    cases["huge"] = (np.random.RandomState(7).uniform(-1, 1, 129) * 3.0e38).astype(np.float32)
    cases["normal_100003"] = np.random.RandomState(3).standard_normal(100003).astype(np.float32)
    return cases


def percol_weight():
    rs = np.random.RandomState(21)
    K, N = 96, 40
    w = (rs.standard_normal((K, N)) * 0.02).astype(np.float32)
    w[:, 3] = 0.0                                                         # all-zero channel
    w[:, 7] = np.float32(0.5) * (np.arange(K, dtype=np.float32) % 5 - 2)  # exact ties
    w[5, 11] = np.float32(9.0)                                            # one outlier
    return w


W8A32_SHAPES = [(37, 200, 53), (1, 16, 1), (64, 784, 256), (5, 32, 130)]


def w8a32_inputs(i):
    M, K, N = W8A32_SHAPES[i]
    rs = np.random.RandomState(300 + i)
    x = rs.uniform(-1, 1, (M, K)).astype(np.float32)
    w = (rs.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    b = (rs.standard_normal(N) * 0.1).astype(np.float32)
    return x, w, b


def mlp_config1_inputs():
    """BASELINE config 1 batch and biases (weights come from Linear(seed=1/2))."""
    x = np.random.RandomState(0).random_sample((64, 784)).astype(np.float32)
    b1 = (np.random.RandomState(1).standard_normal(256) * 0.05).astype(np.float32)
    b2 = (np.random.RandomState(2).standard_normal(10) * 0.05).astype(np.float32)
    return x, b1, b2


LAYERNORM_SHAPES = [(2, 48, 256), (3, 5, 100), (64, 7)]


def layernorm_inputs(i):
    """(x, residual, gamma, beta) for LayerNorm case i; x has a non-zero mean
    and a spread that keeps the ordered sums away from exact arithmetic."""
    shape = LAYERNORM_SHAPES[i]
    d = shape[-1]
    rs = np.random.RandomState(300 + i)
    x = (rs.standard_normal(shape) * 3 + 1).astype(np.float32)
    res = rs.standard_normal(shape).astype(np.float32)
    gamma = rs.uniform(0.5, 1.5, d).astype(np.float32)
    beta = (rs.standard_normal(d) * 0.1).astype(np.float32)
    return x, res, gamma, beta


# (batch, seq_q, seq_k, d_model, heads, mask kind): self-attention with the
# causal mask across a 64-row tile edge, cross-attention with a broadcast
# random additive mask, no mask, and head widths 32 / 64 / 128
ATTENTION_CASES = [(2, 24, 24, 128, 4, "causal"), (2, 67, 67, 128, 2, "causal"), (1, 5, 70, 64, 2, "mask"),
                   (3, 9, 130, 32, 1, "none"), (1, 80, 80, 128, 1, "mask")]


def attention_inputs(i):
    """(q, k, v, mask or None) for attention case i: q [B, Sq, D], k and v
    [B, Sk, D]; the causal mask is causal_mask()'s [1, 1, S, S] (-1e9 above the
    diagonal), the random one [B, 1, Sq, Sk] with about a third of its
    entries negative."""
    B, Sq, Sk, D, H, kind = ATTENTION_CASES[i]
    rs = np.random.RandomState(700 + i)
    q = (rs.standard_normal((B, Sq, D)) * 2).astype(np.float32)
    k = (rs.standard_normal((B, Sk, D)) * 2).astype(np.float32)
    v = rs.standard_normal((B, Sk, D)).astype(np.float32)
    if kind == "causal":
        mask = np.triu(np.full((Sq, Sk), -1e9, np.float32), 1)[None, None]
    elif kind == "mask":
        mask = (rs.uniform(-3, 0, (B, 1, Sq, Sk)) * (rs.uniform(size=(B, 1, Sq, Sk)) < 0.3)).astype(np.float32)
    else:
        mask = None
    return q, k, v, mask
