"""Generate the golden fixtures in this directory from the REFERENCE itself.

Run where the reference checkout is present (it is not on the GPU box):

    make -C oracle ref && python tests/golden/gen_golden.py

Every output array written here comes from the reference's own, unmodified
Python (python/kansai/quantize.py, nn.py, optim.py, distributed.py) running
over the reference's own C++ core compiled from source (oracle/ref_core_py.cpp).
Inputs come from tests/golden/inputs.py (numpy's frozen legacy RandomState)
or from the reference's own `randn(seed=...)`; fixtures store each input's
sha256 so a drifting generator is caught instead of silently compared.

Fixtures:
  quantize_cases.npz  quantize_symmetric / dequantize (quantize.py:50-77) on the
                      cases of tests/test_quantize.py:41-72 plus ties, near-ties,
                      subnormal, huge, all-zero and large random tensors.
  percol_cases.npz    per-output-channel quantization, defined as the reference's
                      quantize_symmetric applied to each column of the [in, out]
                      weight.
  w8a32_cases.npz     qlinear (quantize.py:115-122) at ragged shapes, with bias,
                      and followed by relu / gelu.
  mlp_config1.npz     config 1: Sequential(QLinear(784->256), ReLU,
                      QLinear(256->10)) on a [64, 784] U[0,1) batch.
  xor_qlinear.npz     tests/test_quantize.py:81-125: the trained XOR model and the
                      quantized model's predictions.
  chunk_cases.npz     _chunk_sizes (distributed.py:157-159) for uneven splits.
  layernorm_cases.npz nn.LayerNorm (nn.py:308-331) with set and default
                      parameters, of x and of x.add(residual), and the
                      quantize_symmetric codes of the result (config 3's
                      LayerNorm -> quantize prologue).
  attention_cases.npz nn.MultiHeadAttention.forward (nn.py:410-427) with
                      identity projections: the attention core with the causal
                      mask, a broadcast additive mask, and none.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))
sys.path.insert(0, HERE)

from oracle.refpkg import import_reference_kansai  # noqa: E402
import inputs  # noqa: E402

kansai = import_reference_kansai()
from kansai_reference import nn, optim  # noqa: E402
from kansai_reference.distributed import _chunk_sizes  # noqa: E402
from kansai_reference.quantize import QLinear, QTensor, dequantize, qlinear, quantize_symmetric  # noqa: E402

core = kansai.core
sha = inputs.sha


def to_np(t):
    return np.asarray(t.tolist(), dtype=np.float32).reshape(list(t.shape))


def from_np(x):
    return core.from_flat(np.asarray(x, np.float32).ravel().tolist(), list(x.shape))


def ref_quantize(x):
    q, s, shape = quantize_symmetric(from_np(x))
    deq = to_np(dequantize(q, s, shape))
    return np.asarray(q, np.int8).reshape(x.shape), float(s), deq


def quantize_cases():
    cases = inputs.quantize_case_inputs()
    big = core.randn([256, 256], std=1.0, seed=1)  # tests/test_quantize.py:66
    cases["randn256_seed1"] = to_np(big)
    out = {}
    names = sorted(cases)
    for name in names:
        x = cases[name]
        q, s, deq = ref_quantize(x)
        out[f"{name}__x_sha256"] = np.asarray(sha(x))
        out[f"{name}__q"] = q
        out[f"{name}__scale"] = np.float64(s)
        if x.size <= 4096:           # dequantize outputs for the small cases
            out[f"{name}__deq"] = deq
    out["names"] = np.asarray(names)
    out["randn256_seed1__nbytes"] = np.int64(QTensor.from_tensor(big).nbytes())
    out["randn256_seed1__first_row"] = cases["randn256_seed1"][0]
    np.savez_compressed(os.path.join(HERE, "quantize_cases.npz"), **out)
    print("quantize_cases.npz:", len(names), "cases")


def percol_cases():
    w = inputs.percol_weight()
    K, N = w.shape
    qT = np.empty((N, K), np.int8)
    scales = np.empty(N, np.float64)
    for n in range(N):
        qT[n], scales[n], _ = ref_quantize(np.ascontiguousarray(w[:, n]))
    np.savez_compressed(os.path.join(HERE, "percol_cases.npz"), w_sha256=np.asarray(sha(w)), qT=qT, scales=scales)
    print("percol_cases.npz: K=%d N=%d" % (K, N))


def w8a32_cases():
    out = {}
    for i, (M, K, N) in enumerate(inputs.W8A32_SHAPES):
        x, w, b = inputs.w8a32_inputs(i)
        qw = QTensor.from_tensor(from_np(w))
        xt, bt = from_np(x), from_np(b)
        out[f"c{i}__inputs_sha256"] = np.asarray(sha(x) + sha(w) + sha(b))
        out[f"c{i}__q"] = np.asarray(qw.q, np.int8).reshape(K, N)
        out[f"c{i}__scale"] = np.float64(qw.scale)
        out[f"c{i}__y"] = to_np(qlinear(xt, qw, bt))
        out[f"c{i}__y_relu"] = to_np(qlinear(xt, qw, bt).relu())
        out[f"c{i}__y_gelu"] = to_np(qlinear(xt, qw, bt).gelu())
    out["count"] = np.int64(len(inputs.W8A32_SHAPES))
    np.savez_compressed(os.path.join(HERE, "w8a32_cases.npz"), **out)
    print("w8a32_cases.npz:", len(inputs.W8A32_SHAPES), "shapes")


def mlp_config1():
    # weights N(0, 1/784) and N(0, 1/256) are nn.Linear's own
    # init (std = 1/sqrt(in_features), nn.py:74-79) with seeds 1 and 2.
    l1 = nn.Linear(784, 256, seed=1)
    l2 = nn.Linear(256, 10, seed=2)
    x, b1, b2 = inputs.mlp_config1_inputs()
    l1.bias, l2.bias = from_np(b1), from_np(b2)
    qmodel = nn.Sequential(QLinear(l1), nn.ReLU(), QLinear(l2))
    xt = from_np(x)
    h = qmodel.layers[1](qmodel.layers[0](xt))
    y = qmodel(xt)
    np.savez_compressed(
        os.path.join(HERE, "mlp_config1.npz"),
        x_sha256=np.asarray(sha(x)), w1_sha256=np.asarray(sha(to_np(l1.weight))),
        w2_sha256=np.asarray(sha(to_np(l2.weight))), w1_first_row=to_np(l1.weight)[0],
        q1=np.asarray(qmodel.layers[0].qweight.q, np.int8).reshape(784, 256),
        s1=np.float64(qmodel.layers[0].qweight.scale),
        q2=np.asarray(qmodel.layers[2].qweight.q, np.int8).reshape(256, 10),
        s2=np.float64(qmodel.layers[2].qweight.scale), h=to_np(h), y=to_np(y))
    print("mlp_config1.npz: y", to_np(y).shape)


def xor_qlinear():
    # tests/test_quantize.py:81-125, same setup
    X = kansai.tensor([[0, 0], [0, 1], [1, 0], [1, 1]])
    Y = kansai.tensor([[0], [1], [1], [0]])
    model = nn.Sequential(nn.Linear(2, 8, seed=3), nn.ReLU(), nn.Linear(8, 1, seed=4))
    opt = optim.SGD(model.parameters(), lr=0.1)
    loss = None
    for _ in range(500):
        diff = model(X).sub(Y)
        loss = diff.mul(diff).mean()
        model.zero_grad()
        loss.backward()
        opt.step()
    float_preds = np.asarray(model(X).tolist(), np.float32)
    qmodel = nn.Sequential(QLinear(model.layers[0]), nn.ReLU(), QLinear(model.layers[2]))
    quant_preds = np.asarray(qmodel(X).tolist(), np.float32)
    np.savez_compressed(
        os.path.join(HERE, "xor_qlinear.npz"),
        w1=to_np(model.layers[0].weight), b1=to_np(model.layers[0].bias),
        w2=to_np(model.layers[2].weight), b2=to_np(model.layers[2].bias),
        x=to_np(X), float_preds=float_preds, quant_preds=quant_preds, final_loss=np.float32(loss.tolist()[0]))
    print("xor_qlinear.npz: quant preds", quant_preds.ravel())


def chunk_cases():
    pairs = [(7, 3), (8, 2), (16384, 8), (10, 4), (3, 5)]
    sizes = [_chunk_sizes(t, n) for t, n in pairs]
    np.savez_compressed(os.path.join(HERE, "chunk_cases.npz"), pairs=np.asarray(pairs, np.int64),
                        lens=np.asarray([len(s) for s in sizes], np.int64),
                        flat=np.asarray([v for s in sizes for v in s], np.int64))
    print("chunk_cases.npz:", sizes)


def layernorm_cases():
    out = {}
    for i, shape in enumerate(inputs.LAYERNORM_SHAPES):
        x, res, gamma, beta = inputs.layernorm_inputs(i)
        d = shape[-1]
        ln = nn.LayerNorm(d)
        ln.weight, ln.bias = from_np(gamma), from_np(beta)
        plain = nn.LayerNorm(d)
        xt = from_np(x)
        total = xt.add(from_np(res))                  # nn.py:476-477 residual add
        y = ln(xt)
        out[f"c{i}__inputs_sha256"] = np.asarray(sha(x) + sha(res) + sha(gamma) + sha(beta))
        out[f"c{i}__y"] = to_np(y)
        out[f"c{i}__y_default"] = to_np(plain(xt))
        out[f"c{i}__sum"] = to_np(total)
        out[f"c{i}__y_sum"] = to_np(ln(total))
        q, s, _ = quantize_symmetric(y)
        out[f"c{i}__q"] = np.asarray(q, np.int8).reshape(shape)
        out[f"c{i}__scale"] = np.float64(s)
    out["count"] = np.int64(len(inputs.LAYERNORM_SHAPES))
    np.savez_compressed(os.path.join(HERE, "layernorm_cases.npz"), **out)
    print("layernorm_cases.npz:", len(inputs.LAYERNORM_SHAPES), "shapes")


def attention_cases():
    """The reference's own MultiHeadAttention.forward (nn.py:410-427) with its
    four projections set to the identity: q, k, v and the merged output pass
    through them unchanged (each projection sum has one non-zero term), so the
    output is the attention core -- scores, scale, mask, softmax, weighted sum
    -- exactly as the reference composes it."""
    out = {}
    for i, (B, Sq, Sk, D, H, kind) in enumerate(inputs.ATTENTION_CASES):
        q, k, v, mask = inputs.attention_inputs(i)
        mha = nn.MultiHeadAttention(D, H)
        eye = from_np(np.eye(D, dtype=np.float32))
        mha.w_q = mha.w_k = mha.w_v = mha.w_o = eye
        y = mha.forward(from_np(q), from_np(k), from_np(v), mask=from_np(mask) if mask is not None else None)
        out[f"c{i}__inputs_sha256"] = np.asarray(sha(q) + sha(k) + sha(v) + (sha(mask) if mask is not None else ""))
        out[f"c{i}__y"] = to_np(y)
    out["count"] = np.int64(len(inputs.ATTENTION_CASES))
    np.savez_compressed(os.path.join(HERE, "attention_cases.npz"), **out)
    print("attention_cases.npz:", len(inputs.ATTENTION_CASES), "cases")


if __name__ == "__main__":
    quantize_cases()
    percol_cases()
    w8a32_cases()
    mlp_config1()
    xor_qlinear()
    chunk_cases()
    layernorm_cases()
    attention_cases()
