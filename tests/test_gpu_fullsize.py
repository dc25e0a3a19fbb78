"""GPU parity at the BASELINE sizes of configs 4 and 5 (configs 1-3 run at
full size in the other files).

Config 4: square int8 GEMMs M = N = K in {2048, 4096, 8192, 16384}, operands
~ U{-127..127}, per-row x per-column scales ~ U[1e-3, 1e-2].  The int32
accumulators of 64 sampled rows (every row-tile band and both ends) must equal
the oracle's integer matmul, and the fused fp32 epilogue of the same rows the
oracle's epilogue, bit for bit.

Config 5 on one GPU: 4 int8 Linear layers [16384 -> 16384], weights
~ N(0, 0.01) per output channel, activations [8192, 16384] ~ N(0, 1) per
tensor.  The stack's own forward is recorded layer by layer: each layer's
input codes and scale must equal the oracle's per-tensor quantize of the fp32
tensor that fed it (the input, or the previous layer's device output), its
weight codes and scales the oracle's per-column quantize (sampled columns),
and sampled rows of its fp32 output the oracle's int8 GEMM + epilogue.
"""
import numpy as np
import pytest
import torch

from oracle import cpu as ocpu

pytestmark = pytest.mark.gpu


def _sample_rows(n, count, seed):
    rows = np.random.RandomState(seed).choice(n, count - 2, replace=False)
    return np.sort(np.concatenate([[0, n - 1], rows]))


@pytest.mark.parametrize("n", [2048, 4096, 8192, 16384])
def test_config4_square_gemm_sampled_rows(cuda_device, n):
    from kansaiml_b200 import quantize as kq
    g = torch.Generator(device="cuda")
    g.manual_seed(400 + n)
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
    rs = torch.rand(n, device="cuda", generator=g) * 9e-3 + 1e-3
    cs = torch.rand(n, device="cuda", generator=g) * 9e-3 + 1e-3
    acc = torch.empty((n, n), dtype=torch.int32, device="cuda")
    kq.gemm_i8_device(a, b, out_i32=acc)
    y, _ = kq.gemm_i8_device(a, b, row_scale=rs, col_scale=cs)
    torch.cuda.synchronize()
    assert kq.device_status() == 0
    rows = _sample_rows(n, 64, n)
    idx = torch.from_numpy(rows).cuda()
    a_rows, b_host = a[idx].cpu().numpy(), b.cpu().numpy()
    acc_o = ocpu.gemm_i8(a_rows, b_host)
    np.testing.assert_array_equal(acc[idx].cpu().numpy(), acc_o)
    y_o = ocpu.epilogue(acc_o, rs[idx].cpu().numpy(), cs.cpu().numpy())
    assert y[idx].cpu().numpy().tobytes() == y_o.tobytes()
    del a, b, acc, y
    torch.cuda.empty_cache()


STACK_M, STACK_D, STACK_L = 8192, 16384, 4


def test_config5_stack_full_size_layerwise(cuda_device, monkeypatch):
    import kansaiml_b200.distributed as kd

    def weight(l):
        g = torch.Generator(device="cuda")
        g.manual_seed(5000 + l)
        return torch.randn((STACK_D, STACK_D), generator=g, device="cuda") * 0.01

    stack = kd.ShardedQLinearStack([weight] * STACK_L)
    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    x = torch.randn((STACK_M, STACK_D), generator=g, device="cuda")
    calls = []
    inner = kd.gemm_i8_device

    def recording(a, b, row_scale=None, col_scale=None, **kw):
        out = inner(a, b, row_scale=row_scale, col_scale=col_scale, **kw)
        calls.append((a, row_scale, b, col_scale, out[0]))
        return out

    monkeypatch.setattr(kd, "gemm_i8_device", recording)
    y_last = stack(x).data
    torch.cuda.synchronize()
    assert len(calls) == STACK_L
    assert torch.equal(calls[-1][4], y_last)
    rows = _sample_rows(STACK_M, 32, 5)
    cols = np.sort(np.random.RandomState(6).choice(STACK_D, 48, replace=False))
    ridx, cidx = torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()
    feed = x
    for l, (a, rs, wq, ws, y) in enumerate(calls):
        # the layer's input codes and scale: the oracle's quantize of what fed it
        a_o, s_o = ocpu.quantize_tensor(feed.cpu().numpy())
        assert float(rs.item()) == np.float32(s_o), l
        np.testing.assert_array_equal(a.reshape(STACK_M, STACK_D).cpu().numpy(), a_o, err_msg=f"layer {l}")
        # weight codes and scales on sampled channels (a column's quantize is its own)
        wq_o, ws_o = ocpu.quantize_cols(weight(l)[:, cidx].cpu().numpy())
        np.testing.assert_array_equal(wq[cidx].cpu().numpy(), wq_o, err_msg=f"layer {l}")
        np.testing.assert_array_equal(ws[cidx].cpu().numpy(), ws_o.astype(np.float32))
        # sampled output rows: int8 GEMM + epilogue
        acc_o = ocpu.gemm_i8(a_o[rows], wq.cpu().numpy())
        y_o = ocpu.epilogue(acc_o, s_o, ws.cpu().numpy())
        assert y[ridx].cpu().numpy().tobytes() == y_o.tobytes(), l
        feed = y
    from kansaiml_b200.quantize import device_status
    assert device_status() == 0
