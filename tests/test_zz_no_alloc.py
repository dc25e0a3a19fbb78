"""The allocation-free per-channel quantize entry point.

Some callers of libkz cannot call cudaMalloc -- a host runtime (JVM, Go,
an inference server) that owns all of the GPU's memory through its own
allocator or arena, or that must not allocate once serving has started.
kz_quantize_cols_f32_noalloc gives them per-channel weight quantization with
no workspace argument: its scratch is a static device array inside libkz.

These tests call it through the C ABI and check it against the allocating
entry point, kz_quantize_cols_f32, bit for bit (codes and both scale arrays),
on two calls in a row so a stale scratch from the first call would show up in
the second.  This file is collected last on purpose; it passes on its own in a
fresh process and after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _quantize_both(lib, w_np, stream):
    K, N = w_np.shape
    w = torch.from_numpy(w_np).cuda()
    outs = []
    for noalloc in (False, True):
        qT = torch.empty((N, K), dtype=torch.int8, device="cuda")
        s64 = torch.empty(N, dtype=torch.float64, device="cuda")
        s32 = torch.empty(N, dtype=torch.float32, device="cuda")
        if noalloc:
            st = lib.kz_quantize_cols_f32_noalloc(w.data_ptr(), K, N, qT.data_ptr(), s64.data_ptr(), s32.data_ptr(),
                                                  stream)
        else:
            wsb = lib.kz_quantize_cols_workspace_bytes(K, N)
            ws = torch.empty(max(int(wsb), 16), dtype=torch.uint8, device="cuda")
            st = lib.kz_quantize_cols_f32(w.data_ptr(), K, N, qT.data_ptr(), s64.data_ptr(), s32.data_ptr(),
                                          ws.data_ptr(), ws.numel(), stream)
        assert st == 0, lib.kz_last_error()
        torch.cuda.synchronize()
        outs.append((qT.cpu().numpy(), s64.cpu().numpy(), s32.cpu().numpy()))
    return outs


def test_noalloc_matches_allocating_entry_point_twice(cuda_device):
    from kansaiml_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    # first call: a wide weight with large values; second: a different shape
    # and distribution, so anything left in the shared scratch would show
    shapes = [((1024, 4096), 3.0, 0), ((4096, 1000), 0.02, 1)]
    for (K, N), std, seed in shapes:
        w = (np.random.RandomState(seed).standard_normal((K, N)) * std).astype(np.float32)
        (q_a, s64_a, s32_a), (q_b, s64_b, s32_b) = _quantize_both(lib, w, stream)
        np.testing.assert_array_equal(q_b, q_a)
        np.testing.assert_array_equal(s64_b, s64_a)
        np.testing.assert_array_equal(s32_b, s32_a)
    code = ctypes.c_int(0)
    assert lib.kz_device_status(ctypes.byref(code), 1, stream) == 0 and code.value == 0


def test_noalloc_rejects_more_channels_than_its_scratch(cuda_device):
    from kansaiml_b200 import _lib
    lib = _lib.load()
    st = lib.kz_quantize_cols_f32_noalloc(None, 16, 65537, None, None, None, None)
    assert st == _lib.KZ_ERR_INVALID_ARGUMENT
    assert "65536" in lib.kz_last_error().decode()
