"""The allocation-free per-channel quantize entry point.

Some callers of libkz cannot call cudaMalloc -- a host runtime (JVM, Go,
an inference server) that owns all of the GPU's memory through its own
allocator or arena, or that must not allocate once serving has started.
kz_quantize_cols_f32_noalloc gives them per-channel weight quantization with
no workspace argument: its scratch is a static device array inside libkz.

These tests call it through the C ABI and check it against the allocating
entry point, kz_quantize_cols_f32, and against the oracle's per-column
quantize, bit for bit (codes and both scale arrays), on calls in a row so a
stale scratch from an earlier call would show up in a later one: wide and
narrow weights, up to 60000 channels against its 65536-word scratch, a
ragged shape (the unvectorised kernels), and K == 0,
where the scratch is cleared instead of written.  This file is collected
last on purpose; it passes on its own in a fresh process and after the rest
of the suite.
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
    from oracle import cpu as ocpu
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    # in a row: a wide weight with large values; a different shape and
    # distribution; 8192 and 60000 channels (the row split count times the
    # channels must fit the 65536-word scratch); a ragged 1000-channel weight
    # (the unvectorised kernels); so anything left in the shared scratch by
    # one call would show in the next
    shapes = [((1024, 4096), 3.0, 0), ((4096, 1024), 0.02, 1), ((4096, 8192), 0.5, 2), ((512, 60000), 1.0, 3),
              ((300, 1000), 0.02, 4)]
    for (K, N), std, seed in shapes:
        w = (np.random.RandomState(seed).standard_normal((K, N)) * std).astype(np.float32)
        (q_a, s64_a, s32_a), (q_b, s64_b, s32_b) = _quantize_both(lib, w, stream)
        np.testing.assert_array_equal(q_b, q_a)
        np.testing.assert_array_equal(s64_b, s64_a)
        np.testing.assert_array_equal(s32_b, s32_a)
        if K * N <= 4096 * 4096:
            q_o, s_o = ocpu.quantize_cols(w)
            np.testing.assert_array_equal(q_b, q_o)
            np.testing.assert_array_equal(s64_b, s_o)
            np.testing.assert_array_equal(s32_b, s_o.astype(np.float32))
    code = ctypes.c_int(0)
    assert lib.kz_device_status(ctypes.byref(code), 1, stream) == 0 and code.value == 0


def test_noalloc_k0_clears_the_scratch(cuda_device):
    """K == 0 after a call that left maxima in the scratch: every channel's
    absmax is 0, so every scale is the reference's 1.0 (quantize.py:68), as
    the allocating entry point gives."""
    from kansaiml_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    w = (np.random.RandomState(5).standard_normal((256, 512)) * 4).astype(np.float32)
    _quantize_both(lib, w, stream)
    (_, s64_a, s32_a), (_, s64_b, s32_b) = _quantize_both(lib, np.zeros((0, 512), np.float32), stream)
    np.testing.assert_array_equal(s64_b, s64_a)
    np.testing.assert_array_equal(s32_b, s32_a)
    assert np.all(s64_b == 1.0)


def test_noalloc_rejects_more_channels_than_its_scratch(cuda_device):
    from kansaiml_b200 import _lib
    lib = _lib.load()
    st = lib.kz_quantize_cols_f32_noalloc(None, 16, 65537, None, None, None, None)
    assert st == _lib.KZ_ERR_INVALID_ARGUMENT
    assert "65536" in lib.kz_last_error().decode()
