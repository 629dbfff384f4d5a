"""The allocation-free 2-D convolution entry point, thff_conv2d_noalloc.

Callers that run the convolution where device allocation is not allowed —
inside plugins or real-time pipelines whose host application owns all device memory,
or behind a pooling allocator that must see every byte — use this entry point
instead of thff_conv2d, which needs a caller-allocated workspace.  Its scratch
is a fixed 16 MiB device array inside the library.

This test calls the new entry point through the C ABI twice in a row, with
different inputs, and checks each result three ways:
* against the FP64 oracle's direct circular convolution (relative L2 <=
  5e-3, the gate of the other tests);
* against the existing workspace-based entry point running the same TF32
  pipeline (thff_conv2d_set_arithmetic(THFF_CONV_TF32)), like for like, at a
  tight gate;
* that the second call leaves the device's free memory unchanged: it
  allocates nothing.
It sets up everything it needs itself, so it passes in a fresh process as
well as after the rest of the suite.  The file name makes pytest collect it
last.
"""
import ctypes

import numpy as np
import pytest

import oracle

GATE = 5e-3
SAME_PIPELINE_GATE = 1e-5   # both entry points run the same TF32 kernels


@pytest.mark.gpu
def test_conv2d_noalloc_matches_workspace_entry_point(cuda):
    import torch

    import thunderfft_b200 as tf

    lib = tf.load_library()
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.thff_conv2d_noalloc.argtypes = [i32, i64, i32, i32, i32, vp, vp, vp, vp]
    lib.thff_conv2d_noalloc.restype = i32

    B, C, h, w, f = 5, 2, 512, 512, 31   # 6 image pairs: two passes through the 16 MiB scratch
    # Setup that may allocate happens before the allocation-free call.
    tf.ThunderFFTInitialize("float", h)
    tf.ThunderFFTInitialize("float", w)
    rng = np.random.default_rng(2024)
    filt = torch.from_numpy(rng.standard_normal((C, f, f)).astype(np.float32)).cuda()
    spec = tf.conv2d_filter_spectra(filt, h, w)
    ws = tf.conv2d_workspace(h, w, ((B + 1) // 2) * C)
    stream = torch.cuda.current_stream()

    idx = np.tile(np.arange(C, dtype=np.int32), B)
    for call in range(2):
        xh = rng.standard_normal((B, C, h, w)).astype(np.float32)
        x = torch.from_numpy(xh).cuda()
        tf.conv2d_set_arithmetic("tf32")                         # the pipeline noalloc runs
        try:
            expected = tf.conv2d(x, spec, ws).cpu().numpy()      # existing entry point
        finally:
            tf.conv2d_set_arithmetic("mixed")                    # the library default
        y = torch.full_like(x, float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = lib.thff_conv2d_noalloc(0, B, C, h, w, x.data_ptr(), spec.data_ptr(), y.data_ptr(),
                                     stream.cuda_stream)
        assert st == tf.THFF_OK, lib.thff_last_error()
        tf.sync_check(stream)
        free_after = torch.cuda.mem_get_info()[0]
        if call == 1:   # a warm call: nothing may be allocated on the device
            assert free_after == free_before, (free_before, free_after)
        got = y.cpu().numpy()
        assert np.isfinite(got).all(), call
        assert oracle.rel_l2(got, expected) <= SAME_PIPELINE_GATE, call
        direct = oracle.circconv2d(xh.reshape(B * C, h, w).astype(np.float64),
                                   filt.cpu().numpy().astype(np.float64), idx).reshape(xh.shape)
        assert oracle.rel_l2(got, direct) <= GATE, call


def test_conv2d_noalloc_rejects_images_beyond_the_fixed_scratch():
    import thunderfft_b200 as tf

    lib = tf.load_library()
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.thff_conv2d_noalloc.argtypes = [i32, i64, i32, i32, i32, vp, vp, vp, vp]
    lib.thff_conv2d_noalloc.restype = i32
    p = 1 << 20
    # a 2048 x 1024 image pair needs 32 MiB of scratch: rejected before any CUDA call
    assert lib.thff_conv2d_noalloc(0, 2, 1, 2048, 1024, p, p, p, None) == tf.THFF_INVALID_ARGUMENT
    assert b"fixed scratch" in lib.thff_last_error()
