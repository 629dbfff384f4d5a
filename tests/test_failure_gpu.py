"""Failure detection without a GPU fault: a device-side wait that can never
be satisfied must give up within its bound, surface as a device-timeout
status / RuntimeError on the host, and leave the CUDA context usable."""
import numpy as np
import pytest

import oracle


@pytest.mark.gpu
def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    import torch

    import thunderfft_b200 as tf

    lib = tf.load_library()
    st = lib.thff_selftest_wait_timeout(20000, None)  # 20 ms bound
    assert st == tf.THFF_DEVICE_TIMEOUT, lib.thff_last_error()
    assert b"timed out" in lib.thff_last_error()
    # the error word was cleared and the context still works
    x = (np.random.default_rng(0).standard_normal((8, 256)) + 0j).astype(np.complex64)
    y = tf.fft(torch.from_numpy(x).cuda())
    assert oracle.rel_l2(y.cpu().numpy(), oracle.fft(x)) <= 5e-3
    tf.sync_check()


def test_selftest_argument_checks():
    import thunderfft_b200 as tf

    lib = tf.load_library()
    assert lib.thff_selftest_wait_timeout(0, None) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_selftest_wait_timeout(2_000_000, None) == tf.THFF_INVALID_ARGUMENT
