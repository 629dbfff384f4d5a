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


def test_inject_hook_argument_checks():
    import thunderfft_b200 as tf

    lib = tf.load_library()
    assert lib.thff_test_inject_cuda_error(-1, 0) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_test_inject_cuda_error(2, -1) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_test_inject_cuda_error(0, 0) == tf.THFF_OK


@pytest.mark.gpu
@pytest.mark.parametrize("skip", [0, 1, 2])
def test_injected_cuda_failure_surfaces_and_library_recovers(cuda, skip):
    """Host-side fault injection: the (skip+1)-th CUDA status the library
    checks reads as cudaErrorMemoryAllocation (2).  The Python mirror must
    raise RuntimeError with the reference's message shape, only on the
    calling thread, and the next call must work."""
    import threading

    import torch

    import thunderfft_b200 as tf

    lib = tf.load_library()
    x = (np.random.default_rng(1).standard_normal((16, 1024)) + 0j).astype(np.complex64)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    tf.ThunderFFT_global("float", 1024, True, xd, yd, 16)
    # armed on another thread: this thread is unaffected
    t = threading.Thread(target=lambda: lib.thff_test_inject_cuda_error(2, 0))
    t.start()
    t.join()
    tf.ThunderFFT_global("float", 1024, True, xd, yd, 16)
    assert lib.thff_test_inject_cuda_error(2, skip) == tf.THFF_OK
    with pytest.raises(RuntimeError) as ei:
        tf.ThunderFFT_global("float", 1024, True, xd, yd, 16)
    lib.thff_test_inject_cuda_error(0, 0)
    msg = str(ei.value)
    assert msg.startswith("[ThunderFFT] ") and msg.endswith(": out of memory"), msg
    yd.zero_()
    tf.ThunderFFT_global("float", 1024, True, xd, yd, 16)
    assert oracle.rel_l2(yd.cpu().numpy(), oracle.fft(x)) <= 5e-3


@pytest.mark.gpu
def test_timeout_on_one_stream_leaves_other_streams_alone(cuda):
    """Each stream has its own device error word.  While a bounded wait runs
    out on stream A (3 ms bound), a queue of C2C launches runs on stream B
    across that moment.  B's kernels must neither abort nor see A's error:
    B's output matches the oracle and B's sync reports OK, while A alone
    reports THFF_DEVICE_TIMEOUT.  The wait is bounded, so no GPU hangs."""
    import threading
    import time

    import torch

    import thunderfft_b200 as tf

    lib = tf.load_library()
    n, batch = 1024, 65536
    rng = np.random.default_rng(7)
    x = (rng.uniform(-1, 1, (batch, n)) + 1j * rng.uniform(-1, 1, (batch, n))).astype(np.complex64)
    tf.ThunderFFTInitialize("float", n)
    sa, sb = torch.cuda.Stream(), torch.cuda.Stream()
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    torch.cuda.synchronize()
    status = {}

    def stall_a():
        status["a"] = lib.thff_selftest_wait_timeout(3000, ctypes_stream(sa))
        status["a_msg"] = lib.thff_last_error()

    t = threading.Thread(target=stall_a)
    t.start()
    time.sleep(0.0005)
    for _ in range(60):   # about 10 ms of transforms, straddling A's timeout
        tf.c2c_async("float", n, True, xd, yd, batch, stream=sb)
    tf.sync_check(sb)     # raises if B saw an error
    t.join()
    assert status["a"] == tf.THFF_DEVICE_TIMEOUT, status
    assert b"timed out" in status["a_msg"]
    sel = rng.choice(batch, 256, replace=False)
    assert oracle.rel_l2(yd.cpu().numpy()[sel], oracle.fft(x[sel])) <= 5e-3
    tf.sync_check(sa)     # A's word was cleared by its own read


def ctypes_stream(stream):
    return stream.cuda_stream
