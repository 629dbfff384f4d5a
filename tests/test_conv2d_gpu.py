"""2-D FFT convolution (reference sample
sample/conv2d/thunder.cu + main.cu) against the oracle's FP64 direct 2-D
circular convolution, relative L2 <= 5e-3."""
import numpy as np
import pytest

import oracle

GATE = 5e-3


@pytest.fixture(params=["tf32", "mixed"])
def arith(request):
    """Both arithmetics of the 2-D convolution; restores the default."""
    import thunderfft_b200 as tf

    tf.conv2d_set_arithmetic(request.param)
    yield request.param
    tf.conv2d_set_arithmetic(DEFAULT_ARITH)


DEFAULT_ARITH = "mixed"


def run(torch, tf, x, filt, pairs_per_pass=None):
    B, C, h, w = x.shape
    dx = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    df = torch.from_numpy(np.ascontiguousarray(filt, dtype=np.float32)).cuda()
    spec = tf.conv2d_filter_spectra(df, h, w)
    pairs = pairs_per_pass or ((B + 1) // 2) * C
    ws = tf.conv2d_workspace(h, w, pairs)
    return tf.conv2d(dx, spec, ws).cpu().numpy()


def reference(x, filt):
    B, C, h, w = x.shape
    idx = np.tile(np.arange(C, dtype=np.int32), B)
    return oracle.circconv2d(x.reshape(B * C, h, w).astype(np.float64), filt.astype(np.float64), idx).reshape(x.shape)


@pytest.mark.gpu
@pytest.mark.parametrize("B,C,h,w,f,pairs", [(2, 1, 128, 128, 3, None), (3, 2, 128, 256, 5, None),
                                             (1, 3, 256, 128, 31, 1), (4, 2, 512, 512, 31, 3),
                                             (5, 1, 256, 256, 1, 2),
                                             # every row length (pair-planar loads: NA = 16 with
                                             # G1 = 4, 2, 1; NA = 32; NA = 64) and column length
                                             # (transposed loads with 8, 4, 2 signals per group;
                                             # 4096 takes the transposing-store path)
                                             (3, 1, 1024, 2048, 5, None), (2, 2, 2048, 1024, 3, 1),
                                             (1, 1, 128, 4096, 3, None), (2, 1, 4096, 128, 3, None)])
def test_conv2d_matches_direct_circular_convolution(cuda, arith, B, C, h, w, f, pairs):
    import torch

    import thunderfft_b200 as tf

    rng = np.random.default_rng(B * 100 + C * 10 + f)
    x = rng.standard_normal((B, C, h, w)).astype(np.float32)
    filt = rng.standard_normal((C, f, f)).astype(np.float32)
    y = run(torch, tf, x, filt, pairs)
    assert np.isfinite(y).all()
    e = oracle.rel_l2(y, reference(x, filt))
    assert e <= GATE, e


@pytest.mark.gpu
def test_config5_full_size(cuda, arith):
    """64 x 32 fp32 N(0,1) 512x512 images, 32 N(0,1) 31x31
    filters (one per channel), circular convolution; sampled images checked
    against the FP64 direct convolution."""
    import torch

    import thunderfft_b200 as tf

    B, C, h, w, f = 64, 32, 512, 512, 31
    g = torch.Generator(device="cuda")
    g.manual_seed(55)
    x = torch.randn(B, C, h, w, device="cuda", generator=g)
    filt = torch.randn(C, f, f, device="cuda", generator=g)
    spec = tf.conv2d_filter_spectra(filt, h, w)
    ws = tf.conv2d_workspace(h, w, 64)
    y = tf.conv2d(x, spec, ws)
    assert torch.isfinite(y).all()
    for b, c in ((0, 0), (1, 0), (63, 31), (30, 17)):
        xs = x[b, c].cpu().double().numpy()[None]
        ref = oracle.circconv2d(xs, filt[c].cpu().double().numpy()[None], np.zeros(1, np.int32))
        assert oracle.rel_l2(y[b, c].cpu().numpy()[None], ref) <= GATE, (b, c)


@pytest.mark.gpu
@pytest.mark.parametrize(
    "xscale,fscale",
    [(1e-7, 1.0), (3e4, 1.0), (1.0, 1e-6), (1.0, 5e3), (2e4, 2e3), (1e-36, 1.0), (1e15, 1e15)],
)
def test_conv2d_range_scaling(cuda, arith, xscale, fscale):
    """Images and filters far from unit scale, plus one spike per image: the
    mixed arithmetic's power-of-two scales keep every half2 intermediate in
    range, so the result meets the same gate as for unit-scale data.  The
    (1e15, 1e15) case takes the last pass's unscale past 2^120 (applied as
    two exact factors); (1e-36, 1) puts the image scale above 2^100."""
    import torch

    import thunderfft_b200 as tf

    B, C, h, w, f = 3, 2, 256, 512, 9
    rng = np.random.default_rng(int(np.log10(xscale) * 10 + np.log10(fscale) * 100) & 0xffff)
    x = (rng.standard_normal((B, C, h, w)) * xscale).astype(np.float32)
    x[:, :, 7, 11] *= 50.0
    filt = (rng.standard_normal((C, f, f)) * fscale).astype(np.float32)
    y = run(torch, tf, x, filt)
    assert np.isfinite(y).all()
    e = oracle.rel_l2(y, reference(x, filt))
    assert e <= GATE, e


def test_conv2d_argument_contract():
    import thunderfft_b200 as tf

    lib = tf.load_library()
    ok_ptr = 1 << 20
    assert lib.thff_conv2d_workspace_bytes(0, 512, 512, 1) == 2 * 512 * 512 * 8
    assert lib.thff_conv2d_workspace_bytes(0, 500, 512, 1) == -1
    assert lib.thff_conv2d_async(0, 2, 1, 512, 300, ok_ptr, ok_ptr, ok_ptr, ok_ptr, 1 << 30, None) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_conv2d_async(0, 2, 1, 512, 512, ok_ptr, ok_ptr, ok_ptr, ok_ptr, 16, None) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_conv2d_async(0, 2, 0, 512, 512, ok_ptr, ok_ptr, ok_ptr, ok_ptr, 1 << 30, None) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_conv2d_async(1, 2, 1, 512, 512, ok_ptr, ok_ptr, ok_ptr, ok_ptr, 1 << 30, None) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_conv2d_async(0, 0, 1, 512, 512, 0, 0, 0, 0, 0, None) == tf.THFF_OK
