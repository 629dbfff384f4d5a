"""Tiled (overlap-save) 1-D convolution — the reference's other conv1d sample
(sample/conv1d/main.cu: 64-point windows advancing by 65 - f, FFT -> x filter
spectrum -> inverse FFT, first 65 - f outputs kept) — against the FP64 valid
correlation of the oracle (main.cu:157-172), relative L2 <= 5e-3."""
import numpy as np
import pytest

import oracle

GATE = 5e-3


def run(torch, tf, x, g, T):
    dg = torch.from_numpy(g.astype(np.complex64)).cuda()
    op = tf.conv1d_tiled_operator(dg, T)
    if T == "float":
        dx = torch.from_numpy(x.astype(np.complex64)).cuda()
        y = tf.conv1d_tiled(dx, op)
        return y.cpu().numpy().astype(np.complex128)
    xs = np.stack([x.real, x.imag], -1).astype(np.float16)
    y = tf.conv1d_tiled(torch.from_numpy(xs).cuda(), op).float().cpu().numpy()
    return y[..., 0] + 1j * y[..., 1]


@pytest.mark.gpu
@pytest.mark.parametrize("T", ["float", "half"])
@pytest.mark.parametrize("L,f,batch", [(1 << 16, 9, 1), (64, 64, 1), (65, 1, 2), (1000, 33, 3),
                                       (4097, 5, 2), (70001, 17, 1), (200, 64, 130), (1 << 15, 3, 2)])
def test_tiled_conv1d_matches_valid_correlation(cuda, T, L, f, batch):
    import torch

    import thunderfft_b200 as tf

    rng = np.random.default_rng(L + f + batch)
    x = rng.uniform(0, 1, (batch, L)) + 1j * rng.uniform(0, 1, (batch, L))   # the sample's inputs: rand() in [0, 1]
    g = rng.uniform(0, 1, f) + 1j * rng.uniform(0, 1, f)
    if T == "half":
        x = x.astype(np.complex64)
        x = (x.real.astype(np.float16).astype(np.float64) + 1j * x.imag.astype(np.float16).astype(np.float64))
    y = run(torch, tf, x, g, T)
    ref = oracle.corr1d_valid(x, g)
    assert y.shape == ref.shape
    assert np.isfinite(y).all()
    e = oracle.rel_l2(y, ref)
    assert e <= GATE, (T, L, f, batch, e)


def test_tiled_conv1d_argument_contract():
    import thunderfft_b200 as tf

    lib = tf.load_library()
    p = 1 << 20
    assert lib.thff_conv1d_tiled_operator_bytes(0) == 128 * 128 * 4
    assert lib.thff_conv1d_tiled_operator_bytes(1) == 128 * 128 * 2
    assert lib.thff_conv1d_tiled_operator_bytes(5) == -1
    assert lib.thff_conv1d_tiled_operator(0, p, 65, p, None) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_conv1d_tiled_operator(0, p, 0, p, None) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_conv1d_tiled_async(0, 8, 9, p, p, p, 1, None) == tf.THFF_INVALID_ARGUMENT   # input < filter
    assert lib.thff_conv1d_tiled_async(0, 64, 9, p, p, p, -1, None) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_conv1d_tiled_async(0, 64, 9, 0, 0, 0, 0, None) == tf.THFF_OK              # batch 0: no-op
    assert lib.thff_conv1d_tiled_async(0, 64, 9, p + 4, p, p, 1, None) == tf.THFF_INVALID_ARGUMENT  # misaligned x
