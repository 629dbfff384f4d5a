"""Host-side checks of the index maps behind the half2 N = 256 device
routine (include/thunderfft/detail/thunderfft_impl_device_fft.cuh,
dfft::run256_h; fragment mfft::frag256_h in thunderfft_impl_device_mma.cuh).

The routine's correctness is tested on the GPU (tests/test_header_api.py and
the reference's validation matrix); these tests pin the layout facts its
comments state, so a change to the maps that breaks one fails on CPU.  The
warp-MMA routines' fragment orders (mfft::frag64, frag128 and the TF32
input/output orders) are checked the same way for coverage.  For N = 256:
  * the fragment covers every (signal, element) of the 16-signal tile once;
  * the two-pass split 256 = 16 x 16 reproduces the DFT (float64 restatement
    of the same index arithmetic);
  * the exchange stays inside the (N + pad_h(N)) * batch workspace, writes
    every slot at most once, and neither its row writes nor its column reads
    put two lanes of a warp in one shared-memory bank.
"""
import numpy as np

N, BATCH, THREADS = 256, 16, 128
PAIR = N + N // 16          # N + pad_h(N): one signal pair's plane rows
PLANE = 8 * PAIR            # eight pairs per plane (real, then imaginary)
ROW = 17                    # odd row stride of the exchange


def frag256_h(t, i):
    """(signal, element) held by fragment register i of block thread t."""
    return 2 * (t >> 4) + (i >> 4), (t & 15) + 16 * (i & 15)


# Every other fragment order of the warp-MMA routines, restated from
# thunderfft_impl_device_mma.cuh: (N, batch, threads, map(t, i) -> (j, n)).
OTHER_ORDERS = {
    "frag64 (half2 N=64 in/out, float2 N=64 in)": (64, 16, 32, lambda t, i: (
        ((t & 31) >> 2) + 8 * (i >> 4), 16 * ((t & 31) & 3) + (i & 15))),
    "frag64_tf32_out": (64, 16, 32, lambda t, i: (
        ((t & 31) >> 2) + 8 * (i >> 4), ((t & 31) & 3) + 4 * (i & 15))),
    "frag128 (N=128 in)": (128, 8, 32, lambda t, i: (
        (t & 31) >> 2, 16 * ((t & 31) & 3) + (i & 15) + 64 * (i >> 4))),
    "frag128_tf32_out": (128, 8, 32, lambda t, i: (
        (t & 31) >> 2, 8 * (i & 15) + 4 * (i >> 4) + ((t & 31) & 3))),
    "frag256_tf32_in": (256, 16, 128, lambda t, i: (
        ((t & 31) >> 2) + 8 * (i >> 4), 16 * (t >> 5) + (i & 15) + 64 * ((t & 31) & 3))),
    "frag256_tf32_out": (256, 16, 128, lambda t, i: (
        ((t & 31) >> 2) + 8 * (i >> 4), 16 * (i & 15) + 4 * ((t & 31) & 3) + (t >> 5))),
}


def test_other_fragment_orders_cover_tile_once():
    for name, (n, batch, threads, f) in OTHER_ORDERS.items():
        seen = np.zeros((batch, n), dtype=np.int64)
        for t in range(threads):
            for i in range(n * batch // threads):
                j, e = f(t, i)
                seen[j, e] += 1
        assert (seen == 1).all(), name


def test_fragment_covers_tile_once():
    seen = np.zeros((BATCH, N), dtype=np.int64)
    for t in range(THREADS):
        for i in range(32):
            j, n = frag256_h(t, i)
            seen[j, n] += 1
    assert (seen == 1).all()


def run256_reference(x, forward=True):
    """The routine's arithmetic in float64 on one (signals, 256) array:
    thread q's pass 1 over elements q + 16 r, the W256^(q k1) twiddle, then
    thread k1's pass 2 over q."""
    sgn = -1.0 if forward else 1.0
    w16 = np.exp(sgn * 2j * np.pi * np.outer(np.arange(16), np.arange(16)) / 16)
    out = np.empty_like(x)
    for j in range(x.shape[0]):
        y = np.empty((16, 16), dtype=complex)                      # y[q][k1]
        for q in range(16):
            y[q] = (w16 @ x[j, q::16]) * np.exp(sgn * 2j * np.pi * q * np.arange(16) / N)
        for k1 in range(16):
            out[j, k1::16] = w16 @ y[:, k1]                        # X[k1 + 16 k2]
    return out


def test_two_pass_split_is_the_dft():
    rng = np.random.default_rng(256)
    x = rng.standard_normal((BATCH, N)) + 1j * rng.standard_normal((BATCH, N))
    np.testing.assert_allclose(run256_reference(x, True), np.fft.fft(x, axis=1), rtol=0, atol=1e-9)
    np.testing.assert_allclose(run256_reference(x, False), np.fft.ifft(x, axis=1) * N, rtol=0, atol=1e-9)


def exchange_write(p, q, k1, plane):
    return plane * PLANE + p * PAIR + ROW * k1 + q


def exchange_read(p, q, qq, plane):
    return plane * PLANE + p * PAIR + ROW * q + qq


def test_exchange_in_bounds_and_bijective():
    written = {}
    for t in range(THREADS):
        p, q = t >> 4, t & 15
        for k1 in range(16):
            for plane in (0, 1):
                a = exchange_write(p, q, k1, plane)
                assert 0 <= a < PAIR * BATCH
                assert a not in written
                written[a] = (p, q, k1, plane)
    for t in range(THREADS):
        p, q = t >> 4, t & 15
        for qq in range(16):
            for plane in (0, 1):
                # thread q of pass 2 (k1 = q) reads what thread qq wrote for k1 = q
                assert written[exchange_read(p, q, qq, plane)] == (p, qq, q, plane)


def test_exchange_bank_conflict_free():
    for warp in range(THREADS // 32):
        lanes = range(32 * warp, 32 * warp + 32)
        for k in range(16):
            wr = {exchange_write(t >> 4, t & 15, k, 0) % 32 for t in lanes}
            rd = {exchange_read(t >> 4, t & 15, k, 0) % 32 for t in lanes}
            assert len(wr) == 32 and len(rd) == 32
