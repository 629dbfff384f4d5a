"""GPU parity of the batched C2C FFT against the FP64 oracle.

Mirrors the reference's correctness matrix (sample/validation/fft_validation.cu:
check_size/check_case, :194-311): 7 lengths x {float/TF32, half/FP16} x
{forward, inverse} x the four seeded input kinds, the reference's partial
batches {1, BPB-1, BPB+1} plus this library's tile boundaries, relative L2
<= 5e-3 against an FP64 transform of the values actually represented by the
input dtype, finite outputs, and an output guard tail that must stay intact.
Full BASELINE sizes are checked through size-independent properties
(round trip / N, linearity) plus sampled oracle comparisons.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

SIZES = (64, 128, 256, 512, 1024, 2048, 4096)
REL_L2 = 5e-3          # the reference's gate (fft_validation.cu:26)
GUARD = 16             # sentinel elements after the output (fft_validation.cu:200-210)
# signals per CTA tile of this library's kernels (tile-boundary partial batches)
TILE = {"float": {64: 128, 128: 32, 256: 16, 512: 8, 1024: 4, 2048: 2, 4096: 1},
        "half": {64: 128, 128: 32, 256: 16, 512: 8, 1024: 4, 2048: 2, 4096: 1}}
BPB = {64: 16, 128: 8, 256: 16, 512: 2, 1024: 1, 2048: 1, 4096: 1}
GOLD = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "golden_fft.npz")


def to_dev(x: np.ndarray, T: str, torch, extra: int = 0):
    """Upload complex x (batch, n) as float2 or half2 storage; returns
    (device tensor, represented complex128 values)."""
    if T == "float":
        xs = np.ascontiguousarray(x.astype(np.complex64))
        rep = xs.astype(np.complex128)
        flat = np.concatenate([xs.reshape(-1), np.zeros(extra, np.complex64)])
        return torch.from_numpy(flat).cuda(), rep
    xr = np.stack([x.real, x.imag], -1).astype(np.float16)
    rep = xr[..., 0].astype(np.float64) + 1j * xr[..., 1].astype(np.float64)
    flat = np.concatenate([xr.reshape(-1), np.zeros(2 * extra, np.float16)])
    return torch.from_numpy(flat).cuda(), rep


def from_dev(t, T: str, count: int) -> np.ndarray:
    a = t.cpu().numpy()
    if T == "float":
        return a[:count].astype(np.complex128)
    return a[: 2 * count : 2].astype(np.float64) + 1j * a[1 : 2 * count : 2].astype(np.float64)


def run(tf, torch, x: np.ndarray, T: str, forward: bool):
    """Transform through the public wrapper with an output guard tail.
    Returns (output complex128 (batch, n), guard intact?)."""
    batch, n = x.shape
    din, rep = to_dev(x, T, torch)
    if T == "float":
        out = torch.full((batch * n + GUARD,), complex(float("nan"), 0), dtype=torch.complex64, device="cuda")
        out[batch * n:] = complex(-271.0, 137.0)
    else:
        out = torch.full((2 * (batch * n + GUARD),), float("nan"), dtype=torch.float16, device="cuda")
        out[2 * batch * n::2] = -271.0
        out[2 * batch * n + 1::2] = 137.0
    tf.ThunderFFT_global(T, n, forward, din, out, batch)
    y = from_dev(out, T, batch * n).reshape(batch, n)
    tail = from_dev(out[batch * n:] if T == "float" else out[2 * batch * n:], T, GUARD)
    guard_ok = bool(np.all(tail == complex(-271.0, 137.0)))
    return y, rep, guard_ok


class _DevicePtr:
    """Wrap a raw device pointer for torch.as_tensor (read-only view)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3}


@pytest.fixture(scope="module")
def tfm(cuda):
    import thunderfft_b200 as tf

    return tf


@pytest.mark.parametrize("T", ["float", "half"])
@pytest.mark.parametrize("n", SIZES)
def test_reference_validation_matrix(tfm, cuda, T, n):
    import torch

    tf = tfm
    tf.ThunderFFTInitialize(T, n)
    tile = TILE[T][n]
    tails = sorted({1, BPB[n] - 1, BPB[n] + 1, tile - 1, tile + 1, 2 * tile + 3} - {0})
    worst = 0.0
    for kind in range(4):
        for batch in [64] + tails:
            x = oracle.make_validation_input(n, batch, kind)
            for fwd in (True, False):
                y, rep, guard_ok = run(tf, torch, x, T, fwd)
                assert np.isfinite(y).all(), (T, n, kind, batch, fwd)
                assert guard_ok, f"output guard overwritten {T} n={n} batch={batch}"
                e = oracle.rel_l2(y, oracle.fft(rep, fwd))
                worst = max(worst, e)
                assert e <= REL_L2, f"{T} n={n} kind={kind} batch={batch} fwd={fwd}: rel-L2 {e:.3e}"
    print(f"{T} N={n}: worst rel-L2 {worst:.3e}")
    tf.ThunderFFTFinalize(T)


@pytest.mark.parametrize("T", ["float", "half"])
def test_golden_fixtures(tfm, cuda, T):
    import torch

    for n in (64, 256, 1024):
        for kind in range(4):
            x = GOLD[f"val_n{n}_k{kind}_x"]
            ref = GOLD[f"val_n{n}_k{kind}_fwd" if T == "float" else f"val_n{n}_k{kind}_fwd_half"]
            y, _, ok = run(tfm, torch, x, T, True)
            assert ok and oracle.rel_l2(y, ref) <= REL_L2


def test_config1_n64_batch16_vs_dft(tfm, cuda):
    """BASELINE config 1 against the FP64 DFT definition and the fixture."""
    import torch

    x = GOLD["cfg1_x"]
    y, rep, ok = run(tfm, torch, x, "float", True)
    assert ok
    assert oracle.rel_l2(y, oracle.dft(rep, True)) <= REL_L2
    assert oracle.rel_l2(y, GOLD["cfg1_fwd"]) <= REL_L2
    yi, _, _ = run(tfm, torch, x, "float", False)
    assert oracle.rel_l2(yi, GOLD["cfg1_inv"]) <= REL_L2


def test_quickstart_fft1d_gate(tfm, cuda):
    """sample/fft1d: float N=64 forward, rel L2 and rel Linf <= 5e-3."""
    import torch

    x = GOLD["fft1d_x"]
    y, _, _ = run(tfm, torch, x, "float", True)
    assert oracle.rel_l2(y, GOLD["fft1d_fwd"]) <= 5e-3
    assert oracle.rel_linf(y, GOLD["fft1d_fwd"]) <= 5e-3


def test_config2_full_size_round_trip(tfm, cuda):
    """N=1024, batch 65536 (512 MiB per buffer), TF32
    forward then unnormalized inverse; round trip / N must reproduce the
    input, and sampled signals must match the oracle."""
    import torch

    tf = tfm
    n, batch = 1024, 65536
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    x = torch.complex(torch.rand(batch, n, device="cuda", generator=g) * 2 - 1,
                      torch.rand(batch, n, device="cuda", generator=g) * 2 - 1)
    y = torch.empty_like(x)
    z = torch.empty_like(x)
    tf.ThunderFFTInitialize("float", n)
    tf.ThunderFFT_global("float", n, True, x, y, batch)
    tf.ThunderFFT_global("float", n, False, y, z, batch)
    num = (z / n - x).abs().pow(2).sum().item()
    den = x.abs().pow(2).sum().item()
    assert np.sqrt(num / den) <= REL_L2
    assert torch.isfinite(torch.view_as_real(z)).all()
    idx = torch.tensor([0, 1, 4097, 33333, batch - 1], device="cuda")
    xs = x[idx].cpu().numpy()
    assert oracle.rel_l2(y[idx].cpu().numpy(), oracle.fft(xs, True)) <= REL_L2


@pytest.mark.parametrize("n", SIZES)
def test_config3_fp16_sweep_full_size(tfm, cuda, n):
    """FP16, batch 2^26/N and 2^26/N - 7 (masking), both
    directions, inputs U[-0.5, 0.5)."""
    import torch

    tf = tfm
    tf.ThunderFFTInitialize("half", n)
    for batch in (2 ** 26 // n, 2 ** 26 // n - 7):
        g = torch.Generator(device="cuda")
        g.manual_seed(n + batch)
        x = (torch.rand(batch, n, 2, device="cuda", generator=g) - 0.5).half()
        y = torch.empty_like(x)
        z = torch.empty_like(x)
        tf.ThunderFFT_global("half", n, True, x, y, batch)
        tf.ThunderFFT_global("half", n, False, y, z, batch)
        xf = x.float()
        e = ((z.float() / n - xf).pow(2).sum() / xf.pow(2).sum()).sqrt().item()
        assert np.isfinite(e) and e <= REL_L2, (n, batch, e)
        sel = [0, batch // 2, batch - 1]
        xs = x[sel].float().cpu().numpy()
        rep = xs[..., 0].astype(np.float64) + 1j * xs[..., 1]
        ys = y[sel].float().cpu().numpy()
        yc = ys[..., 0] + 1j * ys[..., 1]
        assert oracle.rel_l2(yc, oracle.fft(rep, True)) <= REL_L2
        del x, y, z
    tf.ThunderFFTFinalize("half")


@pytest.mark.parametrize("T", ["float", "half"])
@pytest.mark.parametrize("n", (64, 1024, 4096))
def test_unaligned_buffers(tfm, cuda, T, n):
    """Input/output pointers off the 16-byte grid take the thread-load /
    plain-store paths; results must not change."""
    import torch

    rng = np.random.default_rng(n)
    batch = 37
    x = rng.uniform(-1, 1, (batch, n)) + 1j * rng.uniform(-1, 1, (batch, n))
    din, rep = to_dev(x, T, torch, extra=1)
    esz = 8 if T == "float" else 4
    nel = batch * n
    src = torch.empty_like(din)
    if T == "float":
        src[1:1 + nel] = din[:nel]
    else:
        src[2:2 + 2 * nel] = din[:2 * nel]
    out = torch.zeros_like(din)
    tfm.ThunderFFT_global(T, n, True, src.data_ptr() + esz, out.data_ptr() + esz, batch)
    y = from_dev(out[1:] if T == "float" else out[2:], T, nel).reshape(batch, n)
    assert oracle.rel_l2(y, oracle.fft(rep, True)) <= REL_L2


@pytest.mark.parametrize("T", ["float", "half"])
def test_linearity(tfm, cuda, T):
    import torch

    n, batch = 2048, 96
    rng = np.random.default_rng(11)
    a = rng.uniform(-0.5, 0.5, (batch, n)) + 1j * rng.uniform(-0.5, 0.5, (batch, n))
    b = rng.uniform(-0.5, 0.5, (batch, n)) + 1j * rng.uniform(-0.5, 0.5, (batch, n))
    ya, ra, _ = run(tfm, torch, a, T, True)
    yb, rb, _ = run(tfm, torch, b, T, True)
    ys, rs, _ = run(tfm, torch, ra + rb, T, True)
    assert oracle.rel_l2(ys, ya + yb) <= 2 * REL_L2


def test_nondefault_stream_and_async(tfm, cuda):
    import torch

    n, batch = 512, 1000
    s = torch.cuda.Stream()
    rng = np.random.default_rng(4)
    x = (rng.uniform(-1, 1, (batch, n)) + 1j * rng.uniform(-1, 1, (batch, n))).astype(np.complex64)
    with torch.cuda.stream(s):
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty_like(dx)
        tfm.c2c_async("float", n, True, dx, dy, batch, s)
        tfm.sync_check(s)
    assert oracle.rel_l2(dy.cpu().numpy(), oracle.fft(x, True)) <= REL_L2


@pytest.mark.parametrize("T", ["float", "half"])
def test_twiddle_cache_lifecycle(tfm, cuda, T):
    """The reference's cache contract (sample/validation/cache_validation.cu:
    check_live/check_lifecycle): one table per (T, device), W[0] = 1+0i,
    W[1] = (cos 2pi/N, sin 2pi/N), same-N init keeps the allocation, another
    N replaces it, finalize clears it, repeated finalize is fine."""
    import torch

    tf = tfm
    tol = 1e-3 if T == "half" else 1e-6

    def live(n):
        p, got_n = tf.twiddle_table(T)
        assert p != 0 and got_n == n
        nbytes = 2 * (4 if T == "half" else 8)
        v = torch.as_tensor(_DevicePtr(p, nbytes), device="cuda").cpu().numpy()
        w = (v.view(np.float16).astype(np.float64) if T == "half" else v.view(np.float32).astype(np.float64))
        assert w[0] == 1.0 and w[1] == 0.0
        assert abs(w[2] - np.cos(2 * np.pi / n)) <= tol and abs(w[3] - np.sin(2 * np.pi / n)) <= tol
        return p

    tf.ThunderFFTInitialize(T, 64)
    first = live(64)
    tf.ThunderFFTInitialize(T, 64)
    assert live(64) == first
    tf.ThunderFFTInitialize(T, 128)
    live(128)
    tf.ThunderFFTFinalize(T)
    assert tf.twiddle_table(T) == (0, 0)
    tf.ThunderFFTFinalize(T)
    assert tf.twiddle_table(T) == (0, 0)
    tf.ThunderFFTInitialize(T, 64)
    live(64)
    tf.ThunderFFTFinalize(T)
    assert tf.twiddle_table(T) == (0, 0)
