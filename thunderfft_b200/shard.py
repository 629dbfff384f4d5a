"""Batch sharding across GPUs (one process per GPU, no collective on the data path).

Every signal of a batched FFT or convolution is independent, so N GPUs each
take a contiguous slice of the batch and run the unchanged single-GPU entry
points on it (the reference has no multi-GPU code; its per-device twiddle
cache, detail/thunderfft_impl_twiddle.cuh:26-36, is what makes this work).
torch.distributed is used only by callers for barriers / timing
reductions, never to move signal data.
"""
from __future__ import annotations


def shard_range(batch: int, world: int, rank: int, align: int = 1):
    """Contiguous slice (start, count) of `batch` items for `rank` of `world`.

    Slices differ in size by at most `align` items, start on multiples of
    `align` (e.g. a kernel tile size, so only the last rank sees a partial
    tile), and together cover [0, batch) exactly once."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    if batch < 0 or align <= 0:
        raise ValueError("need batch >= 0 and align > 0")
    units = (batch + align - 1) // align
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    start = min(u0 * align, batch)
    stop = min(u1 * align, batch)
    return start, stop - start


def conv2d_image_shard(batch_images: int, world: int, rank: int, scaling: str = "strong"):
    """Batch images [b0, b0 + nb) that `rank` convolves in the 2-D convolution.

    strong: the batch is split by image pair (images b and b + 1 of a channel
    share one complex transform), so every slice starts on an even image and
    only the batch's odd last image can stand alone; weak: every rank takes
    the whole batch."""
    if scaling == "weak":
        return 0, batch_images
    if scaling != "strong":
        raise ValueError("scaling must be 'strong' or 'weak'")
    return shard_range(batch_images, world, rank, align=2)


def weak_scaling_value(bytes_per_rank: float, max_ms: float, world: int) -> float:
    """Whole-job throughput (GB/s) when every rank moves `bytes_per_rank`
    bytes and the slowest rank took `max_ms` milliseconds."""
    return world * bytes_per_rank / (max_ms / 1e3) / 1e9


def fft_local_shard(T: str, n: int, forward: bool, x_full, y_full, world: int, rank: int, stream=None):
    """Transform this rank's slice of x_full into y_full (both CUDA tensors on
    this rank's device holding the whole batch, rows = signals)."""
    from . import c2c_async

    batch = x_full.shape[0]
    start, count = shard_range(batch, world, rank)
    if count:
        c2c_async(T, n, forward, x_full[start:start + count], y_full[start:start + count], count, stream)
    return start, count
