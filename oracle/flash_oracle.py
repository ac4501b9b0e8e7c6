"""CPU oracle of Flash token compression (model/flash.py).

TEST INFRASTRUCTURE ONLY. Only ``tests/`` may import this module; the product
path never does, and nothing here runs on a GPU.

Restates, in numpy:
  * ``spatial_layout`` (model/flash.py:6-33): which packed rows the compressed
    blocks keep, and for every row the compressed row it takes its update from;
  * the ``compress`` hook's row selection (model/flash.py:71-79);
  * the ``restore`` hook's arithmetic (model/flash.py:81-84).

Parity pinning: ``tests/test_oracle_flash.py`` checks these against golden
vectors made by running the reference's own ``spatial_layout`` and
``configure_flash`` hooks on the CPU (``tests/golden/make_golden_flash.py``).
"""
from __future__ import annotations

import numpy as np

from .w8a8_oracle import bf16_round, F32


def retained_ranks(count: int, stride: int) -> np.ndarray:
    """Ranks of a sorted coordinate alphabet of ``count`` values that survive
    stride-``stride`` selection: every stride-th value from the first, plus the
    last value (model/flash.py:17-20)."""
    keep = np.zeros(count, bool)
    keep[::stride] = True
    keep[count - 1] = True
    return keep


def spatial_layout(positions: np.ndarray, tags: np.ndarray, stride: int = 2):
    """(keep, inverse) of model/flash.py:6-33.

    positions [S, 3] (time, row, column), tags [S] (0 = video). Non-video rows
    are always kept; a video row is kept when both its row and its column
    coordinate survive stride selection over the video rows' coordinate
    alphabets. ``keep`` lists the kept rows in order; ``inverse[t]`` is the
    compressed row of kept row t, or, for a dropped row, that of its nearest
    same-time kept video row (Euclidean over row/column in fp32, first one on
    ties, anchor 0 if none shares the time)."""
    positions = np.asarray(positions)
    tags = np.asarray(tags)
    if positions.ndim != 2 or tags.ndim != 1 or positions.shape != (tags.size, 3):
        raise ValueError("Flash requires a single shared packed layout")
    video = tags == 0
    if not video.any():
        raise ValueError("Flash requires video tokens")
    spatial = np.ones(tags.size, bool)
    for axis in (1, 2):
        alphabet = np.unique(positions[video, axis])
        ok = retained_ranks(alphabet.size, stride)
        rank = np.searchsorted(alphabet, positions[:, axis])
        inside = rank < alphabet.size
        member = np.zeros(tags.size, bool)
        member[inside] = (alphabet[rank[inside]] == positions[inside, axis]) & ok[rank[inside]]
        spatial &= member
    mask = ~video | spatial
    keep = np.flatnonzero(mask).astype(np.int64)
    inverse = np.zeros(tags.size, np.int64)
    inverse[keep] = np.arange(keep.size, dtype=np.int64)
    dropped = np.flatnonzero(video & ~mask)
    anchors = np.flatnonzero(video & mask)
    if dropped.size:
        inverse[dropped] = inverse[anchors[nearest_anchor(positions.astype(F32), dropped, anchors)]]
    return keep, inverse


def nearest_anchor(pos32: np.ndarray, dropped: np.ndarray, anchors: np.ndarray, chunk: int = 1024):
    """Index into ``anchors`` of each dropped row's nearest same-time anchor
    (model/flash.py:27-32): distance = fp32 sqrt of the squared distance,
    masked to +inf across times, first minimum (numpy's argmin, like torch's)."""
    if anchors.size == 0:
        raise ValueError("dropped rows but no anchors")
    target = pos32[anchors].astype(np.float64)
    out = np.empty(dropped.size, np.int64)
    for lo in range(0, dropped.size, chunk):
        src = pos32[dropped[lo:lo + chunk]].astype(np.float64)
        d2 = ((src[:, None, 1] - target[None, :, 1]) ** 2 + (src[:, None, 2] - target[None, :, 2]) ** 2)
        dist = np.sqrt(d2.astype(F32))
        dist[src[:, None, 0].astype(F32) != target[None, :, 0].astype(F32)] = np.inf
        out[lo:lo + chunk] = np.argmin(dist, axis=1)
    return out


def gather_rows(src: np.ndarray, index: np.ndarray, axis: int) -> np.ndarray:
    """``Tensor.index_select(axis, index)`` (model/flash.py:73,76-79)."""
    return np.take(src, index, axis=axis)


def restore(full, compressed, compressed_input, inverse, gain: float = 1.0) -> np.ndarray:
    """model/flash.py:81-84 on float32 arrays holding bf16 values [B, S|K, D]:
    out = bf16(full + bf16(bf16(compressed - input) * gain)[:, inverse])."""
    delta = bf16_round(np.asarray(compressed, F32) - np.asarray(compressed_input, F32))
    delta = bf16_round(delta * F32(gain))
    return bf16_round(np.asarray(full, F32) + np.take(delta, inverse, axis=1))
