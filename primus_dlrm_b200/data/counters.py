"""Sliding-window counter features (``primus_dlrm/data/counters.py``).

For every event position (in per-user, time-ordered flat arrays) and every
window of ``w`` days, the counters are ``log1p`` of how many listen+ /
like / skip events at earlier positions fall in the ``w`` days before it:

* user counters   [N, 3W]  -- over the user's own earlier events;
* item counters   [N, 3W]  -- over previous events on the same item (all users);
* cross counters  [N, 9W]  -- user x (same item | same artist | same album).

Each count is a two-pointer sweep over events sorted by (key, time): the
window's left edge only moves forward, so every event is visited O(1)
times per window.  Kernels are numba-parallel over contiguous key segments
(falls back to plain Python loops without numba).
"""
from __future__ import annotations

import numpy as np

try:
    import numba as nb
    _jit = nb.njit(parallel=True, cache=False)
    _prange = nb.prange
except ImportError:  # pragma: no cover
    nb = None

    def _jit(f):
        return f
    _prange = range

SECONDS_PER_DAY = 86400


@_jit
def _window_counts(seg_starts, seg_ends, ts, lp, like, skip, windows_s, out, col0):
    """Within each segment (events of one key in time order), position i gets
    log1p of the listen+/like/skip events at earlier positions j < i whose
    timestamp is >= ts[i] - w (events sharing i's timestamp but earlier in
    the order count; the window's lower edge is inclusive)."""
    n_seg = seg_starts.shape[0]
    n_w = windows_s.shape[0]
    for s in _prange(n_seg):
        a = seg_starts[s]
        b = seg_ends[s]
        for w in range(n_w):
            lo = a
            c_lp = 0
            c_like = 0
            c_skip = 0
            for i in range(a, b):
                edge = ts[i] - windows_s[w]
                while lo < i and ts[lo] < edge:
                    c_lp -= lp[lo]
                    c_like -= like[lo]
                    c_skip -= skip[lo]
                    lo += 1
                out[i, col0 + 3 * w] = np.log1p(c_lp)
                out[i, col0 + 3 * w + 1] = np.log1p(c_like)
                out[i, col0 + 3 * w + 2] = np.log1p(c_skip)
                c_lp += lp[i]
                c_like += like[i]
                c_skip += skip[i]


def _segments(keys_sorted: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    if keys_sorted.size == 0:
        return np.zeros(0, np.int64), np.zeros(0, np.int64)
    change = np.flatnonzero(np.diff(keys_sorted)) + 1
    starts = np.concatenate([[0], change]).astype(np.int64)
    ends = np.concatenate([change, [keys_sorted.size]]).astype(np.int64)
    return starts, ends


def _by_key(keys, ts, lp, like, skip, windows_days, n_cols, col0, out):
    order = np.lexsort((ts, keys))          # stable: time order within each key
    k, t = keys[order], ts[order]
    s, e = _segments(k)
    tmp = np.zeros((keys.size, n_cols), dtype=np.float32)
    _window_counts(s, e, t.astype(np.int64), lp[order].astype(np.int64), like[order].astype(np.int64),
                   skip[order].astype(np.int64), np.asarray(windows_days, np.int64) * SECONDS_PER_DAY, tmp, col0)
    out[order] = tmp
    return out


def precompute_user_counters(uid, ts, is_lp, is_like, is_skip, windows_days) -> np.ndarray:
    W = len(windows_days)
    out = np.zeros((uid.size, 3 * W), dtype=np.float32)
    return _by_key(uid, ts, is_lp, is_like, is_skip, windows_days, 3 * W, 0, out)


def precompute_item_counters(item, ts, is_lp, is_like, is_skip, windows_days) -> np.ndarray:
    W = len(windows_days)
    out = np.zeros((item.size, 3 * W), dtype=np.float32)
    return _by_key(item, ts, is_lp, is_like, is_skip, windows_days, 3 * W, 0, out)


def precompute_cross_counters(uid, item, ts, is_lp, is_like, is_skip, item_to_artist, item_to_album,
                              windows_days) -> np.ndarray:
    """Layout per window w (9 columns): user x item (lp, like, skip), user x
    artist (lp, like, skip), user x album (lp, like, skip)."""
    W = len(windows_days)
    n = uid.size
    out = np.zeros((n, 9 * W), dtype=np.float32)
    artist = item_to_artist[item]
    album = item_to_album[item]
    for j, other in enumerate((item, artist, album)):
        key = uid.astype(np.int64) * (int(other.max()) + 1 if other.size else 1) + other.astype(np.int64)
        part = np.zeros((n, 3 * W), dtype=np.float32)
        _by_key(key, ts, is_lp, is_like, is_skip, windows_days, 3 * W, 0, part)
        for w in range(W):
            out[:, 9 * w + 3 * j: 9 * w + 3 * j + 3] = part[:, 3 * w: 3 * w + 3]
    return out
