"""Yambda datasets (``primus_dlrm/data/dataset.py``) on numpy + pyarrow.

On-disk contract (shared with the reference so processed data and caches
carry over):

* ``<root>/processed[_<size>]/``: ``train_sessions.parquet`` (uid,
  session_id, item_ids[], timestamps[], event_types[], is_organic[],
  played_ratio_pct[], track_length_seconds[]), ``test_events.parquet``,
  ``item_popularity.npy``, ``split_meta.json``;
* ``<root>/shared_metadata/``: ``{artist,album}_item_mapping.parquet``,
  ``embeddings.parquet`` (item_id, normalized_embed);
* ``<root>/cache[_<size>]/<key>/``: the flat event store as ``.npy`` files
  (flat_uid, flat_item_ids, flat_timestamps, flat_event_types,
  flat_played_ratio, flat_is_listen_plus, flat_is_like, flat_is_skip,
  flat_is_organic, user_start, user_end, unique_uids, optional counters)
  plus ``store_meta.json`` and ``positions_L{L}.npy``.

Samples: for a training position (an event after at least L earlier events of
its user) the history is split into listen+ / like / skip pools from the
previous 500 events, each left-padded with id 0 to its length, with artist /
album ids looked up per item; labels listen_plus (listen with
played_ratio >= 50), like, dislike, listen_pct.  Per-group lengths
(``data.history_lengths``) are honoured.

``.npy`` arrays are opened with a shared read-only mapping (no copy-on-write
commit charge), so 8 ranks can share a 5B-event cache.
"""
from __future__ import annotations

import json
import logging
import math
import mmap
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch
from torch.utils.data import Dataset, Sampler

from primus_dlrm_b200.config import Config, DataConfig

logger = logging.getLogger(__name__)

EVENT_TYPE_MAP = {"listen": 0, "like": 1, "dislike": 2, "unlike": 3, "undislike": 4}
LISTEN, LIKE, DISLIKE = 0, 1, 2
LISTEN_PLUS_THRESHOLD = 50
SECONDS_PER_DAY = 86400
HISTORY_SCAN = 500
POOLS = ("lp", "like", "skip")
STORE_ARRAYS = ("flat_uid", "flat_item_ids", "flat_timestamps", "flat_event_types", "flat_played_ratio",
                "flat_is_listen_plus", "flat_is_like", "flat_is_skip", "flat_is_organic",
                "user_start", "user_end", "unique_uids")


def load_npy_shared(path: str | Path) -> np.ndarray:
    """Read-only ``.npy`` view over a MAP_SHARED mapping."""
    path = Path(path)
    with open(path, "rb") as f:
        major, _ = np.lib.format.read_magic(f)
        hdr = np.lib.format.read_array_header_1_0 if major == 1 else np.lib.format.read_array_header_2_0
        shape, fortran, dtype = hdr(f)
        offset = f.tell()
    fd = os.open(str(path), os.O_RDONLY)
    try:
        size = os.fstat(fd).st_size
        buf = mmap.mmap(fd, 0, access=mmap.ACCESS_READ) if size else b""
    finally:
        os.close(fd)
    arr = np.ndarray(shape, dtype=dtype, buffer=buf, offset=offset, order="F" if fortran else "C")
    arr.flags.writeable = False
    return arr


@dataclass(frozen=True)
class DataPaths:
    data_root: Path
    dataset_size: str

    @classmethod
    def from_config(cls, config: DataConfig, data_root=None) -> "DataPaths":
        return cls(Path(data_root) if data_root is not None else Path(config.data_dir), config.dataset_size)

    @property
    def raw(self) -> Path:
        return self.data_root / "raw" / self.dataset_size

    @property
    def metadata(self) -> Path:
        return self.data_root / "shared_metadata"

    @property
    def processed(self) -> Path:
        return self.data_root / ("processed" if self.dataset_size == "50m" else f"processed_{self.dataset_size}")

    @property
    def cache(self) -> Path:
        return self.data_root / ("cache" if self.dataset_size == "50m" else f"cache_{self.dataset_size}")


def cache_key(split: str, windows: list[int] | None) -> str:
    return f"{split}_counters_{'_'.join(map(str, windows))}" if windows else f"{split}_nocounters"


# ---------------------------------------------------------------------------
# flat event store
# ---------------------------------------------------------------------------

class EventStore:
    """All training events as flat per-user, time-ordered arrays."""

    @classmethod
    def from_sessions(cls, sessions_path: Path, enable_counters=False, item_to_artist=None, item_to_album=None,
                      windows: list[int] | None = None) -> "EventStore":
        import pyarrow.compute as pc
        import pyarrow.parquet as pq
        t = pq.read_table(sessions_path)
        t = t.sort_by([("uid", "ascending"), ("session_id", "ascending")])
        lens = pc.list_value_length(t.column("item_ids")).to_numpy(zero_copy_only=False)
        st = cls.__new__(cls)
        st.flat_uid = np.repeat(t.column("uid").to_numpy(), lens).astype(np.int64)

        def flat(col, dt):
            return pc.list_flatten(t.column(col)).to_numpy(zero_copy_only=False).astype(dt)
        st.flat_item_ids = flat("item_ids", np.int64)
        st.flat_timestamps = flat("timestamps", np.int64)
        st.flat_event_types = flat("event_types", np.int64)
        st.flat_played_ratio = np.nan_to_num(flat("played_ratio_pct", np.float32), nan=0.0)
        st.flat_is_organic = flat("is_organic", np.int8) if "is_organic" in t.column_names else \
            np.zeros_like(st.flat_item_ids, dtype=np.int8)
        st._finish(enable_counters, item_to_artist, item_to_album, windows)
        return st

    @classmethod
    def from_arrays(cls, uid, item, ts, etype, played, organic=None, enable_counters=False, item_to_artist=None,
                    item_to_album=None, windows=None) -> "EventStore":
        order = np.lexsort((ts, uid))
        st = cls.__new__(cls)
        st.flat_uid = np.asarray(uid, np.int64)[order]
        st.flat_item_ids = np.asarray(item, np.int64)[order]
        st.flat_timestamps = np.asarray(ts, np.int64)[order]
        st.flat_event_types = np.asarray(etype, np.int64)[order]
        st.flat_played_ratio = np.asarray(played, np.float32)[order]
        st.flat_is_organic = (np.asarray(organic, np.int8)[order] if organic is not None
                              else np.zeros(order.size, np.int8))
        st._finish(enable_counters, item_to_artist, item_to_album, windows)
        return st

    def _finish(self, enable_counters, item_to_artist, item_to_album, windows) -> None:
        listen = self.flat_event_types == LISTEN
        self.flat_is_listen_plus = listen & (self.flat_played_ratio >= LISTEN_PLUS_THRESHOLD)
        self.flat_is_like = self.flat_event_types == LIKE
        self.flat_is_skip = listen & (self.flat_played_ratio < LISTEN_PLUS_THRESHOLD)
        n = self.flat_uid.size
        change = np.flatnonzero(np.diff(self.flat_uid)) + 1
        starts = np.concatenate([[0], change]).astype(np.int64)
        ends = np.concatenate([change, [n]]).astype(np.int64)
        uids = self.flat_uid[starts] if n else np.zeros(0, np.int64)
        size = int(uids.max()) + 1 if uids.size else 1
        self.user_start = np.full(size, -1, np.int64)
        self.user_end = np.full(size, -1, np.int64)
        self.user_start[uids] = starts
        self.user_end[uids] = ends
        self.unique_uids = uids
        self.num_users = int(uids.size)
        self.total_events = int(n)
        self.enable_counters = bool(enable_counters)
        self.counter_windows_days = list(windows or [])
        if enable_counters:
            from primus_dlrm_b200.data import counters as C
            w = self.counter_windows_days
            self.user_counters = C.precompute_user_counters(self.flat_uid, self.flat_timestamps,
                                                            self.flat_is_listen_plus, self.flat_is_like,
                                                            self.flat_is_skip, w)
            self.item_counters = C.precompute_item_counters(self.flat_item_ids, self.flat_timestamps,
                                                            self.flat_is_listen_plus, self.flat_is_like,
                                                            self.flat_is_skip, w)
            self.cross_counters = C.precompute_cross_counters(self.flat_uid, self.flat_item_ids,
                                                              self.flat_timestamps, self.flat_is_listen_plus,
                                                              self.flat_is_like, self.flat_is_skip,
                                                              item_to_artist, item_to_album, w)

    def user_slice(self, uid: int) -> tuple[int, int]:
        if uid < 0 or uid >= self.user_start.size:
            return -1, -1
        return int(self.user_start[uid]), int(self.user_end[uid])

    def save(self, d: Path) -> None:
        d = Path(d)
        d.mkdir(parents=True, exist_ok=True)
        for name in STORE_ARRAYS:
            np.save(d / f"{name}.npy", getattr(self, name))
        if self.enable_counters:
            for name in ("user_counters", "item_counters", "cross_counters"):
                np.save(d / f"{name}.npy", getattr(self, name))
        with open(d / "store_meta.json", "w") as f:
            json.dump({"num_users": self.num_users, "total_events": self.total_events,
                       "enable_counters": self.enable_counters,
                       "counter_windows_days": self.counter_windows_days}, f)

    @classmethod
    def load(cls, d: Path, in_memory: bool = False) -> "EventStore":
        d = Path(d)
        with open(d / "store_meta.json") as f:
            meta = json.load(f)
        st = cls.__new__(cls)
        st.num_users, st.total_events = meta["num_users"], meta["total_events"]
        st.enable_counters = meta["enable_counters"]
        st.counter_windows_days = meta.get("counter_windows_days", [])
        names = list(STORE_ARRAYS) + (["user_counters", "item_counters", "cross_counters"] if st.enable_counters else [])
        for name in names:
            p = d / f"{name}.npy"
            if not p.exists():
                raise FileNotFoundError(f"cache {d} lacks {name}.npy (rebuild the cache)")
            a = load_npy_shared(p)
            setattr(st, name, np.array(a) if in_memory else a)
        return st


def _load_metadata(paths: DataPaths, n_items: int):
    import pyarrow.parquet as pq
    to_artist = np.zeros(n_items, np.int64)
    to_album = np.zeros(n_items, np.int64)
    n_art = n_alb = 1
    for fname, arr, key in (("artist_item_mapping.parquet", to_artist, "artist_id"),
                            ("album_item_mapping.parquet", to_album, "album_id")):
        p = paths.metadata / fname
        if p.exists():
            t = pq.read_table(p)
            it = t.column("item_id").to_numpy()
            v = t.column(key).to_numpy()
            ok = it < n_items
            arr[it[ok]] = v[ok]
            if key == "artist_id":
                n_art = int(v.max()) + 1
            else:
                n_alb = int(v.max()) + 1
    audio = None
    ep = paths.metadata / "embeddings.parquet"
    if ep.exists():
        t = pq.read_table(ep)
        ids = t.column("item_id").to_numpy()
        emb = np.stack(t.column("normalized_embed").to_numpy(zero_copy_only=False))
        audio = np.zeros((n_items, emb.shape[1]), np.float32)
        ok = ids < n_items
        audio[ids[ok]] = emb[ok]
    if audio is None:
        audio = np.zeros((n_items, 128), np.float32)
    return to_artist, to_album, n_art, n_alb, audio


def _split_history(store, pos_end: int, user_start: int, lengths: dict[str, int], to_artist, to_album):
    """Per pool: the last L item ids among the previous <=500 events, left-padded with 0."""
    s = max(user_start, pos_end - HISTORY_SCAN)
    items = store.flat_item_ids[s:pos_end]
    masks = {"lp": store.flat_is_listen_plus[s:pos_end], "like": store.flat_is_like[s:pos_end],
             "skip": store.flat_is_skip[s:pos_end]}
    out = {}
    for pool in POOLS:
        L = lengths[pool]
        sel = items[masks[pool]][-L:] if L > 0 else items[:0]
        padded = np.zeros(L, np.int64)
        if sel.size:
            padded[L - sel.size:] = sel
        out[f"{pool}_items"] = padded
        out[f"{pool}_artists"] = to_artist[padded]
        out[f"{pool}_albums"] = to_album[padded]
    return out


def _pool_lengths(config: Config) -> dict[str, int]:
    return {p: config.data.group_length(f"hist_{p}") for p in POOLS}


class _YambdaBase(Dataset):
    def _init_common(self, config: Config, paths: DataPaths, split: str):
        self.config = config
        self.paths = paths
        self.item_popularity = np.load(paths.processed / "item_popularity.npy")
        self.num_items = int(self.item_popularity.shape[0])
        (self.item_to_artist, self.item_to_album, self.num_artists, self.num_albums,
         self.audio_embeddings) = _load_metadata(paths, self.num_items)
        self.audio_dim = self.audio_embeddings.shape[1]
        dc = config.data
        windows = dc.counter_windows_days if dc.enable_counters else None
        cdir = paths.cache / cache_key(split, windows)
        if dc.use_cache and (cdir / "store_meta.json").exists():
            self.store = EventStore.load(cdir)
        else:
            self.store = EventStore.from_sessions(paths.processed / "train_sessions.parquet", dc.enable_counters,
                                                  self.item_to_artist, self.item_to_album, windows)
            if dc.use_cache:
                self.store.save(cdir)
        self._lengths = _pool_lengths(config)
        self._cross = [s for s in (config.model.cross_features or []) if s.enabled]


class YambdaTrainDataset(_YambdaBase):
    """Scoring pairs: (user history before an event, the event's item, its labels)."""

    def __init__(self, config: Config, paths: DataPaths):
        self._init_common(config, paths, "train")
        with open(paths.processed / "split_meta.json") as f:
            self.split_meta = json.load(f)
        L = max(self._lengths.values())
        windows = config.data.counter_windows_days if config.data.enable_counters else None
        pos_path = paths.cache / cache_key("train", windows) / f"positions_L{L}.npy"
        if pos_path.exists():
            self._positions = load_npy_shared(pos_path)
        else:
            st = self.store
            counts = np.maximum(st.user_end - st.user_start - L, 0)
            counts[st.user_start < 0] = 0
            idx = np.repeat(np.arange(counts.size), counts)
            first = np.repeat(st.user_start + L - np.cumsum(np.concatenate([[0], counts[:-1]])), counts)
            self._positions = (first + np.arange(int(counts.sum()))).astype(np.int64)
            del idx
            if config.data.use_cache:
                pos_path.parent.mkdir(parents=True, exist_ok=True)
                np.save(pos_path, self._positions)
        logger.info("Yambda train: %d positions, %d items, %d users", len(self._positions), self.num_items,
                    self.store.num_users)

    def __len__(self) -> int:
        return int(len(self._positions))

    def __getitem__(self, idx: int) -> dict:
        st = self.store
        pos = int(self._positions[idx])
        uid = int(st.flat_uid[pos])
        hist = _split_history(st, pos, int(st.user_start[uid]), self._lengths, self.item_to_artist,
                              self.item_to_album)
        item = int(st.flat_item_ids[pos])
        et = int(st.flat_event_types[pos])
        played = float(st.flat_played_ratio[pos])
        out = {f"hist_{p}_{k}_ids": hist[f"{p}_{k}s"] for p in POOLS for k in ("item", "artist", "album")}
        out.update(uid=uid, item_id=item, artist_id=int(self.item_to_artist[item]),
                   album_id=int(self.item_to_album[item]), audio_embed=self.audio_embeddings[item],
                   listen_plus=float(et == LISTEN and played >= LISTEN_PLUS_THRESHOLD), like=float(et == LIKE),
                   dislike=float(et == DISLIKE), listen_pct=min(played / 100.0, 1.0) if et == LISTEN else 0.0)
        if st.enable_counters:
            out["user_counters"] = np.asarray(st.user_counters[pos])
            out["item_counters"] = np.asarray(st.item_counters[pos])
            out["cross_counters"] = np.asarray(st.cross_counters[pos])
        if self._cross:
            from primus_dlrm_b200.data.hashing import cross_hash_nway
            src = {"uid": uid, "item_id": item, "artist_id": out["artist_id"], "album_id": out["album_id"],
                   "hour_of_day": int(st.flat_timestamps[pos] // 3600 % 24),
                   "is_organic": int(st.flat_is_organic[pos])}
            for s in self._cross:
                out[f"{s.name}_id"] = cross_hash_nway([src[k] for k in s.keys], s.num_embeddings, s.salt)
        return out


def collate_to_dict(samples: list[dict]) -> dict[str, torch.Tensor]:
    """Stack samples into the batch-dict contract (``dataset.py:890-923``)."""
    out = {}
    for k in samples[0]:
        v = [s[k] for s in samples]
        if isinstance(v[0], np.ndarray):
            out[k] = torch.from_numpy(np.stack(v))
        elif isinstance(v[0], float):
            out[k] = torch.tensor(v, dtype=torch.float32)
        else:
            out[k] = torch.tensor(v, dtype=torch.int64)
    for k in ("audio_embed", "user_counters", "item_counters", "cross_counters"):
        if k in out:
            out[k] = out[k].float()
    return out


class _CandidateMixin:
    """Device batches for candidate scoring (shared by the real and synthetic eval sets).

    A counter block is emitted whenever the model consumes it (the config
    declares that dense feature), zero-filled when the data has no counters."""

    def _wants(self, name: str) -> bool:
        return any(d.name == name for d in self.config.feature.dense_features)

    def _dense_dim(self, name: str, default: int) -> int:
        for d in self.config.feature.dense_features:
            if d.name == name:
                return d.dim
        return default

    def _counters_on(self) -> bool:
        st = getattr(self, "store", None)
        return bool(self.config.data.enable_counters and st is not None and st.enable_counters)

    def user_batch(self, sample: dict, device) -> dict[str, torch.Tensor]:
        h = sample["history"]
        out = {f"hist_{p}_{k}_ids": torch.from_numpy(np.asarray(h[f"{p}_{k}s"])).long().unsqueeze(0).to(device)
               for p in POOLS for k in ("item", "artist", "album")}
        out["uid"] = torch.tensor([sample["uid"]], dtype=torch.long, device=device)
        if self._wants("user_counters"):
            out["user_counters"] = torch.from_numpy(self.get_user_counters(sample["uid"])).float().unsqueeze(0).to(device)
        return out

    def candidate_batch(self, items: np.ndarray, device) -> dict[str, torch.Tensor]:
        items = np.asarray(items, np.int64)
        out = {"item_id": torch.from_numpy(items).to(device),
               "artist_id": torch.from_numpy(self.item_to_artist[items]).to(device),
               "album_id": torch.from_numpy(self.item_to_album[items]).to(device),
               "audio_embed": torch.from_numpy(self.audio_embeddings[items]).float().to(device)}
        if self._wants("item_counters"):
            out["item_counters"] = torch.from_numpy(self.get_item_counters_batch(items)).float().to(device)
        return out

    def with_user_features(self, cand: dict, sample: dict, items, device) -> dict[str, torch.Tensor]:
        out = dict(cand)
        if self._wants("cross_counters"):
            out["cross_counters"] = torch.from_numpy(
                self.get_cross_counters_batch(sample["uid"], np.asarray(items, np.int64))).float().to(device)
        return out


class YambdaEvalDataset(_YambdaBase, _CandidateMixin):
    """Test users with ground truth sets; histories from the training events."""

    def __init__(self, config: Config, paths: DataPaths):
        import pyarrow.parquet as pq
        self._init_common(config, paths, "eval")
        t = pq.read_table(paths.processed / "test_events.parquet")
        uid = t.column("uid").to_numpy()
        item = t.column("item_id").to_numpy()
        et = t.column("event_type").to_numpy()
        played = t.column("played_ratio_pct").to_numpy(zero_copy_only=False) if "played_ratio_pct" in \
            t.column_names else np.zeros(uid.size)
        played = np.nan_to_num(played.astype(np.float64), nan=-1)
        gt: dict[int, dict[str, set]] = {}
        for u, i, e, p in zip(uid.tolist(), item.tolist(), et.tolist(), played.tolist()):
            d = gt.setdefault(u, {"listen_plus": set(), "like": set()})
            if e == LISTEN and p >= LISTEN_PLUS_THRESHOLD:
                d["listen_plus"].add(i)
            if e == LIKE:
                d["like"].add(i)
        self.test_ground_truth = gt
        self.test_uids = sorted(gt)
        if config.data.enable_counters:
            self._eval_item_counters()

    def __len__(self) -> int:
        return len(self.test_uids)

    def __getitem__(self, idx: int) -> dict:
        uid = self.test_uids[idx]
        d = {"uid": uid, "history": self.get_user_history(uid)}
        for task, s in self.test_ground_truth[uid].items():
            d[f"ground_truth_{task}"] = s
        return d

    def get_user_history(self, uid: int) -> dict:
        s, e = self.store.user_slice(uid)
        if s < 0:
            return {f"{p}_{k}s": np.zeros(self._lengths[p], np.int64) for p in POOLS for k in ("item", "artist", "album")}
        return _split_history(self.store, e, s, self._lengths, self.item_to_artist, self.item_to_album)

    def get_user_train_items(self, uid: int) -> np.ndarray:
        s, e = self.store.user_slice(uid)
        return np.unique(self.store.flat_item_ids[s:e]) if s >= 0 else np.zeros(0, np.int64)

    def _eval_item_counters(self) -> None:
        st = self.store
        W = len(self.config.data.counter_windows_days)
        self.eval_item_counters = np.zeros((self.num_items, 3 * W), np.float32)
        t_max = int(st.flat_timestamps.max()) if st.total_events else 0
        for w, days in enumerate(self.config.data.counter_windows_days):
            m = st.flat_timestamps >= t_max - days * SECONDS_PER_DAY
            it = st.flat_item_ids[m]
            for c, flag in enumerate((st.flat_is_listen_plus, st.flat_is_like, st.flat_is_skip)):
                cnt = np.bincount(it, weights=flag[m].astype(np.float64), minlength=self.num_items)
                self.eval_item_counters[:, 3 * w + c] = np.log1p(cnt[: self.num_items])

    def get_user_counters(self, uid: int) -> np.ndarray:
        s, e = self.store.user_slice(uid)
        if s < 0 or not self._counters_on():
            return np.zeros(self._dense_dim("user_counters", 3 * len(self.config.data.counter_windows_days)),
                            np.float32)
        return np.asarray(self.store.user_counters[e - 1]).copy()

    def get_item_counters_batch(self, items: np.ndarray) -> np.ndarray:
        if not self._counters_on():
            W = len(self.config.data.counter_windows_days)
            return np.zeros((len(items), self._dense_dim("item_counters", 3 * W)), np.float32)
        return self.eval_item_counters[items]

    def get_cross_counters_batch(self, uid: int, items: np.ndarray) -> np.ndarray:
        W = len(self.config.data.counter_windows_days)
        if not self._counters_on():
            return np.zeros((len(items), self._dense_dim("cross_counters", 9 * W)), np.float32)
        out = np.zeros((len(items), 9 * W), np.float32)
        s, e = self.store.user_slice(uid)
        if s < 0:
            return out
        st = self.store
        t_max = int(st.flat_timestamps[e - 1])
        it = st.flat_item_ids[s:e]
        ts = st.flat_timestamps[s:e]
        flags = (st.flat_is_listen_plus[s:e], st.flat_is_like[s:e], st.flat_is_skip[s:e])
        for w, days in enumerate(self.config.data.counter_windows_days):
            m = ts >= t_max - days * SECONDS_PER_DAY
            for j, (own, cand) in enumerate(((it[m], items), (self.item_to_artist[it[m]], self.item_to_artist[items]),
                                             (self.item_to_album[it[m]], self.item_to_album[items]))):
                for c, flag in enumerate(flags):
                    keys, cnt = np.unique(own[flag[m]], return_counts=True)
                    pos = np.searchsorted(keys, cand)
                    hit = (pos < keys.size) & (keys[np.minimum(pos, max(keys.size - 1, 0))] == cand) \
                        if keys.size else np.zeros(len(items), bool)
                    vals = np.where(hit, cnt[np.minimum(pos, max(keys.size - 1, 0))] if keys.size else 0, 0)
                    out[:, 9 * w + 3 * j + c] = np.log1p(vals)
        return out


class SyntheticEvalDataset(Dataset, _CandidateMixin):
    """Synthetic users for ranking eval over random candidates (the reference
    skips eval for synthetic data).  Histories come from the training
    generator's distributions; ground truth is a random item set per user."""

    def __init__(self, config: Config, num_users: int = 64, num_items_with_history: int = 1000, seed: int = 7,
                 gt_size: int = 20):
        from primus_dlrm_b200.data.synthetic import generate_batch
        self.config = config
        sizes = {t.name: t.num_embeddings for t in config.model.embedding_tables}
        self.num_items = sizes.get("item", max(sizes.values()))
        g = np.random.default_rng(seed)
        self.item_to_artist = g.integers(0, sizes.get("artist", 1), self.num_items, dtype=np.int64)
        self.item_to_album = g.integers(0, sizes.get("album", 1), self.num_items, dtype=np.int64)
        dims = {d.name: d.dim for d in config.feature.dense_features}
        self.audio_embeddings = g.standard_normal((self.num_items, dims.get("audio_embed", 1))).astype(np.float32)
        self.item_popularity = np.sort(g.zipf(1.3, self.num_items))[::-1].astype(np.float64)
        b = generate_batch(config, num_users, seed=seed)
        f2k = config.feature_to_batch_key()
        self._users = []
        for u in range(num_users):
            hist = {}
            for p in POOLS:
                for k in ("item", "artist", "album"):
                    key = f2k.get(f"hist_{p}_{k}", f"hist_{p}_{k}")
                    hist[f"{p}_{k}s"] = b[key][u].numpy() if key in b else np.zeros(1, np.int64)
            uid_key = f2k.get("uid", "uid")
            uid = int(b[uid_key][u]) if uid_key in b else u
            gt = set(g.choice(min(num_items_with_history, self.num_items), gt_size, replace=False).tolist())
            self._users.append({"uid": uid, "history": hist, "ground_truth_" + config.task_names[0]: gt})
        self._counter_dims = {d.name: d.dim for d in config.feature.dense_features if "counter" in d.name}

    def __len__(self) -> int:
        return len(self._users)

    def __getitem__(self, idx: int) -> dict:
        return self._users[idx]

    def get_user_train_items(self, uid: int) -> np.ndarray:
        return np.arange(min(200, self.num_items))

    def get_user_counters(self, uid: int) -> np.ndarray:
        return np.zeros(self._counter_dims.get("user_counters", 0), np.float32)

    def get_item_counters_batch(self, items):
        return np.zeros((len(items), self._counter_dims.get("item_counters", 0)), np.float32)

    def get_cross_counters_batch(self, uid, items):
        return np.zeros((len(items), self._counter_dims.get("cross_counters", 0)), np.float32)


class LargeDatasetSampler(Sampler):
    """O(1)-memory distributed sampler for billion-sample datasets: shuffled =
    seeded sampling with replacement, else strided ``i * W + rank``
    (``scripts/run_distributed.py:25-69``)."""

    def __init__(self, dataset, num_replicas: int, rank: int, shuffle: bool = False, seed: int = 0):
        self.n = len(dataset)
        self.world, self.rank, self.shuffle, self.seed, self.epoch = num_replicas, rank, shuffle, seed, 0
        self.num_samples = math.ceil(self.n / self.world)

    def set_epoch(self, epoch: int) -> None:
        self.epoch = epoch

    def __len__(self) -> int:
        return self.num_samples

    def __iter__(self):
        if self.shuffle:
            g = torch.Generator().manual_seed(self.seed + self.epoch + 7919 * self.rank)
            chunk = 1 << 16
            left = self.num_samples
            while left > 0:
                k = min(chunk, left)
                yield from torch.randint(0, self.n, (k,), generator=g).tolist()
                left -= k
        else:
            for i in range(self.num_samples):
                yield (i * self.world + self.rank) % self.n
