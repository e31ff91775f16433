"""Yambda preprocessing (``primus_dlrm/data/preprocessing.py``) on pyarrow + numpy.

raw ``multi_event.parquet`` (uid, item_id, timestamp, event_type, is_organic,
played_ratio_pct, track_length_seconds) ->

* global temporal split (GTS): the last ``test_days`` form the test window,
  a ``gap_minutes`` gap precedes it, and the ``train_days`` before that are
  training; test events are kept only for users seen in training;
* training events segmented into sessions per user at an inactivity gap of
  ``session_gap_seconds``;
* ``train_sessions.parquet``, ``test_events.parquet``, ``session_index.parquet``,
  ``item_popularity.npy`` (train event counts per item), ``split_meta.json``;
  shared metadata files are copied to ``shared_metadata/``.

Large inputs are read in row groups so memory stays bounded.
"""
from __future__ import annotations

import json
import logging
import shutil
from pathlib import Path

import numpy as np

logger = logging.getLogger(__name__)

EVENT_TYPE_MAP = {"listen": 0, "like": 1, "dislike": 2, "unlike": 3, "undislike": 4}
SECONDS_PER_DAY = 86400
_COLS = ("uid", "item_id", "timestamp", "event_type", "is_organic", "played_ratio_pct", "track_length_seconds")


def split_boundaries(t_max: int, train_days: int, gap_minutes: int, test_days: int) -> tuple[int, int, int, int]:
    """(train_start, train_end, test_start, test_end) counted back from t_max."""
    test_end = t_max
    test_start = test_end - test_days * SECONDS_PER_DAY
    train_end = test_start - gap_minutes * 60
    train_start = train_end - train_days * SECONDS_PER_DAY
    return train_start, train_end, test_start, test_end


def _read_events(path: Path) -> dict[str, np.ndarray]:
    import pyarrow.parquet as pq
    pf = pq.ParquetFile(path)
    cols = [c for c in _COLS if c in pf.schema_arrow.names]
    parts = {c: [] for c in cols}
    for rg in range(pf.num_row_groups):
        t = pf.read_row_group(rg, columns=cols)
        for c in cols:
            col = t.column(c)
            if c == "event_type" and str(col.type) in ("string", "large_string") or \
                    (c == "event_type" and "dictionary" in str(col.type)):
                vals = np.array([EVENT_TYPE_MAP[v] for v in col.to_pylist()], np.uint8)
            else:
                vals = col.to_numpy(zero_copy_only=False)
            parts[c].append(vals)
    ev = {c: np.concatenate(v) if v else np.zeros(0) for c, v in parts.items()}
    n = ev["uid"].size
    ev.setdefault("is_organic", np.zeros(n, np.int8))
    ev.setdefault("played_ratio_pct", np.zeros(n, np.float32))
    ev.setdefault("track_length_seconds", np.zeros(n, np.float32))
    return ev


def _take(ev: dict, m: np.ndarray) -> dict:
    return {k: v[m] for k, v in ev.items()}


def build_sessions(ev: dict, gap_s: int):
    """Session id per event (per user, time ordered) and the session table columns."""
    order = np.lexsort((ev["timestamp"], ev["uid"]))
    ev = {k: v[order] for k, v in ev.items()}
    uid, ts = ev["uid"], ev["timestamp"]
    new_user = np.concatenate([[True], uid[1:] != uid[:-1]]) if uid.size else np.zeros(0, bool)
    gap = np.concatenate([[0], np.diff(ts)]) > gap_s
    brk = new_user | gap
    sess_global = np.cumsum(brk) - 1                        # global session number
    user_first_sess = np.maximum.accumulate(np.where(new_user, sess_global, 0))
    session_id = sess_global - user_first_sess              # 0.. within each user
    starts = np.flatnonzero(brk)
    return ev, session_id, starts


def preprocess(raw_dir: str | Path, out_dir: str | Path, dataset_size: str = "50m", session_gap_seconds: int = 1800,
               train_days: int = 300, gap_minutes: int = 30, test_days: int = 1,
               metadata_out: str | Path | None = None) -> Path:
    import pyarrow as pa
    import pyarrow.parquet as pq
    raw_dir, out_dir = Path(raw_dir), Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    ev = _read_events(raw_dir / dataset_size / "multi_event.parquet")
    n = ev["uid"].size
    logger.info("loaded %d events", n)
    t_min, t_max = int(ev["timestamp"].min()), int(ev["timestamp"].max())
    tr0, tr1, te0, te1 = split_boundaries(t_max, train_days, gap_minutes, test_days)
    train = _take(ev, (ev["timestamp"] >= tr0) & (ev["timestamp"] < tr1))
    test = _take(ev, (ev["timestamp"] >= te0) & (ev["timestamp"] < te1))
    test = _take(test, np.isin(test["uid"], np.unique(train["uid"])))
    sev, sid, starts = build_sessions(train, session_gap_seconds)
    ends = np.concatenate([starts[1:], [sev["uid"].size]]).astype(np.int64)
    offsets = pa.array(np.concatenate([starts, [sev["uid"].size]]).astype(np.int32))

    def lst(a):
        return pa.ListArray.from_arrays(offsets, pa.array(a))
    sessions = pa.table({
        "uid": pa.array(sev["uid"][starts]), "session_id": pa.array(sid[starts].astype(np.int64)),
        "item_ids": lst(sev["item_id"]), "timestamps": lst(sev["timestamp"]), "event_types": lst(sev["event_type"]),
        "is_organic": lst(sev["is_organic"]), "played_ratio_pct": lst(sev["played_ratio_pct"]),
        "track_length_seconds": lst(sev["track_length_seconds"])})
    pq.write_table(sessions, out_dir / "train_sessions.parquet")
    pq.write_table(pa.table({k: pa.array(v) for k, v in test.items() if k != "track_length_seconds"}),
                   out_dir / "test_events.parquet")
    lens = ends - starts
    su = sev["uid"][starts]
    ubreak = np.flatnonzero(np.concatenate([[True], su[1:] != su[:-1]])) if su.size else np.zeros(0, np.int64)
    uoff = pa.array(np.concatenate([ubreak, [su.size]]).astype(np.int32))
    cum = np.zeros_like(lens)
    for a, b in zip(ubreak, np.concatenate([ubreak[1:], [su.size]])):
        cum[a:b] = np.cumsum(lens[a:b])
    index = pa.table({"uid": pa.array(su[ubreak]),
                      "session_ids": pa.ListArray.from_arrays(uoff, pa.array(sid[starts].astype(np.int64))),
                      "session_lens": pa.ListArray.from_arrays(uoff, pa.array(lens)),
                      "session_offsets": pa.ListArray.from_arrays(uoff, pa.array(cum))})
    pq.write_table(index, out_dir / "session_index.parquet")
    n_items = int(max(ev["item_id"].max() if n else 0, 0)) + 1
    pop = np.bincount(train["item_id"].astype(np.int64), minlength=n_items).astype(np.int64)
    np.save(out_dir / "item_popularity.npy", pop)
    meta_dst = Path(metadata_out) if metadata_out else out_dir.parent / "shared_metadata"
    meta_dst.mkdir(parents=True, exist_ok=True)
    for f in ("embeddings.parquet", "artist_item_mapping.parquet", "album_item_mapping.parquet"):
        for src in (raw_dir / f, raw_dir / dataset_size / f):
            if src.exists() and not (meta_dst / f).exists():
                shutil.copy(src, meta_dst / f)
    meta = {"t_min": t_min, "t_max": t_max, "train_start": tr0, "train_end": tr1, "test_start": te0,
            "test_end": te1, "train_days": train_days, "gap_minutes": gap_minutes, "test_days": test_days,
            "session_gap_seconds": session_gap_seconds, "num_train_events": int(train["uid"].size),
            "num_test_events": int(test["uid"].size), "num_sessions": int(starts.size),
            "num_users": int(ubreak.size)}
    with open(out_dir / "split_meta.json", "w") as f:
        json.dump(meta, f, indent=2)
    logger.info("preprocessing done: %s", meta)
    return out_dir
