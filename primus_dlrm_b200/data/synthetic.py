"""Seeded synthetic batches of the configured feature schema.

Behaviour of the reference generator (``primus_dlrm/data/synthetic.py``):
uniform ``randint`` ids, uniform dense features, one Bernoulli rate for every
task, one history length, optional variable lengths (``<key>__lengths``).
This module keeps that behaviour as the default and adds the distributions
the benchmark configs name:

* ``id_distribution: zipf`` -- Zipf(alpha) ranks drawn by inverse-CDF of the
  continuous power law, scattered over the id space by a bijective affine map
  ``id = (a * rank + b) mod N`` (``gcd(a, N) = 1``) so hot ids are not all
  small integers;
* ``data.history_lengths`` -- one length per sequence group;
* ``task_positive_rates`` and ``train.regression_tasks`` -- per-task
  Bernoulli rates and U[0,1] regression labels;
* ``dense_distribution`` -- uniform / normal / lognormal.

Ids are emitted as int64 like the reference; the packed host->device batch
(``primus_dlrm_b200.data.batch``) narrows them to int32 on the wire.
"""
from __future__ import annotations

import copy
import logging
import math
from typing import Iterator

import torch
from torch.utils.data import Dataset

from primus_dlrm_b200.config import Config

logger = logging.getLogger(__name__)


def table_size_by_feature(config: Config) -> dict[str, int]:
    out: dict[str, int] = {}
    for t in config.model.embedding_tables:
        for f in t.features:
            out[f] = t.num_embeddings
    return out


def _coprime_multiplier(n: int) -> int:
    """A large odd multiplier coprime with ``n`` (for the rank -> id scatter)."""
    a = 2654435761 % max(n, 1) or 1
    while math.gcd(a, n) != 1:
        a += 1
    return a


def zipf_ids(n_rows: int, shape, alpha: float, gen: torch.Generator,
             lo: int = 0) -> torch.Tensor:
    """Zipf(alpha)-distributed ids in ``[lo, n_rows)``.

    Rank r in [1, N] is drawn from the continuous power law p(x) ~ x^-alpha by
    inverse CDF, then mapped through the bijection r -> (a*r + b) mod N.
    """
    n = max(n_rows - lo, 1)
    u = torch.rand(shape, generator=gen, dtype=torch.float64)
    if abs(alpha - 1.0) < 1e-9:
        x = torch.pow(float(n), u)
    else:
        one_m = 1.0 - alpha
        x = torch.pow((math.pow(n, one_m) - 1.0) * u + 1.0, 1.0 / one_m)
    rank = (x.floor().to(torch.int64) - 1).clamp_(0, n - 1)
    a = _coprime_multiplier(n)
    b = 97 % n
    return (rank * a + b).remainder_(n) + lo


def _draw_ids(n_rows: int, shape, syn, gen: torch.Generator) -> torch.Tensor:
    hi = syn.sparse_id_max if syn.sparse_id_max > 0 else n_rows
    lo = syn.sparse_id_min
    if syn.id_distribution == "zipf":
        return zipf_ids(hi, shape, syn.zipf_alpha, gen, lo=lo)
    return torch.randint(lo, hi, shape, generator=gen)


def _draw_dense(shape, df, syn, gen: torch.Generator) -> torch.Tensor:
    if syn.dense_distribution == "normal":
        return torch.randn(shape, generator=gen)
    if syn.dense_distribution == "lognormal":
        return torch.randn(shape, generator=gen).exp_()
    lo, hi = df.value_range_min, df.value_range_max
    return torch.rand(shape, generator=gen) * (hi - lo) + lo


def _draw_labels(config: Config, task: str, n: int, syn, gen: torch.Generator) -> torch.Tensor:
    if task in config.train.regression_tasks:
        return torch.rand(n, generator=gen)
    rate = syn.task_positive_rates.get(task, syn.label_positive_rate)
    return (torch.rand(n, generator=gen) < rate).float()


def generate_batch(
    config: Config,
    batch_size: int,
    seed: int = 42,
    label_positive_rate: float | None = None,
    sparse_id_min: int | None = None,
    sparse_id_max: int | None = None,
    sparse_len_min: int | None = None,
    sparse_len_max: int | None = None,
) -> dict[str, torch.Tensor]:
    """One full random batch as a dict of CPU tensors.

    Keys follow ``config.feature_to_batch_key()``: scalar ids ``[B]``,
    sequence ids ``[B, L_group]`` (or flat values + ``<key>__lengths`` when a
    variable length range is set), dense ``[B, dim]`` float32, task labels
    ``[B]`` float32.  Reference signature: ``primus_dlrm/data/synthetic.py:195``.
    """
    syn = copy.copy(config.data.synthetic)
    if label_positive_rate is not None:
        syn.label_positive_rate = label_positive_rate
    if sparse_id_min is not None:
        syn.sparse_id_min = sparse_id_min
    if sparse_id_max is not None:
        syn.sparse_id_max = sparse_id_max
    if sparse_len_min is not None:
        syn.sparse_len_min = sparse_len_min
    if sparse_len_max is not None:
        syn.sparse_len_max = sparse_len_max
    gen = torch.Generator().manual_seed(seed)
    sizes = table_size_by_feature(config)
    f2k = config.feature_to_batch_key()
    fc = config.feature
    B = batch_size
    var_len = syn.sparse_len_min > 0 or syn.sparse_len_max > 0
    out: dict[str, torch.Tensor] = {}

    for feat in fc.scalar_feature_names:
        out[f2k.get(feat, feat)] = _draw_ids(sizes[feat], (B,), syn, gen)

    for group, feats in fc.sequence_groups.items():
        L = config.data.group_length(group)
        for feat in feats:
            key = f2k.get(feat, feat)
            if var_len:
                lens = torch.randint(syn.sparse_len_min, syn.sparse_len_max + 1, (B,),
                                     generator=gen, dtype=torch.int32)
                out[key] = _draw_ids(sizes[feat], (int(lens.sum()),), syn, gen)
                out[key + "__lengths"] = lens
            else:
                out[key] = _draw_ids(sizes[feat], (B, L), syn, gen)

    for df in fc.dense_features:
        out[df.name] = _draw_dense((B, df.dim), df, syn, gen)

    for task in config.task_names:
        out[task] = _draw_labels(config, task, B, syn, gen)
    return out


class SyntheticDataset(Dataset):
    """Per-sample synthetic dataset (``primus_dlrm/data/synthetic.py:40-90``).

    Sample ``idx`` is a pure function of ``seed + idx``; ``num_samples <= 0``
    makes the dataset effectively infinite.
    """

    def __init__(self, config: Config):
        self.config = config
        self._syn = config.data.synthetic
        self._infinite = self._syn.num_samples <= 0

    def __len__(self) -> int:
        return 10_000_000 if self._infinite else self._syn.num_samples

    def __getitem__(self, idx: int) -> dict[str, torch.Tensor]:
        b = generate_batch(self.config, 1, seed=self._syn.seed + idx)
        return {k: v[0] if not k.endswith("__lengths") else v for k, v in b.items()}


def collate_synthetic(samples: list[dict[str, torch.Tensor]]) -> dict[str, torch.Tensor]:
    return {k: torch.stack([s[k] for s in samples]) for k in samples[0]}


class SyntheticDataPipe:
    """Infinite iterator of synthetic batches.

    ``num_prebatched > 0`` pre-generates that many batches and cycles over
    them (cheap per step); ``0`` draws a fresh batch every step.
    Reference: ``primus_dlrm/data/synthetic.py:250-311``.
    """

    def __init__(self, config: Config, batch_size: int, num_prebatched: int = 16,
                 seed: int = 42, **kw):
        self._config = config
        self._batch_size = batch_size
        self._seed = seed
        self._kw = kw
        self._idx = 0
        self.sampler = None
        if num_prebatched > 0:
            logger.info("pre-generating %d synthetic batches (B=%d)", num_prebatched, batch_size)
            self._batches = [generate_batch(config, batch_size, seed=seed + i, **kw)
                             for i in range(num_prebatched)]
        else:
            self._batches = None

    def __len__(self) -> int:
        return 10_000_000

    def __iter__(self) -> Iterator[dict[str, torch.Tensor]]:
        return self

    def __next__(self) -> dict[str, torch.Tensor]:
        self._idx += 1
        if self._batches is not None:
            return self._batches[(self._idx - 1) % len(self._batches)]
        return generate_batch(self._config, self._batch_size, seed=self._seed + self._idx, **self._kw)
