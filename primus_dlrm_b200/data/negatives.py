"""Negative samplers (``primus_dlrm/data/negatives.py``; deprecated by the
reference's config but kept for API parity): uniform, popularity-weighted,
and a uniform/popularity mixture, each without replacement and with an
optional exclusion set."""
from __future__ import annotations

import numpy as np


class NegativeSampler:
    def __init__(self, num_items: int, seed: int = 42):
        self.num_items = num_items
        self.rng = np.random.default_rng(seed)
        self.probs: np.ndarray | None = None

    def sample(self, n: int, exclude: set[int] | None = None) -> np.ndarray:
        if not exclude:
            return self.rng.choice(self.num_items, size=n, replace=False, p=self.probs).astype(np.int64)
        # draw without replacement from the allowed ids, renormalising weights
        allowed = np.setdiff1d(np.arange(self.num_items), np.fromiter(exclude, dtype=np.int64))
        p = None
        if self.probs is not None:
            p = self.probs[allowed]
            p = p / p.sum()
        k = min(n, allowed.size)
        return self.rng.choice(allowed, size=k, replace=False, p=p).astype(np.int64)


class UniformSampler(NegativeSampler):
    pass


class PopularitySampler(NegativeSampler):
    def __init__(self, num_items: int, item_counts: np.ndarray, seed: int = 42):
        super().__init__(num_items, seed)
        c = np.asarray(item_counts, dtype=np.float64)
        self.probs = c / c.sum()


class MixedSampler(NegativeSampler):
    def __init__(self, num_items: int, item_counts: np.ndarray, uniform_ratio: float = 0.5, seed: int = 42):
        super().__init__(num_items, seed)
        self.uniform_ratio = uniform_ratio
        self.uniform = UniformSampler(num_items, seed=seed)
        self.popularity = PopularitySampler(num_items, item_counts, seed=seed + 1)

    def sample(self, n: int, exclude: set[int] | None = None) -> np.ndarray:
        nu = int(n * self.uniform_ratio)
        out = np.concatenate([self.uniform.sample(nu, exclude), self.popularity.sample(n - nu, exclude)])
        self.rng.shuffle(out)
        return out
