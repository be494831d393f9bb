"""Categorical distribution on CUDA (``crates/tynx-python/python/tynx/distributions.py:47-104``).

Logits are normalised with ``log_softmax``; ``probs = exp(logits)``;
``log_prob`` gathers the normalised log-probability of each action;
``entropy = -sum(probs * logits)``.
"""

from __future__ import annotations

from typing import Optional

import numpy as np

from ._core import Tensor


class Categorical:
    def __init__(self, probs: Optional[Tensor] = None, logits: Optional[Tensor] = None):
        if (probs is None) == (logits is None):
            raise ValueError("Categorical requires exactly one of probs or logits")
        if logits is not None:
            self.logits = logits.log_softmax(dim=-1)
            self.probs = self.logits.exp()
        else:
            normalized = probs / probs.sum(dim=-1, keepdim=True)
            self.probs = normalized
            self.logits = normalized.log()

    def log_prob(self, value: Tensor) -> Tensor:
        if value.shape != self.logits.shape[:-1]:
            raise NotImplementedError("Categorical.log_prob on CUDA needs one action per row")
        return self.logits.gather(-1, value.unsqueeze(-1)).squeeze(-1)

    def entropy(self) -> Tensor:
        return -(self.probs * self.logits).sum(dim=-1)

    def sample(self, sample_shape: tuple = (), *, seed: Optional[int] = None) -> Tensor:
        """Detached int64 samples (inverse-CDF on the host from the device probabilities)."""
        probs = self.probs.numpy()
        rng = np.random.default_rng(seed)
        flat = probs.reshape(-1, probs.shape[-1])
        draws = rng.random((int(np.prod(sample_shape)) if sample_shape else 1, flat.shape[0]))
        cdf = np.cumsum(flat, axis=-1)
        idx = (draws[..., None] > cdf[None]).sum(-1).clip(0, flat.shape[-1] - 1)
        out = idx.reshape(tuple(sample_shape) + probs.shape[:-1]).astype(np.int64)
        return Tensor(out, dtype="int64", device=self.probs.device)


__all__ = ["Categorical"]
