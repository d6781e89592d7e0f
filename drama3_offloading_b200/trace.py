"""Synthetic router traces for the offloaded-decode and fetch benchmarks.

The reference measures its cache on real router traces
(``notes/route-trace-512.json``, written by ``RouterTrace`` in
``bin/offload.py:44-79``) and replays them offline in
``bin/simulate_cache.py:64-97``.  Real traces need the 37 GiB checkpoint, so the
benchmarks here use a seeded synthetic stand-in with the same shape: per layer,
expert popularity follows Zipf(s) over a seeded permutation of the experts, and
each decode step draws top-k experts *without replacement* by the Gumbel-top-k
trick (exact sampling without replacement from the Zipf weights).  The order of
the k ids in a row is descending perturbed score, which is the order a sorted
``torch.topk`` returns and therefore the order the slot allocator sees them.

Layout: ``int16 [steps, layers, k]``.  Deterministic for a given seed.
"""
from __future__ import annotations

import numpy as np

__all__ = ["zipf_trace", "TRACE_SEED"]

TRACE_SEED = 0


def zipf_trace(steps: int = 4096, layers: int = 40, experts: int = 256, k: int = 8,
               s: float = 1.1, seed: int = TRACE_SEED, chunk: int = 512) -> np.ndarray:
    """Return an ``int16 [steps, layers, k]`` routing trace.

    ``p(rank r) ∝ r^-s`` over ``rng.permutation(experts)`` drawn once per layer,
    then per (step, layer) ``ids = perm[argsort(-(log p + Gumbel))[:k]]``.
    """
    if not (0 < k <= experts):
        raise ValueError(f"need 0 < k <= experts, got k={k} experts={experts}")
    rng = np.random.default_rng(seed)
    perms = np.stack([rng.permutation(experts) for _ in range(layers)]).astype(np.int64)
    logp = -s * np.log(np.arange(1, experts + 1, dtype=np.float64))
    out = np.empty((steps, layers, k), dtype=np.int16)
    for lo in range(0, steps, chunk):
        hi = min(steps, lo + chunk)
        keys = logp[None, None, :] + rng.gumbel(size=(hi - lo, layers, experts))
        # top-k ranks, then order them by descending key (sorted topk order)
        part = np.argpartition(-keys, k - 1, axis=-1)[..., :k]
        pk = np.take_along_axis(keys, part, axis=-1)
        order = np.argsort(-pk, axis=-1, kind="stable")
        ranks = np.take_along_axis(part, order, axis=-1)
        ids = np.take_along_axis(np.broadcast_to(perms[None], (hi - lo, layers, experts)),
                                 ranks, axis=-1)
        out[lo:hi] = ids.astype(np.int16)
    return out


def uniform_trace(steps: int, tokens: int, layers: int = 40, experts: int = 256, k: int = 8,
                  seed: int = 1) -> np.ndarray:
    """Uniform-random top-k without replacement, ``int16 [steps, layers, tokens, k]``
    (the expert-parallel resident configuration routes uniformly)."""
    rng = np.random.default_rng(seed)
    out = np.empty((steps, layers, tokens, k), dtype=np.int16)
    for s in range(steps):
        keys = rng.random((layers, tokens, experts))
        out[s] = np.argpartition(keys, k - 1, axis=-1)[..., :k]
    return out
