"""Final-logit sampling oracle in numpy — test infrastructure only.

Reference algorithms restated here (runtime/model/inference_kernels.py):

* ``counter_uniform``               :24-33  stateless counter hash -> U(0, 1)
* ``sample_cdf``                    :35-40  inverse-CDF pick with a counter uniform
* ``top_k_top_p_distribution``      :42-58
* ``sample_top_k_top_p_counter``    :73-88  (top_k == 1 is greedy argmax)
* ``presence_penalty``              :1104-1114

All hash arithmetic is on uint32 with wrap-around (the reference masks int64
products with 0xFFFFFFFF, which is the same thing).
"""
from __future__ import annotations

import numpy as np

M32 = 0xFFFFFFFF


def counter_uniform(attempt_ids, steps, seed, stream=0, dtype=np.float32):
    ids = np.asarray(attempt_ids).astype(np.int64) & M32
    st = np.asarray(steps).astype(np.int64) & M32
    ids = ids.astype(np.uint64)
    st = np.broadcast_to(st, ids.shape).astype(np.uint64)
    state = (ids * np.uint64(747796405) + st * np.uint64(289133645)
             + np.uint64((int(seed) & M32) * 277803737)
             + np.uint64((int(stream) & M32) * 144269504)) & np.uint64(M32)
    shift = (state >> np.uint64(28)) + np.uint64(4)
    word = (((state >> shift) ^ state) * np.uint64(277803737)) & np.uint64(M32)
    word = ((word >> np.uint64(22)) ^ word) & np.uint64(M32)
    u = ((word.astype(np.float64) + 0.5) / 4294967296.0).astype(dtype)
    limit = dtype(1.0 - np.finfo(dtype).eps / 2)
    return np.minimum(u, limit)


def sample_cdf(probabilities, attempt_ids, steps, seed, stream=0):
    """First index whose running sum reaches ``u * total`` (clamped just below
    the total), per row."""
    p = np.asarray(probabilities, dtype=np.float32)
    cum = np.cumsum(p, axis=-1, dtype=np.float32)
    total = cum[:, -1:]
    u = counter_uniform(attempt_ids, steps, seed, stream, dtype=np.float32)[:, None]
    threshold = np.minimum(u * total, np.nextafter(total, np.float32(0)))
    return np.array([[np.searchsorted(cum[r], threshold[r, 0], side='left')] for r in range(p.shape[0])],
                    dtype=np.int64)


def _topk(values, k):
    """Top-k per row, larger first; equal values in ascending index order."""
    order = np.argsort(-values, axis=-1, kind='stable')[:, :k]
    return np.take_along_axis(values, order, -1), order


def top_k_top_p_distribution(scores, temperature, top_k, top_p):
    s = np.asarray(scores, dtype=np.float32)
    if temperature == 1.0:
        vals, idx = _topk(s, top_k)
    else:
        vals, idx = _topk(s / np.float32(temperature), top_k)
    vals = vals.astype(np.float32)
    e = np.exp(vals - vals.max(-1, keepdims=True))
    probs = e / e.sum(-1, keepdims=True)
    keep = (np.cumsum(probs, -1, dtype=np.float32) - probs) < np.float32(top_p)
    probs = probs * keep
    probs = probs / probs.sum(-1, keepdims=True)
    return idx, probs.astype(np.float32)


def greedy(scores):
    """Index of the first maximum per row, ``[B, 1]`` int64."""
    return np.argmax(np.asarray(scores, dtype=np.float32), axis=-1)[:, None].astype(np.int64)


def sample_top_k_top_p_counter(scores, attempt_ids, steps, seed, temperature, top_k, top_p, stream=0):
    s = np.asarray(scores, dtype=np.float32)
    if top_k <= 0 and top_p == 1.0:
        z = s / np.float32(temperature)
        e = np.exp(z - z.max(-1, keepdims=True))
        return sample_cdf(e / e.sum(-1, keepdims=True), attempt_ids, steps, seed, stream)
    if top_k == 1:
        return greedy(s)
    idx, probs = top_k_top_p_distribution(s, temperature, top_k if top_k > 0 else s.shape[-1], top_p)
    ranks = sample_cdf(probs / probs.sum(-1, keepdims=True), attempt_ids, steps, seed, stream)
    return np.take_along_axis(idx, ranks, 1).astype(np.int64)


def presence_penalty(scores, seen, penalty):
    s = np.asarray(scores, dtype=np.float32)
    return s - np.float32(penalty) * np.asarray(seen, dtype=np.float32)
