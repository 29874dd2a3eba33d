"""Sliding-window attention decode over the physical ring cache, in numpy —
test infrastructure only.

Reference algorithms restated here (paths inside the reference project):

* ``ring_update``        runtime/model/inference_kernels.py:1828-1879: the
  new token's key / value go to ring position ``index`` of every (row, KV
  head), its validity to ``valid[:, index]``, then ``index`` advances
  modulo the ring width (one index for the whole batch);
* ``decode_attention``   runtime/model/inference_kernels.py:1881-1897: one
  query per row attends to every ring position (softmax over the positions
  whose ``valid`` is set), scale ``D ** -0.5``, grouped-query (query head
  ``h`` reads KV head ``h // (QH / KVH)``).

Shapes: query ``[B, 1, QH, D]``; ring key / value ``[B, KVH, W, D]``; valid
``[B, W]`` bool; new key / value ``[B, KVH, 1, D]``, new valid ``[B, 1]``.
"""
from __future__ import annotations

import numpy as np


def ring_update(ring_key, ring_value, ring_valid, index, key, value, valid):
    """Returns (ring_key, ring_value, ring_valid, next_index) after one write."""
    rk, rv, rval = np.array(ring_key), np.array(ring_value), np.array(ring_valid)
    i = int(index)
    rk[:, :, i] = np.asarray(key)[:, :, 0]
    rv[:, :, i] = np.asarray(value)[:, :, 0]
    rval[:, i] = np.asarray(valid)[:, 0]
    W = rk.shape[2]
    return rk, rv, rval, (i + 1) % W


def decode_attention(query, ring_key, ring_value, valid, dtype=np.float64):
    q = np.asarray(query, dtype)[:, 0]                  # [B, QH, D]
    k = np.asarray(ring_key, dtype)
    v = np.asarray(ring_value, dtype)
    B, QH, D = q.shape
    KVH = k.shape[1]
    R = QH // KVH
    kk = np.repeat(k, R, axis=1)                          # [B, QH, W, D]
    vv = np.repeat(v, R, axis=1)
    logits = np.einsum('bhd,bhwd->bhw', q, kk) / np.sqrt(D)
    logits = np.where(np.asarray(valid)[:, None, :], logits, -np.inf)
    m = logits.max(-1, keepdims=True)
    e = np.exp(logits - m)
    w = e / e.sum(-1, keepdims=True)
    return np.einsum('bhw,bhwd->bhd', w, vv)[:, None]     # [B, 1, QH, D]
