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
  ``h`` reads KV head ``h // (QH / KVH)``); a row with no valid position
  gives zeros, as torch's SDPA does for a fully masked row (torch >= 2.5,
  the version the reference runs on here);
* ``prefill_attention``  modeling_yanchor.py:412-427 (``reference_swa``):
  causal sliding-window attention of a prompt, absolute positions, optional
  key validity and a query offset (keys of a cached window before the
  prompt);
* ``flash_prefill``      modeling_yanchor.py:429-449 (``flash_swa``): the
  same over each row's valid tokens in order (the window counts valid
  tokens).

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
    any_valid = np.asarray(valid).any(-1)[:, None, None]
    logits = np.where(np.asarray(valid)[:, None, :], logits, -np.inf)
    logits = np.where(any_valid, logits, 0.0)             # fully masked rows: weights 0 below
    m = logits.max(-1, keepdims=True)
    e = np.exp(logits - m)
    w = np.where(any_valid, e / e.sum(-1, keepdims=True), 0.0)
    return np.einsum('bhw,bhwd->bhd', w, vv)[:, None]     # [B, 1, QH, D]


def prefill_attention(query, key, value, window, key_valid=None, query_start=0, dtype=np.float64):
    """modeling_yanchor.py:412-427 (``reference_swa``): queries ``[B, Tq, QH, D]``
    at absolute positions ``query_start .. query_start + Tq - 1`` attend to keys
    ``[B, Tk, KVH, D]`` at positions ``0 .. Tk - 1`` with ``q_pos - window < k_pos
    <= q_pos`` and ``key_valid[b, k_pos]``; scale ``D ** -0.5``, grouped-query;
    the output of a query whose own ``key_valid`` entry is False is zero.  A row
    with no admitted key gives zeros."""
    q = np.asarray(query, dtype)
    k = np.asarray(key, dtype)
    v = np.asarray(value, dtype)
    B, Tq, QH, D = q.shape
    Tk, KVH = k.shape[1], k.shape[2]
    R = QH // KVH
    qpos = np.arange(Tq) + int(query_start)
    kpos = np.arange(Tk)
    allowed = (kpos[None, :] <= qpos[:, None]) & (kpos[None, :] >= qpos[:, None] - int(window) + 1)
    allowed = np.broadcast_to(allowed, (B, Tq, Tk))
    if key_valid is not None:
        allowed = allowed & np.asarray(key_valid, bool)[:, None, :]
    kk = np.repeat(k, R, axis=2).transpose(0, 2, 3, 1)             # [B, QH, D, Tk]
    vv = np.repeat(v, R, axis=2).transpose(0, 2, 1, 3)             # [B, QH, Tk, D]
    logits = np.matmul(q.transpose(0, 2, 1, 3), kk) / np.sqrt(D)    # [B, QH, Tq, Tk]
    logits = np.where(allowed[:, None], logits, -np.inf)
    m = logits.max(-1, keepdims=True)
    e = np.where(np.isfinite(m), np.exp(logits - np.where(np.isfinite(m), m, 0.0)), 0.0)
    den = e.sum(-1, keepdims=True)
    w = np.where(den > 0, e / np.where(den > 0, den, 1.0), 0.0)
    out = np.matmul(w, vv).transpose(0, 2, 1, 3)                   # [B, Tq, QH, D]
    if key_valid is not None:
        qv = np.asarray(key_valid, bool)[:, int(query_start):int(query_start) + Tq]
        out = out * qv[:, :, None, None]
    return out


def flash_prefill(query, key, value, window, attention_mask=None, dtype=np.float64):
    """modeling_yanchor.py:429-449 (``flash_swa``): causal sliding window of
    ``window`` tokens over each row's valid tokens taken in order (the
    reference unpads them into one variable-length batch), so the window
    counts valid tokens only; padded positions give zeros."""
    q = np.asarray(query, dtype)
    B, T = q.shape[:2]
    if attention_mask is None:
        return prefill_attention(query, key, value, window, dtype=dtype)
    mask = np.asarray(attention_mask, bool)[:, -T:]
    out = np.zeros_like(q)
    for b in range(B):
        idx = np.nonzero(mask[b])[0]
        if idx.size == 0:
            continue
        sub = prefill_attention(q[b:b + 1, idx], np.asarray(key, dtype)[b:b + 1, idx],
                                np.asarray(value, dtype)[b:b + 1, idx], window, dtype=dtype)
        out[b, idx] = sub[0]
    return out
