"""Anchor-memory (independent GQA memory) oracle in numpy — test infrastructure only.

Reference algorithms restated here (paths inside the reference project):

* ``select_topk`` / ``merge_topk``   modeling_yanchor.py:51-63
* ``exclusive_prefix_topk``          modeling_yanchor.py:65-78
* ``indexed_gqa``                    modeling_yanchor.py:22-42 (torch) and
                                     runtime/model/independent_memory.py:6-45 (Triton)
* ``decode_read``                    modeling_yanchor.py:283-290 (torch) and
                                     runtime/model/independent_memory.py:47-88,177-188
* ``commit_decode``                  modeling_yanchor.py:291-312 (torch) and
                                     runtime/model/independent_memory.py:90-201
* ``sequence`` (prefill read + write) modeling_yanchor.py:178-275

The memory state is a dict with the fields of ``IndependentMemoryState``
(modeling_yanchor.py:80-120): keys/values ``[B, G, CAP, D]``, scores
``[B, G, CAP]`` float32, positions ``[B, G, CAP]`` int32, pending_keys /
pending_values ``[B, G, PC, D]``, pending_scores ``[B, G, PC]`` float32,
count / total ``[B]`` int64.

Ordering used for every top-CAP selection: score descending (NaN first),
then position ascending with invalid entries (reference < 0) last, then
candidate order.
Invalid entries come out as (score -inf, position -1, reference -1).
"""
from __future__ import annotations

import math

import numpy as np

INT64_MAX = np.iinfo(np.int64).max


def select_topk(scores, positions, references, capacity):
    """Top-``capacity`` of the last axis.  Returns (scores, positions, references)."""
    scores = np.asarray(scores, dtype=np.float32)
    references = np.asarray(references, dtype=np.int64)
    positions = np.where(references < 0, -1, np.asarray(positions, dtype=np.int64))
    pos_key = np.where(references < 0, INT64_MAX, positions)
    lead = scores.shape[:-1]
    n = scores.shape[-1]
    flat_s = scores.reshape(-1, n)
    flat_p = pos_key.reshape(-1, n)
    out_s = np.full((flat_s.shape[0], capacity), -math.inf, dtype=np.float32)
    out_p = np.full((flat_s.shape[0], capacity), -1, dtype=np.int64)
    out_r = np.full((flat_s.shape[0], capacity), -1, dtype=np.int64)
    flat_pos = positions.reshape(-1, n)
    flat_ref = references.reshape(-1, n)
    idx = np.arange(n)
    take = min(capacity, n)
    for row in range(flat_s.shape[0]):
        # np.lexsort: last key is primary.  NaN scores rank first and tie with
        # each other (torch's descending sort treats NaN as the largest value);
        # -score puts larger scores first; -0.0 and 0.0 compare equal, as in a
        # stable float sort.
        nan = np.isnan(flat_s[row])
        order = np.lexsort((idx, flat_p[row], np.where(nan, 0.0, -flat_s[row]), ~nan))[:take]
        out_s[row, :take] = flat_s[row, order]
        out_p[row, :take] = flat_pos[row, order]
        out_r[row, :take] = flat_ref[row, order]
    shape = lead + (capacity,)
    return out_s.reshape(shape), out_p.reshape(shape), out_r.reshape(shape)


def merge_topk(left, right, capacity):
    return select_topk(*(np.concatenate((a, b), -1) for a, b in zip(left, right)), capacity)


def exclusive_prefix_topk(scores, positions, references, capacity):
    """Inputs ``[B, blocks, G, chunk]``; output ``[B, blocks + 1, G, capacity]``
    where entry ``i`` is the top-``capacity`` over blocks ``0 .. i-1`` and entry
    ``blocks`` covers every block."""
    scores = np.asarray(scores, dtype=np.float32)
    B, blocks, G, chunk = scores.shape
    out = []
    empty = (np.full((B, G, capacity), -math.inf, np.float32),
             np.full((B, G, capacity), -1, np.int64), np.full((B, G, capacity), -1, np.int64))
    acc = empty
    out.append(acc)
    for i in range(blocks):
        acc = merge_topk(acc, (scores[:, i], positions[:, i], references[:, i]), capacity)
        out.append(acc)
    return tuple(np.stack([o[j] for o in out], 1) for j in range(3))


def _softmax_with_null(logits):
    """Softmax over ``logits`` plus one extra logit 0 (the null slot whose value
    is zero); returns the weights of the real entries only."""
    m = np.maximum(np.max(logits, axis=-1, keepdims=True), 0.0)
    e = np.exp(logits - m)
    den = e.sum(-1, keepdims=True) + np.exp(-m)
    return e / den


def indexed_gqa(query, key, value, references):
    """Prefill anchor read.  query ``[B, blocks, chunk, H, D]``; key / value
    ``[KB, S, G, D]`` (KB is 1 or B); references ``[B, blocks, G, CAP]`` int64
    (-1 = empty).  Each query row attends to its group's referenced rows plus
    the always-valid null slot, with scale ``D ** -0.5``."""
    q = np.asarray(query, dtype=np.float32)
    kk = np.asarray(key, dtype=np.float32)
    vv = np.asarray(value, dtype=np.float32)
    refs = np.asarray(references, dtype=np.int64)
    B, blocks, chunk, H, D = q.shape
    G, CAP = refs.shape[-2:]
    R = H // G
    out = np.zeros_like(q)
    for b in range(B):
        kb = 0 if kk.shape[0] == 1 else b
        for blk in range(blocks):
            for g in range(G):
                r = refs[b, blk, g]
                valid = r >= 0
                keys = kk[kb, np.clip(r, 0, None), g]          # [CAP, D]
                vals = vv[kb, np.clip(r, 0, None), g]
                qs = q[b, blk, :, g * R:(g + 1) * R]            # [chunk, R, D]
                logits = (qs @ keys.T) / math.sqrt(D)
                logits = np.where(valid, logits, -np.inf)
                w = _softmax_with_null(logits)
                out[b, blk, :, g * R:(g + 1) * R] = w @ vals
    return out


def decode_read(query, keys, values, positions, indices=None):
    """Decode anchor read.  query ``[B, 1, H, D]``; keys / values
    ``[BS, G, CAP, D]``; positions ``[BS, G, CAP]`` (< 0 = empty slot).
    ``indices`` (optional, ``[B]``) maps row -> state row, -1 = skip (zeros)."""
    q = np.asarray(query, dtype=np.float32)
    K = np.asarray(keys, dtype=np.float32)
    Vv = np.asarray(values, dtype=np.float32)
    P = np.asarray(positions)
    B, _, H, D = q.shape
    G = K.shape[1]
    R = H // G
    out = np.zeros_like(q)
    for b in range(B):
        s = b if indices is None else int(indices[b])
        if s < 0:
            continue
        for g in range(G):
            qs = q[b, 0, g * R:(g + 1) * R]                     # [R, D]
            logits = qs @ K[s, g].T / math.sqrt(D)
            logits = np.where(P[s, g][None, :] < 0, -np.inf, logits)
            w = _softmax_with_null(logits)
            out[b, 0, g * R:(g + 1) * R] = w @ Vv[s, g]
    return out


def commit_decode(key, value, scores, active, chunk, state, indices=None):
    """Decode write: push (key, value, score) into the pending slot ``count``;
    when the pending chunk fills (``count + 1 == chunk``) merge bank and pending
    into a new top-CAP bank; advance count / total.  Mutates ``state`` (a dict
    of numpy arrays) in place."""
    key = np.asarray(key)
    value = np.asarray(value)
    scores = np.asarray(scores, dtype=np.float32)
    active = np.asarray(active, dtype=bool)
    B = key.shape[0]
    G, CAP = state['keys'].shape[1:3]
    for row in range(B):
        s = row if indices is None else int(indices[row])
        if s < 0 or not active[row]:
            continue
        count = int(state['count'][s])
        total = int(state['total'][s])
        state['pending_keys'][s, :, count] = key[row, 0]
        state['pending_values'][s, :, count] = value[row, 0]
        state['pending_scores'][s, :, count] = scores[row, 0]
        nxt = count + 1
        if nxt == chunk:
            for g in range(G):
                bank_ref = np.where(state['positions'][s, g] < 0, -1, np.arange(CAP))
                pidx = np.arange(chunk)
                p_scores = np.where(pidx >= nxt, -np.inf, state['pending_scores'][s, g, :chunk])
                p_pos = total - count + pidx
                p_ref = np.where(pidx >= nxt, -1, pidx + CAP)
                sel_s, sel_p, sel_r = merge_topk(
                    (state['scores'][s, g], state['positions'][s, g], bank_ref),
                    (p_scores, p_pos, p_ref), CAP)
                src_k = np.concatenate((state['keys'][s, g], state['pending_keys'][s, g, :chunk]), 0)
                src_v = np.concatenate((state['values'][s, g], state['pending_values'][s, g, :chunk]), 0)
                pick = np.clip(sel_r, 0, None)
                state['keys'][s, g] = src_k[pick]
                state['values'][s, g] = src_v[pick]
                state['scores'][s, g] = sel_s
                state['positions'][s, g] = sel_p.astype(state['positions'].dtype)
            state['count'][s] = 0
        else:
            state['count'][s] = nxt
        state['total'][s] = total + 1
    return state


def empty_state(batch, groups, capacity, pending, dim, dtype=np.float32):
    """Fresh state, as ``IndependentMemoryState.empty`` (modeling_yanchor.py:92-96)."""
    return {
        'keys': np.zeros((batch, groups, capacity, dim), dtype),
        'values': np.zeros((batch, groups, capacity, dim), dtype),
        'scores': np.full((batch, groups, capacity), -np.inf, np.float32),
        'positions': np.full((batch, groups, capacity), -1, np.int32),
        'pending_keys': np.zeros((batch, groups, pending, dim), dtype),
        'pending_values': np.zeros((batch, groups, pending, dim), dtype),
        'pending_scores': np.full((batch, groups, pending), -np.inf, np.float32),
        'count': np.zeros((batch,), np.int64),
        'total': np.zeros((batch,), np.int64),
    }


def sequence(query, scores, key_all, value_all, valid, chunk, state=None, capacity=None):
    """Prefill anchor read and write, ``IndependentGQAMemory._sequence``
    (modeling_yanchor.py:178-275), restated step by step.

    query ``[B, T, H, D]``; scores ``[B, T, G]`` float32; ``key_all`` /
    ``value_all`` ``[B, T, G, D]``: the writer's key / value for every token
    (the reference evaluates the writer only on the tokens it keeps; the
    writer works row by row, so those rows are the same); ``valid`` ``[B, T]``
    bool or None; ``state``: a state dict (mutated in place) or None, in which
    case ``capacity`` gives CAP and nothing is written.  Returns the read
    ``[B, T, H, D]``.

    The prompt is laid on a timeline of ``extent`` slots: with a state, the
    first ``count`` slots are the state's pending tokens and the new tokens
    follow.  Each chunk-sized block of the timeline reads the top-CAP of the
    blocks before it (plus the state's bank); only tokens that some block can
    read, or that stay pending afterwards, get a key / value row.
    """
    q_in = np.asarray(query, np.float32)
    s_in = np.asarray(scores, np.float32)
    B, T, H, D = q_in.shape
    G = s_in.shape[-1]
    CAP = state['keys'].shape[2] if state is not None else int(capacity)
    bi = np.arange(B)[:, None]
    if valid is None:
        order = None
        q, s = q_in, s_in
        counts = np.full(B, T, np.int64)
    else:
        valid = np.asarray(valid, bool)
        order = np.argsort(~valid, axis=1, kind='stable')          # valid tokens first, stable
        q, s = q_in[bi, order], s_in[bi, order]
        counts = valid.sum(1).astype(np.int64)
    old_count = np.zeros(B, np.int64) if state is None else state['count'].astype(np.int64)
    old_total = np.zeros(B, np.int64) if state is None else state['total'].astype(np.int64)
    prefix_length = 0 if state is None else chunk
    extent = -(-(T + prefix_length) // chunk) * chunk
    at = np.arange(extent)[None, :].repeat(B, 0)
    limit = old_count + counts
    valid_extent = at < limit[:, None]
    if state is None:
        q = np.concatenate((q, np.zeros((B, extent - T, H, D), np.float32)), 1)
        s = np.concatenate((s, np.full((B, extent - T, G), -np.inf, np.float32)), 1)
        shift = 0
    else:
        select = np.where(at < old_count[:, None], at, chunk + at - old_count[:, None])
        select = np.minimum(select, chunk + T - 1)
        q = np.concatenate((np.zeros((B, chunk, H, D), np.float32), q), 1)[bi, select]
        pend = np.asarray(state['pending_scores'], np.float32).transpose(0, 2, 1)[:, :chunk]
        s = np.concatenate((pend, s), 1)[bi, select]
        shift = CAP
    s = np.where(valid_extent[..., None], s, -np.inf).astype(np.float32)
    positions = (old_total - old_count)[:, None] + at
    refs = np.where(valid_extent, at + shift, -1)
    blocks = extent // chunk

    def blocked(x):
        x = x if x.ndim == 3 else np.repeat(x[..., None], G, -1)
        return x.reshape(B, blocks, chunk, G).transpose(0, 1, 3, 2)

    prefix = exclusive_prefix_topk(blocked(s), blocked(positions), blocked(refs), CAP)
    if state is not None:
        bank_ref = np.where(state['positions'] < 0, -1, np.arange(CAP)[None, None])
        initial = (state['scores'], state['positions'], bank_ref)
        prefix = merge_topk(prefix, tuple(np.repeat(x[:, None], blocks + 1, 1) for x in initial), CAP)
    boundary = (np.arange(1, blocks + 1) * chunk)[None, :, None, None]
    entrant = prefix[2][:, 1:] - shift
    if state is None:
        used = boundary < limit[:, None, None, None]
    else:
        used = boundary <= limit[:, None, None, None]
    take = (entrant >= boundary - chunk) & (entrant < boundary) & used
    needed = np.zeros((B, extent + 1), bool)
    target = np.where(take, entrant, extent).reshape(B, -1)
    needed[np.repeat(np.arange(B), target.shape[1]), target.ravel()] = True
    if state is not None:
        full = limit // chunk
        needed[:, :extent] |= valid_extent & (at >= full[:, None] * chunk)
    needed = needed[:, :extent] & valid_extent & (at >= old_count[:, None])
    sel_b, sel_pos = np.nonzero(needed)
    original = sel_pos - old_count[sel_b]
    if order is not None:
        original = order[sel_b, original]
    k = np.asarray(key_all)[sel_b, original]
    v = np.asarray(value_all)[sel_b, original]
    references = np.full((B, shift + extent), -1, np.int64)
    source_k, source_v = k, v
    offset = 0
    if state is not None:
        offset = B * (CAP + chunk)
        old_k = np.concatenate((state['keys'], state['pending_keys'][:, :, :chunk]), 2).transpose(0, 2, 1, 3)
        old_v = np.concatenate((state['values'], state['pending_values'][:, :, :chunk]), 2).transpose(0, 2, 1, 3)
        source_k = np.concatenate((old_k.reshape(-1, G, D), k), 0)
        source_v = np.concatenate((old_v.reshape(-1, G, D), v), 0)
        base = np.arange(B)[:, None] * (CAP + chunk)
        references[:, :shift] = base + np.arange(shift)[None]
        references[:, shift:] = np.where(at < old_count[:, None], base + CAP + at, -1)
    references[sel_b, shift + sel_pos] = offset + np.arange(len(k))
    zero = np.zeros((1, G, D), source_k.dtype)
    source_k = np.concatenate((source_k, zero), 0)
    source_v = np.concatenate((source_v, zero), 0)
    pre_refs = prefix[2][:, :-1]
    read_refs = np.where(pre_refs < 0, -1, references[np.arange(B)[:, None, None, None], np.maximum(pre_refs, 0)])
    read = indexed_gqa(q.reshape(B, blocks, chunk, H, D), source_k[None], source_v[None], read_refs)
    read = read.reshape(B, extent, H, D)
    if state is None:
        output = read[:, :T]
    else:
        output = read[bi, np.minimum(old_count[:, None] + np.arange(T)[None], extent - 1)]
    if order is not None:
        output = output[bi, np.argsort(order, axis=1)] * valid[..., None, None]
    if state is not None:
        rows = np.arange(B)
        score, position, reference = (x[rows, full] for x in prefix)       # [B, G, CAP]
        g = np.arange(G)[None, :, None]
        compact = references[rows[:, None, None], np.maximum(reference, 0)]
        empty = (reference < 0)[..., None]
        state['keys'][...] = np.where(empty, 0, source_k[np.maximum(compact, 0), g])
        state['values'][...] = np.where(empty, 0, source_v[np.maximum(compact, 0), g])
        state['scores'][...] = score
        state['positions'][...] = position
        pc = state['pending_keys'].shape[2]
        pending = full[:, None] * chunk + np.arange(pc)[None]
        remaining = limit % chunk
        mask = np.arange(pc)[None] < remaining[:, None]
        pending = np.minimum(pending, extent - 1)
        compact = np.maximum(references[bi, pending + shift], 0)
        state['pending_keys'][...] = np.where(mask[..., None, None], source_k[compact], 0).transpose(0, 2, 1, 3)
        state['pending_values'][...] = np.where(mask[..., None, None], source_v[compact], 0).transpose(0, 2, 1, 3)
        state['pending_scores'][...] = np.where(mask[..., None], s[bi, pending], -np.inf).transpose(0, 2, 1)
        state['count'][...] = remaining
        state['total'][...] = old_total + counts
    return output.astype(np.float32)
