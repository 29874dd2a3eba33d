"""Prefill side of the anchor memory: top-CAP selection and the prefill
read / write orchestration, with the reference's call signatures.

    select_topk(scores, positions, references, capacity)       modeling_yanchor.py:51-60
    merge_topk(left, right, capacity)                           modeling_yanchor.py:62-63
    exclusive_prefix_topk(scores, positions, references, capacity, initial=None)
                                                                modeling_yanchor.py:65-78
    sequence(query, scores, write_kv, valid, chunk, state=None, capacity=None)
                                                                modeling_yanchor.py:178-275

The selections run on libyanchor_b200.so's sort / merge kernels and the read
on its indexed-read kernel, which addresses the prompt's own query and output
through the timeline; the index work between them (timeline, slot table,
read references, new state) runs on its prefill orchestration kernels.
There is no CPU path.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._torch import dtype_code, require_cuda, stream_ptr
from .independent_memory import indexed_gqa

_I32, _I64 = 3, 4   # yb_dtype codes for positions


def _positions(p: torch.Tensor):
    if p.dtype == torch.int32:
        return p.contiguous(), _I32
    return p.to(torch.int64).contiguous(), _I64


def select_topk(scores, positions, references, capacity):
    """Top-``capacity`` along the last axis: score descending (NaN first),
    then position ascending with invalid references (< 0) last, then index.
    Returns (scores, positions int64 with -1 where the reference is < 0,
    references), each ``lead + (capacity,)``; short rows are padded with
    (-inf, -1, -1)."""
    require_cuda(scores, positions, references)
    if not (scores.shape == positions.shape == references.shape):
        raise ValueError('scores, positions and references must share a shape')
    capacity = int(capacity)
    lead, n = scores.shape[:-1], scores.shape[-1]
    s32 = scores.to(torch.float32).contiguous()
    pos, pcode = _positions(positions)
    refs = references.to(torch.int64).contiguous()
    rows = math.prod(lead)
    out_s = torch.empty(lead + (capacity,), device=scores.device, dtype=torch.float32)
    out_p = torch.empty(lead + (capacity,), device=scores.device, dtype=torch.int64)
    out_r = torch.empty(lead + (capacity,), device=scores.device, dtype=torch.int64)
    rc = _lib.lib().yb_mem_select_topk(s32.data_ptr(), pos.data_ptr(), pcode, refs.data_ptr(), rows, n, capacity,
                                       out_s.data_ptr(), out_p.data_ptr(), out_r.data_ptr(),
                                       stream_ptr(scores.device))
    _lib.check(rc, 'select_topk')
    return out_s.to(scores.dtype), out_p, out_r.to(references.dtype)


def merge_topk(left, right, capacity):
    """Top-``capacity`` of two candidate sets (the concatenation along the
    last axis, ``left`` first)."""
    return select_topk(*(torch.cat((a, b), -1) for a, b in zip(left, right)), capacity)


def exclusive_prefix_topk(scores, positions, references, capacity, initial=None):
    """Inputs ``[B, blocks, G, chunk]``; returns (scores, positions,
    references), each ``[B, blocks + 1, G, capacity]``: entry ``i`` is the
    top-``capacity`` over blocks ``0 .. i-1`` and entry ``blocks`` over all.

    ``initial`` (an extension): a bank ``(scores, positions[, references])``
    of ``[B, G, capacity]`` that joins every entry, equal to the reference's
    ``merge_topk(prefix, bank expanded over the entries)`` in ``_sequence``
    (references default to the slot index where the position is >= 0).
    Matches the reference whenever valid positions are distinct within a
    (row, group) and invalid references are -1, as in the prefill
    orchestration."""
    require_cuda(scores, positions, references)
    if scores.dim() != 4 or not (scores.shape == positions.shape == references.shape):
        raise ValueError('scores, positions and references must be [B, blocks, G, chunk]')
    B, blocks, G, chunk = scores.shape
    capacity = int(capacity)
    s32 = scores.to(torch.float32).contiguous()
    pos, pcode = _positions(positions)
    refs = references.to(torch.int64).contiguous()
    shape = (B, blocks + 1, G, capacity)
    out_s = torch.empty(shape, device=scores.device, dtype=torch.float32)
    out_p = torch.empty(shape, device=scores.device, dtype=torch.int64)
    out_r = torch.empty(shape, device=scores.device, dtype=torch.int64)
    init_s = init_p = init_r = None
    icode = _I64
    if initial is not None:
        init_s = initial[0].to(torch.float32).contiguous()
        init_p, icode = _positions(initial[1])
        if len(initial) > 2 and initial[2] is not None:
            init_r = initial[2].to(torch.int64).contiguous()
        for t in (init_s, init_p) + ((init_r,) if init_r is not None else ()):
            if t.shape != (B, G, capacity):
                raise ValueError('initial bank must be [B, G, capacity]')
    ptr = lambda t: 0 if t is None else t.data_ptr()  # noqa: E731
    rc = _lib.lib().yb_mem_exclusive_prefix_topk(
        s32.data_ptr(), pos.data_ptr(), pcode, refs.data_ptr(), B, blocks, G, chunk, capacity,
        ptr(init_s), ptr(init_p), icode, ptr(init_r), out_s.data_ptr(), out_p.data_ptr(), out_r.data_ptr(),
        stream_ptr(scores.device))
    _lib.check(rc, 'exclusive_prefix_topk')
    return out_s.to(scores.dtype), out_p, out_r.to(references.dtype)


def _read_timeline(query, old_k, old_v, n_old, new_k, new_v, refs, shift, lo, hi, blocks, chunk, zero_fill):
    """indexed read of the prompt's ``[B, T, H, D]`` query through the
    timeline (slot s of row b = token s + shift[b]), writing slots [lo, hi).
    References below ``n_old`` read rows of ``old_k / old_v``, the others
    rows of ``new_k / new_v`` (the writer's rows, read where they are)."""
    query = query.contiguous()
    B, T, H, D = query.shape
    G, CAP = refs.shape[-2:]
    out = torch.zeros_like(query) if zero_fill else torch.empty_like(query)
    old_k, old_v, new_k, new_v = (x.contiguous() for x in (old_k, old_v, new_k, new_v))
    refs = refs.contiguous()
    shift, lo, hi = (x.to(torch.int64).contiguous() for x in (shift, lo, hi))
    n_new = new_k.shape[0]
    rc = _lib.lib().yb_mem_indexed_read_timeline(
        query.data_ptr(), old_k.data_ptr(), old_v.data_ptr(), new_k.data_ptr() if n_new else None,
        new_v.data_ptr() if n_new else None, refs.data_ptr(), out.data_ptr(), B, T, blocks, chunk, H, G, D, n_old,
        n_new, 1, CAP, shift.data_ptr(), lo.data_ptr(), hi.data_ptr(), dtype_code(query), stream_ptr(query.device))
    _lib.check(rc, 'indexed_gqa (timeline)')
    return out


def sequence(query, scores, write_kv, valid, chunk, state=None, capacity=None, *, capture_safe=False,
             mask_is_run=None):
    """Prefill anchor read and write (``IndependentGQAMemory._sequence``,
    modeling_yanchor.py:178-275).

    query ``[B, T, H, D]``; scores ``[B, T, G]`` (admission scores);
    ``write_kv(batch_index, token_index) -> (key, value)`` gives the writer's
    ``[N, G, D]`` rows for the listed tokens (called once, only for the tokens
    that some block reads or that stay pending); ``valid`` ``[B, T]`` bool or
    None; ``state`` an ``IndependentMemoryState``-like object, updated in
    place, or None (then ``capacity`` gives CAP and nothing is kept).  Returns
    the read ``[B, T, H, D]`` (zero on invalid tokens).

    Each row's tokens (valid ones first, in order) are laid on a timeline
    after the state's ``count`` pending tokens and padded to whole blocks of
    ``chunk``.  Block ``i`` reads the top-CAP over the state's bank and
    blocks ``0 .. i-1``; afterwards the bank becomes the top-CAP over all
    complete blocks and the incomplete tail becomes the pending chunk.

    By default this follows the reference's data flow, which has two host
    synchronisations: the writer runs only on the tokens some block reads or
    that stay pending (a ``nonzero`` over the timeline sizes that list), and
    the read's fast path is chosen by checking on the host that each row's
    valid tokens form one run.  With ``capture_safe=True`` neither happens,
    so the call can be captured in a CUDA graph: the writer runs on every
    slot of the timeline (``B * extent`` rows, entries that no block reads
    are computed and left unused; results are identical), and the caller
    states whether each row's valid tokens are one run (``mask_is_run``;
    not needed without a mask).
    """
    require_cuda(query, scores)
    if capture_safe and valid is not None and mask_is_run is None:
        raise ValueError('capture_safe=True with a mask needs mask_is_run (is every row\'s valid run contiguous?)')
    B, T, H, D = query.shape
    G = scores.shape[-1]
    dev = query.device
    cap = int(state.keys.shape[2]) if state is not None else int(capacity)
    if T == 0:
        return query.new_zeros(query.shape)                   # nothing to read or add
    i64 = dict(device=dev, dtype=torch.int64)
    L = _lib.lib()
    stream = stream_ptr(dev)
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731

    # ---- timeline: [the state's pending tokens | new tokens, valid first], on the device ----
    if valid is None:
        order = n_new = None
    else:
        valid = valid.to(device=dev, dtype=torch.bool)
        order = torch.argsort((~valid).to(torch.int8), dim=1, stable=True).contiguous()   # valid first, stable
        n_new = valid.sum(1).to(torch.int64).contiguous()
    lead = 0 if state is None else chunk
    extent = -(-(T + lead) // chunk) * chunk
    blocks = extent // chunk
    shift = 0 if state is None else cap
    has_state = state is not None
    if has_state:
        _check_state_layout(state, chunk)
        pc = int(state.pending_keys.shape[2])
        count, total, pscores = state.count, state.total, state.pending_scores
        count_s0, pmeta_s0 = count.stride(0), pscores.stride(0)
    else:
        pc, count, total, pscores, count_s0, pmeta_s0 = 0, None, None, None, 0, 0
    snap = torch.empty(3, B, **i64)
    s_blk = torch.empty(B, blocks, G, chunk, device=dev, dtype=torch.float32)
    pos_blk = torch.empty(B, blocks, G, chunk, **i64)
    ref_blk = torch.empty(B, blocks, G, chunk, **i64)
    tok = torch.empty(B, extent, **i64)
    s32 = scores.to(torch.float32).contiguous()
    _lib.check(L.yb_mem_prefill_timeline(s32.data_ptr(), ptr(order), ptr(n_new), ptr(count), ptr(total), count_s0,
                                         ptr(pscores), pmeta_s0, B, T, G, chunk, extent, shift, pc, snap.data_ptr(),
                                         s_blk.data_ptr(), pos_blk.data_ptr(), ref_blk.data_ptr(), tok.data_ptr(),
                                         stream), 'sequence (timeline)')
    c0, fill = snap[0], snap[0] + snap[2]

    initial = None if state is None else (state.scores, state.positions)
    pre_s, pre_p, pre_r = exclusive_prefix_topk(s_blk, pos_blk, ref_blk, cap, initial=initial)

    # ---- which new tokens get a key / value row, and the slot -> source-row table ----
    needed = torch.empty(B, extent, device=dev, dtype=torch.uint8)
    table = torch.empty(B, shift + extent, **i64)
    read_refs = torch.empty(B, blocks, G, cap, **i64)
    _lib.check(L.yb_mem_prefill_table(pre_r.data_ptr(), snap.data_ptr(), B, G, chunk, extent, cap, int(has_state),
                                      int(capture_safe), needed.data_ptr(), table.data_ptr(), read_refs.data_ptr(),
                                      stream), 'sequence (table)')
    offset = B * (cap + chunk) if has_state else 0
    if capture_safe:
        # every slot of the timeline gets a writer row (row b * extent + slot); no list to size
        sel_b = torch.arange(B, **i64)[:, None].expand(B, extent).reshape(-1)
        k_new, v_new = write_kv(sel_b, tok.reshape(-1))
    else:
        sel_b, sel_slot = needed.nonzero(as_tuple=True)
        k_new, v_new = write_kv(sel_b, tok[sel_b, sel_slot])
        table[sel_b, shift + sel_slot] = offset + torch.arange(sel_b.numel(), **i64)
        _lib.check(L.yb_mem_prefill_read_references(pre_r.data_ptr(), table.data_ptr(), B, G, chunk, extent, cap,
                                                    int(has_state), read_refs.data_ptr(), stream),
                   'sequence (read references)')
    k_new = k_new.to(query.dtype).reshape(-1, G, D).contiguous()
    v_new = v_new.to(query.dtype).reshape(-1, G, D).contiguous()

    # ---- the two row sources: [old bank + pending rows (a copy: the state is rewritten below) | new rows] ----
    if has_state:
        old_k = torch.cat((state.keys, state.pending_keys[:, :, :chunk]), 2).transpose(1, 2)
        old_v = torch.cat((state.values, state.pending_values[:, :, :chunk]), 2).transpose(1, 2)
        old_k = old_k.reshape(-1, G, D).to(query.dtype).contiguous()
        old_v = old_v.reshape(-1, G, D).to(query.dtype).contiguous()
    else:
        old_k = old_v = query.new_zeros(1, G, D)   # no old rows: a placeholder no reference reaches

    # ---- read: block i attends to prefix entry i ----
    run = True                                                # each row's valid tokens are one run
    if order is not None:
        if mask_is_run is not None:
            run = bool(mask_is_run)
        else:
            v8 = valid.to(torch.int8)
            run = bool((((v8[:, 1:] > v8[:, :-1]).sum(1) + v8[:, 0]) <= 1).all())
    if run:
        # the read kernel addresses the prompt's own rows: slot s of row b is
        # token s - count + first valid token; only new, live slots are written
        first = torch.zeros(B, **i64) if order is None else valid.to(torch.int8).argmax(1)
        out = _read_timeline(query, old_k, old_v, offset, k_new, v_new, read_refs, first - c0, c0, fill, blocks,
                             chunk, zero_fill=order is not None)
    else:
        # whole (token, all heads) rows move with index_select on flattened views
        rows = torch.arange(B, **i64)[:, None]
        q_slot = query.reshape(B * T, H * D).index_select(0, (rows * T + tok).flatten())
        zero = query.new_zeros(1, G, D)                       # keeps the source non-empty; never referenced
        src_k = torch.cat((old_k[:offset], k_new, zero), 0)
        src_v = torch.cat((old_v[:offset], v_new, zero), 0)
        read = indexed_gqa(q_slot.view(B, blocks, chunk, H, D), src_k[None], src_v[None], read_refs)
        rank = torch.argsort(order, dim=1)                    # token -> its rank among the reordered tokens
        at = (c0[:, None] + rank).clamp(max=extent - 1)
        out = read.view(B * extent, H * D).index_select(0, (rows * extent + at).flatten()).view(B, T, H, D)
        out.masked_fill_(~valid[..., None, None], 0)

    # ---- new state: bank = top-CAP over all complete blocks, tail = pending ----
    if has_state:
        n_rows = k_new.shape[0]
        _lib.check(L.yb_mem_prefill_state(
            pre_s.data_ptr(), pre_p.data_ptr(), pre_r.data_ptr(), table.data_ptr(), snap.data_ptr(),
            s_blk.data_ptr(), old_k.data_ptr(), old_v.data_ptr(), k_new.data_ptr() if n_rows else None,
            v_new.data_ptr() if n_rows else None, state.keys.data_ptr(), state.values.data_ptr(),
            state.keys.stride(0), state.scores.data_ptr(), state.positions.data_ptr(), state.scores.stride(0),
            state.pending_keys.data_ptr(), state.pending_values.data_ptr(), state.pending_keys.stride(0),
            state.pending_scores.data_ptr(), state.pending_scores.stride(0), state.count.data_ptr(),
            state.total.data_ptr(), state.count.stride(0), B, G, chunk, extent, cap, pc, D, dtype_code(query),
            stream), 'sequence (state)')
    return out


def _check_state_layout(state, chunk):
    """The device orchestration reads and writes the state's fields at their
    batch strides with every inner dimension contiguous (as the state's own
    allocation and the vLLM page views are), in the query's dtype for the
    rows, float32 scores, int32 positions and int64 counters."""
    B, G, cap, D = state.keys.shape
    pc = state.pending_keys.shape[2]
    inner = lambda t, n: all(t.stride(i) == math.prod(t.shape[i + 1:]) for i in range(1, n))  # noqa: E731
    ok = (state.values.shape == state.keys.shape and state.values.stride() == state.keys.stride()
          and state.pending_values.shape == state.pending_keys.shape
          and state.pending_values.stride() == state.pending_keys.stride() and pc >= chunk
          and inner(state.keys, 4) and inner(state.pending_keys, 4) and inner(state.scores, 3)
          and state.positions.stride() == state.scores.stride() and inner(state.pending_scores, 3)
          and state.scores.dtype == torch.float32 and state.pending_scores.dtype == torch.float32
          and state.positions.dtype == torch.int32 and state.count.dtype == torch.int64
          and state.total.dtype == torch.int64 and state.count.stride() == state.total.stride())
    if not ok:
        raise ValueError('memory state: fields must be batch-strided with contiguous inner dimensions '
                         '(float32 scores, int32 positions, int64 count / total)')
