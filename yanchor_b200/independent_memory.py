"""Anchor-memory operators with the reference's call signatures.

Drop-in for ``runtime/model/independent_memory.py`` (the module that
``modeling_yanchor.py:19-20`` loads as ``model.independent_memory`` when
``config.backend == 'cuda'``):

    indexed_gqa(query, key, value, references)            -> read   (prefill)
    committed_gqa(query, state, indices=None)             -> read   (decode)
    commit_decode(key, value, scores, active, chunk, state, indices=None)
                                                          -> None   (decode write)
    decode_step(query, key, value, scores, active, chunk, state, indices=None)
                                                          -> read   (read + write, one launch)

``state`` is any object with the fields of ``IndependentMemoryState``
(``modeling_yanchor.py:80-120``): keys / values ``[B, G, CAP, D]``, scores
``[B, G, CAP]`` float32, positions ``[B, G, CAP]`` int32, pending_keys /
pending_values ``[B, G, PC, D]``, pending_scores ``[B, G, PC]`` float32, count
/ total ``[B]`` int64.  The batch axis of every field may be strided (a slot
pool view, as vLLM and SGLang pass); ``indices`` selects pool rows per request
(-1 = skip).  ``commit_decode`` mutates the state in place.

All three run on libyanchor_b200.so's CUDA kernels; there is no CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr



@dataclass
class MemoryState:
    """Device state of one anchor-memory layer, field for field the layout of
    ``IndependentMemoryState`` (``modeling_yanchor.py:80-120``); any object
    with these fields works with the operators below."""
    keys: torch.Tensor
    values: torch.Tensor
    scores: torch.Tensor
    positions: torch.Tensor
    pending_keys: torch.Tensor
    pending_values: torch.Tensor
    pending_scores: torch.Tensor
    count: torch.Tensor
    total: torch.Tensor

    @classmethod
    def empty(cls, batch, groups, capacity, chunk, dim, device, dtype):
        bank, pend = (batch, groups, capacity, dim), (batch, groups, chunk, dim)
        z = dict(device=device, dtype=dtype)
        return cls(torch.zeros(bank, **z), torch.zeros(bank, **z),
                   torch.full(bank[:-1], float('-inf'), device=device, dtype=torch.float32),
                   torch.full(bank[:-1], -1, device=device, dtype=torch.int32),
                   torch.zeros(pend, **z), torch.zeros(pend, **z),
                   torch.full(pend[:-1], float('-inf'), device=device, dtype=torch.float32),
                   torch.zeros(batch, device=device, dtype=torch.int64),
                   torch.zeros(batch, device=device, dtype=torch.int64))


def vllm_page_shapes(groups, capacity, chunk, dim):
    """Per-slot shapes of the vLLM plugin's memory page: (values, meta)
    (vllm_yanchor.py:19-22).  values hold keys, values, pending keys and
    pending values in the model dtype; meta holds float32 scores, int32
    positions, float32 pending scores and int64 count / total."""
    return (2 * groups * (capacity + chunk) * dim,), (groups * (2 * capacity + chunk) + 4,)


def state_from_vllm_page(values, meta, groups, capacity, chunk, dim):
    """A ``MemoryState`` of views into a pool of vLLM memory pages
    ``values [P, 2*G*(CAP+chunk)*D]`` and ``meta [P, G*(2*CAP+chunk)+4]``
    float32, laid out as the plugin's ``YANchorMemory.state``
    (vllm_yanchor.py:47-62): no copy — every operator here reads and writes
    the pages in place (each field is batch-strided by the page size), and
    ``indices`` pick the page of each request."""
    P = values.shape[0]
    if tuple(values.shape[1:]) != vllm_page_shapes(groups, capacity, chunk, dim)[0] or \
            tuple(meta.shape[1:]) != vllm_page_shapes(groups, capacity, chunk, dim)[1] or meta.shape[0] != P:
        raise ValueError('pages do not match the memory shape')
    if meta.dtype != torch.float32:
        raise TypeError('the meta page is float32')
    fields, off = [], 0
    for width in (capacity, capacity, chunk, chunk):
        size = groups * width * dim
        fields.append(values[:, off:off + size].view(P, groups, width, dim))
        off += size
    w = groups * capacity
    scores = meta[:, :w].view(P, groups, capacity)
    positions = meta[:, w:2 * w].view(torch.int32).view(P, groups, capacity)
    pending_scores = meta[:, 2 * w:-4].view(P, groups, chunk)
    count = meta[:, -4:-2].view(torch.int64).squeeze(-1)
    total = meta[:, -2:].view(torch.int64).squeeze(-1)
    return MemoryState(fields[0], fields[1], scores, positions, fields[2], fields[3], pending_scores, count, total)


def reset_vllm_page_(state, pages=None):
    """Empty the given pages (all when None), as ``IndependentMemoryState.reset_``
    (modeling_yanchor.py:110-118) does for a state."""
    for name in ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values', 'pending_scores',
                 'count', 'total'):
        t = getattr(state, name)
        fill = float('-inf') if 'scores' in name else -1 if name == 'positions' else 0
        if pages is None:
            t.fill_(fill)
        else:
            t.index_fill_(0, pages.to(t.device), fill)


def _inner_contiguous(t: torch.Tensor, ndim_inner: int) -> bool:
    expected = 1
    for d in range(t.dim() - 1, t.dim() - 1 - ndim_inner, -1):
        if t.stride(d) != expected:
            return False
        expected *= t.shape[d]
    return True


def _check_state(state):
    for name in ('keys', 'values', 'pending_keys', 'pending_values'):
        t = getattr(state, name)
        if not _inner_contiguous(t, 3):
            raise ValueError(f'state.{name} must be contiguous inside each batch row')
    for name in ('scores', 'positions', 'pending_scores'):
        if not _inner_contiguous(getattr(state, name), 2):
            raise ValueError(f'state.{name} must be contiguous inside each batch row')
    if state.keys.stride(0) != state.values.stride(0):
        raise ValueError('state.keys and state.values must share a batch stride')
    if state.pending_keys.stride(0) != state.pending_values.stride(0):
        raise ValueError('pending keys and values must share a batch stride')
    if state.scores.stride(0) != state.positions.stride(0):
        raise ValueError('state.scores and state.positions must share a batch stride')
    if state.count.stride(0) != state.total.stride(0):
        raise ValueError('state.count and state.total must share a stride')
    if state.positions.dtype != torch.int32 or state.scores.dtype != torch.float32:
        raise TypeError('positions must be int32 and scores float32')
    if state.count.dtype != torch.int64 or state.total.dtype != torch.int64:
        raise TypeError('count and total must be int64')


def _indices(indices, device):
    if indices is None:
        return None
    return indices.to(device=device, dtype=torch.int64).contiguous()


def indexed_gqa(query, key, value, references):
    """Prefill read (``independent_memory.py:38``): query ``[B, blocks, chunk,
    H, D]`` attends to ``key/value[KB, S, G, D]`` rows listed in
    ``references[B, blocks, G, CAP]`` (-1 = empty) plus the null slot."""
    require_cuda(query, key, value, references)
    query, key, value = query.contiguous(), key.contiguous(), value.contiguous()
    references = references.to(torch.int64).contiguous()
    B, blocks, chunk, H, D = query.shape
    G, CAP = references.shape[-2:]
    if key.shape != value.shape or key.shape[2] != G or key.shape[3] != D:
        raise ValueError('key/value must be [KB, S, G, D] matching the query and references')
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise TypeError('query, key and value must share a dtype')
    out = torch.empty_like(query)
    rc = _lib.lib().yb_mem_indexed_read(query.data_ptr(), key.data_ptr(), value.data_ptr(), references.data_ptr(),
                                        out.data_ptr(), B, blocks, chunk, H, G, D, key.shape[1], key.shape[0], CAP,
                                        dtype_code(query), stream_ptr(query.device))
    _lib.check(rc, 'indexed_gqa')
    return out


def committed_gqa(query, state, indices=None):
    """Decode read (``independent_memory.py:177``): query ``[B, 1, H, D]``
    attends to the committed bank of its state row plus the null slot."""
    require_cuda(query, state.keys)
    _check_state(state)
    query = query.contiguous()
    b, _, h, d = query.shape
    g, cap = state.keys.shape[1:3]
    if state.keys.dtype != query.dtype:
        raise TypeError('query and memory keys must share a dtype')
    idx = _indices(indices, query.device)
    out = torch.empty_like(query)
    rc = _lib.lib().yb_mem_decode_read(query.data_ptr(), state.keys.data_ptr(), state.values.data_ptr(),
                                       state.positions.data_ptr(), ptr(idx), out.data_ptr(), b, h, g, cap, d,
                                       state.keys.stride(0), state.positions.stride(0), dtype_code(query),
                                       stream_ptr(query.device))
    _lib.check(rc, 'committed_gqa')
    return out


_ARRIVE = {}
_ARRIVE_RETIRED = []


def _arrive(batch, device):
    """B zeroed int32 counters per device for ``decode_step`` (every call
    leaves them zero).  When a larger batch comes, a larger buffer replaces
    the current one, but the old one is kept alive for the life of the
    process: a CUDA graph captured at a smaller batch still holds its address
    and must never see that memory handed to another tensor."""
    t = _ARRIVE.get(device)
    if t is None or t.numel() < batch:
        if t is not None:
            _ARRIVE_RETIRED.append(t)
        t = _ARRIVE[device] = torch.zeros(max(batch, 64), device=device, dtype=torch.int32)
    return t


def decode_step(query, key, value, scores, active, chunk, state, indices=None, arrive=None):
    """One decode step of a memory layer: ``committed_gqa(query, state)`` then
    ``commit_decode(key, value, scores, active, chunk, state)`` — the reference
    decode layer's order (``modeling_yanchor.py:283-312``) — with identical
    results, in one launch on the tensor-core read path.  Returns the read.
    ``arrive`` is an optional int32 tensor of at least B zeroed counters that
    the caller owns (every call leaves them zero); by default the module keeps
    one buffer per device.  Calls that overlap on the GPU must not share
    counters."""
    require_cuda(query, key, value, scores, active, state.keys)
    _check_state(state)
    if state.positions.stride(0) != state.scores.stride(0):
        out = committed_gqa(query, state, indices)
        commit_decode(key, value, scores, active, chunk, state, indices)
        return out
    query = query.contiguous()
    key, value = key.contiguous(), value.contiguous()
    scores = scores.to(torch.float32).contiguous()
    active = active.to(torch.bool).contiguous()
    b, _, h, d = query.shape
    g, cap = state.keys.shape[1:3]
    pc = state.pending_keys.shape[2]
    if state.keys.dtype != query.dtype or key.dtype != state.keys.dtype or value.dtype != state.values.dtype:
        raise TypeError('query, key, value and the memory must share a dtype')
    idx = _indices(indices, query.device)
    if arrive is None:
        arr = _arrive(b, query.device)
    else:
        if arrive.dtype != torch.int32 or not arrive.is_contiguous() or arrive.numel() < b \
                or arrive.device != query.device:
            raise ValueError('arrive must be a contiguous int32 tensor of at least B counters on the query device')
        arr = arrive
    out = torch.empty_like(query)
    rc = _lib.lib().yb_mem_decode_step(
        query.data_ptr(), out.data_ptr(), key.data_ptr(), value.data_ptr(), scores.data_ptr(), active.data_ptr(),
        int(chunk), state.keys.data_ptr(), state.values.data_ptr(), state.scores.data_ptr(),
        state.positions.data_ptr(), state.pending_keys.data_ptr(), state.pending_values.data_ptr(),
        state.pending_scores.data_ptr(), state.count.data_ptr(), state.total.data_ptr(), ptr(idx),
        arr.data_ptr(), b, h, g, cap, pc, d, state.keys.stride(0), state.scores.stride(0),
        state.pending_keys.stride(0), state.pending_scores.stride(0), state.count.stride(0), dtype_code(query),
        stream_ptr(query.device))
    _lib.check(rc, 'decode_step')
    return out


def commit_decode(key, value, scores, active, chunk, state, indices=None):
    """Decode write (``independent_memory.py:190``): push (key, value, score)
    of every active row into its pending chunk; when the chunk fills, merge
    bank and pending into the new top-CAP bank."""
    require_cuda(key, value, scores, active, state.keys)
    _check_state(state)
    key, value = key.contiguous(), value.contiguous()
    scores = scores.to(torch.float32).contiguous()
    active = active.to(torch.bool).contiguous()
    b = key.shape[0]
    g, cap, d = state.keys.shape[1:]
    pc = state.pending_keys.shape[2]
    if key.dtype != state.keys.dtype or value.dtype != state.values.dtype:
        raise TypeError('key/value must match the memory dtype')
    idx = _indices(indices, key.device)
    rc = _lib.lib().yb_mem_decode_commit(
        key.data_ptr(), value.data_ptr(), scores.data_ptr(), active.data_ptr(), int(chunk),
        state.keys.data_ptr(), state.values.data_ptr(), state.scores.data_ptr(), state.positions.data_ptr(),
        state.pending_keys.data_ptr(), state.pending_values.data_ptr(), state.pending_scores.data_ptr(),
        state.count.data_ptr(), state.total.data_ptr(), ptr(idx), b, g, cap, pc, d,
        state.keys.stride(0), state.scores.stride(0), state.pending_keys.stride(0), state.pending_scores.stride(0),
        state.count.stride(0), dtype_code(key), stream_ptr(key.device))
    _lib.check(rc, 'commit_decode')
