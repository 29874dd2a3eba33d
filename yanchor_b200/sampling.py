"""Final-logit sampling with the reference's call signature.

``sample_top_k_top_p_counter(scores, attempt_ids, steps, *, seed, temperature,
top_k, top_p, stream=0) -> [B, 1] int64`` mirrors
``runtime/model/inference_kernels.py:73-88`` (and its fused top-20 variant at
:1147-1167): top_k == 1 is greedy argmax; otherwise top-k (k <= 256) of
scores / temperature, softmax, top-p truncation and an inverse-CDF pick driven
by the stateless counter uniform of (attempt id, step, seed, stream).  Ties
inside the top-k are ordered by ascending token id.

``apply_dense_presence_penalty_`` mirrors inference_kernels.py:1104-1114.
All run on libyanchor_b200.so's CUDA kernels; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib
from ._torch import dtype_code, require_cuda, stream_ptr


def _rows(scores):
    if scores.dim() != 2:
        raise ValueError('sampling scores must have shape [batch, vocabulary]')
    if scores.stride(-1) != 1:
        scores = scores.contiguous()
    return scores


def workspace_bytes(batch: int, vocab: int, top_k: int = 1) -> int:
    return int(_lib.lib().yb_sample_workspace_bytes(batch, vocab, top_k))


def greedy(scores, workspace=None):
    """argmax over the last axis, ``[B, 1]`` int64 (first maximum wins)."""
    require_cuda(scores)
    scores = _rows(scores)
    B, V = scores.shape
    out = torch.empty((B, 1), device=scores.device, dtype=torch.int64)
    need = workspace_bytes(B, V, 1)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=scores.device, dtype=torch.uint8)
    rc = _lib.lib().yb_sample_greedy(scores.data_ptr(), scores.stride(0), B, V, dtype_code(scores), out.data_ptr(),
                                     workspace.data_ptr(), workspace.numel(), stream_ptr(scores.device))
    _lib.check(rc, 'greedy')
    return out


def greedy_noalloc(scores, out=None):
    """argmax like ``greedy``, for callers that cannot allocate device memory
    when they sample: it needs no workspace (the library keeps a fixed 64 KiB
    device array for the partial results, enough for 4096 rows).  With a
    preallocated ``out`` ([B, 1] or [B] int64, contiguous, on the scores'
    device) and scores whose last stride is 1, the call allocates nothing at
    all; scores with another last stride are refused rather than copied.
    Calls that may run concurrently on the GPU share that array and race; make
    the first call on each device before capturing a CUDA graph."""
    if scores.dim() != 2:
        raise ValueError('sampling scores must have shape [batch, vocabulary]')
    if scores.stride(-1) != 1:
        raise ValueError('greedy_noalloc needs scores with unit stride along the vocabulary '
                         '(a copy would allocate)')
    B, V = scores.shape
    if out is not None:
        if out.dtype != torch.int64:
            raise ValueError('greedy_noalloc: out must be int64')
        if not out.is_contiguous():
            raise ValueError('greedy_noalloc: out must be contiguous')
        if out.numel() < B:
            raise ValueError(f'greedy_noalloc: out holds {out.numel()} ids, {B} rows need one each')
        if out.device != scores.device:
            raise ValueError('greedy_noalloc: out must be on the scores\' device')
    require_cuda(scores)
    if out is None:
        out = torch.empty((B, 1), device=scores.device, dtype=torch.int64)
    rc = _lib.lib().yb_sample_greedy_noalloc(scores.data_ptr(), scores.stride(0), B, V, dtype_code(scores),
                                             out.data_ptr(), stream_ptr(scores.device))
    _lib.check(rc, 'greedy_noalloc')
    return out


def sample_top_k_top_p_counter(scores, attempt_ids, steps, *, seed, temperature, top_k, top_p, stream=0,
                               workspace=None):
    require_cuda(scores)
    scores = _rows(scores)
    if temperature <= 0.0 or not 0.0 < top_p <= 1.0:
        raise ValueError('invalid top-k/top-p sampling parameters')
    B, V = scores.shape
    if top_k > V:
        raise ValueError('top-k exceeds the vocabulary')
    if attempt_ids.shape != scores.shape[:1]:
        raise ValueError('attempt ids must contain one id per probability row')
    if attempt_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError('attempt ids must be integer tensors')
    ids = attempt_ids.to(device=scores.device, dtype=torch.int64).contiguous()
    if isinstance(steps, torch.Tensor):
        if steps.numel() == 1 and steps.dim() == 0:
            steps_t, scalar = None, int(steps.item())
        else:
            if steps.shape != scores.shape[:1]:
                raise ValueError('one integer step per row is required')
            steps_t, scalar = steps.to(device=scores.device, dtype=torch.int64).contiguous(), 0
    else:
        steps_t, scalar = None, int(steps)
    out = torch.empty((B, 1), device=scores.device, dtype=torch.int64)
    need = workspace_bytes(B, V, int(top_k))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=scores.device, dtype=torch.uint8)
    rc = _lib.lib().yb_sample_top_k_top_p_counter(
        scores.data_ptr(), scores.stride(0), B, V, dtype_code(scores), ids.data_ptr(),
        None if steps_t is None else steps_t.data_ptr(), scalar, int(seed), int(stream), float(temperature),
        int(top_k), float(top_p), out.data_ptr(), workspace.data_ptr(), workspace.numel(),
        stream_ptr(scores.device))
    _lib.check(rc, 'sample_top_k_top_p_counter')
    return out


def apply_dense_presence_penalty_(scores, seen, penalty):
    """scores -= penalty * seen, in place (seen: bool, same shape)."""
    if penalty == 0.0:
        return
    if scores.shape != seen.shape or seen.dtype != torch.bool:
        raise ValueError('dense presence state must be a boolean scores-shaped tensor')
    require_cuda(scores, seen)
    if not scores.is_contiguous() or not seen.is_contiguous():
        raise ValueError('scores and seen must be contiguous')
    rc = _lib.lib().yb_presence_penalty(scores.data_ptr(), seen.data_ptr(), scores.numel(), float(penalty),
                                        dtype_code(scores), stream_ptr(scores.device))
    _lib.check(rc, 'apply_dense_presence_penalty_')
