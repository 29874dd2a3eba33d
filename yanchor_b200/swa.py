"""Sliding-window attention decode over the physical ring cache, with the
reference's call shapes.

    physical_ring_update_(ring_key, ring_value, ring_valid, ring_index, key, value, valid)
        runtime/model/inference_kernels.py:1828-1879
        (`triton_fixed_memory_swa_physical_ring_update`): the new token goes
        to ring position ``ring_index`` and the index advances modulo W
    physical_ring_decode_attention(query, ring_key, ring_value, valid)
        runtime/model/inference_kernels.py:1881-1897
        (`fixed_memory_physical_ring_decode_attention`)

Ring key / value ``[B, KVH, W, D]`` (positions contiguous inside each head),
valid ``[B, W]`` bool, ring_index a device int64 scalar tensor.
"""
from __future__ import annotations

import torch

from . import _lib
from ._torch import dtype_code, require_cuda, stream_ptr


def _ring_checks(ring_key, ring_value, valid):
    if ring_key.dim() != 4 or ring_key.shape != ring_value.shape or ring_key.stride() != ring_value.stride():
        raise ValueError('ring key / value must share a [B, KVH, W, D] geometry and layout')
    if ring_key.stride(3) != 1 or ring_key.stride(2) != ring_key.shape[3]:
        raise ValueError('ring positions must be contiguous rows of D inside each head')
    B, _, W, _ = ring_key.shape
    if valid.shape != (B, W) or valid.dtype != torch.bool or valid.stride(1) != 1:
        raise ValueError('ring valid must be a [B, W] bool tensor with contiguous positions')


def physical_ring_update_(ring_key, ring_value, ring_valid, ring_index, key, value, valid):
    """Write one token per row into the ring and advance the index, in place;
    returns ``(ring_key, ring_value, ring_valid)``."""
    require_cuda(ring_key, ring_value, ring_valid, ring_index, key, value, valid)
    _ring_checks(ring_key, ring_value, ring_valid)
    B, KVH, W, D = ring_key.shape
    if key.shape != (B, KVH, 1, D) or value.shape != key.shape or key.dtype != ring_key.dtype:
        raise ValueError('the new key / value must be [B, KVH, 1, D] in the ring dtype')
    if key.stride(3) != 1 or value.stride() != key.stride():
        key, value = key.contiguous(), value.contiguous()
    if ring_index.dtype != torch.int64 or ring_index.numel() != 1:
        raise TypeError('ring_index must be a one-element int64 tensor')
    v = valid.reshape(B).to(torch.bool).contiguous()
    rc = _lib.lib().yb_swa_ring_write(key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1), v.data_ptr(),
                                      ring_key.data_ptr(), ring_value.data_ptr(), ring_key.stride(0),
                                      ring_key.stride(1), ring_valid.data_ptr(), ring_valid.stride(0),
                                      ring_index.data_ptr(), B, KVH, W, D, dtype_code(ring_key),
                                      stream_ptr(ring_key.device))
    _lib.check(rc, 'physical_ring_update_')
    return ring_key, ring_value, ring_valid


def workspace_bytes(B, KVH, QH, W, D):
    return int(_lib.lib().yb_swa_decode_workspace_bytes(B, KVH, QH, W, D))


def physical_ring_decode_attention(query, ring_key, ring_value, valid, *, reproducible=False, workspace=None):
    """One decode query per row over the ring: ``[B, 1, QH, D]`` out.
    ``reproducible`` is accepted for the reference's signature; this kernel
    is deterministic either way."""
    require_cuda(query, ring_key, ring_value, valid)
    if query.dim() != 4 or query.shape[1] != 1:
        raise ValueError('physical-ring attention accepts one decode query')
    _ring_checks(ring_key, ring_value, valid)
    B, KVH, W, D = ring_key.shape
    QH = query.shape[2]
    if query.shape != (B, 1, QH, D) or QH % KVH:
        raise ValueError('query heads must be a multiple of physical-ring KV heads')
    if query.dtype != ring_key.dtype:
        raise TypeError('query and ring must share a dtype')
    q = query.contiguous()
    out = torch.empty_like(q)
    need = workspace_bytes(B, KVH, QH, W, D)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), device=q.device, dtype=torch.uint8)
    rc = _lib.lib().yb_swa_decode_attention(q.data_ptr(), ring_key.data_ptr(), ring_value.data_ptr(),
                                            ring_key.stride(0), ring_key.stride(1), valid.data_ptr(), valid.stride(0),
                                            out.data_ptr(), B, QH, KVH, W, D, dtype_code(q), workspace.data_ptr(),
                                            workspace.numel(), stream_ptr(q.device))
    _lib.check(rc, 'physical_ring_decode_attention')
    return out
