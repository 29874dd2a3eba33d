"""Sliding-window attention decode over the physical ring cache, with the
reference's call shapes.

    physical_ring_update_(ring_key, ring_value, ring_valid, ring_index, key, value, valid)
        runtime/model/inference_kernels.py:1828-1879
        (`triton_fixed_memory_swa_physical_ring_update`): the new token goes
        to ring position ``ring_index`` and the index advances modulo W
    physical_ring_decode_attention(query, ring_key, ring_value, valid)
        runtime/model/inference_kernels.py:1881-1897
        (`fixed_memory_physical_ring_decode_attention`)
    layer_ring_update(layer_cache, key, value, valid)
        the same update on a layer cache object, with the reference's
        signature (runtime/model/inference_kernels.py:1861-1879,
        `triton_fixed_memory_swa_physical_ring_update`): the ring lives in the
        cache's ``_qwen35_swa_physical_ring_*`` attributes and is built on
        first use as the reference builds it (`initialize_physical_ring`,
        same file :555-598)

    reference_swa(q, k, v, *, window, key_valid=None, query_start=0)
        modeling_yanchor.py:412-427: sliding-window attention over a prompt
        (tcgen05 kernel)
    flash_swa(q, k, v, *, window, attention_mask)
        modeling_yanchor.py:429-449: the same over each row's valid tokens

Ring key / value ``[B, KVH, W, D]`` (positions contiguous inside each head),
valid ``[B, W]`` bool, ring_index a device int32 (as the reference keeps it)
or int64 scalar tensor.
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
    if ring_index.dtype not in (torch.int32, torch.int64) or ring_index.numel() != 1:
        raise TypeError('ring_index must be a one-element int32 or int64 tensor')
    v = valid.reshape(B).to(torch.bool).contiguous()
    rc = _lib.lib().yb_swa_ring_write(key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1), v.data_ptr(),
                                      ring_key.data_ptr(), ring_value.data_ptr(), ring_key.stride(0),
                                      ring_key.stride(1), ring_valid.data_ptr(), ring_valid.stride(0),
                                      ring_index.data_ptr(), 3 if ring_index.dtype == torch.int32 else 4,
                                      B, KVH, W, D, dtype_code(ring_key),
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


_RING = '_qwen35_swa_physical_ring_'


def initialize_physical_ring(layer_cache):
    """Build the ring from a chronological window cache (``keys`` / ``values``
    ``[B, KVH, keep, D]``, ``valid [B, keep]``): ring width keep + 1, the
    cached positions at 0 .. keep - 1, the write index at keep (int32).  With
    ``_qwen35_swa_shared_ring_storage`` the cache's fields become views into
    the ring.  Host-issued copies only (cache set-up, as the reference's)."""
    tensors = (layer_cache.keys, layer_cache.values, layer_cache.valid)
    if any(t is None or not t.is_cuda for t in tensors):
        raise ValueError('physical SWA ring requires CUDA cache tensors')
    keep = int(layer_cache.keys.shape[-2])
    window = keep + 1
    if getattr(layer_cache, '_qwen35_swa_shared_ring_storage', False):
        for field, dim in (('keys', 2), ('values', 2), ('valid', 1)):
            source = getattr(layer_cache, field)
            shape = list(source.shape)
            shape[dim] = window
            target = getattr(layer_cache, _RING + field, None)
            if target is not None and target.shape == tuple(shape) and source.data_ptr() == target.data_ptr():
                target.narrow(dim, keep, 1).zero_()
            else:
                target = source.new_zeros(shape)
                target.narrow(dim, 0, keep).copy_(source)
            setattr(layer_cache, _RING + field, target)
            setattr(layer_cache, field, target.narrow(dim, 0, keep))
    else:
        for field, source in (('keys', layer_cache.keys), ('values', layer_cache.values),
                              ('valid', layer_cache.valid)):
            shape = (*source.shape[:-2], window, source.shape[-1]) if field != 'valid' else (source.shape[0], window)
            target = getattr(layer_cache, _RING + field, None)
            if target is None or target.shape != shape or target.device != source.device:
                target = source.new_zeros(shape)
                setattr(layer_cache, _RING + field, target)
            else:
                target.zero_()
            if field == 'valid':
                target[:, :keep].copy_(source)
            else:
                target[:, :, :keep].copy_(source)
    index = getattr(layer_cache, _RING + 'index', None)
    if index is None or index.device != layer_cache.keys.device:
        setattr(layer_cache, _RING + 'index', torch.tensor(keep, dtype=torch.int32, device=layer_cache.keys.device))
    else:
        index.fill_(keep)


def layer_ring_update(layer_cache, key, value, valid):
    """One decode token into the layer cache's ring (built on first use);
    returns ``(ring_key, ring_value, ring_valid)`` as the reference does."""
    require_cuda(key, value, valid)
    if key.shape[-2] != 1 or value.shape[-2] != 1 or valid.shape[-1] != 1:
        raise ValueError('physical SWA ring accepts one token')
    if key.shape != value.shape or key.stride(-1) != 1 or value.stride(-1) != 1:
        raise ValueError('physical SWA ring requires matching contiguous KV heads')
    if not hasattr(layer_cache, _RING + 'index'):
        initialize_physical_ring(layer_cache)
    return physical_ring_update_(getattr(layer_cache, _RING + 'keys'), getattr(layer_cache, _RING + 'values'),
                                 getattr(layer_cache, _RING + 'valid'), getattr(layer_cache, _RING + 'index'),
                                 key, value, valid)


def reference_swa(q, k, v, *, window, key_valid=None, query_start=0):
    """Sliding-window attention over a prompt, modeling_yanchor.py:412-427:
    queries ``[B, Tq, QH, D]`` at positions ``query_start ..`` attend to keys
    ``[B, Tk, KVH, D]`` at positions ``0 .. Tk - 1`` within ``window`` (causal),
    masked by ``key_valid [B, Tk]``; a query whose own ``key_valid`` entry is
    False gives zeros.  One tcgen05 kernel launch (bf16, D = 256)."""
    require_cuda(q, k, v, key_valid)
    if q.dim() != 4 or k.dim() != 4 or k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[3] != k.shape[3]:
        raise ValueError('reference_swa expects q [B, Tq, QH, D] and k, v [B, Tk, KVH, D]')
    if q.shape[2] % k.shape[2]:
        raise ValueError('query heads must be a multiple of key heads')
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError('q, k, v must share a dtype')
    B, Tq, QH, D = q.shape
    Tk, KVH = k.shape[1], k.shape[2]
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    kv = None
    if key_valid is not None:
        if key_valid.shape != (B, Tk):
            raise ValueError('key_valid must be [B, Tk]')
        kv = key_valid.to(torch.bool).contiguous()
    out = torch.empty_like(q)
    rc = _lib.lib().yb_swa_prefill_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                             None if kv is None else kv.data_ptr(), Tk, out.data_ptr(), B, Tq, Tk,
                                             QH, KVH, D, int(window), int(query_start), dtype_code(q),
                                             stream_ptr(q.device))
    _lib.check(rc, 'reference_swa')
    return out


def flash_swa(q, k, v, *, window, attention_mask):
    """The prefill SWA of the CUDA path, modeling_yanchor.py:429-449: causal
    window of ``window`` tokens; with ``attention_mask`` ([B, >= T], the last T
    columns belong to this prompt) over each row's valid tokens in order, as
    the reference's unpad / variable-length FlashAttention call does, padded
    positions giving zeros.  Rows whose valid tokens form one run (left or
    right padding) run in place; other rows are packed valid-first, run, and
    scattered back."""
    require_cuda(q, k, v)
    if attention_mask is None:
        return reference_swa(q, k, v, window=window)
    B, T = q.shape[:2]
    mask = attention_mask[:, -T:].to(device=q.device, dtype=torch.bool)
    m8 = mask.to(torch.int8)
    starts = (m8[:, 1:] > m8[:, :-1]).sum(1) + m8[:, 0]
    if bool((starts <= 1).all()):
        return reference_swa(q, k, v, window=window, key_valid=mask)
    order = torch.argsort((~mask).to(torch.int8), dim=1, stable=True)          # valid tokens first, in order
    n = mask.sum(1)
    packed_valid = torch.arange(T, device=q.device)[None, :] < n[:, None]

    def pack(x):
        return torch.gather(x, 1, order[:, :, None, None].expand(x.shape))
    out_packed = reference_swa(pack(q), pack(k), pack(v), window=window, key_valid=packed_valid)
    out = torch.zeros_like(q)
    out.scatter_(1, order[:, :, None, None].expand(out.shape), out_packed)
    return out
