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
        cache's ``_qwen35_swa_physical_ring_*`` attributes; a cache without
        one gets it from the reference's own initialiser (same file :555-598)

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


def _reference_ring_initializer():
    """The reference's own ring set-up, ``initialize_fixed_memory_swa_physical_ring``
    (runtime/model/inference_kernels.py:555-598), from the module the
    reference model imports (``model.inference_kernels``).  A layer cache
    with the ``_qwen35_swa_physical_ring_*`` fields only exists inside the
    reference's decode path, where that module is importable; the ring it
    builds is exactly the layout the kernels here read and write."""
    import importlib
    try:
        return importlib.import_module('model.inference_kernels').initialize_fixed_memory_swa_physical_ring
    except (ImportError, AttributeError) as e:
        raise RuntimeError('this layer cache has no physical ring yet, and the reference\'s '
                           'initialize_fixed_memory_swa_physical_ring (model.inference_kernels) that builds it '
                           'is not importable') from e


def layer_ring_update(layer_cache, key, value, valid):
    """One decode token into the layer cache's ring; returns ``(ring_key,
    ring_value, ring_valid)`` as the reference does.  A cache without a ring
    yet gets one from the reference's own initialiser first."""
    require_cuda(key, value, valid)
    if key.shape[-2] != 1 or value.shape[-2] != 1 or valid.shape[-1] != 1:
        raise ValueError('physical SWA ring accepts one token')
    if key.shape != value.shape or key.stride(-1) != 1 or value.stride(-1) != 1:
        raise ValueError('physical SWA ring requires matching contiguous KV heads')
    if not hasattr(layer_cache, _RING + 'index'):
        _reference_ring_initializer()(layer_cache)
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
    window of ``window`` tokens, the queries aligned to the last keys as
    FlashAttention aligns them (a decode query over a cached window attends
    to the window's last ``window`` keys); with ``attention_mask`` ([B, >= T], the last T
    columns belong to this prompt) over each row's valid tokens in order, as
    the reference's unpad / variable-length FlashAttention call does, padded
    positions giving zeros.  Rows whose valid tokens form one run (left or
    right padding) run in place; other rows are packed valid-first, run, and
    scattered back."""
    require_cuda(q, k, v)
    if attention_mask is None:
        # FlashAttention's causal mask is aligned to the end of the keys: the
        # last query sits at the last key (a decode query over a cached window)
        return reference_swa(q, k, v, window=window, query_start=k.shape[1] - q.shape[1])
    if k.shape[1] != q.shape[1]:
        raise ValueError('flash_swa with an attention mask needs as many keys as queries')
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
