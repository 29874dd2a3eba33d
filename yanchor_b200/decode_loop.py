"""Decode-loop plumbing around the hot path: the per-step bookkeeping kernel
and the CUDA-graph driver of the fixed-memory decode, with the reference's
call shapes.

    update_fixed_decode_state_(...)
        runtime/model/inference_kernels.py:1206-1208 (`_update_fixed_decode_state_`,
        Triton kernel :1169-1204; torch statements :1701-1717): one launch
        of ``yb_decode_state_update``
    resolve_recurrent_state_storage(storage, batch_size)
        same file :428-435
    snapshot_cuda_graph_cache(cache) / restore_cuda_graph_cache(cache, snap)
        same file :388-426: device copies of every cache tensor, so that the
        warm-up and capture forwards leave the cache as they found it
    FixedMemoryDecodeGraph(model, cache, token, position, ...)
        same file :437-553: warm up, capture one decode forward (and the
        position increment) into a CUDA graph, then ``replay(token,
        position_ids)`` copies the new ids in and replays

The graph driver is model-agnostic: ``model`` is called as the reference
calls it (``input_ids``, ``position_ids``, ``past_key_values``,
``use_cache=True``, ``logits_to_keep=1``) and must return an object with
``.logits [B, 1, vocab]``.  The reference's two model hooks (switching its
layers to graph mode, converting the recurrent-state storage) are optional
callables here.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._torch import require_cuda, stream_ptr

YB_I32, YB_I64 = 3, 4


def _vector(t, name, dtype, n):
    if t.dtype != dtype or t.numel() != n or (n > 1 and t.dim() == 1 and t.stride(0) != 1):
        raise ValueError(f'{name} must be {n} contiguous {dtype} values')
    return t


def update_fixed_decode_state_(sampled_token, storage, dense_seen, generated_lengths, finished_by_eos, finished,
                               slot_rows, sink_rows, slot_caps, row_steps, row_positions, decode_ids,
                               decode_useful_events, *, maximum_new_tokens, pad_token_id, eos_token_ids):
    """In-place bookkeeping after one sampled token per slot (one launch)."""
    require_cuda(sampled_token, storage, dense_seen, generated_lengths, finished_by_eos, finished, slot_rows,
                 sink_rows, slot_caps, row_steps, row_positions, decode_ids, decode_useful_events)
    slots = sampled_token.shape[0]
    if sampled_token.dim() != 2 or sampled_token.shape[1] != 1 or sampled_token.dtype != torch.int64:
        raise ValueError('sampled tokens must be [slots, 1] int64')
    if decode_ids.shape != (slots, 1) or decode_ids.dtype != torch.int64:
        raise ValueError('decode ids must be [slots, 1] int64')
    if storage.dim() != 2 or storage.dtype not in (torch.int32, torch.int64) or storage.stride(1) != 1:
        raise ValueError('storage must be a row-major [rows, max_new_tokens + 1] int32 / int64 table')
    if dense_seen.dim() != 2 or dense_seen.shape[0] != slots or dense_seen.dtype != torch.bool or \
            dense_seen.stride(1) != 1:
        raise ValueError('dense_seen must be a row-major [slots, vocab] bool table')
    rows = storage.shape[0]
    _vector(generated_lengths, 'generated_lengths', torch.int64, rows)
    _vector(finished_by_eos, 'finished_by_eos', torch.bool, rows)
    for name, t, dt in (('finished', finished, torch.bool), ('slot_rows', slot_rows, torch.int64),
                        ('sink_rows', sink_rows, torch.int64), ('slot_caps', slot_caps, torch.int64),
                        ('row_steps', row_steps, torch.int64), ('row_positions', row_positions, torch.int64)):
        _vector(t, name, dt, slots)
    _vector(decode_useful_events, 'decode_useful_events', torch.int64, 1)
    eos = [int(e) for e in eos_token_ids]
    eos_arr = (ctypes.c_int64 * max(len(eos), 1))(*eos)
    rc = _lib.lib().yb_decode_state_update(
        sampled_token.data_ptr(), sampled_token.stride(0), storage.data_ptr(),
        YB_I32 if storage.dtype == torch.int32 else YB_I64, rows, storage.shape[1], storage.stride(0),
        dense_seen.data_ptr(), dense_seen.stride(0), dense_seen.shape[1], generated_lengths.data_ptr(),
        finished_by_eos.data_ptr(), finished.data_ptr(), slot_rows.data_ptr(), sink_rows.data_ptr(),
        slot_caps.data_ptr(), row_steps.data_ptr(), row_positions.data_ptr(), decode_ids.data_ptr(),
        decode_ids.stride(0), decode_useful_events.data_ptr(), slots, int(maximum_new_tokens), int(pad_token_id),
        ctypes.cast(eos_arr, ctypes.c_void_p), len(eos), stream_ptr(storage.device))
    _lib.check(rc, 'update_fixed_decode_state_')


def resolve_recurrent_state_storage(storage: str, batch_size: int) -> str:
    if batch_size <= 0:
        raise ValueError('recurrent-state storage requires a positive batch')
    if storage == 'fp16_non_anchor_auto_b64':
        return 'fp16_non_anchor' if batch_size >= 64 else 'fp32'
    if storage not in {'fp32', 'bf16_non_anchor', 'fp16_non_anchor'}:
        raise ValueError(f'unsupported GDN recurrent state storage: {storage}')
    return storage


STATE_DTYPES = {'fp32': torch.float32, 'bf16_non_anchor': torch.bfloat16, 'fp16_non_anchor': torch.float16}

_RING_PREFIXES = ('_qwen35_swa_scratch_', '_qwen35_swa_physical_ring_')


def _cache_tensors(cache, include_ring_backing):
    found = []
    for li, layer in enumerate(cache.layers):
        for name, value in vars(layer).items():
            if not include_ring_backing and name.startswith(_RING_PREFIXES):
                continue
            if isinstance(value, torch.Tensor):
                found.append((f'{li}.{name}', value))
            elif isinstance(value, dict):
                found.extend((f'{li}.{name}.{k}', v) for k, v in value.items() if isinstance(v, torch.Tensor))
            elif name == 'memory_state' and value is not None:
                found.extend((f'{li}.memory_state.{k}', v) for k, v in vars(value).items()
                             if isinstance(v, torch.Tensor))
    return found


def snapshot_cuda_graph_cache(cache, *, include_ring_backing=False):
    return {'entries': [(n, t, t.clone()) for n, t in _cache_tensors(cache, include_ring_backing)],
            'include_ring_backing': bool(include_ring_backing),
            'seen_tokens': getattr(cache, '_seen_tokens', None),
            'layer_metadata': [{'cumulative_length': getattr(layer, 'cumulative_length', None),
                                'all_valid_host': getattr(layer, 'all_valid_host', None)} for layer in cache.layers]}


def restore_cuda_graph_cache(cache, snapshot, *, reset_ring=None):
    """Copy the saved values back into the same tensors (a tensor that the
    forward replaced by a new object is an error: a graph would keep the old
    one).  ``reset_ring(layer)`` runs for layers holding a physical ring when
    the ring backing was not saved."""
    current = dict(_cache_tensors(cache, snapshot.get('include_ring_backing', False)))
    for name, tensor, saved in snapshot['entries']:
        if current.get(name) is not tensor:
            raise RuntimeError(f'CUDA Graph capture replaced cache tensor {name}')
        tensor.copy_(saved)
    if snapshot['seen_tokens'] is not None:
        cache._seen_tokens = int(snapshot['seen_tokens'])
    for layer, meta in zip(cache.layers, snapshot['layer_metadata']):
        for name, value in meta.items():
            if hasattr(layer, name):
                setattr(layer, name, value)
        if not snapshot.get('include_ring_backing', False) and reset_ring is not None and \
                hasattr(layer, '_qwen35_swa_physical_ring_index'):
            reset_ring(layer)


class FixedMemoryDecodeGraph:
    """One captured decode forward, replayed once per generated token."""

    @torch.no_grad()
    def __init__(self, model, cache, token, position, scores_dtype=torch.float32, consume_capture_steps=False, *,
                 set_graph_decode=None, convert_state_storage=None, state_storage=None, reset_ring=None):
        if token.ndim != 2 or token.shape[1] != 1 or not token.is_cuda:
            raise ValueError('fixed-memory CUDA Graph requires CUDA [batch, 1] tokens')
        if scores_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError('decode scores must use FP32 or BF16')
        self.model, self.cache, self._reset_ring = model, cache, reset_ring
        storage = resolve_recurrent_state_storage(
            state_storage or str(getattr(getattr(model, 'config', None), 'gdn_recurrent_state_storage', 'fp32')),
            int(token.shape[0]))
        self.recurrent_state_storage_receipt = (convert_state_storage(cache, STATE_DTYPES[storage])
                                                if convert_state_storage is not None else None)
        self.static_ids = token.clone()
        if isinstance(position, torch.Tensor):
            pv = position.to(device=token.device, dtype=torch.long)
            if pv.ndim == 1:
                pv = pv[:, None]
            if pv.shape not in (token.shape, (4, *token.shape)):
                raise ValueError('decode positions require one value per token row')
            self.static_position_ids = pv.clone()
        else:
            self.static_position_ids = torch.full((token.shape[0], 1), int(position), dtype=torch.long,
                                                  device=token.device)
        initial = self.static_position_ids.clone()
        self.replays = 0
        self.graph = None
        self.scores = None
        self._pending_scores = None
        self.consume_capture_steps = bool(consume_capture_steps)
        self._set_graph_decode = set_graph_decode
        if set_graph_decode is not None:
            set_graph_decode(model, cache, True)
        if self.consume_capture_steps:
            # the warm-up forward is a real decode step: its scores are handed
            # out by the first replay, and the graph is captured on that replay
            host = self._snapshot_host_metadata()
            out = self._forward()
            self.scores = out.logits[:, -1].to(dtype=scores_dtype)
            self._pending_scores = self.scores
            self.static_position_ids.add_(1)
            self._restore_host_metadata(host)
            self.replays += 1
            torch.cuda.synchronize(token.device)
            return
        warm = snapshot_cuda_graph_cache(cache)
        self._forward()
        torch.cuda.synchronize(token.device)
        restore_cuda_graph_cache(cache, warm, reset_ring=reset_ring)
        del warm
        snap = snapshot_cuda_graph_cache(cache)
        self.static_position_ids.copy_(initial)
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(token.device)
        with torch.cuda.graph(self.graph):
            out = self._forward()
            self.scores = out.logits[:, -1].to(dtype=scores_dtype)
            self.static_position_ids.add_(1)
        torch.cuda.synchronize(token.device)
        restore_cuda_graph_cache(cache, snap, reset_ring=reset_ring)
        self.static_position_ids.copy_(initial)

    def _forward(self):
        return self.model(input_ids=self.static_ids, position_ids=self.static_position_ids,
                          past_key_values=self.cache, use_cache=True, logits_to_keep=1)

    def _snapshot_host_metadata(self):
        return (getattr(self.cache, '_seen_tokens', None),
                [(getattr(layer, 'cumulative_length', None), getattr(layer, 'all_valid_host', None))
                 for layer in self.cache.layers])

    def _restore_host_metadata(self, snapshot):
        seen, layers = snapshot
        if seen is not None:
            self.cache._seen_tokens = int(seen)
        for layer, (cum, valid) in zip(self.cache.layers, layers):
            if cum is not None and hasattr(layer, 'cumulative_length'):
                layer.cumulative_length = cum
            if valid is not None and hasattr(layer, 'all_valid_host'):
                layer.all_valid_host = valid

    def _copy_position_ids(self, position_ids):
        if position_ids is None:
            return
        pv = position_ids.to(device=self.static_position_ids.device, dtype=torch.long)
        if pv.ndim == 1:
            pv = pv[:, None]
        if pv.shape != self.static_position_ids.shape:
            raise ValueError('decode positions require one value per captured row')
        self.static_position_ids.copy_(pv)

    @torch.no_grad()
    def replay(self, token, position_ids=None):
        if self._pending_scores is not None:
            if not torch.equal(token, self.static_ids):
                raise RuntimeError('capture-consuming warm token changed before use')
            scores, self._pending_scores = self._pending_scores, None
            return scores
        self.static_ids.copy_(token)
        self._copy_position_ids(position_ids)
        if self.graph is None:
            # first replay after a capture-consuming warm-up: capture now, then
            # replay, so this step's forward runs exactly once
            self.graph = torch.cuda.CUDAGraph()
            host = self._snapshot_host_metadata()
            torch.cuda.synchronize(token.device)
            with torch.cuda.graph(self.graph):
                out = self._forward()
                self.scores = out.logits[:, -1].to(dtype=self.scores.dtype)
                self.static_position_ids.add_(1)
            self._restore_host_metadata(host)
            self.graph.replay()
            torch.cuda.synchronize(token.device)
            self.replays += 1
            return self.scores
        self.graph.replay()
        self.replays += 1
        return self.scores

    def close(self):
        """Release the graph (and the hook's graph mode)."""
        self.graph = None
        if self._set_graph_decode is not None:
            self._set_graph_decode(self.model, self.cache, False)
