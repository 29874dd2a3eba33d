"""Decode-loop plumbing around the hot path: the per-step bookkeeping kernel
and a CUDA-graph driver for decode steps built from this package's ops.

    update_fixed_decode_state_(...)
        runtime/model/inference_kernels.py:1206-1208 (`_update_fixed_decode_state_`,
        Triton kernel :1169-1204; torch statements :1701-1717): one launch
        of ``yb_decode_state_update``
    prepare_capture(device, max_batch)
        the one-time set-up of every lazily initialised piece of this package
        on a device, so that a step made of its ops can be captured without
        first running it
    StepGraphs(step, batch_sizes)
        one CUDA graph of ``step(batch)`` per batch size, captured largest
        first into one shared memory pool; ``replay(batch)`` runs the graph
        of the smallest captured size that holds ``batch`` rows

The reference's own driver (`FixedMemoryDecodeGraph`,
runtime/model/inference_kernels.py:437-553) runs warm-up forwards before
capture and therefore snapshots and restores the whole cache around them.
The ops here need no warm-up forward: ``prepare_capture`` does their set-up
without touching any caller state, and capturing records the step without
executing it, so the caller's recurrent, memory and ring state is exactly as
it was when the graphs are ready.  The reference's driver can also drive
these ops unchanged (it calls the rebound kernels).
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



def prepare_capture(device=None, max_batch: int = 4096) -> None:
    """Set up, once, everything in this package that is initialised on first
    use, so that a decode step built from its ops can be captured in a CUDA
    graph without running it first: the library is loaded, the anchor-memory
    step's arrival counters are sized for ``max_batch`` rows, and the
    no-allocation sampler has looked up its scratch address.  Touches no
    caller state; must not run during a capture."""
    from . import independent_memory, sampling
    device = torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)
    _lib.lib()
    independent_memory._arrive(int(max_batch), device)
    with torch.cuda.device(device):
        sampling.greedy_noalloc(torch.zeros((1, 1), device=device), out=torch.empty(1, device=device,
                                                                                    dtype=torch.int64))
    torch.cuda.synchronize(device)


class StepGraphs:
    """CUDA graphs of one decode step, one per batch size.

    ``step(batch)`` is the caller's function for ``batch`` rows: it reads its
    inputs from tensors the caller owns and keeps at fixed addresses (token
    ids, positions, the recurrent / memory / ring state of the first
    ``batch`` rows) and returns the step's outputs (tensors, or a tuple of
    them).  Each size is captured once, largest first, into one shared pool,
    so smaller sizes reuse the largest graph's activation memory; nothing is
    executed while capturing.  ``replay(batch)`` runs the graph of the
    smallest captured size >= ``batch`` and returns that graph's outputs
    (rows beyond ``batch`` belong to padding rows the caller keeps inactive).
    Call ``close()`` (or drop the object) before tearing the process group or
    the device down.

    ``warm``, if given, runs once before the first capture: the place for
    set-up of code outside this package (e.g. cuBLAS handles of the caller's
    projections) that must not run inside a capture."""

    def __init__(self, step, batch_sizes, *, device=None, warm=None):
        sizes = sorted({int(b) for b in batch_sizes})
        if not sizes or sizes[0] <= 0:
            raise ValueError('StepGraphs needs positive batch sizes')
        self.device = torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)
        prepare_capture(self.device, sizes[-1])
        if warm is not None:
            warm()
            torch.cuda.synchronize(self.device)
        self.sizes = sizes
        self.pool = torch.cuda.graph_pool_handle()
        self.graphs = {}
        self.outputs = {}
        for b in reversed(sizes):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.pool):
                out = step(b)
            self.graphs[b], self.outputs[b] = g, out

    def bucket(self, batch: int) -> int:
        for b in self.sizes:
            if b >= batch:
                return b
        raise ValueError(f'no captured decode step holds {batch} rows (largest: {self.sizes[-1]})')

    def replay(self, batch: int):
        b = self.bucket(int(batch))
        self.graphs[b].replay()
        return self.outputs[b]

    def close(self):
        self.graphs.clear()
        self.outputs.clear()
