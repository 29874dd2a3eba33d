"""Decode-loop bookkeeping after each sampled token, in numpy — test
infrastructure only (the checker of ``yb_decode_state_update``).

Restates the per-step state update of the reference's fixed-memory decode
loop: runtime/model/inference_kernels.py:1700-1717 (the torch path) and the
equivalent one-launch Triton kernel ``_qwen35_decode_state_update_kernel``
(same file :1169-1204, wrapper :1206-1208):

* a row is ``active`` when it is not finished and holds a slot
  (``slot_rows >= 0``); an inactive row's token becomes ``pad``, and its
  write goes to its private sink row at column ``maximum_new_tokens``;
* ``storage[write_row, write_column] = token``;
  ``dense_seen[row, token] = True`` (the pad token too, for inactive rows);
* ``next_step = step + active``; the write row's generated length becomes
  ``next_step`` when active;
* ``finished_by_eos[write_row] |= active & is_eos``;
  ``finished |= active & (is_eos | next_step >= slot_cap)``;
* ``row_steps = next_step``; ``row_positions += active``;
  ``decode_ids = pad if finished else token``;
  ``decode_useful_events += sum(active)``.

Fixtures: tests/golden/decode_state.npz, made by running the reference's
torch path (tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np


def update_decode_state(sampled_token, storage, dense_seen, generated_lengths, finished_by_eos, finished, slot_rows,
                        sink_rows, slot_caps, row_steps, row_positions, decode_ids, decode_useful_events, *,
                        maximum_new_tokens, pad_token_id, eos_token_ids):
    """In place on the numpy arrays, as the reference mutates its tensors.
    ``sampled_token`` / ``decode_ids`` are ``[slots, 1]``; ``decode_useful_events``
    a 0-d or one-element array."""
    tok = np.asarray(sampled_token).reshape(-1).astype(np.int64)
    active = ~finished.astype(bool) & (slot_rows >= 0)
    tok = np.where(active, tok, np.int64(pad_token_id))
    write_rows = np.where(active, slot_rows, sink_rows)
    write_cols = np.where(active, row_steps, np.int64(maximum_new_tokens))
    storage[write_rows, write_cols] = tok.astype(storage.dtype)
    dense_seen[np.arange(tok.shape[0]), tok] = True
    next_steps = row_steps + active.astype(row_steps.dtype)
    generated_lengths[write_rows] = np.where(active, next_steps, generated_lengths[write_rows])
    is_eos = np.zeros(tok.shape[0], bool)
    for e in eos_token_ids:
        is_eos |= tok == int(e)
    finished_by_eos[write_rows] |= active & is_eos
    finished |= active & (is_eos | (next_steps >= slot_caps))
    row_steps[:] = next_steps
    row_positions += active.astype(row_positions.dtype)
    decode_ids.reshape(-1)[:] = np.where(finished, np.int64(pad_token_id), tok)
    decode_useful_events.reshape(-1)[0] += int(active.sum())
