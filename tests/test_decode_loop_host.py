"""Decode-loop host logic, no GPU: the bookkeeping oracle against the
fixtures made by running the reference's torch statements
(runtime/model/inference_kernels.py:1701-1717), and the argument checks of
the C entry point."""
import os
import numpy as np
import pytest
import torch

from conftest import ROOT
from oracle import decode_state as od

GOLDEN = os.path.join(ROOT, 'tests', 'golden', 'decode_state.npz')
FIELDS = ('storage', 'dense_seen', 'generated_lengths', 'finished_by_eos', 'finished', 'slot_rows', 'sink_rows',
          'slot_caps', 'row_steps', 'row_positions', 'decode_ids', 'decode_useful_events')


def replay_fixture(d, update):
    """Run every step of the fixture through ``update`` and compare each field
    after each step."""
    st = {k: d['ds_init_' + k].copy() for k in FIELDS}
    mx, pad, e0, e1, _ = (int(x) for x in d['ds_meta'])
    for t in range(d['ds_tokens'].shape[0]):
        if t == 4:
            st['slot_rows'][3] = -1
        st = update(d['ds_tokens'][t], st, mx, pad, (e0, e1))
        for k in FIELDS:
            np.testing.assert_array_equal(st[k], d[f'ds_{t}_{k}'], err_msg=f'step {t} {k}')


def test_oracle_matches_reference_bookkeeping():
    def update(tok, st, mx, pad, eos):
        od.update_decode_state(tok, *(st[k] for k in FIELDS), maximum_new_tokens=mx, pad_token_id=pad,
                               eos_token_ids=eos)
        return st
    replay_fixture(np.load(GOLDEN), update)


def test_fixture_exercises_every_branch():
    d = np.load(GOLDEN)
    last = {k: d[f'ds_6_{k}'] for k in FIELDS}
    assert last['finished_by_eos'].any()                          # an EOS finish
    assert (last['row_steps'] >= d['ds_init_slot_caps']).any()    # a cap finish
    assert (d['ds_init_slot_rows'] < 0).any() and d['ds_init_finished'].any()
    assert (last['storage'][d['ds_init_sink_rows']] == int(d['ds_meta'][1])).all()


def test_c_entry_rejects_bad_arguments():
    """Host-side checks return a status before any launch."""
    from yanchor_b200 import _lib
    lib = _lib.lib()
    ok = dict(tok=16, ts=1, storage=16, sdt=3, rows=4, cols=3, sstride=3, seen=16, seen_stride=10, vocab=10,
              gl=16, fe=16, fin=16, sr=16, sk=16, caps=16, steps=16, pos=16, ids=16, ids_stride=1, ev=16, slots=2,
              max_new=2, pad=0, eos=None, neos=0, stream=None)
    for bad in (dict(sdt=0), dict(sstride=2), dict(seen_stride=9), dict(slots=-1), dict(neos=1),
                dict(storage=None), dict(ev=None)):
        args = dict(ok, **bad)
        assert lib.yb_decode_state_update(*args.values()) == _lib.YB_ERR_ARGUMENT, bad
    import ctypes
    nine = (ctypes.c_int64 * 9)(*range(9))
    args = dict(ok, eos=ctypes.cast(nine, ctypes.c_void_p), neos=9)
    assert lib.yb_decode_state_update(*args.values()) == _lib.YB_ERR_UNSUPPORTED
