"""Decode-loop host logic, no GPU: the bookkeeping oracle against the
fixtures made by running the reference's torch statements
(runtime/model/inference_kernels.py:1701-1717), the recurrent-state storage
resolver (:428-435), the cache snapshot / restore (:388-426), and the
argument checks of the C entry point."""
import os
from types import SimpleNamespace

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


@pytest.mark.parametrize('storage,batch,want', [('fp32', 1, 'fp32'), ('bf16_non_anchor', 8, 'bf16_non_anchor'),
                                                ('fp16_non_anchor_auto_b64', 63, 'fp32'),
                                                ('fp16_non_anchor_auto_b64', 64, 'fp16_non_anchor')])
def test_resolve_recurrent_state_storage(storage, batch, want):
    import yanchor_b200 as yb
    assert yb.resolve_recurrent_state_storage(storage, batch) == want == od.resolve_recurrent_state_storage(
        storage, batch)


@pytest.mark.parametrize('storage,batch', [('fp8', 4), ('fp32', 0)])
def test_resolve_recurrent_state_storage_rejects(storage, batch):
    import yanchor_b200 as yb
    with pytest.raises(ValueError):
        yb.resolve_recurrent_state_storage(storage, batch)


def fake_cache():
    mem = SimpleNamespace(keys=torch.arange(6.0), count=torch.tensor([2]))
    l0 = SimpleNamespace(recurrent_states=torch.ones(2, 3), conv={'a': torch.zeros(4), 'n': 3},
                         cumulative_length=5, all_valid_host=True)
    l1 = SimpleNamespace(keys=torch.full((3,), 7.0), memory_state=mem, _qwen35_swa_physical_ring_index=torch.tensor(2),
                         _qwen35_swa_physical_ring_keys=torch.zeros(2))
    return SimpleNamespace(layers=[l0, l1], _seen_tokens=11)


def test_snapshot_restore_roundtrip():
    import yanchor_b200 as yb
    c = fake_cache()
    snap = yb.snapshot_cuda_graph_cache(c)
    names = [n for n, _, _ in snap['entries']]
    assert names == ['0.recurrent_states', '0.conv.a', '1.keys', '1.memory_state.keys', '1.memory_state.count']
    c.layers[0].recurrent_states.add_(1)
    c.layers[0].conv['a'].fill_(9)
    c.layers[1].memory_state.count.add_(1)
    c.layers[1]._qwen35_swa_physical_ring_keys.fill_(5)         # ring backing: not saved by default
    c._seen_tokens, c.layers[0].cumulative_length = 12, 6
    resets = []
    yb.restore_cuda_graph_cache(c, snap, reset_ring=resets.append)
    assert (c.layers[0].recurrent_states == 1).all() and (c.layers[0].conv['a'] == 0).all()
    assert int(c.layers[1].memory_state.count) == 2 and c._seen_tokens == 11 and c.layers[0].cumulative_length == 5
    assert (c.layers[1]._qwen35_swa_physical_ring_keys == 5).all() and resets == [c.layers[1]]


def test_restore_rejects_replaced_tensor():
    import yanchor_b200 as yb
    c = fake_cache()
    snap = yb.snapshot_cuda_graph_cache(c)
    c.layers[0].recurrent_states = torch.ones(2, 3)
    with pytest.raises(RuntimeError, match='replaced cache tensor'):
        yb.restore_cuda_graph_cache(c, snap)


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
