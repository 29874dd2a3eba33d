"""GPU parity of the decode-loop plumbing: the bookkeeping kernel against the
reference fixtures and the oracle (bit-exact: integer work), and the CUDA
graph driver against eager decode steps of a small recurrent model built on
this package's kernels."""
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import ROOT
from oracle import decode_state as od

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(ROOT, 'tests', 'golden', 'decode_state.npz')
FIELDS = ('storage', 'dense_seen', 'generated_lengths', 'finished_by_eos', 'finished', 'slot_rows', 'sink_rows',
          'slot_caps', 'row_steps', 'row_positions', 'decode_ids', 'decode_useful_events')


@pytest.fixture(scope='module')
def yb():
    import yanchor_b200
    return yanchor_b200


def gpu_update(yb):
    def update(tok, st, mx, pad, eos):
        dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in st.items()}
        yb.update_fixed_decode_state_(torch.from_numpy(np.ascontiguousarray(tok)).cuda(), *(dev[k] for k in FIELDS),
                                      maximum_new_tokens=mx, pad_token_id=pad, eos_token_ids=eos)
        return {k: v.cpu().numpy() for k, v in dev.items()}
    return update


def test_state_update_matches_reference_fixture(yb):
    from test_decode_loop_host import replay_fixture
    replay_fixture(np.load(GOLDEN), gpu_update(yb))
    assert yb.lib().yb_device_error(1) == 0


@pytest.mark.parametrize('slots,storage_dtype,eos', [(300, np.int32, (5, 9, 11)), (33, np.int64, ()),
                                                      (1, np.int32, (2,))])
def test_state_update_random_trajectory(yb, slots, storage_dtype, eos):
    """A long run with more slots than one block's threads, int32 and int64
    storage, 0-3 EOS ids; slots empty and caps end rows along the way.  The
    device state stays on the device across steps."""
    rng = np.random.default_rng(slots)
    total, max_new, vocab, pad = 2 * slots, 40, 64, 1
    st = {
        'storage': np.full((total + slots, max_new + 1), pad, storage_dtype),
        'dense_seen': np.zeros((slots, vocab), bool),
        'generated_lengths': np.zeros(total + slots, np.int64),
        'finished_by_eos': np.zeros(total + slots, bool),
        'finished': rng.random(slots) < 0.1,
        'slot_rows': np.where(rng.random(slots) < 0.9, rng.permutation(total)[:slots], -1).astype(np.int64),
        'sink_rows': (total + np.arange(slots)).astype(np.int64),
        'slot_caps': rng.integers(1, max_new + 1, slots).astype(np.int64),
        'row_steps': np.ones(slots, np.int64),
        'row_positions': rng.integers(0, 5000, slots).astype(np.int64),
        'decode_ids': rng.integers(0, vocab, (slots, 1)).astype(np.int64),
        'decode_useful_events': np.zeros((), np.int64),
    }
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in st.items()}
    for t in range(max_new + 2):
        tok = rng.integers(0, vocab, (slots, 1)).astype(np.int64)
        od.update_decode_state(tok, *(st[k] for k in FIELDS), maximum_new_tokens=max_new, pad_token_id=pad,
                               eos_token_ids=eos)
        yb.update_fixed_decode_state_(torch.from_numpy(tok).cuda(), *(dev[k] for k in FIELDS),
                                      maximum_new_tokens=max_new, pad_token_id=pad, eos_token_ids=eos)
    for k in FIELDS:
        np.testing.assert_array_equal(dev[k].cpu().numpy(), st[k], err_msg=k)
    assert (st['finished'] | (st['slot_rows'] < 0)).all()       # slots without a row stay idle, unfinished
    assert yb.lib().yb_device_error(1) == 0


def test_state_update_out_of_vocabulary_token_is_reported(yb):
    """A sampled id outside the vocabulary skips its seen-table store and sets
    the device error word; every other field is updated as the oracle does."""
    slots, vocab = 4, 16
    dev = dict(storage=torch.zeros((2 * slots, 5), dtype=torch.int32), dense_seen=torch.zeros((slots, vocab),
                                                                                               dtype=torch.bool),
               generated_lengths=torch.zeros(2 * slots, dtype=torch.int64),
               finished_by_eos=torch.zeros(2 * slots, dtype=torch.bool), finished=torch.zeros(slots, dtype=torch.bool),
               slot_rows=torch.arange(slots), sink_rows=slots + torch.arange(slots),
               slot_caps=torch.full((slots,), 4), row_steps=torch.ones(slots, dtype=torch.int64),
               row_positions=torch.zeros(slots, dtype=torch.int64), decode_ids=torch.zeros((slots, 1),
                                                                                           dtype=torch.int64),
               decode_useful_events=torch.zeros((), dtype=torch.int64))
    dev = {k: v.cuda() for k, v in dev.items()}
    yb.lib().yb_device_error(1)
    tok = torch.tensor([[3], [vocab + 5], [0], [7]]).cuda()
    yb.update_fixed_decode_state_(tok, *(dev[k] for k in FIELDS), maximum_new_tokens=4, pad_token_id=0,
                                  eos_token_ids=())
    torch.cuda.synchronize()
    assert yb.lib().yb_device_error(1) == 0x401
    assert dev['dense_seen'][1].sum().item() == 0 and dev['dense_seen'][0, 3].item()
    assert dev['storage'][1, 1].item() == vocab + 5 and int(dev['decode_useful_events']) == slots


class TinyRecurrentLM:
    """A one-layer recurrent decoder on this package's kernels: embedding ->
    q, k, v, gates -> in-place GDN decode step -> logits.  The cache holds the
    recurrent state (one layer), so the graph driver's snapshot covers it."""

    def __init__(self, vocab=97, H=2, HV=4, K=128, V=128, seed=0):
        g = torch.Generator(device='cuda').manual_seed(seed)
        self.H, self.HV, self.K, self.V = H, HV, K, V
        self.emb = torch.randn(vocab, (2 * H * K + HV * V + 2 * HV), generator=g, device='cuda') * 0.3
        self.out = torch.randn(HV * V, vocab, generator=g, device='cuda') * 0.05
        self.config = SimpleNamespace(gdn_recurrent_state_storage='fp32')
        import yanchor_b200
        self.yb = yanchor_b200

    def __call__(self, input_ids, position_ids, past_key_values, use_cache, logits_to_keep):
        H, HV, K, V = self.H, self.HV, self.K, self.V
        B = input_ids.shape[0]
        x = self.emb[input_ids[:, 0]] + 1e-3 * position_ids.to(torch.float32)
        q, k, v, a, b = torch.split(x, [H * K, H * K, HV * V, HV, HV], dim=-1)
        q = q.reshape(B, 1, H, K).to(torch.bfloat16)
        k = k.reshape(B, 1, H, K).to(torch.bfloat16)
        v = v.reshape(B, 1, HV, V).to(torch.bfloat16)
        g = torch.nn.functional.logsigmoid(a).reshape(B, 1, HV)
        beta = torch.sigmoid(b).reshape(B, 1, HV).to(torch.bfloat16)
        state = past_key_values.layers[0].recurrent_states
        o, _ = self.yb.fused_recurrent_gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=state,
                                                        output_final_state=True, use_qk_l2norm_in_kernel=True,
                                                        inplace=True)
        return SimpleNamespace(logits=(o.reshape(B, HV * V).float() @ self.out)[:, None])


def fresh_cache(B, HV=4, K=128, V=128, seed=1):
    g = torch.Generator(device='cuda').manual_seed(seed)
    return SimpleNamespace(layers=[SimpleNamespace(recurrent_states=torch.randn(B, HV, K, V, generator=g,
                                                                                  device='cuda') * 0.02)])


@pytest.mark.parametrize('consume', [False, True])
def test_decode_graph_matches_eager_steps(yb, consume):
    """Greedy decoding through FixedMemoryDecodeGraph (with the bookkeeping
    kernel after each step) equals the same loop run eagerly, token for token
    and state for state."""
    B, steps = 6, 12
    model = TinyRecurrentLM()
    first = torch.randint(0, 97, (B, 1), device='cuda', generator=torch.Generator(device='cuda').manual_seed(3))
    pos0 = torch.arange(100, 100 + B, device='cuda')

    def run(use_graph):
        cache = fresh_cache(B)
        ids, pos = first.clone(), pos0.clone()
        toks = []
        graph = yb.FixedMemoryDecodeGraph(model, cache, ids, pos, consume_capture_steps=consume) if use_graph \
            else None
        for _ in range(steps):
            if use_graph:
                scores = graph.replay(ids, position_ids=pos)
            else:
                scores = model(input_ids=ids, position_ids=pos[:, None], past_key_values=cache, use_cache=True,
                               logits_to_keep=1).logits[:, -1]
            ids = yb.greedy(scores)
            pos = pos + 1
            toks.append(ids.clone())
        if graph is not None:
            graph.close()
        return torch.cat(toks, 1), cache.layers[0].recurrent_states

    t_eager, s_eager = run(False)
    t_graph, s_graph = run(True)
    assert torch.equal(t_eager, t_graph)
    assert torch.equal(s_eager, s_graph)


def test_decode_graph_capture_leaves_cache_unchanged(yb):
    """Without capture-consuming steps the warm-up and capture forwards are
    undone: the cache equals its value before the driver was built."""
    cache = fresh_cache(3)
    before = cache.layers[0].recurrent_states.clone()
    model = TinyRecurrentLM()
    graph = yb.FixedMemoryDecodeGraph(model, cache, torch.zeros((3, 1), dtype=torch.long, device='cuda'), 5)
    assert torch.equal(cache.layers[0].recurrent_states, before)
    assert int(graph.static_position_ids[0]) == 5
    graph.replay(torch.ones((3, 1), dtype=torch.long, device='cuda'))
    assert not torch.equal(cache.layers[0].recurrent_states, before)
    graph.close()
