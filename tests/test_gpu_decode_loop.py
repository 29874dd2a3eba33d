"""GPU parity of the decode-loop plumbing: the bookkeeping kernel against the
reference fixtures and the oracle (bit-exact: integer work), and the CUDA
graph driver against eager decode steps of a small recurrent model built on
this package's kernels."""
import os

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
    q, k, v, gates -> in-place GDN decode step -> logits -> greedy, with the
    state, token ids and positions in tensors at fixed addresses."""

    def __init__(self, rows, vocab=97, H=2, HV=4, K=128, V=128, seed=0):
        g = torch.Generator(device='cuda').manual_seed(seed)
        self.H, self.HV, self.K, self.V = H, HV, K, V
        self.emb = torch.randn(vocab, (2 * H * K + HV * V + 2 * HV), generator=g, device='cuda') * 0.3
        self.out = torch.randn(HV * V, vocab, generator=g, device='cuda') * 0.05
        self.state = torch.randn(rows, HV, K, V, generator=g, device='cuda') * 0.02
        self.ids = torch.randint(0, vocab, (rows, 1), device='cuda', generator=g)
        self.pos = torch.arange(100, 100 + rows, device='cuda')
        import yanchor_b200
        self.yb = yanchor_b200

    def step(self, b):
        """One decode step of the first b rows, in place: returns the ids."""
        H, HV, K, V = self.H, self.HV, self.K, self.V
        x = self.emb[self.ids[:b, 0]] + 1e-3 * self.pos[:b, None].to(torch.float32)
        q, k, v, a, beta = torch.split(x, [H * K, H * K, HV * V, HV, HV], dim=-1)
        q = q.reshape(b, 1, H, K).to(torch.bfloat16)
        k = k.reshape(b, 1, H, K).to(torch.bfloat16)
        v = v.reshape(b, 1, HV, V).to(torch.bfloat16)
        g = torch.nn.functional.logsigmoid(a).reshape(b, 1, HV)
        beta = torch.sigmoid(beta).reshape(b, 1, HV).to(torch.bfloat16)
        o, _ = self.yb.fused_recurrent_gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=self.state[:b],
                                                        output_final_state=True, use_qk_l2norm_in_kernel=True,
                                                        inplace=True)
        scores = o.reshape(b, HV * V).float() @ self.out
        self.ids[:b].copy_(self.yb.greedy(scores))
        self.pos[:b].add_(1)
        return self.ids[:b]

    def warm(self):
        torch.randn(8, 8, device='cuda') @ torch.randn(8, 8, device='cuda')   # cuBLAS set-up


def test_step_graphs_match_eager_steps(yb):
    """Greedy decoding through StepGraphs equals the same loop run eagerly,
    token for token and state for state; capturing leaves the state, ids and
    positions untouched (nothing runs during capture), and a batch between
    two captured sizes replays the larger graph."""
    rows, steps = 8, 12
    eager, graphed = TinyRecurrentLM(rows), TinyRecurrentLM(rows)
    before = (graphed.state.clone(), graphed.ids.clone(), graphed.pos.clone())
    graphs = yb.StepGraphs(graphed.step, [2, 6, 8], warm=graphed.warm)
    assert torch.equal(graphed.state, before[0]) and torch.equal(graphed.ids, before[1])
    assert torch.equal(graphed.pos, before[2])
    assert graphs.bucket(5) == 6 and graphs.bucket(6) == 6 and graphs.bucket(7) == 8
    with pytest.raises(ValueError):
        graphs.bucket(9)
    toks_e, toks_g = [], []
    for t in range(steps):
        b = 6 if t < 5 else 8
        toks_e.append(eager.step(b).clone())
        toks_g.append(graphs.replay(b).clone())
    graphs.close()
    for t, (a, b) in enumerate(zip(toks_e, toks_g)):
        assert torch.equal(a, b), t
    assert torch.equal(eager.state, graphed.state)
    assert torch.equal(eager.pos, graphed.pos)
