"""GPU parity of the prefill side of the anchor memory: top-CAP selection
(select / merge / exclusive prefix) bit-exact against the reference fixtures
and the oracle, and the prefill read / write orchestration against the
reference's ``_sequence`` fixtures (fp32) and the oracle (bf16, YANchor
shape).  Selections, positions, counts and copied rows compare exactly;
reads at 2e-5 (fp32) or 2e-2 (bf16)."""
import numpy as np
import pytest
import torch

from oracle import memory as omem

pytestmark = pytest.mark.gpu

FIELDS = ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values', 'pending_scores', 'count',
          'total')


@pytest.fixture(scope='module')
def yb():
    import yanchor_b200
    return yanchor_b200


def cuda(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t if dtype is None else t.to(dtype)


def host(t):
    return t.detach().cpu().numpy() if t.dtype in (torch.int32, torch.int64, torch.bool) else \
        t.detach().float().cpu().numpy()


def same(got, want):
    for g, w in zip(got, want):
        np.testing.assert_array_equal(host(g), np.asarray(w))


# ---------------------------------------------------------------- selection --
@pytest.mark.parametrize('case,cap', [('sel', 10), ('selpad', 28), ('seledge', 9)])
def test_select_topk_golden(yb, golden, case, cap):
    d = golden('memory')
    src = 'seledge' if case == 'seledge' else 'sel'
    got = yb.select_topk(cuda(d[f'{src}_scores_in']), cuda(d[f'{src}_pos_in']), cuda(d[f'{src}_refs_in']), cap)
    same(got, (d[f'{case}_scores'], d[f'{case}_pos'], d[f'{case}_refs']))


@pytest.mark.parametrize('case,cap', [('pre', 6), ('pre2', 16)])
def test_exclusive_prefix_topk_golden(yb, golden, case, cap):
    d = golden('memory')
    got = yb.exclusive_prefix_topk(cuda(d[f'{case}_scores_in']), cuda(d[f'{case}_pos_in']),
                                   cuda(d[f'{case}_refs_in']), cap)
    same(got, (d[f'{case}_scores'], d[f'{case}_pos'], d[f'{case}_refs']))


def _candidates(rng, B, blocks, G, chunk, invalid=0.2):
    s = (rng.standard_normal((B, blocks, G, chunk)) * 3).round().astype(np.float32) / 2     # many ties
    pos = np.broadcast_to(np.arange(blocks * chunk).reshape(1, blocks, 1, chunk) + 100,
                          (B, blocks, G, chunk)).astype(np.int64).copy()
    refs = pos.copy()
    bad = rng.random(refs.shape) < invalid
    refs[bad] = -1
    s[bad] = -np.inf
    return s, pos, refs


@pytest.mark.parametrize('blocks,chunk,cap', [(37, 64, 64), (5, 100, 64), (9, 16, 40), (1, 64, 64), (0, 64, 64)])
def test_exclusive_prefix_topk_vs_oracle(yb, blocks, chunk, cap):
    rng = np.random.default_rng(blocks * 1000 + chunk + cap)
    B, G = 2, 4
    s, pos, refs = _candidates(rng, B, blocks, G, chunk)
    got = yb.exclusive_prefix_topk(cuda(s), cuda(pos), cuda(refs), cap)
    same(got, omem.exclusive_prefix_topk(s, pos, refs, cap))


def test_exclusive_prefix_topk_with_bank(yb):
    """A seeded bank equals the reference's merge of every prefix entry with it."""
    rng = np.random.default_rng(5)
    B, blocks, G, chunk, cap = 3, 11, 4, 64, 64
    s, pos, refs = _candidates(rng, B, blocks, G, chunk)
    bank_s = (rng.standard_normal((B, G, cap)) * 3).round().astype(np.float32) / 2
    bank_p = rng.integers(0, 100, (B, G, cap)).astype(np.int32)     # older positions
    for b in range(B):
        for g in range(G):
            bank_p[b, g] = rng.permutation(100)[:cap]
    bank_p[rng.random(bank_p.shape) < 0.3] = -1
    bank_s[bank_p < 0] = -np.inf
    got = yb.exclusive_prefix_topk(cuda(s), cuda(pos), cuda(refs), cap, initial=(cuda(bank_s), cuda(bank_p)))
    pre = omem.exclusive_prefix_topk(s, pos, refs, cap)
    bank_r = np.where(bank_p < 0, -1, np.arange(cap)[None, None])
    want = omem.merge_topk(pre, tuple(np.repeat(x[:, None], blocks + 1, 1) for x in (bank_s, bank_p, bank_r)), cap)
    same(got, want)


def test_merge_topk_vs_oracle(yb):
    rng = np.random.default_rng(9)
    a = _candidates(rng, 6, 1, 4, 64)
    b = _candidates(rng, 6, 1, 4, 64)
    b = (b[0], b[1] + 10_000, b[2] + 10_000)
    got = yb.merge_topk(tuple(cuda(x) for x in a), tuple(cuda(x) for x in b), 64)
    same(got, omem.merge_topk(a, b, 64))


def test_select_topk_nan_and_int32(yb):
    s = np.array([[1.0, np.nan, -0.0, 0.0, -np.inf, 2.0, np.nan, 7.0]], np.float32)
    p = np.array([[5, 3, 9, 1, 0, 4, 2, 8]], np.int32)
    r = np.array([[0, 1, 2, 3, 4, 5, 6, -1]], np.int64)
    same(yb.select_topk(cuda(s), cuda(p), cuda(r), 10), omem.select_topk(s, p, r, 10))


# ------------------------------------------------------------ orchestration --
def _state(yb, B, G, CAP, PC, D, dtype):
    return yb.MemoryState.empty(B, G, CAP, PC, D, torch.device('cuda'), dtype)


def test_sequence_golden(yb, golden):
    """The reference's _sequence on a fresh state with a left-padded mask, a
    continuation and the stateless form (fp32)."""
    d = golden('memory')
    B, _, G, D = d['seq1_k'].shape
    CAP, PC = d['seq1_state_keys'].shape[2], d['seq1_state_pending_keys'].shape[2]
    state = _state(yb, B, G, CAP, PC, D, torch.float32)
    for name, stateful in (('seq1', True), ('seq2', True), ('seq3', False)):
        K, V = cuda(d[f'{name}_k']), cuda(d[f'{name}_v'])
        valid = cuda(d[f'{name}_valid']) if f'{name}_valid' in d else None
        o = yb.sequence(cuda(d[f'{name}_q']), cuda(d[f'{name}_scores']), lambda b, t: (K[b, t], V[b, t]), valid,
                        PC, state if stateful else None, capacity=CAP)
        np.testing.assert_allclose(host(o), d[f'{name}_o'], atol=2e-5)
        if stateful:
            for f in FIELDS:
                got, want = host(getattr(state, f)), d[f'{name}_state_{f}']
                if f in ('keys', 'values', 'pending_keys', 'pending_values'):
                    np.testing.assert_allclose(got, want, atol=1e-6, err_msg=f'{name} {f}')
                else:
                    np.testing.assert_array_equal(got, want, err_msg=f'{name} {f}')


def test_sequence_bf16_yanchor_shape(yb):
    """YANchor memory shape (H=16, G=4, D=256, CAP=64, chunk 64), bf16,
    against the oracle: a left-padded first prefill, a left-padded
    continuation (pending tokens and padding in the same block), unmasked
    continuations, and a mask with holes (the gather path)."""
    rng = np.random.default_rng(77)
    B, H, G, D, CAP, CH = 3, 16, 4, 256, 64, 64
    bf = torch.bfloat16
    state = _state(yb, B, G, CAP, CH, D, bf)
    st = omem.empty_state(B, G, CAP, CH, D)
    calls = [(300, 'left'), (150, 'left'), (64, None), (77, 'holes'), (129, None)]
    for T, mask in calls:
        q = cuda(rng.standard_normal((B, T, H, D)).astype(np.float32), bf)
        sc = cuda((rng.standard_normal((B, T, G)) * 2).round().astype(np.float32) / 2)
        K = cuda(rng.standard_normal((B, T, G, D)).astype(np.float32), bf)
        V = cuda(rng.standard_normal((B, T, G, D)).astype(np.float32), bf)
        valid = None
        if mask == 'left':
            vm = np.ones((B, T), bool)
            vm[1, :37] = False
            vm[2, :T - 70] = False
            valid = cuda(vm)
        elif mask == 'holes':
            vm = rng.random((B, T)) > 0.3
            vm[0] = False                                   # a row with nothing new
            valid = cuda(vm)
        o = yb.sequence(q, sc, lambda b, t: (K[b, t], V[b, t]), valid, CH, state)
        want = omem.sequence(host(q), host(sc), host(K), host(V), None if valid is None else host(valid), CH, st)
        assert np.abs(host(o) - want).max() <= 2e-2, f'T={T} {mask}'
        for f in FIELDS:
            np.testing.assert_array_equal(host(getattr(state, f)), st[f].astype(host(getattr(state, f)).dtype),
                                          err_msg=f'T={T} {mask} {f}')


def test_sequence_capture_safe_matches_and_graphs(yb):
    """capture_safe=True (the writer on every timeline slot, the mask kind
    given by the caller, no host synchronisation) gives results identical to
    the default path over the same calls as the YANchor-shape test, and a
    left-padded call captured in a CUDA graph and replayed gives them too."""
    rng = np.random.default_rng(78)
    B, H, G, D, CAP, CH = 3, 16, 4, 256, 64, 64
    bf = torch.bfloat16
    st_a, st_b = _state(yb, B, G, CAP, CH, D, bf), _state(yb, B, G, CAP, CH, D, bf)
    calls = [(300, 'left'), (150, 'left'), (64, None), (77, 'holes'), (129, None)]
    for T, mask in calls:
        q = cuda(rng.standard_normal((B, T, H, D)).astype(np.float32), bf)
        sc = cuda((rng.standard_normal((B, T, G)) * 2).round().astype(np.float32) / 2)
        K = cuda(rng.standard_normal((B, T, G, D)).astype(np.float32), bf)
        V = cuda(rng.standard_normal((B, T, G, D)).astype(np.float32), bf)
        valid, run = None, None
        if mask == 'left':
            vm = np.ones((B, T), bool)
            vm[1, :37] = False
            vm[2, :T - 70] = False
            valid, run = cuda(vm), True
        elif mask == 'holes':
            vm = rng.random((B, T)) > 0.3
            vm[0] = False
            valid, run = cuda(vm), False
        writer = lambda b, t: (K[b, t], V[b, t])  # noqa: E731
        o_a = yb.sequence(q, sc, writer, valid, CH, st_a)
        o_b = yb.sequence(q, sc, writer, valid, CH, st_b, capture_safe=True, mask_is_run=run)
        assert torch.equal(o_a, o_b), f'T={T} {mask}'
        for f in FIELDS:
            assert torch.equal(getattr(st_a, f), getattr(st_b, f)), f'T={T} {mask} {f}'
    # a graph of one left-padded call on a copy of the state, replayed: the same as the eager call
    T = 200
    q = cuda(rng.standard_normal((B, T, H, D)).astype(np.float32), bf)
    sc = cuda((rng.standard_normal((B, T, G)) * 2).round().astype(np.float32) / 2)
    K = cuda(rng.standard_normal((B, T, G, D)).astype(np.float32), bf)
    V = cuda(rng.standard_normal((B, T, G, D)).astype(np.float32), bf)
    vm = np.ones((B, T), bool)
    vm[0, :20] = False
    valid = cuda(vm)
    writer = lambda b, t: (K[b, t], V[b, t])  # noqa: E731
    st_g = yb.MemoryState(*(getattr(st_b, f).clone() for f in FIELDS))
    saved = [getattr(st_g, f).clone() for f in FIELDS]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):      # warm-up (library set-up, allocator pools) on the copy
        yb.sequence(q, sc, writer, valid, CH, st_g, capture_safe=True, mask_is_run=True)
    torch.cuda.current_stream().wait_stream(side)
    for f, t in zip(FIELDS, saved):
        getattr(st_g, f).copy_(t)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o_g = yb.sequence(q, sc, writer, valid, CH, st_g, capture_safe=True, mask_is_run=True)
    graph.replay()
    o_a = yb.sequence(q, sc, writer, valid, CH, st_a)
    torch.cuda.synchronize()
    assert torch.equal(o_g, o_a)
    for f in FIELDS:
        assert torch.equal(getattr(st_g, f), getattr(st_a, f)), f
    del graph
