"""GPU parity of the anchor-memory kernels against the reference fixtures and
the CPU oracle.  Integer state (positions, count, total) and copied rows
(bank keys / values, scores) must match exactly; reads are float and compare
at 1e-5 (fp32) or 2e-2 (bf16)."""
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


def to_device_state(yb, st, dtype):
    return yb.MemoryState(*(cuda(st[f], dtype if st[f].dtype == np.float32 and 'score' not in f else None)
                            for f in FIELDS))


def test_decode_sequence_matches_reference(yb, golden):
    """Replay the reference's 41-step decode (fixed ties, inactive rows,
    several commits) on the GPU."""
    d = golden('memory')
    B, G, D = d['dec_k'].shape[1], d['dec_k'].shape[3], d['dec_k'].shape[4]
    CAP, PC = d['dec_final_keys'].shape[2], d['dec_final_pending_keys'].shape[2]
    st = yb.MemoryState.empty(B, G, CAP, PC, D, 'cuda', torch.float32)
    for t in range(d['dec_q'].shape[0]):
        read = yb.committed_gqa(cuda(d['dec_q'][t]), st) * cuda(d['dec_valid'][t])[..., None, None]
        np.testing.assert_allclose(host(read), d['dec_reads'][t], atol=1e-5, err_msg=f'step {t}')
        yb.commit_decode(cuda(d['dec_k'][t]), cuda(d['dec_v'][t]), cuda(d['dec_scores'][t]),
                         cuda(d['dec_valid'][t][:, 0]), 8, st)
        if t in (7, 20):
            for f in FIELDS:
                np.testing.assert_array_equal(host(getattr(st, f)), d[f'dec_t{t}_{f}'], err_msg=f'{f} @ {t}')
    for f in FIELDS:
        np.testing.assert_array_equal(host(getattr(st, f)), d[f'dec_final_{f}'], err_msg=f)


def test_decode_yanchor_shape_bf16_with_pool_indices(yb):
    """YANchor-4B memory shape (G=4, H=16, D=256, CAP=64, chunk=64), bf16,
    requests mapped into a larger slot pool through indices (-1 = skip)."""
    rng = np.random.default_rng(40)
    B, POOL, G, H, D, CAP, CH, STEPS = 6, 9, 4, 16, 256, 64, 64, 150
    indices = np.array([3, 0, -1, 8, 5, 1], dtype=np.int64)
    st_np = omem.empty_state(POOL, G, CAP, CH, D)
    bf = torch.bfloat16
    st = to_device_state(yb, st_np, bf)
    for t in range(STEPS):
        q = rng.standard_normal((B, 1, H, D)).astype(np.float32)
        k = rng.standard_normal((B, 1, G, D)).astype(np.float32)
        v = rng.standard_normal((B, 1, G, D)).astype(np.float32)
        sc = np.round(rng.standard_normal((B, 1, G)) * 4).astype(np.float32) / 4   # frequent ties
        act = rng.random(B) > 0.1
        qb, kb, vb = cuda(q, bf), cuda(k, bf), cuda(v, bf)
        read = yb.committed_gqa(qb, st, cuda(indices))
        ref_read = omem.decode_read(host(qb), st_np['keys'], st_np['values'], st_np['positions'], indices)
        assert np.abs(host(read) - ref_read).max() <= 2e-2, t
        yb.commit_decode(kb, vb, cuda(sc), cuda(act), CH, st, cuda(indices))
        omem.commit_decode(host(kb), host(vb), sc, act, CH, st_np, indices)
    for f in FIELDS:
        np.testing.assert_array_equal(host(getattr(st, f)), st_np[f].astype(host(getattr(st, f)).dtype),
                                      err_msg=f)


def test_decode_strided_pool_view(yb):
    """State fields that are views into a wider page (batch stride larger than
    the row), as the vLLM adapter passes."""
    rng = np.random.default_rng(41)
    B, G, H, D, CAP, CH = 4, 2, 4, 64, 16, 8
    st_np = omem.empty_state(B, G, CAP, CH, D)
    pad = lambda x, extra: torch.cat([x, torch.zeros((x.shape[0], extra) + x.shape[2:], dtype=x.dtype,  # noqa: E731
                                                                 device=x.device)], 1)[:, :x.shape[1]]
    base = to_device_state(yb, st_np, torch.float32)
    st = yb.MemoryState(*(pad(getattr(base, f), 3) if getattr(base, f).dim() > 1 else getattr(base, f)
                          for f in FIELDS))
    assert st.keys.stride(0) != G * CAP * D
    for t in range(20):
        q = rng.standard_normal((B, 1, H, D)).astype(np.float32)
        k = rng.standard_normal((B, 1, G, D)).astype(np.float32)
        v = rng.standard_normal((B, 1, G, D)).astype(np.float32)
        sc = rng.standard_normal((B, 1, G)).astype(np.float32)
        act = np.ones(B, bool)
        read = yb.committed_gqa(cuda(q), st)
        np.testing.assert_allclose(host(read), omem.decode_read(q, st_np['keys'], st_np['values'],
                                                                st_np['positions']), atol=1e-5)
        yb.commit_decode(cuda(k), cuda(v), cuda(sc), cuda(act), CH, st)
        omem.commit_decode(k, v, sc, act, CH, st_np)
    for f in FIELDS:
        np.testing.assert_array_equal(host(getattr(st, f)), st_np[f].astype(host(getattr(st, f)).dtype))


@pytest.mark.parametrize('R,D,pool,dt', [(4, 256, False, torch.bfloat16), (2, 128, True, torch.bfloat16),
                                         (8, 64, False, torch.float16), (1, 256, True, torch.float16)])
def test_memory_decode_step_matches_read_then_commit(yb, R, D, pool, dt):
    """The one-launch decode step of a memory layer against committed_gqa
    then commit_decode on a copy of the same state, bit for bit, over 170
    steps (two commits at chunk 64 for rows active in 128 of them, the second
    merging a full bank with a full chunk): tied scores, inactive rows, and (pool)
    requests mapped into a larger slot pool with one skipped request."""
    rng = np.random.default_rng(90 + D + R)
    B, G, CAP, chunk = 6, 4, 64, 64
    H = G * R
    bf = dt
    rows = 9 if pool else B
    idx = cuda(np.array([3, 0, -1, 8, 5, 1], np.int64)) if pool else None
    st_a = yb.MemoryState.empty(rows, G, CAP, chunk, D, 'cuda', bf)
    st_b = yb.MemoryState.empty(rows, G, CAP, chunk, D, 'cuda', bf)
    for t in range(170):
        q = cuda(rng.standard_normal((B, 1, H, D)), bf)
        k = cuda(rng.standard_normal((B, 1, G, D)), bf)
        v = cuda(rng.standard_normal((B, 1, G, D)), bf)
        sc = cuda(np.round(rng.standard_normal((B, 1, G)) * 2).astype(np.float32) / 2)   # ties
        act = cuda(rng.random(B) > 0.15)
        out_a = yb.memory_decode_step(q, k, v, sc, act, chunk, st_a, indices=idx)
        out_b = yb.committed_gqa(q, st_b, indices=idx)
        yb.commit_decode(k, v, sc, act, chunk, st_b, indices=idx)
        assert torch.equal(out_a, out_b), f'read @ {t}'
        if t in (62, 63, 64, 127, 150, 169):
            for f in FIELDS:
                assert torch.equal(getattr(st_a, f), getattr(st_b, f)), f'{f} @ {t}'
    assert int(st_a.positions.max()) >= 64   # the bank holds rows from the second chunk
    assert yb.lib().yb_device_error(1) == 0


@pytest.mark.parametrize('CAP,chunk', [(64, 64), (40, 24), (64, 96)])
def test_memory_decode_step_nan_scores_match_oracle(yb, CAP, chunk):
    """Merges with NaN admission scores among tied ones: NaN ranks ahead of
    every number and NaNs tie with each other (torch's descending sort),
    then position, then candidate index.  The one-launch step (its commit
    warps rank one candidate each: 64 + 64 and 40 + 24 here; 64 + 96 has
    more candidates than commit threads and takes the two launches) against
    the read and commit launches and the oracle, every state field bit for
    bit."""
    rng = np.random.default_rng(7 * CAP + chunk)
    B, G, H, D = 4, 4, 16, 256
    bf = torch.bfloat16
    st_a = yb.MemoryState.empty(B, G, CAP, chunk, D, 'cuda', bf)
    st_b = yb.MemoryState.empty(B, G, CAP, chunk, D, 'cuda', bf)
    st_np = omem.empty_state(B, G, CAP, chunk, D)
    for t in range(2 * chunk + 5):
        q = cuda(rng.standard_normal((B, 1, H, D)), bf)
        k = cuda(rng.standard_normal((B, 1, G, D)), bf)
        v = cuda(rng.standard_normal((B, 1, G, D)), bf)
        sc = np.round(rng.standard_normal((B, 1, G)) * 2).astype(np.float32) / 2
        sc[rng.random((B, 1, G)) < 0.1] = np.nan
        act = rng.random(B) > 0.1
        out_a = yb.memory_decode_step(q, k, v, cuda(sc), cuda(act), chunk, st_a)
        out_b = yb.committed_gqa(q, st_b)
        yb.commit_decode(k, v, cuda(sc), cuda(act), chunk, st_b)
        omem.commit_decode(host(k), host(v), sc, act, chunk, st_np)
        assert torch.equal(out_a, out_b), f'read @ {t}'
    for f in FIELDS:
        a, b = host(getattr(st_a, f)), host(getattr(st_b, f))
        np.testing.assert_array_equal(a, b, err_msg=f)
        np.testing.assert_array_equal(a, st_np[f].astype(a.dtype), err_msg=f)
    assert np.isnan(host(st_a.scores)).any()   # NaN entries made it into the banks
    assert yb.lib().yb_device_error(1) == 0


def test_indexed_read_golden(yb, golden):
    d = golden('memory')
    out = yb.indexed_gqa(cuda(d['idx_q']), cuda(d['idx_k']), cuda(d['idx_v']), cuda(d['idx_refs']))
    np.testing.assert_allclose(host(out), d['idx_out'], atol=1e-5)


@pytest.mark.parametrize('kb', [1, 2])
def test_indexed_read_bf16_yanchor_shape(yb, kb):
    rng = np.random.default_rng(42 + kb)
    B, blocks, chunk, H, G, D, S, CAP = 2, 3, 64, 16, 4, 256, 300, 64
    q = rng.standard_normal((B, blocks, chunk, H, D)).astype(np.float32)
    k = rng.standard_normal((kb, S, G, D)).astype(np.float32)
    v = rng.standard_normal((kb, S, G, D)).astype(np.float32)
    refs = rng.integers(0, S, (B, blocks, G, CAP)).astype(np.int64)
    refs[rng.random(refs.shape) < 0.2] = -1
    refs[1, 2, 3] = -1
    bf = torch.bfloat16
    qb, kb_, vb = cuda(q, bf), cuda(k, bf), cuda(v, bf)
    out = yb.indexed_gqa(qb, kb_, vb, cuda(refs))
    ref = omem.indexed_gqa(host(qb), host(kb_), host(vb), refs)
    assert np.abs(host(out) - ref).max() <= 2e-2
    assert not host(out)[1, 2, :, 12:16].any()      # no anchors: only the null slot


def test_vllm_page_pool_decode(yb):
    """The decode read + commit on a pool of vLLM memory pages (views, no
    copies) with state indices (one request skipped) equal the oracle."""
    from yanchor_b200 import independent_memory as im
    rng = np.random.default_rng(8)
    B, H, G, D, CAP, CH, P, steps = 4, 16, 4, 256, 64, 64, 6, 70
    vs, ms = im.vllm_page_shapes(G, CAP, CH, D)
    values = torch.empty((P,) + vs, device='cuda', dtype=torch.bfloat16)
    meta = torch.empty((P,) + ms, device='cuda')
    st = im.state_from_vllm_page(values, meta, G, CAP, CH, D)
    im.reset_vllm_page_(st)
    idx = np.array([3, 0, -1, 5], np.int64)
    pool_np = omem.empty_state(P, G, CAP, CH, D)
    for t in range(steps):
        q = rng.standard_normal((B, 1, H, D)).astype(np.float32)
        k = rng.standard_normal((B, 1, G, D)).astype(np.float32)
        v = rng.standard_normal((B, 1, G, D)).astype(np.float32)
        sc = (rng.standard_normal((B, 1, G)) * 2).round().astype(np.float32) / 2
        act = rng.random(B) > 0.1
        bf = torch.bfloat16
        qb, kb, vb = cuda(q, bf), cuda(k, bf), cuda(v, bf)
        r = yb.committed_gqa(qb, st, cuda(idx))
        er = omem.decode_read(host(qb), pool_np['keys'], pool_np['values'], pool_np['positions'], idx)
        assert np.abs(host(r) - er).max() <= 2e-2
        yb.commit_decode(kb, vb, cuda(sc), cuda(act), CH, st, cuda(idx))
        omem.commit_decode(host(kb), host(vb), sc, act, CH, pool_np, idx)
    for f in FIELDS:
        np.testing.assert_array_equal(host(getattr(st, f)), pool_np[f].astype(host(getattr(st, f)).dtype),
                                      err_msg=f)


@pytest.mark.parametrize('R,D,CAP', [(1, 64, 16), (2, 128, 40), (4, 256, 64), (8, 128, 64), (4, 64, 1)])
@pytest.mark.parametrize('dt', [torch.bfloat16, torch.float16])
def test_decode_read_16bit_shapes(yb, R, D, CAP, dt):
    """The 16-bit decode read (tensor-core path for banks of <= 64 slots):
    head groups of 1-8, head dims 64-256, partly empty banks, a bank with no
    entry (only the null slot), pool indices with a skipped request."""
    rng = np.random.default_rng(R * 1000 + D + CAP)
    B, G, POOL = 5, 3, 7
    H = G * R
    st = omem.empty_state(POOL, G, CAP, 4, D)
    st['keys'][:] = rng.standard_normal(st['keys'].shape) * 2
    st['values'][:] = rng.standard_normal(st['values'].shape)
    st['positions'][:] = np.where(rng.random(st['positions'].shape) < 0.7,
                                  rng.integers(0, 1000, st['positions'].shape), -1)
    st['positions'][2, 1] = -1                          # nothing stored: the null slot only
    dev = to_device_state(yb, st, dt)
    q = rng.standard_normal((B, 1, H, D)).astype(np.float32)
    idx = np.array([2, 0, -1, 6, 3], np.int64)
    qd = cuda(q, dt)
    out = yb.committed_gqa(qd, dev, cuda(idx))
    ref = omem.decode_read(host(qd), host(dev.keys), host(dev.values), st['positions'], idx)
    assert np.abs(host(out) - ref).max() <= 2e-2
    assert not host(out)[2].any()


def test_memory_decode_step_graph_survives_counter_growth(yb):
    """A CUDA graph captured around memory_decode_step at B=8 keeps the
    arrival counters it was captured with.  An eager call at B=128 makes the
    module grow its counter buffer; the captured graph must still replay
    correctly afterwards (its counters are never freed or reused), over 70
    steps that cross one commit at chunk 64, bit-exact against the oracle
    (modeling_yanchor.py:277-313 restated in oracle/memory.py)."""
    rng = np.random.default_rng(77)
    B, G, H, D, CAP, CH = 8, 4, 16, 256, 64, 64
    bf = torch.bfloat16
    st_np = omem.empty_state(B, G, CAP, CH, D)
    st = to_device_state(yb, st_np, bf)
    q = torch.zeros(B, 1, H, D, device='cuda', dtype=bf)
    k = torch.zeros(B, 1, G, D, device='cuda', dtype=bf)
    v = torch.zeros(B, 1, G, D, device='cuda', dtype=bf)
    sc = torch.zeros(B, 1, G, device='cuda')
    act = torch.ones(B, device='cuda', dtype=torch.bool)
    # warm up on a scratch state (the first call may set up the module), then capture
    scratch = yb.MemoryState.empty(B, G, CAP, CH, D, 'cuda', bf)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        yb.memory_decode_step(q, k, v, sc, act, CH, scratch)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = yb.memory_decode_step(q, k, v, sc, act, CH, st)
    # an eager call at a larger batch grows the module's counter buffer
    big = yb.MemoryState.empty(128, G, CAP, CH, D, 'cuda', bf)
    yb.memory_decode_step(torch.randn(128, 1, H, D, device='cuda').to(bf), torch.randn(128, 1, G, D, device='cuda').to(bf),
                          torch.randn(128, 1, G, D, device='cuda').to(bf), torch.randn(128, 1, G, device='cuda'),
                          torch.ones(128, device='cuda', dtype=torch.bool), CH, big)
    filler = [torch.full((1 << 16,), 7, device='cuda', dtype=torch.int32) for _ in range(8)]   # reuse freed memory
    torch.cuda.synchronize()
    for t in range(70):
        qn = rng.standard_normal((B, 1, H, D)).astype(np.float32)
        kn = rng.standard_normal((B, 1, G, D)).astype(np.float32)
        vn = rng.standard_normal((B, 1, G, D)).astype(np.float32)
        sn = np.round(rng.standard_normal((B, 1, G)) * 2).astype(np.float32) / 2
        q.copy_(cuda(qn, bf))
        k.copy_(cuda(kn, bf))
        v.copy_(cuda(vn, bf))
        sc.copy_(cuda(sn))
        graph.replay()
        ref = omem.decode_read(host(q), st_np['keys'], st_np['values'], st_np['positions'])
        assert np.abs(host(out) - ref).max() <= 2e-2, t
        omem.commit_decode(host(k), host(v), sn, np.ones(B, bool), CH, st_np)
    for f in FIELDS:
        np.testing.assert_array_equal(host(getattr(st, f)), st_np[f].astype(host(getattr(st, f)).dtype), err_msg=f)
    assert all(int(x.min()) == 7 for x in filler)
    del graph
