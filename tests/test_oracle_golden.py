"""Pin the numpy oracle to fixtures produced by the reference's own torch code
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest

from oracle import gdn, memory, sampling


def close(a, b, atol, rtol=0.0):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    fin = np.isfinite(a) & np.isfinite(b)
    err = np.abs(a - b)[fin].max() if fin.any() else 0.0
    assert np.allclose(a, b, atol=atol, rtol=rtol), f'max abs err {err}'


# ---------------------------------------------------------------- GDN ------
def test_l2norm(golden):
    d = golden('gdn')
    close(gdn.l2norm(d['small_q'])[:, :8], d['small_l2q_head'], 1e-6)


@pytest.mark.parametrize('form', ['chunk', 'rec'])
def test_gdn_small(golden, form):
    d = golden('gdn')
    fn = gdn.chunk_gated_delta_rule if form == 'chunk' else gdn.recurrent_gated_delta_rule
    o, s = fn(d['small_q'], d['small_k'], d['small_v'], d['small_g'], d['small_beta'],
              initial_state=d['small_h0'], use_qk_l2norm=True)
    close(o, d[f'small_{form}_o'], 2e-5)
    close(s, d[f'small_{form}_s'], 2e-5)


def test_gdn_config0_recipe(golden):
    """Config-0 recipe: q, k normalised up front, zero initial state."""
    d = golden('gdn')
    q, k = gdn.l2norm(d['small_q']), gdn.l2norm(d['small_k'])
    o, s = gdn.chunk_gated_delta_rule(q, k, d['small_v'], d['small_g'], d['small_beta'])
    close(o, d['small_chunk0_o'], 2e-5)
    close(s, d['small_chunk0_s'], 2e-5)


@pytest.mark.parametrize('form', ['chunk', 'rec'])
def test_gdn_gva_varlen(golden, form):
    d = golden('gdn')
    fn = gdn.chunk_gated_delta_rule if form == 'chunk' else gdn.recurrent_gated_delta_rule
    o, s = fn(d['var_q'], d['var_k'], d['var_v'], d['var_g'], d['var_beta'], initial_state=d['var_h0'],
              use_qk_l2norm=True, cu_seqlens=d['var_cu'])
    close(o, d[f'var_{form}_o'], 2e-5)
    close(s, d[f'var_{form}_s'], 2e-5)


def test_chunk_equals_recurrent_float64(golden):
    d = golden('gdn')
    args = (d['var_q'], d['var_k'], d['var_v'], d['var_g'], d['var_beta'])
    kw = dict(initial_state=d['var_h0'], use_qk_l2norm=True, cu_seqlens=d['var_cu'], dtype=np.float64)
    o1, s1 = gdn.chunk_gated_delta_rule(*args, **kw)
    o2, s2 = gdn.recurrent_gated_delta_rule(*args, **kw)
    close(o1, o2, 1e-10)
    close(s1, s2, 1e-10)


def test_transposed_state_layout(golden):
    d = golden('gdn')
    args = (d['var_q'], d['var_k'], d['var_v'], d['var_g'], d['var_beta'])
    h0t = d['var_h0'].swapaxes(-1, -2)
    o, s = gdn.recurrent_gated_delta_rule(*args, initial_state=h0t, use_qk_l2norm=True,
                                          cu_seqlens=d['var_cu'], transpose_state=True)
    close(o, d['var_rec_o'], 2e-5)
    close(s.swapaxes(-1, -2), d['var_rec_s'], 2e-5)


def test_gates(golden):
    d = golden('gdn')
    g, beta = gdn.gdn_gates(d['gate_a'], d['gate_b'], d['gate_A_log'], d['gate_dt_bias'])
    close(g, d['gate_g'], 1e-5, 1e-6)
    close(beta, d['gate_beta'], 1e-6)


def test_rmsnorm_gated(golden):
    d = golden('gdn')
    close(gdn.rmsnorm_gated(d['norm_x'], d['norm_z'], d['norm_w']), d['norm_out'], 1e-5)


# ------------------------------------------------------------- memory ------
def test_select_topk(golden):
    d = golden('memory')
    s, p, r = memory.select_topk(d['sel_scores_in'], d['sel_pos_in'], d['sel_refs_in'], 10)
    np.testing.assert_array_equal(s, d['sel_scores'])
    np.testing.assert_array_equal(p, d['sel_pos'])
    np.testing.assert_array_equal(r, d['sel_refs'])
    s, p, r = memory.select_topk(d['sel_scores_in'], d['sel_pos_in'], d['sel_refs_in'], 28)
    np.testing.assert_array_equal(s, d['selpad_scores'])
    np.testing.assert_array_equal(p, d['selpad_pos'])
    np.testing.assert_array_equal(r, d['selpad_refs'])


def test_exclusive_prefix_topk(golden):
    d = golden('memory')
    s, p, r = memory.exclusive_prefix_topk(d['pre_scores_in'], d['pre_pos_in'], d['pre_refs_in'], 6)
    np.testing.assert_array_equal(s, d['pre_scores'])
    np.testing.assert_array_equal(p, d['pre_pos'])
    np.testing.assert_array_equal(r, d['pre_refs'])


def test_select_topk_edges(golden):
    """NaN scores rank first, invalid references keep finite scores, int32 positions."""
    d = golden('memory')
    s, p, r = memory.select_topk(d['seledge_scores_in'], d['seledge_pos_in'], d['seledge_refs_in'], 9)
    np.testing.assert_array_equal(s, d['seledge_scores'])
    np.testing.assert_array_equal(p, d['seledge_pos'])
    np.testing.assert_array_equal(r, d['seledge_refs'])


def test_exclusive_prefix_topk_odd_blocks(golden):
    d = golden('memory')
    s, p, r = memory.exclusive_prefix_topk(d['pre2_scores_in'], d['pre2_pos_in'], d['pre2_refs_in'], 16)
    np.testing.assert_array_equal(s, d['pre2_scores'])
    np.testing.assert_array_equal(p, d['pre2_pos'])
    np.testing.assert_array_equal(r, d['pre2_refs'])


SEQ_FIELDS = ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values', 'pending_scores',
              'count', 'total')


def test_sequence_prefill(golden):
    """Prefill read + write against the reference's _sequence: a fresh state
    with a left-padded mask, a continuation, and the stateless form."""
    d = golden('memory')
    B, G, D = d['seq1_k'].shape[0], d['seq1_k'].shape[2], d['seq1_k'].shape[3]
    CAP, CHUNK = d['seq1_state_keys'].shape[2], d['seq1_state_pending_keys'].shape[2]
    state = memory.empty_state(B, G, CAP, CHUNK, D)
    for name, stateful in (('seq1', True), ('seq2', True), ('seq3', False)):
        valid = d.get(f'{name}_valid')
        o = memory.sequence(d[f'{name}_q'], d[f'{name}_scores'], d[f'{name}_k'], d[f'{name}_v'], valid, CHUNK,
                            state if stateful else None, capacity=CAP)
        close(o, d[f'{name}_o'], 2e-5)
        if stateful:
            for f in SEQ_FIELDS:
                if state[f].dtype.kind == 'f':
                    close(state[f], d[f'{name}_state_{f}'], 2e-5)
                else:
                    np.testing.assert_array_equal(state[f], d[f'{name}_state_{f}'], err_msg=f'{name} {f}')


def test_indexed_gqa(golden):
    d = golden('memory')
    out = memory.indexed_gqa(d['idx_q'], d['idx_k'], d['idx_v'], d['idx_refs'])
    close(out, d['idx_out'], 2e-5)


def _replay_decode(d, upto):
    B, G, D = d['dec_k'].shape[1], d['dec_k'].shape[3], d['dec_k'].shape[4]
    CAP = d['dec_final_keys'].shape[2]
    PC = d['dec_final_pending_keys'].shape[2]
    st = memory.empty_state(B, G, CAP, PC, D)
    reads = []
    for t in range(upto):
        k0 = st['keys'].copy()
        reads.append(memory.decode_read(d['dec_q'][t], st['keys'], st['values'], st['positions'])
                     * d['dec_valid'][t][..., None, None])
        memory.commit_decode(d['dec_k'][t], d['dec_v'][t], d['dec_scores'][t], d['dec_valid'][t][:, 0], 8, st)
        del k0
    return st, np.stack(reads)


def test_decode_read_commit_sequence(golden):
    d = golden('memory')
    steps = d['dec_q'].shape[0]
    for t in (7, 20):
        st, _ = _replay_decode(d, t + 1)
        for f in st:
            np.testing.assert_allclose(st[f], d[f'dec_t{t}_{f}'], atol=0, err_msg=f)
    st, reads = _replay_decode(d, steps)
    close(reads, d['dec_reads'], 2e-5)
    for f in st:
        np.testing.assert_allclose(st[f], d[f'dec_final_{f}'], atol=0, err_msg=f)


# ----------------------------------------------------------- sampling ------
def test_counter_uniform(golden):
    d = golden('sampling')
    for seed, stream in ((0, 0), (1234, 0), (2**32 + 99, 3)):
        u = sampling.counter_uniform(d['cu_ids'], d['cu_steps'], seed, stream)
        np.testing.assert_array_equal(u, d[f'cu_u_{seed}_{stream}'])


def test_sampler(golden):
    d = golden('sampling')
    for i in range(sum(1 for k in d if k.startswith('samp_case'))):
        temp, tk, tp = d[f'samp_case{i}']
        got = sampling.sample_top_k_top_p_counter(d['samp_scores'], d['samp_attempt'], d['samp_steps'], 77,
                                                  float(temp), int(tk), float(tp))
        np.testing.assert_array_equal(got, d[f'samp_out{i}'], err_msg=f'case {i}')


# --------------------------------------------------------------- conv1d ------
def test_conv_update(golden):
    from oracle import conv
    d = golden('conv')
    y, st = conv.conv_update(d['conv_upd_x'], d['conv_upd_state'], d['conv_w'])
    close(y, d['conv_upd_y'], 1e-5)
    close(st, d['conv_upd_state_after'], 0.0)


@pytest.mark.parametrize('name,cached', [('conv_pre', False), ('conv_prec', True), ('conv_pres', False)])
def test_conv_prefill(golden, name, cached):
    from oracle import conv
    d = golden('conv')
    y, st = conv.conv_fwd(d[f'{name}_x'], d['conv_w'], initial_state=d['conv_prec_state_in'] if cached else None)
    close(y, d[f'{name}_y'], 1e-5)
    close(st, d[f'{name}_state'], 0.0)


# ------------------------------------------------------------------ SWA ------
def test_swa_decode_attention(golden):
    from oracle import swa
    d = golden('swa')
    close(swa.decode_attention(d['swa_q'], d['swa_k'], d['swa_v'], d['swa_valid']), d['swa_out'], 2e-6)


def test_swa_decode_attention_empty_row_matches_reference():
    """A ring row with no valid position: the reference's own decode attention
    (runtime/model/inference_kernels.py:1881-1897, run here on the CPU from
    its install) gives zeros for it under the installed torch; the oracle
    does the same, and the other rows agree."""
    import _reference
    if not _reference.available():
        pytest.skip('SKIPPED, NOT PASSED: the reference install (baseline/_ref) is absent')
    import torch
    from oracle import swa
    ik = _reference.inference_kernels()
    rng = np.random.default_rng(3)
    B, QH, KVH, W, D = 3, 4, 2, 9, 16
    q = rng.standard_normal((B, 1, QH, D))
    k = rng.standard_normal((B, KVH, W, D))
    v = rng.standard_normal((B, KVH, W, D))
    valid = rng.random((B, W)) > 0.4
    valid[1] = False
    ref = ik.fixed_memory_physical_ring_decode_attention(*(torch.from_numpy(x) for x in (q, k, v, valid))).numpy()
    assert np.all(ref[1] == 0)
    close(swa.decode_attention(q, k, v, valid), ref, 1e-12)


@pytest.mark.parametrize('case', ['a', 'b', 'c'])
def test_swa_prefill_attention(golden, case):
    """reference_swa: plain causal window, left padding through key validity,
    a query block after a cached window with holes."""
    from oracle import swa
    d = golden('swa_prefill')
    window, qs = (int(x) for x in d[f'sp{case}_meta'])
    kv = d[f'sp{case}_valid'] if f'sp{case}_valid' in d else None
    close(swa.prefill_attention(d[f'sp{case}_q'], d[f'sp{case}_k'], d[f'sp{case}_v'], window, kv, qs),
          d[f'sp{case}_out'], 2e-6)


def test_flash_prefill_matches_reference_swa_on_contiguous_masks(golden):
    """flash_swa counts valid tokens only; on left-padded rows (one contiguous
    valid run per row) that is the same as reference_swa's absolute positions."""
    from oracle import swa
    d = golden('swa_prefill')
    window, _ = (int(x) for x in d['spb_meta'])
    close(swa.flash_prefill(d['spb_q'], d['spb_k'], d['spb_v'], window, d['spb_valid']), d['spb_out'], 2e-6)
