"""GPU parity of the gated-delta-rule kernels against the CPU oracle and the
reference-generated fixtures.

Tolerances: fp32 inputs compare at 1e-4 (chunk, recurrent) against the fp32
reference outputs; bf16 inputs use the north-star bar — max abs error
<= 2e-2 on outputs and <= 1e-3 relative (Frobenius) on the fp32 state —
against a float64 oracle."""
import numpy as np
import pytest
import torch

from oracle import gdn as ogdn

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2
STATE_RTOL = 1e-3


@pytest.fixture(scope='module')
def yb():
    import yanchor_b200
    assert torch.cuda.is_available()
    return yanchor_b200


def cuda(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t if dtype is None else t.to(dtype)


def host(t):
    return t.detach().float().cpu().numpy()


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def make_inputs(rng, B, T, H, HV, K, V, h0_std=0.02, N=None):
    q = rng.standard_normal((B, T, H, K)).astype(np.float32)
    k = rng.standard_normal((B, T, H, K)).astype(np.float32)
    v = rng.standard_normal((B, T, HV, V)).astype(np.float32)
    g = np.log(1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))).astype(np.float32)   # logsigmoid
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))).astype(np.float32)
    h0 = (h0_std * rng.standard_normal((N or B, HV, K, V))).astype(np.float32)
    return q, k, v, g, beta, h0


# ---------------------------------------------------------------- golden ----
@pytest.mark.parametrize('form', ['chunk', 'rec'])
def test_golden_small_fp32(yb, golden, form):
    d = golden('gdn')
    fn = yb.chunk_gated_delta_rule if form == 'chunk' else yb.fused_recurrent_gated_delta_rule
    o, s = fn(cuda(d['small_q']), cuda(d['small_k']), cuda(d['small_v']), g=cuda(d['small_g']),
              beta=cuda(d['small_beta']), initial_state=cuda(d['small_h0']), output_final_state=True,
              use_qk_l2norm_in_kernel=True)
    np.testing.assert_allclose(host(o), d[f'small_{form}_o'], atol=1e-4)
    np.testing.assert_allclose(host(s), d[f'small_{form}_s'], atol=1e-4)


@pytest.mark.parametrize('form', ['chunk', 'rec'])
def test_golden_gva_varlen_fp32(yb, golden, form):
    d = golden('gdn')
    fn = yb.chunk_gated_delta_rule if form == 'chunk' else yb.fused_recurrent_gated_delta_rule
    o, s = fn(cuda(d['var_q']), cuda(d['var_k']), cuda(d['var_v']), g=cuda(d['var_g']), beta=cuda(d['var_beta']),
              initial_state=cuda(d['var_h0']), output_final_state=True, use_qk_l2norm_in_kernel=True,
              cu_seqlens=cuda(d['var_cu']))
    np.testing.assert_allclose(host(o), d[f'var_{form}_o'], atol=1e-4)
    np.testing.assert_allclose(host(s), d[f'var_{form}_s'], atol=1e-4)


def test_golden_config0_recipe(yb, golden):
    d = golden('gdn')
    q, k = ogdn.l2norm(d['small_q']), ogdn.l2norm(d['small_k'])
    o, s = yb.chunk_gated_delta_rule(cuda(q), cuda(k), cuda(d['small_v']), cuda(d['small_g']),
                                     cuda(d['small_beta']), output_final_state=True)
    np.testing.assert_allclose(host(o), d['small_chunk0_o'], atol=1e-4)
    np.testing.assert_allclose(host(s), d['small_chunk0_s'], atol=1e-4)


# ------------------------------------------------------------ decode bf16 ---
@pytest.mark.parametrize('trans', [False, True])
def test_decode_bf16_yanchor_shape(yb, trans):
    """One decode step at the YANchor-4B GDN shape (H=16, HV=32, K=V=128)."""
    rng = np.random.default_rng(10)
    q, k, v, g, beta, h0 = make_inputs(rng, 16, 1, 16, 32, 128, 128, h0_std=0.05)
    qb, kb, vb = (cuda(x, torch.bfloat16) for x in (q, k, v))
    h0d = cuda(h0.swapaxes(-1, -2).copy() if trans else h0)
    o, s = yb.fused_recurrent_gated_delta_rule(qb, kb, vb, g=cuda(g), beta=cuda(beta, torch.bfloat16),
                                               initial_state=h0d, output_final_state=True,
                                               use_qk_l2norm_in_kernel=True, transpose_state_layout=trans)
    eo, es = ogdn.recurrent_gated_delta_rule(host(qb), host(kb), host(vb), g, host(cuda(beta, torch.bfloat16)),
                                             initial_state=h0, use_qk_l2norm=True, dtype=np.float64)
    sd = host(s)
    if trans:
        sd = sd.swapaxes(-1, -2)
    assert np.abs(host(o) - eo).max() <= BF16_ATOL
    assert rel(sd, es) <= STATE_RTOL


def test_decode_inplace_state_and_steps(yb):
    """In-place state (h0 is ht) over 24 decode steps equals the oracle run."""
    rng = np.random.default_rng(11)
    B, H, HV, K, V, steps = 8, 16, 32, 128, 128, 24
    q, k, v, g, beta, h0 = make_inputs(rng, B, steps, H, HV, K, V, h0_std=0.05)
    state = cuda(h0)
    outs = []
    for t in range(steps):
        o, s = yb.fused_recurrent_gated_delta_rule(
            cuda(q[:, t:t + 1], torch.bfloat16), cuda(k[:, t:t + 1], torch.bfloat16),
            cuda(v[:, t:t + 1], torch.bfloat16), g=cuda(g[:, t:t + 1]), beta=cuda(beta[:, t:t + 1]),
            initial_state=state, output_final_state=True, use_qk_l2norm_in_kernel=True, inplace=True)
        assert s is state
        outs.append(host(o))
    rb = lambda x: host(cuda(x, torch.bfloat16))  # noqa: E731
    eo, es = ogdn.recurrent_gated_delta_rule(rb(q), rb(k), rb(v), g, beta, initial_state=h0, use_qk_l2norm=True,
                                             dtype=np.float64)
    assert np.abs(np.concatenate(outs, 1) - eo).max() <= BF16_ATOL
    assert rel(host(state), es) <= STATE_RTOL


@pytest.mark.parametrize('sdtype', [torch.float16, torch.bfloat16])
@pytest.mark.parametrize('trans', [False, True])
def test_decode_16bit_state_storage(yb, sdtype, trans):
    """The reference's reduced-precision state storage: a bf16 / fp16 state
    updated in place over 8 decode calls (fp32 inside a call, rounded to
    nearest on store) against the oracle with the same rounding after every
    call."""
    rng = np.random.default_rng(40 + trans)
    B, H, HV, K, V, steps = 4, 16, 32, 128, 128, 8
    q, k, v, g, beta, h0 = make_inputs(rng, B, steps, H, HV, K, V, h0_std=0.05)
    if trans:
        h0 = np.ascontiguousarray(h0.transpose(0, 1, 3, 2))
    store = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(sdtype).float().numpy()  # noqa: E731
    state = cuda(h0).to(sdtype)
    es = store(h0)
    outs, eouts = [], []
    rb = lambda x: host(cuda(x, torch.bfloat16))  # noqa: E731
    for t in range(steps):
        sl = slice(t, t + 1)
        o, s = yb.fused_recurrent_gated_delta_rule(
            cuda(q[:, sl], torch.bfloat16), cuda(k[:, sl], torch.bfloat16), cuda(v[:, sl], torch.bfloat16),
            g=cuda(g[:, sl]), beta=cuda(beta[:, sl]), initial_state=state, output_final_state=True,
            use_qk_l2norm_in_kernel=True, transpose_state_layout=trans, inplace=True)
        assert s is state and s.dtype == sdtype
        outs.append(host(o))
        eo, es = ogdn.recurrent_gated_delta_rule(rb(q[:, sl]), rb(k[:, sl]), rb(v[:, sl]), g[:, sl], beta[:, sl],
                                                 initial_state=es, use_qk_l2norm=True, transpose_state=trans,
                                                 dtype=np.float64)
        es = store(es)
        eouts.append(eo)
    assert np.abs(np.concatenate(outs, 1) - np.concatenate(eouts, 1)).max() <= BF16_ATOL
    assert rel(host(state), es) <= STATE_RTOL


@pytest.mark.parametrize('sdtype', [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize('B,H,HV', [(6, 16, 32), (3, 1, 1)])
@pytest.mark.parametrize('norm', [False, True])
def test_decode_staged_path_matches_generic(yb, sdtype, B, H, HV, norm):
    """One token per sequence with the state in place runs the staged kernel
    (the state copied into shared memory by bulk copies); the same inputs
    laid out as varlen sequences of length 1 run the generic kernel.  Both do
    the same fp32 operations in the same order, so outputs and states agree
    bit for bit, for fp32 and 16-bit states, at the YANchor head counts and
    at one head, with and without the fused gates and gated RMSNorm."""
    rng = np.random.default_rng(91)
    K, V = 128, 128
    q, k, v, g, beta, h0 = make_inputs(rng, B, 1, H, HV, K, V, h0_std=0.05)
    bf = torch.bfloat16
    sa = cuda(h0).to(sdtype)
    sb = sa.clone()
    extra = {}
    if norm:
        extra = dict(use_gate_in_kernel=True, A_log=cuda(np.log(rng.uniform(1, 16, HV)).astype(np.float32)),
                     dt_bias=cuda(rng.standard_normal(HV).astype(np.float32)), use_beta_sigmoid_in_kernel=True,
                     norm_weight=cuda((1 + 0.1 * rng.standard_normal(V)).astype(np.float32), bf))
        z = rng.standard_normal((B, 1, HV, V)).astype(np.float32)
    oa, _ = yb.fused_recurrent_gated_delta_rule(cuda(q, bf), cuda(k, bf), cuda(v, bf), g=cuda(g), beta=cuda(beta),
                                                initial_state=sa, output_final_state=True,
                                                use_qk_l2norm_in_kernel=True, inplace=True,
                                                **(dict(extra, z=cuda(z, bf)) if norm else {}))
    cu = torch.arange(B + 1, device='cuda', dtype=torch.int64)
    flat = lambda x, dt=None: cuda(x, dt).reshape(1, B, *x.shape[2:]) if dt else cuda(x).reshape(1, B, *x.shape[2:])  # noqa: E731
    ob, _ = yb.fused_recurrent_gated_delta_rule(flat(q, bf), flat(k, bf), flat(v, bf), g=flat(g), beta=flat(beta),
                                                initial_state=sb, output_final_state=True,
                                                use_qk_l2norm_in_kernel=True, inplace=True, cu_seqlens=cu,
                                                **(dict(extra, z=flat(z, bf)) if norm else {}))
    torch.cuda.synchronize()
    assert torch.equal(sa, sb)
    assert torch.equal(oa.reshape(-1), ob.reshape(-1))


def test_decode_16bit_state_not_inplace_returns_fp32(yb):
    """Without ``inplace`` a 16-bit initial state is read and a new float32
    final state returned, as fla does."""
    rng = np.random.default_rng(3)
    q, k, v, g, beta, h0 = make_inputs(rng, 2, 1, 16, 32, 128, 128, h0_std=0.05)
    st16 = cuda(h0).half()
    o, s = yb.fused_recurrent_gated_delta_rule(cuda(q, torch.bfloat16), cuda(k, torch.bfloat16),
                                               cuda(v, torch.bfloat16), g=cuda(g), beta=cuda(beta),
                                               initial_state=st16, output_final_state=True,
                                               use_qk_l2norm_in_kernel=True)
    assert s.dtype == torch.float32 and s is not st16
    rb = lambda x: host(cuda(x, torch.bfloat16))  # noqa: E731
    eo, es = ogdn.recurrent_gated_delta_rule(rb(q), rb(k), rb(v), g, beta, initial_state=host(st16),
                                             use_qk_l2norm=True, dtype=np.float64)
    assert rel(host(s), es) <= STATE_RTOL


def test_decode_gates_and_norm_in_kernel(yb):
    """use_gate_in_kernel + beta logits + the fused gated RMSNorm epilogue."""
    rng = np.random.default_rng(12)
    B, H, HV, K, V = 8, 16, 32, 128, 128
    q, k, v, _, _, h0 = make_inputs(rng, B, 1, H, HV, K, V, h0_std=0.05)
    a = (2 * rng.standard_normal((B, 1, HV))).astype(np.float32)
    blog = rng.standard_normal((B, 1, HV)).astype(np.float32)
    A_log = np.log(rng.uniform(1, 16, HV)).astype(np.float32)
    dt_bias = rng.standard_normal(HV).astype(np.float32)
    z = rng.standard_normal((B, 1, HV, V)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(V)).astype(np.float32)
    bf = torch.bfloat16
    o, s = yb.fused_recurrent_gated_delta_rule(
        cuda(q, bf), cuda(k, bf), cuda(v, bf), g=cuda(a), beta=cuda(blog, bf), initial_state=cuda(h0),
        output_final_state=True, use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=cuda(A_log),
        dt_bias=cuda(dt_bias), use_beta_sigmoid_in_kernel=True, z=cuda(z, bf), norm_weight=cuda(w, bf))
    g, beta = ogdn.gdn_gates(a, host(cuda(blog, bf)), A_log, dt_bias, dtype=np.float64)
    rb = lambda x: host(cuda(x, bf))  # noqa: E731
    beta = rb(beta.astype(np.float32))   # beta = sigmoid(b) is stored in the input dtype (modeling_qwen3_5.py:500)
    eo, es = ogdn.recurrent_gated_delta_rule(rb(q), rb(k), rb(v), g, beta, initial_state=h0, use_qk_l2norm=True,
                                             dtype=np.float64)
    en = ogdn.rmsnorm_gated(eo, rb(z), rb(w), dtype=np.float64)
    # The norm divides by rms(o) per head (o is small here), so compare
    # relative to the output scale: the kernel rounds o, the normalised value
    # and weight * value to bf16 exactly where Qwen3_5RMSNormGated does.
    assert rel(host(o), en) <= 1e-2
    assert np.abs(host(o) - en).max() <= 0.1
    assert rel(host(s), es) <= STATE_RTOL


@pytest.mark.parametrize('sdtype,trans,T', [(torch.float32, False, 1), (torch.float16, False, 1),
                                            (torch.float32, True, 1), (torch.float32, False, 3),
                                            (torch.bfloat16, True, 2)])
def test_fused_decode_layer_vs_oracle(yb, sdtype, trans, T):
    """The one-launch GDN decode core (conv -> gates -> L2 norm -> recurrence
    -> gated RMSNorm), 4 calls, against the reference chain in the oracle:
    conv outputs and beta rounded to bf16 as the reference stores them, the
    state rounded to its storage dtype after every call."""
    from oracle import conv as oconv
    rng = np.random.default_rng(70 + T + trans)
    B, H, HV, K, V, calls = 4, 16, 32, 128, 128, 4
    C = 2 * H * K + HV * V
    bf = torch.bfloat16
    rb = lambda x: host(cuda(np.ascontiguousarray(x, np.float32), bf))  # noqa: E731
    store = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(sdtype).float().numpy()  # noqa: E731
    w_conv = (0.5 * rng.standard_normal((C, 4))).astype(np.float32)
    cst = rb(rng.standard_normal((B, C, 4)))
    A_log = np.log(rng.uniform(1, 16, HV)).astype(np.float32)
    dt_bias = rng.standard_normal(HV).astype(np.float32)
    wn = rb(1 + 0.1 * rng.standard_normal(V))
    h0 = (0.05 * rng.standard_normal((B, HV, K, V))).astype(np.float32)
    if trans:
        h0 = np.ascontiguousarray(h0.transpose(0, 1, 3, 2))
    conv_state = cuda(cst, bf)
    state = cuda(h0).to(sdtype)
    es, ecs = store(h0), cst
    for _ in range(calls):
        mixed = rb(rng.standard_normal((B, T, C)))
        z = rb(rng.standard_normal((B, T, HV, V)))
        a = rb(2 * rng.standard_normal((B, T, HV)))
        blog = rb(rng.standard_normal((B, T, HV)))
        o = yb.fused_gdn_decode(cuda(mixed, bf), cuda(z, bf), cuda(a, bf), cuda(blog, bf), conv_state, cuda(w_conv),
                                None, state, cuda(A_log), cuda(dt_bias), cuda(wn, bf), num_k_heads=H,
                                transpose_state_layout=trans)
        outs = []
        for t in range(T):
            y, ecs = oconv.conv_update(mixed[:, t, :, None], ecs, w_conv)
            y = rb(y[:, :, 0])[:, None]                               # stored as bf16 by the conv update
            q = y[..., :H * K].reshape(B, 1, H, K)
            k = y[..., H * K:2 * H * K].reshape(B, 1, H, K)
            v = y[..., 2 * H * K:].reshape(B, 1, HV, V)
            g, beta = ogdn.gdn_gates(a[:, t:t + 1], blog[:, t:t + 1], A_log, dt_bias, dtype=np.float64)
            beta = rb(beta)                                           # stored in b's dtype
            eo, es = ogdn.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=es, use_qk_l2norm=True,
                                                     transpose_state=trans, dtype=np.float64)
            outs.append(ogdn.rmsnorm_gated(eo, z[:, t:t + 1], wn, dtype=np.float64))
        es = store(es)
        en = np.concatenate(outs, 1)
        assert rel(host(o), en) <= 1e-2
        assert np.abs(host(o) - en).max() <= 0.1
    np.testing.assert_array_equal(host(conv_state), rb(ecs))
    assert rel(host(state), es) <= STATE_RTOL


def test_fused_decode_staged_pair_matches_pair(yb):
    """Two one-token calls (the staged paired kernel: state in shared memory,
    conv under the state copy) against one two-token call (the register
    paired kernel) from the same fp32 state: the same arithmetic in the same
    order, so outputs, state and conv state agree bit for bit."""
    rng = np.random.default_rng(77)
    B, T, H, HV, K, V = 3, 2, 16, 32, 128, 128
    C = 2 * H * K + HV * V
    bf = torch.bfloat16
    mixed = cuda(rng.standard_normal((B, T, C)), bf)
    z = cuda(rng.standard_normal((B, T, HV, V)), bf)
    a = cuda(2 * rng.standard_normal((B, T, HV)), bf)
    blog = cuda(rng.standard_normal((B, T, HV)), bf)
    f32 = lambda x: cuda(np.float32(x))  # noqa: E731
    w_conv = f32(0.5 * rng.standard_normal((C, 4)))
    A_log = f32(np.log(rng.uniform(1, 16, HV)))
    dt_bias = f32(rng.standard_normal(HV))
    wn = cuda(1 + 0.1 * rng.standard_normal(V), bf)
    cs0 = cuda(rng.standard_normal((B, C, 4)), bf)
    h0 = f32(0.05 * rng.standard_normal((B, HV, K, V)))

    cs_pair, st_pair = cs0.clone(), h0.clone()
    o_pair = yb.fused_gdn_decode(mixed, z, a, blog, cs_pair, w_conv, None, st_pair, A_log, dt_bias, wn,
                                 num_k_heads=H)
    cs_st, st_st = cs0.clone(), h0.clone()
    o_st = [yb.fused_gdn_decode(mixed[:, t:t + 1].contiguous(), z[:, t:t + 1].contiguous(),
                                a[:, t:t + 1].contiguous(), blog[:, t:t + 1].contiguous(), cs_st, w_conv, None,
                                st_st, A_log, dt_bias, wn, num_k_heads=H) for t in range(T)]
    torch.cuda.synchronize()
    assert yb.lib().yb_device_error(1) == 0
    assert torch.equal(torch.cat(o_st, 1), o_pair)
    assert torch.equal(st_st, st_pair)
    assert torch.equal(cs_st, cs_pair)


def test_gdn_gates_kernel(yb, golden):
    d = golden('gdn')
    beta, g = yb.gdn_gates(cuda(d['gate_b']), cuda(d['gate_a']), cuda(d['gate_A_log']), cuda(d['gate_dt_bias']))
    np.testing.assert_allclose(host(g), d['gate_g'], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(beta), d['gate_beta'], atol=1e-6)


# ------------------------------------------------------------ prefill bf16 --
@pytest.mark.parametrize('H', [16, 32])
def test_chunk_bf16_vs_oracle(yb, H):
    """bf16 chunked prefill with a ragged tail and a nonzero initial state."""
    rng = np.random.default_rng(20 + H)
    B, T, HV, K, V = 2, 300, 32, 128, 128
    q, k, v, g, beta, h0 = make_inputs(rng, B, T, H, HV, K, V)
    bf = torch.bfloat16
    o, s = yb.chunk_gated_delta_rule(cuda(q, bf), cuda(k, bf), cuda(v, bf), cuda(g), cuda(beta, bf),
                                     initial_state=cuda(h0), output_final_state=True, use_qk_l2norm_in_kernel=True)
    rb = lambda x: host(cuda(x, bf))  # noqa: E731
    eo, es = ogdn.chunk_gated_delta_rule(rb(q), rb(k), rb(v), g, rb(beta), initial_state=h0, use_qk_l2norm=True,
                                         dtype=np.float64)
    assert np.abs(host(o) - eo).max() <= BF16_ATOL
    assert rel(host(s), es) <= STATE_RTOL


def test_chunk_varlen_bf16_vs_oracle(yb):
    rng = np.random.default_rng(30)
    cu = np.array([0, 1, 64, 65, 200, 333, 512], dtype=np.int64)
    H, HV, K, V = 16, 32, 128, 128
    q, k, v, g, beta, h0 = make_inputs(rng, 1, int(cu[-1]), H, HV, K, V, N=len(cu) - 1)
    bf = torch.bfloat16
    o, s = yb.chunk_gated_delta_rule(cuda(q, bf), cuda(k, bf), cuda(v, bf), cuda(g), cuda(beta, bf),
                                     initial_state=cuda(h0), output_final_state=True, use_qk_l2norm_in_kernel=True,
                                     cu_seqlens=cuda(cu))
    rb = lambda x: host(cuda(x, bf))  # noqa: E731
    eo, es = ogdn.chunk_gated_delta_rule(rb(q), rb(k), rb(v), g, rb(beta), initial_state=h0, use_qk_l2norm=True,
                                         cu_seqlens=cu, dtype=np.float64)
    assert np.abs(host(o) - eo).max() <= BF16_ATOL
    assert rel(host(s), es) <= STATE_RTOL


def test_empty_and_zero_length(yb):
    bf = torch.bfloat16
    q = torch.zeros(1, 0, 16, 128, device='cuda', dtype=bf)
    v = torch.zeros(1, 0, 32, 128, device='cuda', dtype=bf)
    g = torch.zeros(1, 0, 32, device='cuda')
    o, s = yb.chunk_gated_delta_rule(q, q, v, g, g.to(bf), output_final_state=True)
    assert o.shape == (1, 0, 32, 128) and s.shape == (1, 32, 128, 128) and not s.abs().any()
    # a zero-length sequence in a varlen batch keeps its initial state
    cu = torch.tensor([0, 0, 5], device='cuda')
    qq = torch.randn(1, 5, 16, 128, device='cuda', dtype=bf)
    vv = torch.randn(1, 5, 32, 128, device='cuda', dtype=bf)
    gg = -torch.rand(1, 5, 32, device='cuda')
    h0 = torch.randn(2, 32, 128, 128, device='cuda')
    for fn in (yb.chunk_gated_delta_rule, yb.fused_recurrent_gated_delta_rule):
        _, s = fn(qq, qq, vv, g=gg, beta=gg.sigmoid().to(bf), initial_state=h0, output_final_state=True,
                  cu_seqlens=cu, use_qk_l2norm_in_kernel=True)
        torch.testing.assert_close(s[0], h0[0], rtol=0, atol=0)


# ------------------------------------------------- full-size properties -----
def test_config1_chunk_equals_recurrent_and_split(yb):
    """At the config-1 shape (B=8, T=8192, H=HV=32, K=V=128, bf16), the
    chunked prefill agrees with the token recurrence, and splitting the
    sequence in two with state passing gives the same final state."""
    torch.manual_seed(0)
    B, T, H, K = 8, 8192, 32, 128
    bf = torch.bfloat16
    q = torch.randn(B, T, H, K, device='cuda', dtype=bf)
    k = torch.randn(B, T, H, K, device='cuda', dtype=bf)
    v = torch.randn(B, T, H, K, device='cuda', dtype=bf)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device='cuda'))
    beta = torch.randn(B, T, H, device='cuda').sigmoid().to(bf)
    h0 = 0.02 * torch.randn(B, H, K, K, device='cuda')
    kw = dict(output_final_state=True, use_qk_l2norm_in_kernel=True)
    o1, s1 = yb.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=h0, **kw)
    o2, s2 = yb.fused_recurrent_gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=h0, **kw)
    assert (o1.float() - o2.float()).abs().max().item() <= BF16_ATOL
    assert ((s1 - s2).norm() / s2.norm()).item() <= STATE_RTOL
    cut = 3000   # not a chunk multiple
    oa, sa = yb.chunk_gated_delta_rule(q[:, :cut], k[:, :cut], v[:, :cut], g[:, :cut], beta[:, :cut],
                                       initial_state=h0, **kw)
    ob, sb = yb.chunk_gated_delta_rule(q[:, cut:], k[:, cut:], v[:, cut:], g[:, cut:], beta[:, cut:],
                                       initial_state=sa, **kw)
    assert (torch.cat([oa, ob], 1).float() - o1.float()).abs().max().item() <= BF16_ATOL
    assert ((sb - s1).norm() / s1.norm()).item() <= STATE_RTOL
