"""Parity at the full sizes of the benchmark configurations, against the CPU
oracle on sampled rows and heads (every (sequence, head) chain and every
decode row is independent, so a sample of them restated on the CPU checks
the full-size launch).

* Config 1 (chunked prefill, B=8, T=8192, H=HV=32, K=V=128, bf16 inputs, fp32
  state, h0 ~ N(0, 0.02)): sampled (row, head) chains over all 8192 tokens
  against the float64 chunk oracle (transformers qwen3_5
  modeling_qwen3_5.py:234-311 restated in oracle/gdn.py).  Bar: max |d o| <=
  2e-2 on the bf16 outputs, ||dS|| / ||S|| <= 1e-3 on the fp32 state.
* Config 2 (batched decode, B=256, one token per step, the YANchor-4B GDN
  and memory shapes): the decode step's kernels — the short conv update, the
  recurrence with gates, L2 norm and gated RMSNorm (state in place), the
  one-launch memory read + commit, greedy — over several steps, sampled rows
  against the oracle.  Bars: the north-star ones for the GDN state / output,
  the conv state and every memory state field bit-exact, reads <= 2e-2, token
  ids exact."""
import numpy as np
import pytest
import torch

from oracle import conv as oconv, gdn as ogdn, memory as omem, sampling as osamp

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2
STATE_RTOL = 1e-3


@pytest.fixture(scope='module')
def yb():
    import yanchor_b200
    return yanchor_b200


def host(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def test_config1_full_size_vs_fp64_oracle(yb):
    """Config 1 at full size: the tensor-core chunked prefill over 8192 tokens
    (128 chunks, the state carried in TMEM and fed back as bf16 each chunk),
    six sampled (row, head) chains against the float64 oracle."""
    gen = torch.Generator(device='cuda').manual_seed(11)
    B, T, H, K = 8, 8192, 32, 128
    bf = torch.bfloat16
    q = torch.randn(B, T, H, K, generator=gen, device='cuda').to(bf)
    k = torch.randn(B, T, H, K, generator=gen, device='cuda').to(bf)
    v = torch.randn(B, T, H, K, generator=gen, device='cuda').to(bf)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=gen, device='cuda'))
    beta = torch.randn(B, T, H, generator=gen, device='cuda').sigmoid().to(bf)
    h0 = 0.02 * torch.randn(B, H, K, K, generator=gen, device='cuda')
    o, s = yb.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True,
                                     use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    for b, h in ((0, 0), (1, 31), (3, 7), (5, 16), (6, 23), (7, 30)):
        sl = lambda t: host(t[b:b + 1, :, h:h + 1])  # noqa: E731
        eo, es = ogdn.chunk_gated_delta_rule(sl(q), sl(k), sl(v), sl(g), sl(beta),
                                             initial_state=host(h0[b:b + 1, h:h + 1]), use_qk_l2norm=True,
                                             dtype=np.float64)
        assert np.abs(sl(o) - eo).max() <= BF16_ATOL, (b, h)
        assert rel(host(s[b:b + 1, h:h + 1]), es) <= STATE_RTOL, (b, h)


def test_config2_b256_decode_step_vs_oracle(yb):
    """Config 2's batch: B=256 rows through the decode step's kernels for one
    GDN layer and one memory layer at the YANchor-4B shapes, 70 steps (the
    memory chunk of 64 fills once), eight sampled rows restated on the CPU."""
    rng = np.random.default_rng(256)
    B, H, HV, K, V, KS = 256, 16, 32, 128, 128, 4
    C = 2 * H * K + HV * V
    G, MH, D, CAP, CH = 4, 16, 256, 64, 64
    rows = np.array([0, 1, 63, 64, 127, 200, 254, 255])
    steps = 70
    bf = torch.bfloat16
    dev = 'cuda'

    def cu(x, dt=None):
        t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
        return t if dt is None else t.to(dt)

    w_conv = (0.5 * rng.standard_normal((C, KS))).astype(np.float32)
    A_log = np.log(rng.uniform(1, 16, HV)).astype(np.float32)
    dt_bias = np.ones(HV, np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(V)).astype(np.float32)
    conv_state = cu(rng.standard_normal((B, C, KS)), bf)
    state = cu((0.02 * rng.standard_normal((B, HV, K, V))).astype(np.float32))
    mem = yb.MemoryState.empty(B, G, CAP, CH, D, dev, bf)
    # the oracle's copies of the sampled rows
    cst_np = host(conv_state)[rows].astype(np.float64)
    s_np = host(state)[rows].astype(np.float64)
    mem_np = omem.empty_state(len(rows), G, CAP, CH, D)
    w_b, nw_b = host(cu(w_conv)), host(cu(norm_w, bf))
    for t in range(steps):
        mixed = cu(rng.standard_normal((B, 1, C)), bf)
        z = cu(rng.standard_normal((B, 1, HV, V)), bf)
        a = cu(rng.standard_normal((B, 1, HV)), bf)
        blog = cu(rng.standard_normal((B, 1, HV)), bf)
        mix = yb.causal_conv1d_update(mixed.transpose(1, 2), conv_state, cu(w_conv), None, 'silu').transpose(1, 2)
        qd = mix[..., :H * K].unflatten(-1, (H, K))
        kd = mix[..., H * K:2 * H * K].unflatten(-1, (H, K))
        vd = mix[..., 2 * H * K:].unflatten(-1, (HV, V))
        o, _ = yb.fused_recurrent_gated_delta_rule(
            qd, kd, vd, g=a, beta=blog, initial_state=state, output_final_state=True,
            use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=cu(A_log), dt_bias=cu(dt_bias),
            use_beta_sigmoid_in_kernel=True, z=z, norm_weight=cu(norm_w, bf), inplace=True)
        mq = cu(rng.standard_normal((B, 1, MH, D)), bf)
        mk = cu(rng.standard_normal((B, 1, G, D)), bf)
        mv = cu(rng.standard_normal((B, 1, G, D)), bf)
        ms = cu(np.round(rng.standard_normal((B, 1, G)) * 2).astype(np.float32) / 2)
        act = cu(rng.random(B) > 0.05)
        read = yb.memory_decode_step(mq, mk, mv, ms, act, CH, mem)
        logits = cu(3 * rng.standard_normal((B, 248320)), bf)
        tok = yb.greedy(logits)
        # --- the oracle on the sampled rows ---
        y, cst_np = oconv.conv_update(host(mixed.transpose(1, 2))[rows], cst_np, w_b)
        y = host(cu(y[:, :, 0].astype(np.float32), bf))          # the reference stores the conv output in bf16
        q_r = y[:, None, :H * K].reshape(-1, 1, H, K)
        k_r = y[:, None, H * K:2 * H * K].reshape(-1, 1, H, K)
        v_r = y[:, None, 2 * H * K:].reshape(-1, 1, HV, V)
        gg, bb = ogdn.gdn_gates(host(a)[rows], host(blog)[rows], A_log, dt_bias, dtype=np.float64)
        bb = host(cu(bb.astype(np.float32), bf))                   # beta in the input dtype
        eo, s_np = ogdn.recurrent_gated_delta_rule(q_r, k_r, v_r, gg, bb, initial_state=s_np, use_qk_l2norm=True,
                                                   dtype=np.float64)
        en = ogdn.rmsnorm_gated(eo, host(z)[rows], nw_b, dtype=np.float64)
        assert rel(host(o)[rows], en) <= 1e-2, t
        ref_read = omem.decode_read(host(mq)[rows], mem_np['keys'], mem_np['values'], mem_np['positions'])
        assert np.abs(host(read)[rows] - ref_read).max() <= BF16_ATOL, t
        omem.commit_decode(host(mk)[rows], host(mv)[rows], host(ms)[rows], host(act)[rows], CH, mem_np)
        np.testing.assert_array_equal(host(tok)[rows], osamp.greedy(host(logits)[rows]))
    assert rel(host(state)[rows], s_np) <= STATE_RTOL
    np.testing.assert_array_equal(host(conv_state)[rows], cst_np.astype(np.float32))
    for f in ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values', 'pending_scores', 'count',
              'total'):
        got = host(getattr(mem, f))[rows]
        np.testing.assert_array_equal(got, mem_np[f].astype(got.dtype), err_msg=f)
    assert int(host(mem.positions)[rows].max()) >= 0        # a commit happened
