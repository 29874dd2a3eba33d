"""The torch custom ops (torch.ops.yanchor_b200.*) on the GPU: torch's own
op checks (the schema's in-place annotations against what the kernel
writes, and the fake implementation against the real outputs), and a
decode step traced whole by torch.compile (fullgraph) that gives the same
results as the plain calls."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def yb():
    import yanchor_b200
    return yanchor_b200


def rnd(*shape, dtype=torch.bfloat16, scale=1.0, gen=None):
    return (torch.randn(*shape, device='cuda', generator=gen) * scale).to(dtype)


def memory_state(yb, B, G=4, CAP=64, PC=64, D=256):
    st = yb.MemoryState.empty(B, G, CAP, PC, D, 'cuda', torch.bfloat16)
    return st


def test_opcheck(yb):
    ops = torch.ops.yanchor_b200
    gen = torch.Generator(device='cuda').manual_seed(0)
    B, T, H, HV, K = 2, 70, 2, 4, 128
    q, k = rnd(B, T, H, K, gen=gen), rnd(B, T, H, K, gen=gen)
    v = rnd(B, T, HV, K, gen=gen)
    g = torch.nn.functional.logsigmoid(rnd(B, T, HV, dtype=torch.float32, gen=gen))
    beta = rnd(B, T, HV, gen=gen).float().sigmoid().to(torch.bfloat16)
    h0 = rnd(B, HV, K, K, dtype=torch.float32, scale=0.02, gen=gen)
    utils = ('test_schema', 'test_faketensor')
    torch.library.opcheck(ops.chunk_gated_delta_rule.default, (q, k, v, g, beta, 0.1, h0, True, True, None, False),
                          test_utils=utils)
    torch.library.opcheck(ops.fused_recurrent_gated_delta_rule_.default,
                          (q[:, :1], k[:, :1], v[:, :1], g[:, :1], beta[:, :1], 0.1, h0.clone(), True, False, None,
                           None, False, None, None, 1e-6), test_utils=utils)
    C = 2 * H * K + HV * K
    torch.library.opcheck(ops.causal_conv1d_update_.default,
                          (rnd(B, C, 1, gen=gen), rnd(B, C, 4, gen=gen), rnd(C, 4, dtype=torch.float32, gen=gen),
                           None, True), test_utils=utils)
    st = memory_state(yb, B)
    fields = (st.keys, st.values, st.scores, st.positions, st.pending_keys, st.pending_values, st.pending_scores,
              st.count, st.total)
    mq, mk, mv = rnd(B, 1, 16, 256, gen=gen), rnd(B, 1, 4, 256, gen=gen), rnd(B, 1, 4, 256, gen=gen)
    ms, act = rnd(B, 1, 4, dtype=torch.float32, gen=gen), torch.ones(B, device='cuda', dtype=torch.bool)
    torch.library.opcheck(ops.memory_decode_step_.default, (mq, mk, mv, ms, act, 64, *fields, None), test_utils=utils)
    torch.library.opcheck(ops.commit_decode_.default, (mk, mv, ms, act, 64, *fields, None), test_utils=utils)
    torch.library.opcheck(ops.committed_gqa.default, (mq, *fields, None), test_utils=utils)
    torch.library.opcheck(ops.greedy.default, (rnd(3, 1000, gen=gen),), test_utils=utils)


def test_compiled_decode_step_matches_plain_calls(yb):
    """One GDN layer (conv update + recurrence, states in place), one memory
    layer (read + commit) and greedy, traced whole by torch.compile through
    the custom ops, against the plain Python API on copies of the states."""
    ops = torch.ops.yanchor_b200
    gen = torch.Generator(device='cuda').manual_seed(1)
    B, H, HV, K = 4, 16, 32, 128
    C = 2 * H * K + HV * K
    conv_w = rnd(C, 4, dtype=torch.float32, scale=0.5, gen=gen)
    A_log = torch.rand(HV, device='cuda', generator=gen).add(1).log()
    dt_bias = torch.ones(HV, device='cuda')
    norm_w = rnd(K, gen=gen)

    def step(mixed, z, a, b, logits, mq, mk, mv, ms, act, conv_state, state, *mem):
        y = ops.causal_conv1d_update_(mixed.transpose(1, 2), conv_state, conv_w, None, True).transpose(1, 2)
        q = y[..., :H * K].unflatten(-1, (H, K))
        k = y[..., H * K:2 * H * K].unflatten(-1, (H, K))
        v = y[..., 2 * H * K:].unflatten(-1, (HV, K))
        o = ops.fused_recurrent_gated_delta_rule_(q, k, v, a, b, K ** -0.5, state, True, True, A_log, dt_bias, True,
                                                  z, norm_w, 1e-6)
        r = ops.memory_decode_step_(mq, mk, mv, ms, act, 64, *mem, None)
        return o, r, ops.greedy(logits)

    compiled = torch.compile(step, fullgraph=True, backend='aot_eager')
    conv_a, conv_b = rnd(B, C, 4, gen=gen), None
    conv_b = conv_a.clone()
    state_a = rnd(B, HV, K, K, dtype=torch.float32, scale=0.02, gen=gen)
    state_b = state_a.clone()
    mem_a, mem_b = memory_state(yb, B), memory_state(yb, B)
    fa = yb.ops.memory_fields(mem_a)
    for t in range(70):
        x = dict(mixed=rnd(B, 1, C, gen=gen), z=rnd(B, 1, HV, K, gen=gen), a=rnd(B, 1, HV, gen=gen),
                 b=rnd(B, 1, HV, gen=gen), logits=rnd(B, 5000, gen=gen), mq=rnd(B, 1, 16, 256, gen=gen),
                 mk=rnd(B, 1, 4, 256, gen=gen), mv=rnd(B, 1, 4, 256, gen=gen),
                 ms=rnd(B, 1, 4, dtype=torch.float32, gen=gen), act=torch.ones(B, device='cuda', dtype=torch.bool))
        o_a, r_a, ids_a = compiled(x['mixed'], x['z'], x['a'], x['b'], x['logits'], x['mq'], x['mk'], x['mv'],
                                   x['ms'], x['act'], conv_a, state_a, *fa)
        y = yb.causal_conv1d_update(x['mixed'].transpose(1, 2), conv_b, conv_w, None, 'silu').transpose(1, 2)
        q = y[..., :H * K].unflatten(-1, (H, K))
        k = y[..., H * K:2 * H * K].unflatten(-1, (H, K))
        v = y[..., 2 * H * K:].unflatten(-1, (HV, K))
        o_b, _ = yb.fused_recurrent_gated_delta_rule(q, k, v, g=x['a'], beta=x['b'], initial_state=state_b,
                                                     output_final_state=True, use_qk_l2norm_in_kernel=True,
                                                     use_gate_in_kernel=True, A_log=A_log, dt_bias=dt_bias,
                                                     use_beta_sigmoid_in_kernel=True, z=x['z'], norm_weight=norm_w,
                                                     inplace=True)
        r_b = yb.memory_decode_step(x['mq'], x['mk'], x['mv'], x['ms'], x['act'], 64, mem_b)
        ids_b = yb.greedy(x['logits'])
        assert torch.equal(o_a, o_b) and torch.equal(r_a, r_b) and torch.equal(ids_a, ids_b), t
    assert torch.equal(conv_a, conv_b) and torch.equal(state_a, state_b)
    for fa_, fb_ in zip(fa, yb.ops.memory_fields(mem_b)):
        assert torch.equal(fa_, fb_)
