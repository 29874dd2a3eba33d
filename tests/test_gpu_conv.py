"""GPU parity of the causal depthwise conv1d (decode update and prefill)
against the reference fixtures (fp32) and the oracle (bf16, the YANchor
channel count).  States are copies of inputs and compare exactly."""
import numpy as np
import pytest
import torch

from oracle import conv as oconv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def yb():
    import yanchor_b200
    return yanchor_b200


def cuda(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t if dtype is None else t.to(dtype)


def host(t):
    return t.detach().float().cpu().numpy()


def token_major(x, dtype=None):
    """[B, C, T] numpy -> a CUDA [B, C, T] view of token-major memory (as the reference passes it)."""
    return cuda(np.ascontiguousarray(np.asarray(x).transpose(0, 2, 1)), dtype).transpose(1, 2)


def test_update_golden(yb, golden):
    d = golden('conv')
    st = cuda(d['conv_upd_state'])
    y = yb.causal_conv1d_update(token_major(d['conv_upd_x']), st, cuda(d['conv_w']), None, 'silu')
    np.testing.assert_allclose(host(y), d['conv_upd_y'], atol=1e-5)
    np.testing.assert_array_equal(host(st), d['conv_upd_state_after'])


@pytest.mark.parametrize('name,cached', [('conv_pre', False), ('conv_prec', True), ('conv_pres', False)])
def test_prefill_golden(yb, golden, name, cached):
    d = golden('conv')
    init = cuda(d['conv_prec_state_in']) if cached else None
    y, st = yb.causal_conv1d_fn(token_major(d[f'{name}_x']), cuda(d['conv_w']), initial_states=init,
                                return_final_states=True, final_states_out=None if not cached else
                                torch.empty_like(init), activation='silu')
    np.testing.assert_allclose(host(y), d[f'{name}_y'], atol=1e-5)
    if cached:
        np.testing.assert_array_equal(host(st), d[f'{name}_state'])
    else:   # width KS - 1 without a cache state: the last KS - 1 inputs
        np.testing.assert_array_equal(host(st), d[f'{name}_state'][:, :, 1:])


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_update_yanchor_shape_steps(yb, dtype):
    """B=64, C = 2*16*128 + 32*128 = 8192, KS=4, bias, 6 decode steps in place."""
    rng = np.random.default_rng(5)
    B, C, KS, steps = 64, 8192, 4, 6
    w = (rng.standard_normal((C, KS)) * 0.5).astype(np.float32)
    bias = (rng.standard_normal(C) * 0.1).astype(np.float32)
    st = cuda(rng.standard_normal((B, C, KS)).astype(np.float32), dtype)
    est = host(st)
    for _ in range(steps):
        x = rng.standard_normal((B, 1, C)).astype(np.float32)
        xt = cuda(x, dtype).transpose(1, 2)                  # [B, C, 1] view of [B, 1, C]
        y = yb.causal_conv1d_update(xt, st, cuda(w), cuda(bias), 'silu')
        ey, est = oconv.conv_update(host(xt), est, w, bias)
        tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
        np.testing.assert_allclose(host(y), ey, atol=tol, rtol=tol)
        np.testing.assert_array_equal(host(st), est.astype(np.float32))


@pytest.mark.parametrize('width', [4, 3])
@pytest.mark.parametrize('T', [300, 3, 1])
def test_prefill_yanchor_shape(yb, width, T):
    """bf16, C=8192, an initial state of width KS (cache) or KS-1 (package),
    final state written in place over the initial one."""
    rng = np.random.default_rng(T + width)
    B, C, KS = 2, 8192, 4
    w = (rng.standard_normal((C, KS)) * 0.5).astype(np.float32)
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    st0 = rng.standard_normal((B, C, width)).astype(np.float32)
    xt = token_major(x, torch.bfloat16)
    st = cuda(st0, torch.bfloat16)
    y, st_out = yb.causal_conv1d_fn(xt, cuda(w), initial_states=st, return_final_states=True,
                                    final_states_out=st, activation='silu')
    assert st_out is st
    full_state = np.concatenate((np.zeros((B, C, KS - width)), host(cuda(st0, torch.bfloat16))), -1)
    ey, est = oconv.conv_fwd(host(xt), w, initial_state=full_state)
    np.testing.assert_allclose(host(y), ey, atol=2e-2, rtol=2e-2)
    np.testing.assert_array_equal(host(st), est[:, :, KS - width:].astype(np.float32))
    assert y.shape == (B, C, T) and y.transpose(1, 2).is_contiguous()


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_state_in_the_reference_cache_layout(yb, dtype):
    """The reference's cache keeps the conv state as F.pad of the transposed
    projection (transformers qwen3_5 modeling_qwen3_5.py:466-467): channels
    contiguous, taps C apart.  Prefill writing that state and decode steps
    updating it in place give the same outputs and states as the packed
    layout, and the oracle's."""
    rng = np.random.default_rng(31)
    B, C, KS, T = 3, 1024, 4, 37
    w = (0.5 * rng.standard_normal((C, KS))).astype(np.float32)
    xp = rng.standard_normal((B, C, T)).astype(np.float32)
    mixed = token_major(xp, dtype)
    # the cache's state: the last KS inputs, in the transposed projection's memory layout
    ref_state = torch.nn.functional.pad(mixed, (KS - T, 0))
    assert ref_state.stride(1) == 1 and ref_state.stride(2) == C
    packed = ref_state.contiguous()
    y_ref = yb.causal_conv1d_fn(mixed, cuda(w), activation='silu')
    ey, est = oconv.conv_fwd(host(mixed), w)
    assert np.abs(host(y_ref) - ey).max() <= (1e-5 if dtype == torch.float32 else 2e-2)
    for t in range(5):
        x1 = token_major(rng.standard_normal((B, C, 1)).astype(np.float32), dtype)
        y_a = yb.causal_conv1d_update(x1, ref_state, cuda(w), None, 'silu')
        y_b = yb.causal_conv1d_update(x1, packed, cuda(w), None, 'silu')
        assert torch.equal(y_a, y_b), t
        assert torch.equal(ref_state, packed), t
        ey1, est = oconv.conv_update(host(x1), est, w)
        assert np.abs(host(y_a) - ey1).max() <= (1e-5 if dtype == torch.float32 else 2e-2)
    np.testing.assert_array_equal(host(ref_state), est.astype(np.float32))
    # a prefill continuing from / writing a state in that layout
    init = ref_state.clone()
    fin = torch.nn.functional.pad(torch.zeros_like(mixed), (KS - T, 0))
    y2, _ = yb.causal_conv1d_fn(mixed, cuda(w), initial_states=init, return_final_states=True,
                                final_states_out=fin, activation='silu')
    y3, fin_p = yb.causal_conv1d_fn(mixed, cuda(w), initial_states=init.contiguous(), return_final_states=True,
                                    activation='silu')
    assert torch.equal(y2, y3) and torch.equal(fin, fin_p)
