"""GPU parity of the sliding-window prefill attention (tcgen05 kernel)
against the CPU oracle, which is pinned to the reference's ``reference_swa``
(tests/golden/swa_prefill.npz).  bf16 outputs compare at 2e-2 absolute."""
import numpy as np
import pytest
import torch

from oracle import swa as oswa

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope='module')
def yb():
    import yanchor_b200
    return yanchor_b200


def rnd(rng, *shape):
    return torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).cuda().to(torch.bfloat16)


def host(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize('B,T,QH,KVH,window', [(2, 200, 16, 4, 64), (1, 150, 4, 4, 100), (2, 97, 8, 4, 300),
                                               (1, 130, 16, 2, 33), (3, 64, 16, 4, 1)])
def test_causal_window(yb, B, T, QH, KVH, window):
    """Head groups of 1, 2, 4, 8; windows shorter and longer than the prompt,
    a window of one token; prompts that end inside a query tile."""
    rng = np.random.default_rng(B * 1000 + T + window)
    q, k, v = rnd(rng, B, T, QH, 256), rnd(rng, B, T, KVH, 256), rnd(rng, B, T, KVH, 256)
    out = yb.reference_swa(q, k, v, window=window)
    ref = oswa.prefill_attention(host(q), host(k), host(v), window, dtype=np.float32)
    assert np.abs(host(out) - ref).max() <= TOL
    assert yb.lib().yb_device_error(1) == 0


def test_window_1024_long_prompt(yb):
    """The YANchor window over a prompt longer than it (17 key tiles per query tile)."""
    rng = np.random.default_rng(3)
    T = 1100
    q, k, v = rnd(rng, 1, T, 16, 256), rnd(rng, 1, T, 4, 256), rnd(rng, 1, T, 4, 256)
    out = yb.reference_swa(q, k, v, window=1024)
    ref = oswa.prefill_attention(host(q), host(k), host(v), 1024, dtype=np.float32)
    assert np.abs(host(out) - ref).max() <= TOL


def test_key_valid_and_cached_window(yb):
    """Left padding, holes and a fully padded row through key_valid; a query
    block after a cached window of 70 keys (query_start)."""
    rng = np.random.default_rng(11)
    B, Tq, start, QH, KVH = 3, 90, 70, 16, 4
    Tk = start + Tq
    q, k, v = rnd(rng, B, Tq, QH, 256), rnd(rng, B, Tk, KVH, 256), rnd(rng, B, Tk, KVH, 256)
    valid = np.ones((B, Tk), bool)
    valid[0, :40] = False                       # left padding inside the cached window
    valid[1] = rng.random(Tk) > 0.3             # holes
    valid[2] = False                            # nothing valid: zeros
    kv = torch.from_numpy(valid).cuda()
    out = yb.reference_swa(q, k, v, window=80, key_valid=kv, query_start=start)
    ref = oswa.prefill_attention(host(q), host(k), host(v), 80, valid, start, dtype=np.float32)
    assert np.abs(host(out) - ref).max() <= TOL
    assert not host(out)[2].any()


@pytest.mark.parametrize('kind', ['left', 'holes'])
def test_flash_swa_masks(yb, kind):
    """flash_swa counts valid tokens: left padding runs in place, holes are
    packed valid-first and scattered back."""
    rng = np.random.default_rng(5 if kind == 'left' else 6)
    B, T = 3, 120
    q, k, v = rnd(rng, B, T, 16, 256), rnd(rng, B, T, 4, 256), rnd(rng, B, T, 4, 256)
    mask = np.ones((B, T + 7), bool)                      # longer than the prompt: the last T columns count
    if kind == 'left':
        mask[0, :7 + 25] = False
        mask[2, :7 + 119] = False
    else:
        mask[:, 7:] = rng.random((B, T)) > 0.35
    out = yb.flash_swa(q, k, v, window=40, attention_mask=torch.from_numpy(mask).cuda())
    ref = oswa.flash_prefill(host(q), host(k), host(v), 40, mask, dtype=np.float32)
    assert np.abs(host(out) - ref).max() <= TOL


def test_unsupported_shape_is_refused(yb):
    q = torch.zeros(1, 8, 4, 128, device='cuda', dtype=torch.bfloat16)
    with pytest.raises(Exception, match='D = 256'):
        yb.reference_swa(q, q, q, window=4)
