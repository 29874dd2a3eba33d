"""Stage-by-stage check of the tensor-core chunk kernel (tests/csrc/tc_debug.cu
builds it with intermediate dumps enabled): every TMEM tile and the fp32
inverse of the first chunk of CTA 0 against numpy, so a failure names the
stage that diverged.  Tolerances reflect bf16 operand rounding."""
import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

LIB = os.path.join(ROOT, 'tests', '_build', 'libyb_tc_debug.so')
DBG = dict(D1=0, W=16384, U=24576, X=32768, Y=40960, O=49152, S1=57344, T=73728, NORM=77824)


def bf(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def hilo(x):
    """x as the kernel feeds it to the tensor cores: bf16 hi + bf16 lo."""
    h = bf(x)
    return h + bf(np.asarray(x, np.float32) - h)


def relerr(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope='module')
def run():
    lib = ctypes.CDLL(LIB)
    f = lib.ybdbg_gdn_chunk_tc
    P, I64, F, I, U = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_uint32
    f.argtypes = [P, P, P, I64, I64, I64, P, P, I64, I64, P, P, P, I64, I64, I64, I64, F, I, I, U, P, P]
    f.restype = I
    lib.ybdbg_last_error.restype = ctypes.c_char_p
    lib.ybdbg_device_error.argtypes = [I]
    rng = np.random.default_rng(7)
    B, T, H, HV, K = 1, 100, 2, 2, 128
    q = bf(rng.standard_normal((B, T, H, K)))
    k = bf(rng.standard_normal((B, T, H, K)))
    v = bf(rng.standard_normal((B, T, HV, K)))
    g = np.log(1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))).astype(np.float32)
    beta = bf(1 / (1 + np.exp(-rng.standard_normal((B, T, HV)))))
    h0 = (0.05 * rng.standard_normal((B, HV, K, K))).astype(np.float32)
    dev = lambda x, dt=torch.bfloat16: torch.from_numpy(x).cuda().to(dt).contiguous()  # noqa: E731
    qd, kd, vd, bd = dev(q), dev(k), dev(v), dev(beta)
    gd, h0d = dev(g, torch.float32), dev(h0, torch.float32)
    ht = torch.zeros_like(h0d)
    o = torch.zeros(B, T, HV, K, device='cuda', dtype=torch.bfloat16)
    dbg = torch.full((80000,), float("nan"), device="cuda")
    scale = K ** -0.5
    rc = f(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), H * K, H * K, HV * K, gd.data_ptr(), bd.data_ptr(), HV, HV,
           h0d.data_ptr(), ht.data_ptr(), o.data_ptr(), B, T, H, HV, scale, 0, 2, 1, dbg.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.ybdbg_last_error()
    torch.cuda.synchronize()
    assert lib.ybdbg_device_error(1) == 0
    return dict(q=q, k=k, v=v, g=g, beta=beta, h0=h0, scale=scale, dbg=dbg.cpu().numpy(), o=o.float().cpu().numpy(),
                ht=ht.cpu().numpy())


def expected(d):
    K_ = d['k'][0, :64, 0]
    Q_ = d['q'][0, :64, 0]
    V_ = d['v'][0, :64, 0]
    G = np.cumsum(d['g'][0, :64, 0].astype(np.float64))
    bt = d['beta'][0, :64, 0].astype(np.float64)
    e = {}
    KQ = np.concatenate([K_, Q_], 0)
    e['D1'] = KQ @ KQ.T
    kn = 1 / np.sqrt(np.diag(K_ @ K_.T) + 1e-6)
    qn = d['scale'] / np.sqrt((Q_ * Q_).sum(1) + 1e-6)
    e['NORM'] = np.concatenate([kn, qn])
    dec = np.exp(np.tril(G[:, None] - G[None, :]))
    L = np.tril(bt[:, None] * kn[:, None] * kn[None, :] * dec * (K_ @ K_.T), -1)
    Tm = np.linalg.inv(np.eye(64) + L)
    e['T'] = Tm
    Tw = hilo(Tm * (bt * np.exp(G) * kn)[None, :])
    Tu = hilo(Tm * bt[None, :])
    e['W'] = K_.T @ Tw.T
    e['U'] = V_.T @ Tu.T
    ST = bf(d['h0'][0, 0].T)
    e['X'] = ST @ bf(e['W'])
    e['Y'] = ST @ Q_.T
    vn = e['U'] - e['X']
    P = bf(np.tril(qn[:, None] * kn[None, :] * dec * (Q_ @ K_.T)))
    e['O'] = bf(vn) @ P.T
    vt = hilo(vn * (np.exp(G[-1] - G) * kn)[None, :])
    e['S1'] = np.exp(G[-1]) * d['h0'][0, 0].T + vt @ K_      # the state after chunk 0 (S^T)
    return e


SHAPES = dict(D1=(128, 128), W=(128, 64), U=(128, 64), X=(128, 64), Y=(128, 64), O=(128, 64), S1=(128, 128),
              T=(64, 64), NORM=(128,))
ORDER = ['D1', 'NORM', 'T', 'W', 'U', 'X', 'Y', 'O', 'S1']
TOL = dict(D1=2e-3, NORM=2e-3, T=2e-3, W=2e-3, U=2e-3, X=2e-2, Y=1e-2, O=2e-2, S1=2e-3)


@pytest.mark.parametrize('stage', ORDER)
def test_stage(run, stage):
    e = expected(run)[stage]
    n = int(np.prod(SHAPES[stage]))
    got = run['dbg'][DBG[stage]:DBG[stage] + n].reshape(SHAPES[stage])
    assert np.isfinite(got).all(), f'{stage}: not written / non-finite'
    err = relerr(got, e)
    assert err <= TOL[stage], f'{stage}: relative error {err:.3e}'


def test_full_chunk_output_vs_oracle(run):
    from oracle import gdn as ogdn
    eo, es = ogdn.chunk_gated_delta_rule(run['q'], run['k'], run['v'], run['g'], run['beta'],
                                         initial_state=run['h0'], use_qk_l2norm=True, dtype=np.float64)
    assert np.abs(run['o'] - eo).max() <= 2e-2
    assert relerr(run['ht'], es) <= 1e-3
