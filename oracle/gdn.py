"""Gated delta rule (GDN) oracle in numpy — test infrastructure only.

Reference algorithms restated here (paths inside the reference project; the
``transformers`` paths are inside the pinned wheel
``wheels/transformers-5.7.0.dev0-py3-none-any.whl``):

* ``l2norm``                 transformers/models/qwen3_5/modeling_qwen3_5.py:228-231
* ``gdn_gates``              transformers/models/qwen3_5/modeling_qwen3_5.py:500-502,
                             runtime/model/inference_kernels.py:668-681
* ``recurrent_gated_delta_rule``
                             transformers/models/qwen3_5/modeling_qwen3_5.py:314-353,
                             with the grouped-value-head (GVA) and ``cu_seqlens``
                             semantics of fla 0.5.1's
                             ``fused_recurrent_gated_delta_rule`` (third-party,
                             ``fla/ops/gated_delta_rule/fused_recurrent.py:291``)
* ``chunk_gated_delta_rule`` transformers/models/qwen3_5/modeling_qwen3_5.py:234-311,
                             same GVA / varlen semantics as fla's
                             ``chunk_gated_delta_rule`` (``chunk.py:365``)
* ``rmsnorm_gated``          transformers/models/qwen3_5/modeling_qwen3_5.py:175-190

Layouts follow the fla operator contract: q, k ``[B, T, H, K]``; v
``[B, T, HV, V]``; g (log decay) and beta ``[B, T, HV]``; state
``[N, HV, K, V]`` (or ``[N, HV, V, K]`` with ``transpose_state``).  Value head
``hv`` reads query/key head ``hv // (HV // H)``.  With ``cu_seqlens`` the batch
is 1 and sequence ``n`` spans tokens ``cu_seqlens[n]:cu_seqlens[n+1]``.

Everything is computed in ``dtype`` (float32 by default, matching the
reference's fp32 arithmetic; float64 gives a high-precision answer).
"""
from __future__ import annotations

import numpy as np


def l2norm(x, eps=1e-6, dtype=np.float32):
    """x * rsqrt(sum(x^2) + eps) over the last axis."""
    x = np.asarray(x, dtype=dtype)
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + dtype(eps))


def softplus(x, threshold=20.0):
    """log(1 + e^x), returning x itself above ``threshold`` (torch default)."""
    x = np.asarray(x)
    out = np.log1p(np.exp(np.minimum(x, threshold)))
    return np.where(x > threshold, x, out).astype(x.dtype)


def gdn_gates(a, b, A_log, dt_bias, dtype=np.float32):
    """Return ``(g, beta)``: g = -exp(A_log) * softplus(a + dt_bias) in fp32 and
    beta = sigmoid(b)."""
    a = np.asarray(a, dtype=dtype)
    b = np.asarray(b, dtype=dtype)
    g = -np.exp(np.asarray(A_log, dtype=dtype)) * softplus(a + np.asarray(dt_bias, dtype=dtype))
    beta = 1.0 / (1.0 + np.exp(-b))
    return g.astype(dtype), beta.astype(dtype)


def _sequences(B, T, cu_seqlens):
    if cu_seqlens is None:
        return [(b, 0, T) for b in range(B)]
    cu = [int(x) for x in np.asarray(cu_seqlens).reshape(-1)]
    if B != 1:
        raise ValueError("cu_seqlens requires batch size 1")
    return [(0, cu[n], cu[n + 1]) for n in range(len(cu) - 1)]


def _prepare(q, k, v, g, beta, scale, use_qk_l2norm, dtype):
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    if use_qk_l2norm:
        q = l2norm(q, dtype=dtype)
        k = l2norm(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    g = np.asarray(g, dtype=dtype)
    beta = np.asarray(beta, dtype=dtype)
    H, K = q.shape[2], q.shape[3]
    HV = v.shape[2]
    if HV % H:
        raise ValueError("HV must be a multiple of H")
    rep = HV // H
    if rep > 1:
        q = np.repeat(q, rep, axis=2)
        k = np.repeat(k, rep, axis=2)
    if scale is None:
        scale = K ** -0.5
    return q, k, v, g, beta, dtype(scale)


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, scale=None,
                               use_qk_l2norm=False, cu_seqlens=None,
                               transpose_state=False, dtype=np.float32):
    """Token-by-token gated delta rule.  Returns ``(o, final_state)``.

    Per token:  S <- S * exp(g);  d = beta * (v - S^T k);  S <- S + k d^T;
    o = S^T q * scale.
    """
    q, k, v, g, beta, scale = _prepare(q, k, v, g, beta, scale, use_qk_l2norm, dtype)
    B, T, HV, K = k.shape
    V = v.shape[3]
    seqs = _sequences(B, T, cu_seqlens)
    N = len(seqs)
    if initial_state is None:
        S = np.zeros((N, HV, K, V), dtype=dtype)
    else:
        S = np.asarray(initial_state, dtype=dtype).copy()
        if transpose_state:
            S = S.swapaxes(-1, -2).copy()
    o = np.zeros((B, T, HV, V), dtype=dtype)
    for n, (b, start, end) in enumerate(seqs):
        state = S[n]
        for t in range(start, end):
            state *= np.exp(g[b, t])[:, None, None]
            kt, qt = k[b, t], q[b, t] * scale
            recalled = np.einsum('hkv,hk->hv', state, kt)
            delta = (v[b, t] - recalled) * beta[b, t][:, None]
            state += kt[:, :, None] * delta[:, None, :]
            o[b, t] = np.einsum('hkv,hk->hv', state, qt)
        S[n] = state
    if transpose_state:
        S = S.swapaxes(-1, -2).copy()
    return o, S


def _unit_lower_inverse(L, dtype):
    """(I + L)^-1 for strictly lower-triangular L (batched over leading axes),
    by forward substitution one row at a time."""
    C = L.shape[-1]
    Tm = np.zeros_like(L)
    eye = np.eye(C, dtype=dtype)
    for i in range(C):
        # row i of the inverse: e_i - sum_{m<i} L[i, m] * row_m
        Tm[..., i, :] = eye[i] - np.einsum('...m,...mj->...j', L[..., i, :i], Tm[..., :i, :])
    return Tm


def chunk_gated_delta_rule(q, k, v, g, beta, initial_state=None, scale=None,
                           use_qk_l2norm=False, cu_seqlens=None, chunk_size=64,
                           transpose_state=False, dtype=np.float32):
    """Chunk-parallel (WY / UT transform) form of the same recurrence.

    For each chunk of ``chunk_size`` tokens with in-chunk cumulative log decay
    G (G_i = g_0 + ... + g_i):
      L[i, j]  = beta_i * (k_i . k_j) * exp(G_i - G_j)          (j < i)
      Tm       = (I + L)^-1
      W        = Tm @ (beta * exp(G) * k),   U = Tm @ (beta * v)
      v_new    = U - W @ S
      o        = scale * [(exp(G) * q) @ S + ((q k^T) * exp(G_i - G_j))_{j<=i} @ v_new]
      S       <- exp(G_last) * S + (exp(G_last - G) * k)^T @ v_new
    A trailing partial chunk is zero-padded (zero k, v, beta and g), which
    leaves the state untouched by the padding.
    """
    q, k, v, g, beta, scale = _prepare(q, k, v, g, beta, scale, use_qk_l2norm, dtype)
    B, T, HV, K = k.shape
    V = v.shape[3]
    C = chunk_size
    seqs = _sequences(B, T, cu_seqlens)
    N = len(seqs)
    if initial_state is None:
        S = np.zeros((N, HV, K, V), dtype=dtype)
    else:
        S = np.asarray(initial_state, dtype=dtype).copy()
        if transpose_state:
            S = S.swapaxes(-1, -2).copy()
    o = np.zeros((B, T, HV, V), dtype=dtype)
    causal = np.tril(np.ones((C, C), dtype=bool))
    strict = np.tril(np.ones((C, C), dtype=bool), -1)
    for n, (b, start, end) in enumerate(seqs):
        state = S[n]                                  # [HV, K, V]
        for c0 in range(start, end, C):
            c1 = min(c0 + C, end)
            m = c1 - c0

            def pad(x):
                out = np.zeros((C,) + x.shape[1:], dtype=dtype)
                out[:m] = x
                return out.swapaxes(0, 1)             # head-major [HV, C, ...]
            qc, kc, vc = pad(q[b, c0:c1]) * scale, pad(k[b, c0:c1]), pad(v[b, c0:c1])
            gc, bc = pad(g[b, c0:c1]), pad(beta[b, c0:c1])   # [HV, C]
            G = np.cumsum(gc, axis=-1)
            decay = np.exp(np.where(causal, G[:, :, None] - G[:, None, :], -np.inf))
            L = np.where(strict, bc[:, :, None] * (kc @ kc.swapaxes(1, 2)) * decay, 0).astype(dtype)
            Tm = _unit_lower_inverse(L, dtype)
            W = Tm @ (kc * (bc * np.exp(G))[:, :, None])
            U = Tm @ (vc * bc[:, :, None])
            v_new = U - W @ state
            attn = (qc @ kc.swapaxes(1, 2)) * decay
            out = (qc * np.exp(G)[:, :, None]) @ state + attn @ v_new
            o[b, c0:c1] = out.swapaxes(0, 1)[:m]
            G_last = G[:, -1]
            k_tail = kc * np.exp(G_last[:, None] - G)[:, :, None]
            state = state * np.exp(G_last)[:, None, None] + k_tail.swapaxes(1, 2) @ v_new
        S[n] = state
    if transpose_state:
        S = S.swapaxes(-1, -2).copy()
    return o, S


def rmsnorm_gated(x, z, weight, eps=1e-6, dtype=np.float32):
    """weight * rmsnorm(x) * silu(z) over the last axis (norm before gate)."""
    x = np.asarray(x, dtype=dtype)
    z = np.asarray(z, dtype=dtype)
    var = (x * x).mean(-1, keepdims=True)
    y = x / np.sqrt(var + dtype(eps))
    y = np.asarray(weight, dtype=dtype) * y
    return y * (z / (1.0 + np.exp(-z)))
