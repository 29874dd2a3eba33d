"""Causal depthwise conv1d before the GDN recurrence, in numpy — test
infrastructure only.

Reference algorithms restated here (paths inside the reference project):

* ``conv_update``  one decode token: runtime/model/inference_kernels.py:339-355
  (``_qwen35_graph_safe_conv_update_kernel``, fp32 arithmetic, one rounding)
  and modeling_yanchor.py:349-353 (``torch_causal_conv1d_update``);
* ``conv_fwd``     a prefill segment: transformers qwen3_5
  modeling_qwen3_5.py:462-480 (``F.silu(conv1d(x)[..., :T])`` with the
  cached state prepended when there is one, and the new state = the last
  ``KS`` inputs, zero-padded on the left).

Shapes: x ``[B, C, T]`` (channels first, as the reference passes it),
conv_state ``[B, C, KS]``, weight ``[C, KS]``, bias ``[C]`` or None.
"""
from __future__ import annotations

import numpy as np


def _act(y, activation):
    if activation in ('silu', 'swish'):
        return y / (1.0 + np.exp(-y))
    if activation is None:
        return y
    raise ValueError(f'unsupported activation {activation!r}')


def conv_update(x, conv_state, weight, bias=None, activation='silu'):
    """One token: returns (out [B, C, 1], new_state [B, C, KS])."""
    x = np.asarray(x, np.float64)
    st = np.asarray(conv_state, np.float64)
    w = np.asarray(weight, np.float64)
    window = np.concatenate((st[:, :, 1:], x[:, :, :1]), -1)          # [B, C, KS]
    y = (window * w[None]).sum(-1, keepdims=True)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :, None]
    return _act(y, activation), window


def conv_fwd(x, weight, bias=None, activation='silu', initial_state=None):
    """A segment: returns (out [B, C, T], final_state [B, C, KS])."""
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    B, C, T = x.shape
    KS = w.shape[1]
    if initial_state is None:
        left = np.zeros((B, C, KS - 1))
        full = np.concatenate((left, x), -1)
        state_src = x
    else:
        st = np.asarray(initial_state, np.float64)
        full = np.concatenate((st[:, :, 1:], x), -1)
        state_src = np.concatenate((st, x), -1)
    y = np.zeros((B, C, T))
    for j in range(KS):
        y += w[None, :, j:j + 1] * full[:, :, j:j + T]
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :, None]
    n = state_src.shape[-1]
    final = np.concatenate((np.zeros((B, C, max(KS - n, 0))), state_src[:, :, max(n - KS, 0):]), -1)
    return _act(y, activation), final
