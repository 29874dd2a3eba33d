"""Causal depthwise conv1d in front of the GDN recurrence, with the call
signatures the reference layer uses.

    causal_conv1d_update(x, conv_state, weight, bias=None, activation=None)
        one decode token; runtime/model/inference_kernels.py:339-376
        (`triton_graph_safe_causal_conv1d_update`) and modeling_yanchor.py:
        349-353 (`torch_causal_conv1d_update`)
    causal_conv1d_fn(x, weight, bias=None, seq_idx=None, initial_states=None,
                     return_final_states=False, final_states_out=None, activation=None)
        a prefill segment; the causal-conv1d package's function as transformers
        qwen3_5 calls it (modeling_qwen3_5.py:470-476)

x is [B, C, T] (channels first); the memory behind it is expected to be
token-major (the reference passes ``mixed_qkv.transpose(1, 2)``), which the
kernels read in place.  Outputs are allocated token-major and returned as the
same [B, C, T] view.  SiLU is applied when ``activation`` is ``'silu'`` or
``'swish'``.  Arithmetic is fp32 with one rounding to the input dtype.
"""
from __future__ import annotations

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr


def _silu(activation):
    if activation in ('silu', 'swish'):
        return 1
    if activation is None:
        return 0
    raise ValueError(f'unsupported causal-convolution activation: {activation}')


def _weight(weight, C):
    w = weight.reshape(weight.shape[0], -1) if weight.dim() == 3 else weight
    if w.dim() != 2 or w.shape[0] != C:
        raise ValueError('weight must be [C, KS] (or [C, 1, KS])')
    return w.to(torch.float32).contiguous()


def _token_major(x):
    """x [B, C, T] whose channels are contiguous (stride 1)."""
    if x.stride(1) != 1:
        x = x.transpose(1, 2).contiguous().transpose(1, 2)
    return x


def _state_strides(st):
    """A conv state [B, C, W] may have any layout whose (channel, tap)
    elements do not overlap: packed per row (the kernels' fast path) or, as
    the reference's cache keeps it after padding a transposed projection,
    channels contiguous with taps C apart."""
    cs, ts = st.stride(1), st.stride(2)
    if cs < 1 or ts < 1 or not (cs >= st.shape[2] * ts or ts >= st.shape[1] * cs):
        raise ValueError('conv_state channel and tap strides overlap')


def causal_conv1d_update(x, conv_state, weight, bias=None, activation=None):
    """One token: x [B, C, 1] (or [B, C]); conv_state [B, C, W] updated in
    place (shifted left, the input appended); returns the output, shaped and
    typed like x."""
    require_cuda(x, conv_state, weight, bias)
    squeeze = x.dim() == 2
    x3 = x[:, :, None] if squeeze else x
    if x3.dim() != 3 or x3.shape[-1] != 1:
        raise ValueError('causal_conv1d_update takes one decode token')
    B, C, _ = x3.shape
    w = _weight(weight, C)
    KS = w.shape[1]
    if conv_state.dim() != 3 or conv_state.shape[:2] != (B, C) or conv_state.shape[2] not in (KS, KS - 1):
        raise ValueError('conv_state must be [B, C, KS] (or [B, C, KS - 1])')
    if conv_state.dtype != x3.dtype:
        raise TypeError('conv_state and x must share a dtype')
    _state_strides(conv_state)
    xin = x3 if x3.stride(1) == 1 else x3.contiguous()
    out = torch.empty((B, C, 1), device=x3.device, dtype=x3.dtype)
    b = None if bias is None else bias.to(torch.float32).contiguous()
    rc = _lib.lib().yb_conv1d_update(xin.data_ptr(), xin.stride(0), conv_state.data_ptr(), conv_state.stride(0),
                                     conv_state.stride(1), conv_state.stride(2), conv_state.shape[2], w.data_ptr(),
                                     ptr(b), out.data_ptr(), out.stride(0), B, C, KS, _silu(activation),
                                     dtype_code(x3), stream_ptr(x3.device))
    _lib.check(rc, 'causal_conv1d_update')
    return out[:, :, 0] if squeeze else out


def causal_conv1d_fn(x, weight, bias=None, seq_idx=None, initial_states=None, return_final_states=False,
                     final_states_out=None, activation=None):
    """A segment: x [B, C, T] -> [B, C, T].  ``initial_states`` [B, C, KS - 1]
    (or [B, C, KS]) holds the inputs before the segment; with
    ``return_final_states`` the last inputs come back in that width (written
    into ``final_states_out`` when given, which may be ``initial_states``)."""
    if seq_idx is not None:
        raise NotImplementedError('seq_idx (packed varlen convolution) is not part of the YANchor path')
    require_cuda(x, weight, bias, initial_states, final_states_out)
    if x.dim() != 3:
        raise ValueError('x must be [B, C, T]')
    B, C, T = x.shape
    w = _weight(weight, C)
    KS = w.shape[1]
    x = _token_major(x)
    W = KS - 1
    for st in (initial_states, final_states_out):
        if st is not None:
            if st.dim() != 3 or st.shape[:2] != (B, C) or st.shape[2] not in (KS, KS - 1):
                raise ValueError('conv states must be [B, C, KS - 1] (or [B, C, KS])')
            if st.dtype != x.dtype:
                raise ValueError('conv states must share the dtype of x')
            _state_strides(st)
            W = st.shape[2]
    if initial_states is not None and final_states_out is not None and \
            (initial_states.shape[2] != final_states_out.shape[2] or
             initial_states.stride() != final_states_out.stride()):
        raise ValueError('initial and final states must share width and strides')
    if return_final_states and final_states_out is None:
        final_states_out = torch.empty((B, C, W), device=x.device, dtype=x.dtype)
    out = torch.empty((B, T, C), device=x.device, dtype=x.dtype).transpose(1, 2)
    b = None if bias is None else bias.to(torch.float32).contiguous()
    st = initial_states if initial_states is not None else final_states_out
    st_strides = st.stride() if st is not None else (0, W, 1)
    rc = _lib.lib().yb_conv1d_fwd(x.data_ptr(), x.stride(0), x.stride(2), ptr(initial_states),
                                  ptr(final_states_out), st_strides[0], st_strides[1], st_strides[2], W, w.data_ptr(),
                                  ptr(b), out.data_ptr(),
                                  out.stride(0), out.stride(2), B, T, C, KS, _silu(activation), dtype_code(x),
                                  stream_ptr(x.device))
    _lib.check(rc, 'causal_conv1d_fn')
    return (out, final_states_out) if return_final_states else out
