"""Gated delta rule operators with the fla call signatures.

``chunk_gated_delta_rule`` and ``fused_recurrent_gated_delta_rule`` accept the
arguments of fla 0.5.1 (``fla/ops/gated_delta_rule/chunk.py:365`` and
``fused_recurrent.py:291``, the third-party package the reference pins), which
is what ``modeling_yanchor.py:397-406`` binds onto every
``Qwen3_5GatedDeltaNet`` and what ``runtime/model/inference_kernels.py:716``
calls for decode.  They also accept the positional torch-path convention of
``transformers`` qwen3_5 (``modeling_qwen3_5.py:508-529``).  Shapes:

    q, k  [B, T, H, K]      v  [B, T, HV, V]      g, beta  [B, T, HV]
    initial_state / final_state  [N, HV, K, V] float32  ([N, HV, V, K] with
    transpose_state_layout);  N = B, or len(cu_seqlens) - 1 with B == 1.

Returns ``(o [B, T, HV, V] in q.dtype, final_state or None)``.  With
``inplace=True`` (recurrent operator only) a contiguous float32
``initial_state`` is updated in place and returned as the final state, the
contract of the reference's in-place decode override
(``inference_kernels.py:147-173``).

Everything runs on the CUDA kernels of libyanchor_b200.so; there is no CPU
path.
"""
from __future__ import annotations

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, scalar_token_view, stream_ptr, token_view


def _validate(q, k, v, g, beta, initial_state, cu_seqlens):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError('q, k, v must be [B, T, H, K] / [B, T, HV, V]')
    if q.shape[2] != k.shape[2]:
        raise ValueError(f'q and k must have the same number of heads, but got q.shape[2]={q.shape[2]} '
                         f'and k.shape[2]={k.shape[2]}')
    H, HV = q.shape[2], v.shape[2]
    if HV % H != 0:
        raise ValueError(f'For GVA, num_v_heads (HV={HV}) must be evenly divisible by num_heads (H={H}), '
                         f'but got HV % H = {HV % H}')
    if q.shape != k.shape or q.shape[:2] != v.shape[:2]:
        raise ValueError('q, k, v batch/time/feature shapes disagree')
    if g is None or beta is None:
        raise ValueError('g and beta are required')
    if g.shape != v.shape[:3] or beta.shape != v.shape[:3]:
        raise ValueError('g and beta must be [B, T, HV] (head-wise beta)')
    if cu_seqlens is not None:
        if q.shape[0] != 1:
            raise ValueError(f'The batch size is expected to be 1 rather than {q.shape[0]} when using '
                             f'`cu_seqlens`.Please flatten variable-length inputs before processing.')
        if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
            raise ValueError(f'The number of initial states is expected to be equal to the number of input '
                             f'sequences, i.e., {len(cu_seqlens) - 1} rather than {initial_state.shape[0]}.')


def _common(q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm_in_kernel, cu_seqlens,
            transpose_state_layout, use_gate_in_kernel, A_log, dt_bias, beta_logits, inplace):
    require_cuda(q, k, v, g, beta, initial_state, cu_seqlens, A_log, dt_bias)
    _validate(q, k, v, g, beta, initial_state, cu_seqlens)
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError('q, k and v must share a dtype')
    if cu_seqlens is not None:
        cu = cu_seqlens.to(device=q.device, dtype=torch.int64).contiguous()
        N = cu.numel() - 1
    else:
        cu = None
        N = B
    if scale is None:
        scale = K ** -0.5
    flags = 0
    if use_qk_l2norm_in_kernel:
        flags |= _lib.GDN_QK_L2NORM
    if transpose_state_layout:
        flags |= _lib.GDN_TRANSPOSE_STATE
    if use_gate_in_kernel:
        if A_log is None:
            raise ValueError('`A_log` must be provided when `use_gate_in_kernel=True`.')
        flags |= _lib.GDN_GATE_IN_KERNEL
        A_log = A_log.to(torch.float32).contiguous()
        dt_bias = None if dt_bias is None else dt_bias.to(torch.float32).contiguous()
    else:
        A_log = dt_bias = None
    if beta_logits:
        flags |= _lib.GDN_BETA_SIGMOID
    q, qs = token_view(q)
    k, ks = token_view(k)
    v, vs = token_view(v)
    g, gs = scalar_token_view(g)
    beta, bs = scalar_token_view(beta)
    state_shape = (N, HV, V, K) if transpose_state_layout else (N, HV, K, V)
    h0 = None
    if initial_state is not None:
        if tuple(initial_state.shape) != state_shape:
            raise ValueError(f'initial_state must have shape {state_shape}, got {tuple(initial_state.shape)}')
        h0 = initial_state
        half_state = h0.dtype in (torch.float16, torch.bfloat16)
        if inplace and half_state and h0.is_contiguous() and h0.data_ptr() % 16 == 0:
            # 16-bit state storage, updated in place in its own dtype
            flags |= _lib.GDN_STATE_F16 if h0.dtype == torch.float16 else _lib.GDN_STATE_BF16
        elif h0.dtype != torch.float32 or not h0.is_contiguous() or h0.data_ptr() % 16:
            h0 = h0.to(torch.float32).contiguous()
            if h0.data_ptr() % 16:
                h0 = h0.clone()
    ht = None
    if output_final_state:
        if inplace and h0 is not None and h0 is initial_state:
            ht = h0
        else:
            ht = torch.empty(state_shape, device=q.device, dtype=torch.float32)
    o = torch.empty((B, T, HV, V), device=q.device, dtype=q.dtype)
    return dict(q=q, k=k, v=v, qs=qs, ks=ks, vs=vs, g=g, gs=gs, beta=beta, bs=bs, A_log=A_log, dt_bias=dt_bias,
                h0=h0, ht=ht, o=o, cu=cu, B=B, T=T, H=H, HV=HV, K=K, V=V, N=N, scale=float(scale), flags=flags)


def fused_recurrent_gated_delta_rule(q, k, v, g=None, gk=None, gv=None, beta=None, scale=None, initial_state=None,
                                     output_final_state=False, use_qk_l2norm_in_kernel=False,
                                     use_gate_in_kernel=False, A_log=None, dt_bias=None, cu_seqlens=None,
                                     transpose_state_layout=False, *, use_beta_sigmoid_in_kernel=False,
                                     z=None, norm_weight=None, norm_eps=1e-6, inplace=False):
    """Per-token gated delta rule (fla ``fused_recurrent_gated_delta_rule``).

    Extra keyword-only arguments: ``use_beta_sigmoid_in_kernel`` (beta holds
    logits); ``z`` / ``norm_weight`` / ``norm_eps`` to fuse the gated RMSNorm
    epilogue (``Qwen3_5RMSNormGated``) into the output; ``inplace`` to write
    the final state into ``initial_state`` (when it is a contiguous float32,
    bfloat16 or float16 tensor) and return that tensor, as the reference's
    in-place decode override does.  A 16-bit state stays 16-bit: it is the
    reference's reduced-precision state storage (``fp16_non_anchor`` /
    ``bf16_non_anchor``), widened to fp32 for the step and rounded to nearest
    when stored.  By default a new float32 final-state tensor is returned, as
    fla does.
    """
    if gk is not None or gv is not None:
        raise NotImplementedError('per-key / per-value decays (gk, gv) are not part of the YANchor path')
    if beta is None:
        beta = torch.ones(v.shape[:3], device=v.device, dtype=q.dtype)
    a = _common(q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm_in_kernel, cu_seqlens,
                transpose_state_layout, use_gate_in_kernel, A_log, dt_bias, use_beta_sigmoid_in_kernel, inplace)
    if (z is None) != (norm_weight is None):
        raise ValueError('z and norm_weight go together')
    if z is not None:
        require_cuda(z, norm_weight)
        if z.shape != a['o'].shape:
            raise ValueError('z must be [B, T, HV, V]')
        z = z.to(q.dtype).contiguous()
        norm_weight = norm_weight.to(q.dtype).contiguous()
    rc = _lib.lib().yb_gdn_recurrent_fwd(
        a['q'].data_ptr(), a['k'].data_ptr(), a['v'].data_ptr(), a['qs'], a['ks'], a['vs'],
        a['g'].data_ptr(), a['beta'].data_ptr(), a['gs'], a['bs'], ptr(a['A_log']), ptr(a['dt_bias']),
        ptr(a['h0']), ptr(a['ht']), a['o'].data_ptr(), ptr(z), ptr(norm_weight), float(norm_eps), ptr(a['cu']),
        a['B'], a['T'], a['H'], a['HV'], a['K'], a['V'], a['N'], a['scale'], dtype_code(a['q']),
        dtype_code(a['g']), dtype_code(a['beta']), a['flags'], stream_ptr(q.device))
    _lib.check(rc, 'fused_recurrent_gated_delta_rule')
    return a['o'], (a['ht'] if output_final_state else None)


def chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None, output_final_state=False,
                           use_qk_l2norm_in_kernel=False, cu_seqlens=None, cu_seqlens_cpu=None, cp_context=None,
                           transpose_state_layout=False, **kwargs):
    """Chunked (64-token) gated delta rule (fla ``chunk_gated_delta_rule``).

    Two CUDA kernels serve it, chosen by the inputs:

    * bf16 q / k / v with K = V = 128 (the YANchor shape): the tcgen05
      tensor-core kernel (``gdn_chunk_tc_kernel``), 1.5 ms at B=8, T=8192,
      H=32 on a B200;
    * anything else (fp16 or fp32 inputs, other head dimensions): the SIMT
      kernel (``gdn_chunk_simt_kernel``), which does the same arithmetic on
      the FP32 pipe, about 20x slower at the YANchor shape. Convert fp16
      inputs to bf16 first where that precision is acceptable.
    """
    if 'head_first' in kwargs:
        raise DeprecationWarning('head_first has been removed. Inputs must be in `[B, T, H, ...]` format.')
    if cp_context is not None:
        raise NotImplementedError('context parallelism is not part of the YANchor path')
    if 'chunk_size' in kwargs and kwargs['chunk_size'] != 64:
        raise NotImplementedError('only chunk_size=64 is built')
    use_gate_in_kernel = kwargs.get('use_gate_in_kernel', False)
    a = _common(q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm_in_kernel, cu_seqlens,
                transpose_state_layout, use_gate_in_kernel, kwargs.get('A_log'), kwargs.get('dt_bias'),
                kwargs.get('use_beta_sigmoid_in_kernel', False), inplace=False)
    L = _lib.lib()
    need = L.yb_gdn_chunk_workspace_bytes(a['B'], a['T'], a['H'], a['HV'], a['K'], a['V'], a['N'],
                                          dtype_code(a['q']))
    ws = torch.empty(max(need, 1), device=q.device, dtype=torch.uint8) if need > 0 else None
    rc = L.yb_gdn_chunk_fwd(
        a['q'].data_ptr(), a['k'].data_ptr(), a['v'].data_ptr(), a['qs'], a['ks'], a['vs'],
        a['g'].data_ptr(), a['beta'].data_ptr(), a['gs'], a['bs'], ptr(a['A_log']), ptr(a['dt_bias']),
        ptr(a['h0']), ptr(a['ht']), a['o'].data_ptr(), ptr(a['cu']),
        a['B'], a['T'], a['H'], a['HV'], a['K'], a['V'], a['N'], a['scale'], dtype_code(a['q']),
        dtype_code(a['g']), dtype_code(a['beta']), a['flags'], ptr(ws), need, stream_ptr(q.device))
    _lib.check(rc, 'chunk_gated_delta_rule')
    return a['o'], (a['ht'] if output_final_state else None)


def gdn_gates(b, a, A_log, dt_bias):
    """beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) for one
    decode token: b, a ``[B, 1, HV]`` (any row stride) -> (beta in b.dtype,
    g float32), as ``runtime/model/inference_kernels.py:683-691``."""
    require_cuda(b, a, A_log, dt_bias)
    if b.shape != a.shape or b.shape[-1] != A_log.numel():
        raise ValueError('fused GDN gates require matching [.., HV] head logits')
    if b.stride(-1) != 1 or a.stride(-1) != 1:
        b, a = b.contiguous(), a.contiguous()
    heads = b.shape[-1]
    rows = b.numel() // heads
    b2, a2 = b.reshape(rows, heads), a.reshape(rows, heads)
    beta = torch.empty(b.shape, device=b.device, dtype=b.dtype)
    g = torch.empty(b.shape, device=b.device, dtype=torch.float32)
    A = A_log.to(torch.float32).contiguous()
    dtb = None if dt_bias is None else dt_bias.to(torch.float32).contiguous()
    rc = _lib.lib().yb_gdn_gates(b2.data_ptr(), a2.data_ptr(), b2.stride(0), a2.stride(0), A.data_ptr(), ptr(dtb),
                                 beta.data_ptr(), g.data_ptr(), rows, heads, dtype_code(b), stream_ptr(b.device))
    _lib.check(rc, 'gdn_gates')
    return beta, g


# names used by fla and by the transformers torch path
fused_recurrent_gdn = fused_recurrent_gated_delta_rule
chunk_gdn = chunk_gated_delta_rule
recurrent_gated_delta_rule = fused_recurrent_gated_delta_rule


def fused_gdn_decode(mixed_qkv, z, a, b, conv_state, conv_weight, conv_bias, recurrent_state, A_log, dt_bias,
                     norm_weight, *, num_k_heads, norm_eps=1e-6, scale=None, transpose_state_layout=False):
    """One GDN layer's decode core, everything between ``in_proj_*`` and
    ``out_proj`` of ``_fused_gdn_gate_native_decode_forward``
    (runtime/model/inference_kernels.py:693-721), in one launch:
    short conv update (SiLU) -> split q | k | v -> gates -> L2 norm -> gated
    delta rule (state in place) -> gated RMSNorm with z.

    mixed_qkv ``[B, T, 2*H*K + HV*V]`` (the in_proj_qkv output, token-major);
    z ``[B, T, HV, V]`` (or ``[B, T, HV*V]``); a, b ``[B, T, HV]`` logits;
    conv_state ``[B, C, 4]`` (activation dtype) and recurrent_state
    ``[B, HV, K, V]`` (float32, bfloat16 or float16) are updated in place;
    conv_weight ``[C, 4]`` (or ``[C, 1, 4]``); returns ``[B, T, HV, V]``.
    K = V = 128, HV / H in {1, 2}.
    """
    require_cuda(mixed_qkv, z, a, b, conv_state, conv_weight, conv_bias, recurrent_state, A_log, dt_bias,
                 norm_weight)
    B, T, C = mixed_qkv.shape
    N, HV = recurrent_state.shape[0], recurrent_state.shape[1]
    K = recurrent_state.shape[3] if transpose_state_layout else recurrent_state.shape[2]
    V = recurrent_state.shape[2] if transpose_state_layout else recurrent_state.shape[3]
    H = int(num_k_heads)
    if N != B or C != 2 * H * K + HV * V:
        raise ValueError('mixed_qkv must be [B, T, 2*H*K + HV*V] for the recurrent state [B, HV, K, V]')
    if mixed_qkv.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError('activations must be bfloat16 or float16')
    for name, t in (('z', z), ('a', a), ('b', b), ('conv_state', conv_state), ('norm_weight', norm_weight)):
        if t.dtype != mixed_qkv.dtype:
            raise TypeError(f'{name} must share the activation dtype')
    if not recurrent_state.is_contiguous() or recurrent_state.data_ptr() % 16:
        raise ValueError('recurrent_state must be contiguous and 16-byte aligned (it is updated in place)')
    if conv_state.shape != (B, C, 4) or conv_state.stride(2) != 1 or conv_state.stride(1) != 4:
        raise ValueError('conv_state must be [B, C, 4], contiguous inside each batch row')
    mixed, ms = token_view(mixed_qkv)
    z = z.reshape(B, T, HV, V)
    z, zs = token_view(z)
    a, abs_ = scalar_token_view(a)
    b, bs_ = scalar_token_view(b)
    if abs_ != bs_:
        b = b.reshape(B, T, HV).contiguous()
        a = a.reshape(B, T, HV).contiguous()
        abs_ = HV
    w = conv_weight.reshape(C, -1).to(torch.float32).contiguous()
    cb = None if conv_bias is None else conv_bias.to(torch.float32).contiguous()
    A_log = A_log.to(torch.float32).contiguous()
    dt_bias = None if dt_bias is None else dt_bias.to(torch.float32).contiguous()
    norm_weight = norm_weight.contiguous()
    o = torch.empty((B, T, HV, V), device=mixed_qkv.device, dtype=mixed_qkv.dtype)
    sd = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[recurrent_state.dtype]
    rc = _lib.lib().yb_gdn_decode_fused(
        mixed.data_ptr(), ms, z.data_ptr(), zs, a.data_ptr(), b.data_ptr(), abs_, conv_state.data_ptr(),
        conv_state.stride(0), 4, w.data_ptr(), ptr(cb), w.shape[1], recurrent_state.data_ptr(), sd, A_log.data_ptr(),
        ptr(dt_bias), norm_weight.data_ptr(), float(norm_eps), o.data_ptr(), B, T, H, HV, K, V,
        float(K ** -0.5 if scale is None else scale), dtype_code(mixed_qkv),
        _lib.GDN_TRANSPOSE_STATE if transpose_state_layout else 0, stream_ptr(mixed_qkv.device))
    _lib.check(rc, 'fused_gdn_decode')
    return o
