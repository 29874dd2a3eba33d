"""The hot-path operators registered as torch custom ops (``torch.ops.yanchor_b200.*``).

The reference's serving hosts trace the model around these calls: vLLM
compiles the decode graph around ``vllm_yanchor.py:49-82``, and
``torch.compile`` needs every op it meets to be either traceable or a
registered custom op with a fake (shape-only) implementation.  Each op below
wraps the same C-ABI call as the Python API in this package and declares
which arguments it writes in place, so a tracer neither looks inside the
CUDA library nor loses the state updates.  Calling through
``torch.ops.yanchor_b200`` gives the same results as the plain functions.

    chunk_gated_delta_rule(q, k, v, g, beta, scale, initial_state,
        output_final_state, use_qk_l2norm_in_kernel, cu_seqlens,
        transpose_state_layout) -> (o, final_state)   # final_state empty if not asked
    fused_recurrent_gated_delta_rule_(q, k, v, g, beta, scale, state,
        use_qk_l2norm_in_kernel, use_gate_in_kernel, A_log, dt_bias,
        beta_logits, z, norm_weight, norm_eps) -> o     # state updated in place
    causal_conv1d_update_(x, conv_state, weight, bias, silu) -> y   # conv_state in place
    indexed_gqa(query, key, value, references) -> out
    committed_gqa(query, <state fields>, indices) -> out
    commit_decode_(key, value, scores, active, chunk, keys, values, bank_scores,
        positions, pending_keys, pending_values, pending_scores, count, total,
        indices) -> ()                                   # the memory state in place
    memory_decode_step_(query, key, value, scores, active, chunk, <state fields>,
        indices) -> out                                  # read, then the commit in place
    greedy(scores) -> ids [B, 1] int64
    sample_top_k_top_p_counter(scores, attempt_ids, steps, seed, temperature,
        top_k, top_p, stream) -> ids [B, 1] int64
"""
from typing import Optional

import torch
from torch import Tensor

from . import conv as _conv
from . import gated_delta_rule as _gdr
from . import independent_memory as _mem
from . import sampling as _samp

_NS = 'yanchor_b200'
_MEM_FIELDS = ('keys', 'values', 'bank_scores', 'positions', 'pending_keys', 'pending_values', 'pending_scores',
               'count', 'total')


def _state(*fields):
    return _mem.MemoryState(*fields)


# ------------------------------------------------------------------- GDN ----
@torch.library.custom_op(f'{_NS}::chunk_gated_delta_rule', mutates_args=())
def chunk_gated_delta_rule(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, scale: float,
                           initial_state: Optional[Tensor], output_final_state: bool, use_qk_l2norm_in_kernel: bool,
                           cu_seqlens: Optional[Tensor], transpose_state_layout: bool) -> tuple[Tensor, Tensor]:
    o, s = _gdr.chunk_gated_delta_rule(q, k, v, g, beta, scale=scale, initial_state=initial_state,
                                       output_final_state=output_final_state,
                                       use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel, cu_seqlens=cu_seqlens,
                                       transpose_state_layout=transpose_state_layout)
    return o, (s if s is not None else q.new_empty((0,), dtype=torch.float32))


@chunk_gated_delta_rule.register_fake
def _(q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm_in_kernel, cu_seqlens,
      transpose_state_layout):
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.shape[0] - 1
    o = q.new_empty((B, T, HV, V))
    if not output_final_state:
        return o, q.new_empty((0,), dtype=torch.float32)
    shape = (N, HV, V, K) if transpose_state_layout else (N, HV, K, V)
    return o, q.new_empty(shape, dtype=torch.float32)


@torch.library.custom_op(f'{_NS}::fused_recurrent_gated_delta_rule_', mutates_args=('state',))
def fused_recurrent_gated_delta_rule_(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, scale: float,
                                      state: Tensor, use_qk_l2norm_in_kernel: bool, use_gate_in_kernel: bool,
                                      A_log: Optional[Tensor], dt_bias: Optional[Tensor], beta_logits: bool,
                                      z: Optional[Tensor], norm_weight: Optional[Tensor],
                                      norm_eps: float) -> Tensor:
    if not state.is_contiguous() or state.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ValueError('the in-place state must be a contiguous float32, float16 or bfloat16 tensor')
    o, _ = _gdr.fused_recurrent_gated_delta_rule(
        q, k, v, g=g, beta=beta, scale=scale, initial_state=state, output_final_state=True,
        use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel, use_gate_in_kernel=use_gate_in_kernel, A_log=A_log,
        dt_bias=dt_bias, use_beta_sigmoid_in_kernel=beta_logits, z=z, norm_weight=norm_weight, norm_eps=norm_eps,
        inplace=True)
    return o


@fused_recurrent_gated_delta_rule_.register_fake
def _(q, k, v, g, beta, scale, state, use_qk_l2norm_in_kernel, use_gate_in_kernel, A_log, dt_bias, beta_logits, z,
      norm_weight, norm_eps):
    B, T = q.shape[:2]
    return q.new_empty((B, T, v.shape[2], v.shape[3]))


@torch.library.custom_op(f'{_NS}::causal_conv1d_update_', mutates_args=('conv_state',))
def causal_conv1d_update_(x: Tensor, conv_state: Tensor, weight: Tensor, bias: Optional[Tensor],
                          silu: bool) -> Tensor:
    return _conv.causal_conv1d_update(x, conv_state, weight, bias, 'silu' if silu else None)


@causal_conv1d_update_.register_fake
def _(x, conv_state, weight, bias, silu):
    return x.new_empty(x.shape)


# ---------------------------------------------------------------- memory ----
@torch.library.custom_op(f'{_NS}::indexed_gqa', mutates_args=())
def indexed_gqa(query: Tensor, key: Tensor, value: Tensor, references: Tensor) -> Tensor:
    return _mem.indexed_gqa(query, key, value, references)


@indexed_gqa.register_fake
def _(query, key, value, references):
    return query.new_empty(query.shape)


@torch.library.custom_op(f'{_NS}::committed_gqa', mutates_args=())
def committed_gqa(query: Tensor, keys: Tensor, values: Tensor, bank_scores: Tensor, positions: Tensor,
                  pending_keys: Tensor, pending_values: Tensor, pending_scores: Tensor, count: Tensor,
                  total: Tensor, indices: Optional[Tensor]) -> Tensor:
    return _mem.committed_gqa(query, _state(keys, values, bank_scores, positions, pending_keys, pending_values,
                                            pending_scores, count, total), indices)


@committed_gqa.register_fake
def _(query, keys, values, bank_scores, positions, pending_keys, pending_values, pending_scores, count, total,
      indices):
    return query.new_empty(query.shape)


@torch.library.custom_op(f'{_NS}::commit_decode_', mutates_args=_MEM_FIELDS)
def commit_decode_(key: Tensor, value: Tensor, scores: Tensor, active: Tensor, chunk: int, keys: Tensor,
                   values: Tensor, bank_scores: Tensor, positions: Tensor, pending_keys: Tensor,
                   pending_values: Tensor, pending_scores: Tensor, count: Tensor, total: Tensor,
                   indices: Optional[Tensor]) -> None:
    _mem.commit_decode(key, value, scores, active, chunk,
                       _state(keys, values, bank_scores, positions, pending_keys, pending_values, pending_scores,
                              count, total), indices)


@commit_decode_.register_fake
def _(key, value, scores, active, chunk, keys, values, bank_scores, positions, pending_keys, pending_values,
      pending_scores, count, total, indices):
    return None


@torch.library.custom_op(f'{_NS}::memory_decode_step_', mutates_args=_MEM_FIELDS)
def memory_decode_step_(query: Tensor, key: Tensor, value: Tensor, scores: Tensor, active: Tensor, chunk: int,
                        keys: Tensor, values: Tensor, bank_scores: Tensor, positions: Tensor, pending_keys: Tensor,
                        pending_values: Tensor, pending_scores: Tensor, count: Tensor, total: Tensor,
                        indices: Optional[Tensor]) -> Tensor:
    return _mem.decode_step(query, key, value, scores, active, chunk,
                            _state(keys, values, bank_scores, positions, pending_keys, pending_values,
                                   pending_scores, count, total), indices)


@memory_decode_step_.register_fake
def _(query, key, value, scores, active, chunk, keys, values, bank_scores, positions, pending_keys, pending_values,
      pending_scores, count, total, indices):
    return query.new_empty(query.shape)


# -------------------------------------------------------------- sampling ----
@torch.library.custom_op(f'{_NS}::greedy', mutates_args=())
def greedy(scores: Tensor) -> Tensor:
    return _samp.greedy(scores)


@greedy.register_fake
def _(scores):
    return scores.new_empty((scores.shape[0], 1), dtype=torch.int64)


@torch.library.custom_op(f'{_NS}::sample_top_k_top_p_counter', mutates_args=())
def sample_top_k_top_p_counter(scores: Tensor, attempt_ids: Tensor, steps: Tensor, seed: int, temperature: float,
                               top_k: int, top_p: float, stream: int) -> Tensor:
    return _samp.sample_top_k_top_p_counter(scores, attempt_ids, steps, seed=seed, temperature=temperature,
                                            top_k=top_k, top_p=top_p, stream=stream)


@sample_top_k_top_p_counter.register_fake
def _(scores, attempt_ids, steps, seed, temperature, top_k, top_p, stream):
    return scores.new_empty((scores.shape[0], 1), dtype=torch.int64)


def memory_fields(state):
    """The memory state's tensors in the order the memory ops take them."""
    return (state.keys, state.values, state.scores, state.positions, state.pending_keys, state.pending_values,
            state.pending_scores, state.count, state.total)
