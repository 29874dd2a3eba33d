"""Bind the B200 operators where the reference looks them up.

* ``bind_gdn_kernels(model)`` sets ``chunk_gated_delta_rule`` and
  ``recurrent_gated_delta_rule`` on every module that has them (the
  ``Qwen3_5GatedDeltaNet`` layers), as ``bind_native_qwen_gdn_kernels`` does
  for fla (``modeling_yanchor.py:392-410``), and their
  ``causal_conv1d_update`` / ``causal_conv1d_fn``.  With ``inplace_decode`` the
  recurrent operator updates the cached state in place, as the reference's
  decode override (``runtime/model/inference_kernels.py:147-184``).
* ``install_memory_module()`` makes ``importlib.import_module(
  "model.independent_memory")`` — the lookup of ``_cuda_module``
  (``modeling_yanchor.py:19-20``) — return ``yanchor_b200.independent_memory``.
* ``bind_memory_prefill(modeling)`` replaces the module-level ``select_topk``
  / ``merge_topk`` / ``exclusive_prefix_topk`` of the given
  ``modeling_yanchor`` module and ``IndependentGQAMemory._sequence``
  (modeling_yanchor.py:51-78, 178-275) with ``yanchor_b200.memory_prefill``.
"""
from __future__ import annotations

import functools
import sys
import types

from . import conv as conv1d, gated_delta_rule, independent_memory, memory_prefill


def bind_gdn_kernels(model, *, inplace_decode: bool = True, conv: bool = True) -> dict:
    recurrent = functools.partial(gated_delta_rule.fused_recurrent_gated_delta_rule, inplace=inplace_decode)
    names = []
    for name, module in model.named_modules():
        if hasattr(module, 'chunk_gated_delta_rule') and hasattr(module, 'recurrent_gated_delta_rule'):
            module.chunk_gated_delta_rule = gated_delta_rule.chunk_gated_delta_rule
            module.recurrent_gated_delta_rule = recurrent
            if conv and hasattr(module, 'causal_conv1d_update'):
                # the layer's short convolution (transformers qwen3_5 modeling_qwen3_5.py:453-476)
                module.causal_conv1d_update = conv1d.causal_conv1d_update
                module.causal_conv1d_fn = conv1d.causal_conv1d_fn
            names.append(name)
    if not names:
        raise RuntimeError('no GDN layers were found')
    return {'backend': 'yanchor_b200', 'native_gdn_layers': names, 'inplace_decode': inplace_decode, 'conv': conv}


def install_memory_module() -> types.ModuleType:
    pkg = sys.modules.get('model')
    if pkg is None:
        pkg = types.ModuleType('model')
        pkg.__path__ = []
        sys.modules['model'] = pkg
    sys.modules['model.independent_memory'] = independent_memory
    pkg.independent_memory = independent_memory
    return independent_memory


def bind_memory_prefill(modeling) -> dict:
    for name in ('select_topk', 'merge_topk', 'exclusive_prefix_topk'):
        setattr(modeling, name, getattr(memory_prefill, name))

    def _sequence(self, u, query, scores, position_embeddings, valid, chunk, state=None):
        def write_kv(batch_index, token_index):
            angles = tuple(x.expand(query.shape[0], -1, -1)[batch_index, token_index] for x in position_embeddings)
            return self._write_kv(u[batch_index, token_index], angles)
        return memory_prefill.sequence(query, scores, write_kv, valid, chunk, state, capacity=self.capacity)

    modeling.IndependentGQAMemory._sequence = _sequence
    return {'backend': 'yanchor_b200', 'memory_prefill': ['select_topk', 'merge_topk', 'exclusive_prefix_topk',
                                                          'IndependentGQAMemory._sequence']}
