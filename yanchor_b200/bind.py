"""Bind the B200 operators where the reference looks them up.

* ``bind_gdn_kernels(model)`` sets ``chunk_gated_delta_rule`` and
  ``recurrent_gated_delta_rule`` on every module that has them (the
  ``Qwen3_5GatedDeltaNet`` layers), as ``bind_native_qwen_gdn_kernels`` does
  for fla (``modeling_yanchor.py:392-410``).  With ``inplace_decode`` the
  recurrent operator updates the cached state in place, as the reference's
  decode override (``runtime/model/inference_kernels.py:147-184``).
* ``install_memory_module()`` makes ``importlib.import_module(
  "model.independent_memory")`` — the lookup of ``_cuda_module``
  (``modeling_yanchor.py:19-20``) — return ``yanchor_b200.independent_memory``.
"""
from __future__ import annotations

import functools
import sys
import types

from . import gated_delta_rule, independent_memory


def bind_gdn_kernels(model, *, inplace_decode: bool = True) -> dict:
    recurrent = functools.partial(gated_delta_rule.fused_recurrent_gated_delta_rule, inplace=inplace_decode)
    names = []
    for name, module in model.named_modules():
        if hasattr(module, 'chunk_gated_delta_rule') and hasattr(module, 'recurrent_gated_delta_rule'):
            module.chunk_gated_delta_rule = gated_delta_rule.chunk_gated_delta_rule
            module.recurrent_gated_delta_rule = recurrent
            names.append(name)
    if not names:
        raise RuntimeError('no GDN layers were found')
    return {'backend': 'yanchor_b200', 'native_gdn_layers': names, 'inplace_decode': inplace_decode}


def install_memory_module() -> types.ModuleType:
    pkg = sys.modules.get('model')
    if pkg is None:
        pkg = types.ModuleType('model')
        pkg.__path__ = []
        sys.modules['model'] = pkg
    sys.modules['model.independent_memory'] = independent_memory
    pkg.independent_memory = independent_memory
    return independent_memory
