"""yanchor_b200 — B200 (sm_100a) kernels for YANchor's data-parallel hot path.

Operators (all CUDA, via the C ABI library libyanchor_b200.so):

* gated delta rule: ``chunk_gated_delta_rule`` (prefill),
  ``fused_recurrent_gated_delta_rule`` (decode), ``gdn_gates``, and the
  short convolution before it: ``causal_conv1d_update`` /
  ``causal_conv1d_fn``
* anchor memory: ``indexed_gqa`` (prefill read), ``committed_gqa`` (decode
  read), ``commit_decode`` (decode write), ``memory_decode_step`` (the read
  and the write of one decode step in one launch), ``select_topk`` / ``merge_topk`` /
  ``exclusive_prefix_topk`` (top-CAP selection) and ``sequence`` (the
  prefill read / write orchestration)
* sliding-window attention decode over the physical ring:
  ``physical_ring_update_``, ``physical_ring_decode_attention``
* sampling: ``greedy``, ``sample_top_k_top_p_counter``,
  ``apply_dense_presence_penalty_``
* decode loop: ``update_fixed_decode_state_`` (per-step bookkeeping in one
  launch), ``prepare_capture`` and ``StepGraphs`` (CUDA graphs of a decode
  step per batch size, captured without warm-up forwards)
* ``bind_gdn_kernels`` / ``install_memory_module`` / ``bind_memory_prefill``
  put them where the reference model code looks them up.
* ``torch.ops.yanchor_b200.*`` (``yanchor_b200.ops``): the same operators
  registered as torch custom ops with fake implementations, for tracers
  such as ``torch.compile``.
"""
from .gated_delta_rule import (chunk_gated_delta_rule, fused_gdn_decode, fused_recurrent_gated_delta_rule,  # noqa: F401
                               gdn_gates)
from .conv import causal_conv1d_fn, causal_conv1d_update  # noqa: F401
from .swa import (flash_swa, layer_ring_update, physical_ring_decode_attention,  # noqa: F401
                  physical_ring_update_, reference_swa)
from .independent_memory import MemoryState, commit_decode, committed_gqa, indexed_gqa  # noqa: F401
from .independent_memory import decode_step as memory_decode_step  # noqa: F401
from .memory_prefill import exclusive_prefix_topk, merge_topk, select_topk, sequence  # noqa: F401
from .sampling import apply_dense_presence_penalty_, greedy, greedy_noalloc, sample_top_k_top_p_counter  # noqa: F401
from .decode_loop import StepGraphs, prepare_capture, update_fixed_decode_state_  # noqa: F401
from .bind import bind_gdn_kernels, bind_memory_prefill, install_memory_module  # noqa: F401
from . import ops  # noqa: F401  (registers torch.ops.yanchor_b200.*)
from ._lib import LIB_PATH, YanchorError, lib  # noqa: F401

__version__ = '0.1.0'
