"""CPU oracle for the YANchor hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithms that the CUDA
kernels of ``yanchor_b200`` replace.  It exists so that the tests, the
``smoke()`` check in ``__graft_entry__`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` have an independent CPU answer to
compare against.  Product code (``yanchor_b200``) never imports it: the
product path fails loudly when its CUDA library is missing instead of falling
back to anything here.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
torch implementation (the pinned transformers wheel's Qwen3.5 GDN functions
and ``modeling_yanchor.py``'s anchor-memory code, plus
``runtime/model/inference_kernels.py``'s counter sampler) on seeded inputs and
commits the outputs as fixtures; ``tests/test_oracle_golden.py`` checks every
function here against them.

Modules:
  gdn       gated delta rule: l2norm, gates, recurrent and chunked forms,
            gated RMSNorm epilogue
  memory    anchor memory: top-k selection, prefix top-k, indexed prefill read,
            decode read, decode commit
  sampling  counter uniform, greedy, top-k/top-p counter sampler, presence
            penalty
"""
