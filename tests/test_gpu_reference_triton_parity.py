"""GPU parity against the reference's own GPU kernels for the anchor memory:
the Triton module runtime/model/independent_memory.py from the reference
install (`committed_gqa` :177, `commit_decode` :190, `indexed_gqa` :38), run
on the same inputs on the same GPU.

The memory state is index and copy work, so after every decode step each
state field must be equal bit for bit; the reads are bf16 outputs of two
different fp32 reductions and must agree within the north-star bar
(2e-2)."""
import importlib.util
import os
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

REF = os.path.join(ROOT, 'baseline', '_ref')
FIELDS = ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values', 'pending_scores', 'count',
          'total')


@pytest.fixture(scope='module')
def ref_mem():
    path = os.path.join(REF, 'runtime', 'model', 'independent_memory.py')
    if not os.path.exists(path):
        pytest.skip('SKIPPED, NOT PASSED: the reference install (baseline/_ref) is absent')
    if REF not in sys.path:
        sys.path.append(REF)   # the module imports modeling_yanchor from the install root
    spec = importlib.util.spec_from_file_location('reference_independent_memory_parity', path)
    mod = importlib.util.module_from_spec(spec)
    try:
        spec.loader.exec_module(mod)
    except Exception as e:  # noqa: BLE001
        pytest.skip(f'SKIPPED, NOT PASSED: the reference memory module does not load ({type(e).__name__}: {e})')
    return mod


@pytest.fixture(scope='module')
def yb():
    import yanchor_b200
    return yanchor_b200


def test_decode_steps_match_reference_triton(yb, ref_mem):
    """70 decode steps (one commit of every row's chunk, some rows inactive)
    through this library's one-launch step and through the reference's
    committed_gqa + commit_decode, each on its own copy of the state."""
    B, G, H, D, CAP, CH = 16, 4, 16, 256, 64, 64
    bf = torch.bfloat16
    gen = torch.Generator(device='cuda').manual_seed(17)
    ours = yb.MemoryState.empty(B, G, CAP, CH, D, 'cuda', bf)
    theirs = yb.MemoryState.empty(B, G, CAP, CH, D, 'cuda', bf)
    for step in range(70):
        q = torch.randn(B, 1, H, D, generator=gen, device='cuda').to(bf)
        k = torch.randn(B, 1, G, D, generator=gen, device='cuda').to(bf)
        v = torch.randn(B, 1, G, D, generator=gen, device='cuda').to(bf)
        s = (torch.randn(B, 1, G, generator=gen, device='cuda') * 2).round() / 2   # ties on purpose
        active = torch.rand(B, generator=gen, device='cuda') > 0.1
        out = yb.memory_decode_step(q, k, v, s, active, CH, ours)
        ref_out = ref_mem.committed_gqa(q, theirs, None)
        ref_mem.commit_decode(k, v, s, active, CH, theirs, None)
        torch.cuda.synchronize()
        assert (out.float() - ref_out.float()).abs().max().item() <= 2e-2, step
    for f in FIELDS:
        assert torch.equal(getattr(ours, f), getattr(theirs, f)), f
    assert int(ours.total.max()) >= CH   # at least one chunk was committed


def test_indexed_read_matches_reference_triton(yb, ref_mem):
    """The prefill read: every block's queries over its referenced rows plus
    the null slot, empty references included."""
    B, blocks, CH, H, G, D, S, CAP = 2, 8, 64, 16, 4, 256, 300, 64
    bf = torch.bfloat16
    gen = torch.Generator(device='cuda').manual_seed(23)
    q = torch.randn(B, blocks, CH, H, D, generator=gen, device='cuda').to(bf)
    kv = torch.randn(2, 1, S, G, D, generator=gen, device='cuda').to(bf)
    refs = torch.randint(0, S, (B, blocks, G, CAP), generator=gen, device='cuda')
    refs[torch.rand(refs.shape, generator=gen, device='cuda') < 0.2] = -1
    out = yb.indexed_gqa(q, kv[0], kv[1], refs)
    ref_out = ref_mem.indexed_gqa(q, kv[0], kv[1], refs)
    torch.cuda.synchronize()
    assert (out.float() - ref_out.float()).abs().max().item() <= 2e-2


def test_top20_sampler_matches_reference_triton(yb):
    """The reference's production sampler on the GPU (the fused top-20 counter
    sampler, runtime/model/inference_kernels.py:1147-1164, selected at :1420)
    against this library's on the same fp32 logits: the same token for every
    row (continuous logits, so no ties inside the top 20)."""
    path = os.path.join(REF, 'runtime', 'model', 'inference_kernels.py')
    if not os.path.exists(path):
        pytest.skip('SKIPPED, NOT PASSED: the reference install (baseline/_ref) is absent')
    import _reference
    ik = _reference.inference_kernels()
    B, vocab = 64, 248320
    gen = torch.Generator(device='cuda').manual_seed(31)
    for step in range(4):
        logits = 3 * torch.randn(B, vocab, generator=gen, device='cuda')   # fp32: no ties in the top 20
        attempt = torch.arange(B, device='cuda', dtype=torch.int64) + 100 * step
        ref_ids = ik._sample_top_k_top_p_counter_triton(logits, attempt, step, seed=1234, temperature=0.7, top_k=20,
                                                        top_p=0.95)
        ids = yb.sample_top_k_top_p_counter(logits, attempt, step, seed=1234, temperature=0.7, top_k=20, top_p=0.95)
        torch.cuda.synchronize()
        assert torch.equal(ids.view(-1).cpu(), ref_ids.view(-1).cpu()), step
