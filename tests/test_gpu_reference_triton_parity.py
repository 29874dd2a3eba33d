"""GPU parity against the reference's own GPU kernels, run from its install
on the same inputs on the same GPU: the anchor memory's Triton module
runtime/model/independent_memory.py (`committed_gqa` :177, `commit_decode`
:190, `indexed_gqa` :38), and from runtime/model/inference_kernels.py the
fused top-20 sampler, the graph-safe conv update, the fused GDN gates and
the decode loop's bookkeeping.

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


def _kernels():
    if not os.path.exists(os.path.join(REF, 'runtime', 'model', 'inference_kernels.py')):
        pytest.skip('SKIPPED, NOT PASSED: the reference install (baseline/_ref) is absent')
    import _reference
    return _reference.inference_kernels()


def test_conv_update_matches_reference_triton(yb):
    """The graph-safe decode convolution (inference_kernels.py:339-376) on the
    cache's own [B, C, 4] state layout: the shifted state bit-identical, the
    bf16 output within one rounding (the two sum the four taps in different
    orders)."""
    ik = _kernels()
    B, C, KS = 64, 8192, 4
    bf = torch.bfloat16
    gen = torch.Generator(device='cuda').manual_seed(41)
    state = torch.randn(B, C, KS, generator=gen, device='cuda').to(bf)
    ref_state = state.clone()
    w = torch.randn(C, KS, generator=gen, device='cuda') * 0.5
    bias = torch.randn(C, generator=gen, device='cuda') * 0.1
    for _ in range(3):
        x = torch.randn(B, C, 1, generator=gen, device='cuda').to(bf)
        y = yb.causal_conv1d_update(x, state, w, bias, 'silu')
        ry = ik.triton_graph_safe_causal_conv1d_update(x, ref_state, w, bias, 'silu')
        torch.cuda.synchronize()
        assert torch.equal(state, ref_state)
        d = (y.float() - ry.float()).abs()
        assert (d <= ry.float().abs() * 2 ** -7 + 1e-6).all()


def test_gates_match_reference_triton(yb):
    """The fused decode gates (inference_kernels.py:668-691): beta = sigmoid(b)
    in bf16 and g = -exp(A_log) softplus(a + dt_bias) in fp32."""
    ik = _kernels()
    B, HV = 64, 32
    gen = torch.Generator(device='cuda').manual_seed(43)
    b = torch.randn(B, 1, HV, generator=gen, device='cuda').to(torch.bfloat16)
    a = (3 * torch.randn(B, 1, HV, generator=gen, device='cuda')).to(torch.bfloat16)
    A_log = torch.log(torch.rand(HV, generator=gen, device='cuda') * 15 + 1)
    dt_bias = torch.randn(HV, generator=gen, device='cuda')
    beta, g = yb.gdn_gates(b, a, A_log, dt_bias)
    rbeta, rg = ik.triton_qwen35_fused_gdn_gates(b, a, A_log, dt_bias)
    torch.cuda.synchronize()
    assert (beta.float() - rbeta.float()).abs().max().item() <= 2 ** -8
    assert ((g - rg).abs() <= rg.abs() * 1e-5 + 1e-7).all()


def test_decode_bookkeeping_matches_reference_triton(yb):
    """The decode loop's per-step bookkeeping (inference_kernels.py:1169-1208)
    over a 42-step trajectory with EOS ids, empty slots and per-row caps:
    every table bit-identical."""
    ik = _kernels()
    slots, total, max_new, vocab, pad, eos = 96, 192, 40, 64, 1, (5, 9)
    gen = torch.Generator(device='cuda').manual_seed(47)
    i64 = dict(device='cuda', dtype=torch.int64)

    def fresh():
        perm = torch.randperm(total, generator=gen, device='cuda')[:slots]
        rows = torch.where(torch.rand(slots, generator=gen, device='cuda') < 0.9, perm, torch.full_like(perm, -1))
        return {
            'storage': torch.full((total + slots, max_new + 1), pad, device='cuda', dtype=torch.int32),
            'dense_seen': torch.zeros(slots, vocab, device='cuda', dtype=torch.bool),
            'generated_lengths': torch.zeros(total + slots, **i64),
            'finished_by_eos': torch.zeros(total + slots, device='cuda', dtype=torch.bool),
            'finished': torch.rand(slots, generator=gen, device='cuda') < 0.1,
            'slot_rows': rows,
            'sink_rows': total + torch.arange(slots, **i64),
            'slot_caps': torch.randint(1, max_new + 1, (slots,), generator=gen, **i64),
            'row_steps': torch.ones(slots, **i64),
            'row_positions': torch.randint(0, 5000, (slots,), generator=gen, **i64),
            'decode_ids': torch.randint(0, vocab, (slots, 1), generator=gen, **i64),
            'decode_useful_events': torch.zeros((), **i64),
        }
    ours = fresh()
    theirs = {k: v.clone() for k, v in ours.items()}
    order = ('storage', 'dense_seen', 'generated_lengths', 'finished_by_eos', 'finished', 'slot_rows', 'sink_rows',
             'slot_caps', 'row_steps', 'row_positions', 'decode_ids', 'decode_useful_events')
    for _ in range(max_new + 2):
        tok = torch.randint(0, vocab, (slots, 1), generator=gen, **i64)
        yb.update_fixed_decode_state_(tok, *(ours[k] for k in order), maximum_new_tokens=max_new,
                                      pad_token_id=pad, eos_token_ids=eos)
        ik._update_fixed_decode_state_(tok, *(theirs[k] for k in order), maximum_new_tokens=max_new,
                                       pad_token_id=pad, eos_token_ids=eos)
    torch.cuda.synchronize()
    for k in order:
        assert torch.equal(ours[k], theirs[k]), k
