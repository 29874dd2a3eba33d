"""Generate golden fixtures from the reference's own torch implementation.

Run once in a container where the reference project is available:

    python tests/golden/make_golden.py --reference /path/to/YANchor

It extracts the pinned transformers wheel (``wheels/transformers-*.whl``, pure
Python) to a scratch directory, puts it and the reference root first on
``sys.path`` and calls:

* ``torch_chunk_gated_delta_rule`` / ``torch_recurrent_gated_delta_rule`` /
  ``l2norm`` / ``Qwen3_5RMSNormGated``
  (transformers/models/qwen3_5/modeling_qwen3_5.py:175-353)
* the gate expression of ``Qwen3_5GatedDeltaNet.forward`` (same file :500-502)
* ``select_topk``, ``merge_topk``, ``exclusive_prefix_topk``,
  ``indexed_gqa_torch``, ``IndependentGQAMemory._write_kv`` / ``_sequence`` /
  ``_decode`` with the torch backend (modeling_yanchor.py:22-313)
* ``counter_uniform`` and ``sample_top_k_top_p_counter``
  (runtime/model/inference_kernels.py:24-88)
* ``torch_causal_conv1d_update`` and the causal ``nn.Conv1d`` of the GDN
  layer (modeling_yanchor.py:349-370)
* ``fixed_memory_physical_ring_decode_attention`` (runtime/model/
  inference_kernels.py:1881-1897)
* the torch statements of the fixed-memory decode loop's per-step
  bookkeeping (runtime/model/inference_kernels.py:1701-1717)
* ``reference_swa`` (modeling_yanchor.py:412-427)

on seeded inputs and writes the inputs and outputs as ``.npz`` files next to
this script.  The GPU box never needs the reference: tests only read the
``.npz`` files.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
import tempfile
import zipfile
from types import SimpleNamespace

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root):
    wheel = [f for f in os.listdir(os.path.join(root, 'wheels')) if f.startswith('transformers') and f.endswith('.whl')][0]
    scratch = tempfile.mkdtemp(prefix='yb_golden_whl_')
    zipfile.ZipFile(os.path.join(root, 'wheels', wheel)).extractall(scratch)
    sys.path[:0] = [scratch, root, os.path.join(root, 'runtime')]
    import torch  # noqa: F401
    from transformers.models.qwen3_5 import modeling_qwen3_5 as qwen
    import modeling_yanchor as my
    import model.inference_kernels as ik
    return qwen, my, ik


def gdn_fixtures(qwen, torch):
    F = torch.nn.functional
    out = {}
    # --- config-0 style, T=160 (two full chunks + a partial one), fp32 ---------
    g0 = torch.Generator().manual_seed(0)
    B, T, H, D = 2, 160, 2, 64
    q = torch.randn(B, T, H, D, generator=g0)
    k = torch.randn(B, T, H, D, generator=g0)
    v = torch.randn(B, T, H, D, generator=g0)
    g = F.logsigmoid(torch.randn(B, T, H, generator=g0))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g0))
    h0 = 0.02 * torch.randn(B, H, D, D, generator=g0)
    out.update(small_q=q, small_k=k, small_v=v, small_g=g, small_beta=beta, small_h0=h0)
    o, s = qwen.torch_chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=h0,
                                             output_final_state=True, use_qk_l2norm_in_kernel=True)
    out.update(small_chunk_o=o, small_chunk_s=s)
    o, s = qwen.torch_recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=h0,
                                                 output_final_state=True, use_qk_l2norm_in_kernel=True)
    out.update(small_rec_o=o, small_rec_s=s)
    # the exact config-0 recipe: pre-normalised q, k; zero initial state
    qn, kn = qwen.l2norm(q), qwen.l2norm(k)
    out.update(small_l2q_head=qn[:, :8])
    o, s = qwen.torch_chunk_gated_delta_rule(qn, kn, v, g, beta, chunk_size=64, initial_state=None,
                                             output_final_state=True)
    out.update(small_chunk0_o=o, small_chunk0_s=s)
    # --- grouped value heads (H=2, HV=4) and varlen packing ------------------
    g1 = torch.Generator().manual_seed(1)
    cu = [0, 37, 100, 165]
    Tt, Hk, HV, Dk = cu[-1], 2, 4, 32
    q = torch.randn(1, Tt, Hk, Dk, generator=g1)
    k = torch.randn(1, Tt, Hk, Dk, generator=g1)
    v = torch.randn(1, Tt, HV, Dk, generator=g1)
    g = F.logsigmoid(torch.randn(1, Tt, HV, generator=g1))
    beta = torch.sigmoid(torch.randn(1, Tt, HV, generator=g1))
    h0 = 0.02 * torch.randn(len(cu) - 1, HV, Dk, Dk, generator=g1)
    out.update(var_q=q, var_k=k, var_v=v, var_g=g, var_beta=beta, var_h0=h0, var_cu=torch.tensor(cu))
    for name, fn in (('chunk', qwen.torch_chunk_gated_delta_rule), ('rec', qwen.torch_recurrent_gated_delta_rule)):
        os_, ss = [], []
        for n in range(len(cu) - 1):
            sl = slice(cu[n], cu[n + 1])
            qq = q[:, sl].repeat_interleave(HV // Hk, dim=2)
            kk = k[:, sl].repeat_interleave(HV // Hk, dim=2)
            kw = dict(initial_state=h0[n:n + 1], output_final_state=True, use_qk_l2norm_in_kernel=True)
            if name == 'chunk':
                kw['chunk_size'] = 64
            o, s = fn(qq, kk, v[:, sl], g[:, sl], beta[:, sl], **kw)
            os_.append(o)
            ss.append(s)
        out[f'var_{name}_o'] = torch.cat(os_, 1)
        out[f'var_{name}_s'] = torch.cat(ss, 0)
    # --- gates and the gated RMSNorm epilogue --------------------------------
    g2 = torch.Generator().manual_seed(2)
    a = 3.0 * torch.randn(5, 3, 8, generator=g2)
    a[0, 0, :4] = torch.tensor([25.0, 21.0, 19.0, -30.0])     # both softplus branches
    b = torch.randn(5, 3, 8, generator=g2)
    A_log = torch.empty(8).uniform_(0, 16, generator=g2).log()
    dt_bias = torch.randn(8, generator=g2)
    beta_ref = b.sigmoid()
    g_ref = -A_log.float().exp() * F.softplus(a.float() + dt_bias)     # modeling_qwen3_5.py:500-502
    out.update(gate_a=a, gate_b=b, gate_A_log=A_log, gate_dt_bias=dt_bias, gate_g=g_ref, gate_beta=beta_ref)
    norm = qwen.Qwen3_5RMSNormGated(64, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(1.0 + 0.1 * torch.randn(64, generator=g2))
    x = torch.randn(12, 64, generator=g2)
    z = torch.randn(12, 64, generator=g2)
    with torch.no_grad():
        out.update(norm_x=x, norm_z=z, norm_w=norm.weight.detach().clone(), norm_out=norm(x, z))
    return out


def memory_fixtures(my, torch):
    out = {}
    g = torch.Generator().manual_seed(3)
    # --- select_topk / merge_topk with ties, -0.0 and invalid references ------
    n, cap = 24, 10
    scores = torch.randint(-3, 4, (4, 3, n), generator=g).float() * 0.5
    scores[0, 0, :3] = torch.tensor([0.0, -0.0, 0.0])
    positions = torch.stack([torch.randperm(100, generator=g)[:n] for _ in range(12)]).reshape(4, 3, n)
    refs = torch.arange(n).expand(4, 3, n).clone()
    refs[torch.rand(4, 3, n, generator=g) < 0.25] = -1
    scores = scores.masked_fill(refs < 0, -math.inf)
    sel = my.select_topk(scores, positions, refs, cap)
    out.update(sel_scores_in=scores, sel_pos_in=positions, sel_refs_in=refs,
               sel_scores=sel[0], sel_pos=sel[1], sel_refs=sel[2])
    sel = my.select_topk(scores, positions, refs, n + 4)      # capacity above n pads
    out.update(selpad_scores=sel[0], selpad_pos=sel[1], selpad_refs=sel[2])
    # --- exclusive prefix top-k over blocks ----------------------------------
    B, blocks, G, chunk, cap = 2, 5, 2, 8, 6
    ps = torch.randn(B, blocks, G, chunk, generator=g)
    pp = torch.arange(blocks * chunk).reshape(1, blocks, 1, chunk).expand(B, blocks, G, chunk).clone()
    pr = pp.clone()
    pr[:, -1, :, 5:] = -1
    ps = ps.masked_fill(pr < 0, -math.inf)
    pre = my.exclusive_prefix_topk(ps, pp, pr, cap)
    out.update(pre_scores_in=ps, pre_pos_in=pp, pre_refs_in=pr,
               pre_scores=pre[0], pre_pos=pre[1], pre_refs=pre[2])
    # --- select_topk edge cases: NaN scores (rank first, as torch's descending
    # sort puts them), invalid references with finite scores, int32 positions
    es = torch.randint(-2, 3, (5, 17), generator=g).float()
    es[0, [2, 9]] = float('nan')
    es[1, :4] = torch.tensor([-0.0, 0.0, float('inf'), float('-inf')])
    ep = torch.stack([torch.randperm(50, generator=g)[:17] for _ in range(5)]).int()
    er = torch.arange(17).expand(5, 17).clone()
    er[torch.rand(5, 17, generator=g) < 0.3] = -1          # invalid, but scores stay finite
    sel = my.select_topk(es, ep, er, 9)
    out.update(seledge_scores_in=es, seledge_pos_in=ep, seledge_refs_in=er,
               seledge_scores=sel[0], seledge_pos=sel[1], seledge_refs=sel[2])
    # --- exclusive prefix top-k: odd block count, chunk = capacity, ties -------
    B, blocks, G, chunk, cap = 2, 7, 3, 16, 16
    ps = (torch.randn(B, blocks, G, chunk, generator=g) * 4).round() / 4
    pp = torch.arange(blocks * chunk).reshape(1, blocks, 1, chunk).expand(B, blocks, G, chunk).clone() + 5
    pr = pp.clone()
    pr[1, -1, :, 9:] = -1
    ps = ps.masked_fill(pr < 0, -math.inf)
    pre = my.exclusive_prefix_topk(ps, pp, pr, cap)
    out.update(pre2_scores_in=ps, pre2_pos_in=pp, pre2_refs_in=pr,
               pre2_scores=pre[0], pre2_pos=pre[1], pre2_refs=pre[2])
    # --- prefill orchestration (_sequence): fresh state with a left-padded
    # mask, a continuation from that state, and the stateless form.  The
    # writer's k / v are recorded for every token (the writer is row-wise), so
    # a restatement can gather the rows the reference computes on demand.
    out.update(sequence_fixtures(my, torch, g))
    # --- indexed_gqa_torch (prefill read) ------------------------------------
    B, blocks, chunk, H, G, D, S, cap = 2, 3, 8, 4, 2, 32, 20, 6
    q = torch.randn(B, blocks, chunk, H, D, generator=g)
    kk = torch.randn(B, S, G, D, generator=g)
    vv = torch.randn(B, S, G, D, generator=g)
    rr = torch.randint(0, S, (B, blocks, G, cap), generator=g)
    rr[torch.rand(B, blocks, G, cap, generator=g) < 0.3] = -1
    rr[0, 0, 0] = -1                                            # a group with no anchors
    out.update(idx_q=q, idx_k=kk, idx_v=vv, idx_refs=rr, idx_out=my.indexed_gqa_torch(q, kk, vv, rr))
    # --- decode read + commit, many steps, torch backend ----------------------
    B, H, G, D, CAP, CHUNK, STEPS = 3, 4, 2, 32, 6, 8, 41
    cfg = SimpleNamespace(backend='torch', hidden_size=16, num_attention_heads=H, num_key_value_heads=G,
                          head_dim=D, rms_norm_eps=1e-6, initializer_range=0.02, fixed_memory_swa_window=64,
                          independent_memory=dict(capacity=CAP, max_commit_chunk=CHUNK, admission_rank=4,
                                                  writer_intermediate_size=8))
    mem = my.IndependentGQAMemory(cfg)
    state = my.IndependentMemoryState.empty(B, G, CAP, CHUNK, D, 'cpu', torch.float32)
    qs = torch.randn(STEPS, B, 1, H, D, generator=g)
    ks = torch.randn(STEPS, B, 1, G, D, generator=g)
    vs = torch.randn(STEPS, B, 1, G, D, generator=g)
    sc = torch.randint(-4, 5, (STEPS, B, 1, G), generator=g).float() * 0.25   # ties on purpose
    valid = torch.rand(STEPS, B, 1, generator=g) > 0.15
    reads = []
    snapshots = {}
    for t in range(STEPS):
        with torch.no_grad():
            r = mem._decode(qs[t], ks[t], vs[t], sc[t], valid[t], CHUNK, state)
        reads.append(r)
        if t in (7, 20):
            for f in ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values',
                      'pending_scores', 'count', 'total'):
                snapshots[f'dec_t{t}_{f}'] = getattr(state, f).clone()
    out.update(dec_q=qs, dec_k=ks, dec_v=vs, dec_scores=sc, dec_valid=valid, dec_reads=torch.stack(reads))
    out.update(snapshots)
    for f in ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values',
              'pending_scores', 'count', 'total'):
        out[f'dec_final_{f}'] = getattr(state, f).clone()
    return out


def sequence_fixtures(my, torch, g):
    B, H, G, D, CAP, CHUNK, ROT, HID = 3, 4, 2, 32, 6, 8, 8, 16
    cfg = SimpleNamespace(backend='torch', hidden_size=HID, num_attention_heads=H, num_key_value_heads=G,
                          head_dim=D, rms_norm_eps=1e-6, initializer_range=0.2, fixed_memory_swa_window=64,
                          independent_memory=dict(capacity=CAP, max_commit_chunk=CHUNK, admission_rank=4,
                                                  writer_intermediate_size=8))
    mem = my.IndependentGQAMemory(cfg)
    out = {}
    state = my.IndependentMemoryState.empty(B, G, CAP, CHUNK, D, 'cpu', torch.float32)
    fields = ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values', 'pending_scores',
              'count', 'total')
    calls = [('seq1', 29, True, True), ('seq2', 13, False, True), ('seq3', 21, False, False)]
    for name, T, masked, stateful in calls:
        u = torch.randn(B, T, HID, generator=g)
        query = torch.randn(B, T, H, D, generator=g)
        scores = (torch.randn(B, T, G, generator=g) * 2).round() / 2       # ties on purpose
        theta = torch.randn(B, T, ROT // 2, generator=g)
        pe = (torch.cat((theta.cos(), theta.cos()), -1), torch.cat((theta.sin(), theta.sin()), -1))
        valid = None
        if masked:
            valid = torch.ones(B, T, dtype=torch.bool)
            valid[1, :5] = False                                           # left padding
            valid[2, :T - 3] = False                                       # a short prompt
        with torch.no_grad():
            k_all, v_all = mem._write_kv(u.reshape(-1, HID), tuple(x.reshape(-1, ROT) for x in pe))
            o = mem._sequence(u, query, scores, pe, valid, CHUNK, state if stateful else None)
        out.update({f'{name}_q': query, f'{name}_scores': scores, f'{name}_o': o,
                    f'{name}_k': k_all.reshape(B, T, G, D), f'{name}_v': v_all.reshape(B, T, G, D)})
        if valid is not None:
            out[f'{name}_valid'] = valid
        if stateful:
            for f in fields:
                out[f'{name}_state_{f}'] = getattr(state, f).clone()
    return out


def conv_fixtures(my, torch):
    """Causal depthwise conv1d: the decode update through the reference's
    ``torch_causal_conv1d_update`` (modeling_yanchor.py:349-353), and
    prefill segments through an ``nn.Conv1d`` built as the reference layer
    builds it (modeling_yanchor.py:369-370) and applied as the qwen3_5
    forward applies it (modeling_qwen3_5.py:462-480): fresh, with a cached
    state prepended, and shorter than the kernel."""
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(11)
    B, C, KS = 3, 40, 4
    w = torch.randn(C, KS, generator=g) * 0.5
    out = {'conv_w': w}
    x = torch.randn(B, C, 1, generator=g)
    st = torch.randn(B, C, KS, generator=g)
    st_after = st.clone()
    y = my.torch_causal_conv1d_update(x, st_after, w, None, 'silu')
    out.update(conv_upd_x=x, conv_upd_state=st, conv_upd_y=y, conv_upd_state_after=st_after)
    layer = torch.nn.Conv1d(C, C, KS, groups=C, padding=KS - 1, bias=False)
    with torch.no_grad():
        layer.weight.copy_(w[:, None])
        for name, T, cached in (('conv_pre', 11, False), ('conv_prec', 9, True), ('conv_pres', 2, False)):
            xs = torch.randn(B, C, T, generator=g)
            mixed = torch.cat([st, xs], -1) if cached else xs
            new_state = F.pad(mixed, (KS - mixed.shape[-1], 0))
            ys = F.silu(layer(mixed)[:, :, :mixed.shape[-1]])
            if cached:
                ys = ys[:, :, -T:]
            out.update({f'{name}_x': xs, f'{name}_y': ys, f'{name}_state': new_state})
    out['conv_prec_state_in'] = st
    return out


def swa_fixtures(ik, torch):
    """The physical-ring decode attention (runtime/model/inference_kernels.py:
    1881-1897) through its reproducible (math SDPA) path: grouped-query, a
    validity mask with holes and a row with a single valid position."""
    g = torch.Generator().manual_seed(13)
    B, QH, KVH, W, D = 3, 8, 2, 24, 32
    q = torch.randn(B, 1, QH, D, generator=g)
    rk = torch.randn(B, KVH, W, D, generator=g)
    rv = torch.randn(B, KVH, W, D, generator=g)
    valid = torch.rand(B, W, generator=g) > 0.3
    valid[2] = False
    valid[2, 5] = True
    out = ik.fixed_memory_physical_ring_decode_attention(q, rk, rv, valid, reproducible=True)
    return {'swa_q': q, 'swa_k': rk, 'swa_v': rv, 'swa_valid': valid, 'swa_out': out}


def swa_prefill_fixtures(my, torch):
    """``reference_swa`` (modeling_yanchor.py:412-427): a plain causal window,
    left-padded rows through key validity, and a query block after a cached
    window (``query_start``), grouped-query."""
    g = torch.Generator().manual_seed(17)
    out = {}
    cases = [
        ('a', 2, 40, 40, 4, 1, 16, 16, 0, None),
        ('b', 3, 37, 37, 4, 2, 16, 50, 0, 'left'),
        ('c', 2, 20, 45, 8, 2, 16, 24, 25, 'holes'),
    ]
    for name, B, Tq, Tk, QH, KVH, D, window, qs, mask in cases:
        q = torch.randn(B, Tq, QH, D, generator=g)
        k = torch.randn(B, Tk, KVH, D, generator=g)
        v = torch.randn(B, Tk, KVH, D, generator=g)
        kv = None
        if mask == 'left':
            kv = torch.ones(B, Tk, dtype=torch.bool)
            kv[1, :5] = False
            kv[2, :36] = False
        elif mask == 'holes':
            kv = torch.rand(B, Tk, generator=g) > 0.25
            kv[:, qs:] |= torch.arange(Tq)[None, :] % 3 == 0
        o = my.reference_swa(q, k, v, window=window, key_valid=kv, query_start=qs)
        out.update({f'sp{name}_q': q, f'sp{name}_k': k, f'sp{name}_v': v, f'sp{name}_out': o,
                    f'sp{name}_meta': torch.tensor([window, qs])})
        if kv is not None:
            out[f'sp{name}_valid'] = kv
    return out


def sampling_fixtures(ik, torch):
    out = {}
    g = torch.Generator().manual_seed(4)
    ids = torch.cat([torch.arange(64), torch.tensor([2**31 - 1, 2**32 - 1, 2**40 + 5, -1, -7])])
    steps = torch.randint(0, 2**33, ids.shape, generator=g)
    out.update(cu_ids=ids, cu_steps=steps)
    for seed, stream in ((0, 0), (1234, 0), (2**32 + 99, 3)):
        out[f'cu_u_{seed}_{stream}'] = ik.counter_uniform(ids, steps, seed=seed, stream=stream)
    B, V = 16, 1000
    scores = torch.randn(B, V, generator=g) * 3.0
    attempt = torch.arange(B) * 7 + 3
    step = torch.randint(0, 10000, (B,), generator=g)
    out.update(samp_scores=scores, samp_attempt=attempt, samp_steps=step)
    # cases 6-8: top-k beyond 256 with and without top-p, and top-p over the whole vocabulary (top_k 0)
    cases = [(1.0, 1, 1.0), (1.0, 20, 0.95), (0.7, 20, 0.9), (1.3, 50, 1.0), (1.0, 5, 0.3), (0.8, 0, 1.0),
             (1.0, 300, 0.9), (0.9, 0, 0.8), (1.1, 600, 1.0)]
    for i, (temp, tk, tp) in enumerate(cases):
        out[f'samp_case{i}'] = torch.tensor([temp, tk, tp])
        out[f'samp_out{i}'] = ik.sample_top_k_top_p_counter(scores, attempt, step, seed=77, temperature=temp,
                                                             top_k=tk, top_p=tp)
    return out


def _decode_loop_update_block(ik):
    """The torch statements of the reference's per-step decode bookkeeping
    (runtime/model/inference_kernels.py:1700-1717): the ``else`` branch of the
    ``if`` that otherwise launches ``_update_fixed_decode_state_``.  Found in the
    module's own source by its syntax tree, compiled, and run as written."""
    import ast
    import inspect
    tree = ast.parse(inspect.getsource(ik))
    for node in ast.walk(tree):
        if isinstance(node, ast.If) and node.orelse and any(
                isinstance(c, ast.Call) and getattr(c.func, 'id', None) == '_update_fixed_decode_state_'
                for st in node.body for c in ast.walk(st)):
            mod = ast.Module(body=node.orelse, type_ignores=[])
            return compile(ast.fix_missing_locations(mod), ik.__file__, 'exec'), node.orelse[0].lineno
    raise RuntimeError('decode-loop update block not found')


def decode_state_fixtures(ik, torch):
    """Several decode steps of the bookkeeping block on a slot table with
    empty slots, finished rows, caps reached mid-run, two EOS ids and a row
    whose slot empties between steps."""
    code, line = _decode_loop_update_block(ik)
    g = torch.Generator().manual_seed(21)
    slots, total, max_new, vocab, pad = 11, 17, 9, 50, 0
    eos = (7, 3)
    st = {
        'storage': torch.full((total + slots, max_new + 1), pad, dtype=torch.int32),
        'dense_seen': torch.zeros(slots, vocab, dtype=torch.bool),
        'generated_lengths': torch.zeros(total + slots, dtype=torch.long),
        'finished_by_eos': torch.zeros(total + slots, dtype=torch.bool),
        'finished': torch.tensor([False] * 8 + [True, False, False]),
        'slot_rows': torch.tensor([0, 4, 2, 9, 11, 5, -1, 16, 3, 7, 1]),
        'sink_rows': total + torch.arange(slots),
        'slot_caps': torch.tensor([9, 3, 9, 5, 9, 2, 0, 9, 9, 4, 9]),
        'row_steps': torch.ones(slots, dtype=torch.long),
        'row_positions': torch.randint(100, 900, (slots,), generator=g),
        'decode_ids': torch.randint(0, vocab, (slots, 1), generator=g),
        'decode_useful_events': torch.zeros((), dtype=torch.long),
    }
    out = {'ds_init_' + k: v.clone() for k, v in st.items()}
    out['ds_meta'] = torch.tensor([max_new, pad, *eos, line])
    steps = 7
    tokens = torch.randint(0, vocab, (steps, slots, 1), generator=g)
    tokens[1, 2, 0], tokens[2, 0, 0], tokens[3, 7, 0] = 7, 3, 7    # EOS hits
    out['ds_tokens'] = tokens
    for t in range(steps):
        if t == 4:
            st['slot_rows'][3] = -1                                      # a slot emptied between steps
        ns = dict(st, torch=torch, next_token=tokens[t].clone(), max_new_tokens=max_new, pad_token_id=pad,
                  eos_token_ids=eos, prefill_context=None)
        exec(code, ns)
        for k in st:
            st[k] = ns[k]
        for k, v in st.items():
            out[f'ds_{t}_{k}'] = v.clone()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True)
    ap.add_argument('--only', nargs='*', help='fixture files to rewrite (default: all)')
    args = ap.parse_args()
    qwen, my, ik = _import_reference(os.path.abspath(args.reference))
    import torch
    torch.manual_seed(0)
    for name, fn in (('gdn', lambda: gdn_fixtures(qwen, torch)), ('memory', lambda: memory_fixtures(my, torch)),
                     ('sampling', lambda: sampling_fixtures(ik, torch)), ('conv', lambda: conv_fixtures(my, torch)),
                     ('swa', lambda: swa_fixtures(ik, torch)), ('decode_state', lambda: decode_state_fixtures(ik, torch)),
                     ('swa_prefill', lambda: swa_prefill_fixtures(my, torch))):
        if args.only and name not in args.only:
            continue
        data = {k: (v.detach().cpu().numpy() if hasattr(v, 'detach') else np.asarray(v)) for k, v in fn().items()}
        path = os.path.join(HERE, f'{name}.npz')
        np.savez_compressed(path, **data)
        print(path, sum(x.nbytes for x in data.values()), 'bytes raw')


if __name__ == '__main__':
    main()
