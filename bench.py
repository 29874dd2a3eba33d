"""Benchmark of the YANchor hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl yanchor_b200|reference]

One step = one decode step of the hot path at the YANchor-4B shape for the
batch on this GPU (weak scaling: every rank owns its own sequences):

  * 24 GDN layers: fused recurrent update (q/k L2 norm, gates from raw a / b,
    fp32 state 32 x 128 x 128 per sequence updated in place, gated RMSNorm
    epilogue) — ``fused_recurrent_gated_delta_rule``
  * 8 anchor-memory layers: decode read + commit (G=4, H=16, D=256,
    CAP=64, chunk=64) — ``committed_gqa`` then ``commit_decode``, in one
    launch (``memory_decode_step``)
  * greedy sampling over the 248,320-token vocabulary — ``greedy``

``value`` is whole-job decode tokens/s (N x batch / step time) with inputs
resident in HBM; the GDN state (3.2 GB per GPU at batch 64) is far larger than
L2, so no L2 flush is needed between steps.  ``e2e`` repeats the step with
the step's activations copied from pinned host memory before it and the
sampled token ids copied back after it; two independent request groups take
turns so that one group's copies overlap the other group's step (the
one-group, copy-then-step figure is reported beside it as ``serial_*``).
``prefill`` reports config 1 (chunked prefill B=8, T=8192, H=HV=32,
K=V=128, plus the anchor prefill of one memory layer) on rank 0.  ``--impl reference`` times the reference algorithm's CPU
restatement (the numpy oracle) on the host cores instead.

The step runs as a captured CUDA graph (the reference's decode loop replays a
graph of the whole model forward too).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = 'decode tok/s/GPU at B=64, 32K gen; chunked-prefill tok/s; % of roofline'

# YANchor-4B hot-path shape (configuration_yanchor.py over Qwen3_5TextConfig
# defaults: 32 layers, every 4th is SWA + anchor memory)
L_GDN, L_MEM = 24, 8
H_K, H_V, DK, DV = 16, 32, 128, 128
CONV_C, CONV_KS = 2 * H_K * DK + H_V * DV, 4     # the short convolution over the fused q/k/v projection
MEM_G, MEM_H, MEM_D, MEM_CAP, MEM_CHUNK = 4, 16, 256, 64, 64
SW_QH, SW_KVH, SW_W, SW_D = 16, 4, 1024, 256       # the SWA layers: window 1024 (modeling_yanchor.py:451)
VOCAB = 248320
GEN_TOKENS = 32768                                # config 3: 32K generated tokens per sequence
PAD_ID, EOS_IDS = 248044, ()                      # fixed-length generation: no end ids (runtime/inference.py:94)


def peaks():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p['hbm_gbs']), float(p['bf16_tflops']), float(p.get('bf16_tflops_sustained', p['bf16_tflops'])), \
            'measured'
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0, 1400.0, 'fallback'


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons through NVML from a
    background thread every few milliseconds while the timed region runs.
    Reading clocks changes nothing on the GPU."""
    REASONS = (('hw_slowdown', 'nvmlClocksEventReasonHwSlowdown'),
               ('hw_thermal_slowdown', 'nvmlClocksEventReasonHwThermalSlowdown'),
               ('sw_thermal_slowdown', 'nvmlClocksEventReasonSwThermalSlowdown'),
               ('sw_power_cap', 'nvmlClocksEventReasonSwPowerCap'),
               ('hw_power_brake', 'nvmlClocksEventReasonHwPowerBrakeSlowdown'))

    def __init__(self, index, interval_s=0.002):
        self.index = index
        self.interval = interval_s
        self.samples = []
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            visible = os.environ.get('CUDA_VISIBLE_DEVICES')
            idx = self.index
            if visible:
                ids = [x for x in visible.split(',') if x.strip()]
                if ids and ids[self.index].strip().isdigit():
                    idx = int(ids[self.index])
            self.nv = nv
            self.handle = nv.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception as e:  # noqa: BLE001
            self.error = repr(e)
            self.nv = None
        return self

    def _run(self):
        nv = self.nv
        getr = getattr(nv, 'nvmlDeviceGetCurrentClocksEventReasons', None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM),
                                     int(getr(self.handle))))
            except Exception as e:  # noqa: BLE001
                self.error = repr(e)
                return
            time.sleep(self.interval)

    def __exit__(self, *exc):
        self._stop.set()
        if self.nv is not None:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': self.max_mhz, 'reasons': ['unsampled'], 'samples': 0,
                    'error': self.error}
        reasons = set()
        for _, bits in self.samples:
            for name, const in self.REASONS:
                if bits & int(getattr(self.nv, const, 0)):
                    reasons.add(name)
        return {'sm_mhz': statistics.median(m for m, _ in self.samples), 'sm_max_mhz': self.max_mhz,
                'reasons': sorted(reasons), 'samples': len(self.samples), 'source': 'NVML, 2 ms polling'}


# ----------------------------------------------------------------- GPU arm --
def build_decode(torch, yb, B, device, n_inputs=4, seed=0, state_dtype=None):
    """Allocate the model-shaped state and `n_inputs` sets of step inputs."""
    gen = torch.Generator(device=device).manual_seed(seed)
    bf = torch.bfloat16

    def rnd(*shape, dtype=bf, scale=1.0):
        return (torch.randn(*shape, generator=gen, device=device) * scale).to(dtype)

    layers = []
    for _ in range(L_GDN):
        layers.append(dict(state=(0.02 * torch.randn(B, H_V, DK, DV, generator=gen, device=device)).to(
                               state_dtype or torch.float32),
                           conv_state=rnd(B, CONV_C, CONV_KS),
                           conv_w=torch.randn(CONV_C, CONV_KS, generator=gen, device=device) * 0.5,
                           A_log=torch.empty(H_V, device=device).uniform_(1, 16, generator=gen).log(),
                           dt_bias=torch.ones(H_V, device=device),
                           norm_w=rnd(DV, scale=0.1) + 1.0))
    mems = [yb.MemoryState.empty(B, MEM_G, MEM_CAP, MEM_CHUNK, MEM_D, device, bf) for _ in range(L_MEM)]
    inputs = []
    for _ in range(n_inputs):
        inputs.append(dict(
            mixed=rnd(L_GDN, B, 1, CONV_C),
            z=rnd(L_GDN, B, 1, H_V, DV), a=rnd(L_GDN, B, 1, H_V), b=rnd(L_GDN, B, 1, H_V),
            mq=rnd(L_MEM, B, 1, MEM_H, MEM_D), mk=rnd(L_MEM, B, 1, MEM_G, MEM_D), mv=rnd(L_MEM, B, 1, MEM_G, MEM_D),
            ms=rnd(L_MEM, B, 1, MEM_G, dtype=torch.float32), logits=rnd(B, VOCAB, scale=3.0)))
    active = torch.ones(B, dtype=torch.bool, device=device)
    ws = torch.empty(yb.sampling.workspace_bytes(B, VOCAB, 1), dtype=torch.uint8, device=device)
    return layers, mems, inputs, active, ws, build_table(torch, B, device)


def build_table(torch, B, device):
    """The decode loop's slot table (runtime/model/inference_kernels.py:1451-1475
    shapes): one slot per sequence, token storage for the 32K-token run,
    the seen-token table over the vocabulary, sink rows for idle slots."""
    i64 = torch.int64
    return dict(storage=torch.zeros((2 * B, GEN_TOKENS + 1), dtype=torch.int32, device=device),
                dense_seen=torch.zeros((B, VOCAB), dtype=torch.bool, device=device),
                generated_lengths=torch.zeros(2 * B, dtype=i64, device=device),
                finished_by_eos=torch.zeros(2 * B, dtype=torch.bool, device=device),
                finished=torch.zeros(B, dtype=torch.bool, device=device),
                slot_rows=torch.arange(B, device=device), sink_rows=B + torch.arange(B, device=device),
                slot_caps=torch.full((B,), GEN_TOKENS, dtype=i64, device=device),
                row_steps=torch.ones(B, dtype=i64, device=device),
                row_positions=torch.full((B,), 1024, dtype=i64, device=device),
                decode_ids=torch.zeros((B, 1), dtype=i64, device=device),
                decode_useful_events=torch.zeros((), dtype=i64, device=device))


TABLE_FIELDS = ('storage', 'dense_seen', 'generated_lengths', 'finished_by_eos', 'finished', 'slot_rows', 'sink_rows',
                'slot_caps', 'row_steps', 'row_positions', 'decode_ids', 'decode_useful_events')


def conv_qkv(yb, L, mixed):
    """The layer's short convolution (in place on its conv state), then q, k, v
    as views of its output, as the reference layer splits them."""
    mix = yb.causal_conv1d_update(mixed.transpose(1, 2), L['conv_state'], L['conv_w'], None, 'silu').transpose(1, 2)
    q = mix[..., :H_K * DK].unflatten(-1, (H_K, DK))
    k = mix[..., H_K * DK:2 * H_K * DK].unflatten(-1, (H_K, DK))
    v = mix[..., 2 * H_K * DK:].unflatten(-1, (H_V, DV))
    return q, k, v


def gdn_layer(yb, L, x, i):
    """One GDN layer's decode core in one launch: conv update, gates, L2 norm,
    recurrence (state in place), gated RMSNorm."""
    return yb.fused_gdn_decode(x['mixed'][i], x['z'][i], x['a'][i], x['b'][i], L['conv_state'], L['conv_w'], None,
                               L['state'], L['A_log'], L['dt_bias'], L['norm_w'], num_k_heads=H_K)


def decode_step(yb, layers, mems, x, active, ws, table, fused=False):
    """One decode step of the hot path, then the decode loop's bookkeeping
    of the sampled token; returns the sampled token ids."""
    for i, L in enumerate(layers):
        if fused:
            gdn_layer(yb, L, x, i)
            continue
        q, k, v = conv_qkv(yb, L, x['mixed'][i])
        yb.fused_recurrent_gated_delta_rule(
            q, k, v, g=x['a'][i], beta=x['b'][i], initial_state=L['state'],
            output_final_state=True, use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=L['A_log'],
            dt_bias=L['dt_bias'], use_beta_sigmoid_in_kernel=True, z=x['z'][i], norm_weight=L['norm_w'],
            inplace=True)
    for i, st in enumerate(mems):   # committed_gqa then commit_decode, in one launch
        yb.memory_decode_step(x['mq'][i], x['mk'][i], x['mv'][i], x['ms'][i], active, MEM_CHUNK, st)
    tok = yb.greedy(x['logits'], workspace=ws)
    yb.update_fixed_decode_state_(tok, *(table[k] for k in TABLE_FIELDS), maximum_new_tokens=GEN_TOKENS,
                                  pad_token_id=PAD_ID, eos_token_ids=EOS_IDS)
    return tok


# conv + recurrence per GDN layer, read + commit (one launch) per memory layer, greedy (2), bookkeeping (1)
LAUNCHES_PER_STEP = 2 * L_GDN + L_MEM + 3


def gdn_bytes_per_launch(B, state_bytes=4):
    """Algorithmic HBM bytes of one recurrence launch (after the conv)."""
    state = B * H_V * DK * DV * state_bytes * 2            # state read + write (fp32, or a 16-bit storage)
    acts = B * (2 * H_K * DK + 3 * H_V * DV) * 2 + B * H_V * 2 * 2   # q, k, v, z, o (bf16) + a, b
    return state + acts


def time_recurrences(torch, yb, layers, x, stream, reps=5):
    """Mean time of one recurrence launch, measured as in the step: one graph
    runs the recurrence over every layer's own state and inputs in turn, so
    the 24 states (3.2 GB fp32, 1.6 GB 16-bit) stream from HBM and no launch
    finds its predecessor's state in L2."""
    qkv = [conv_qkv(yb, L, x['mixed'][i]) for i, L in enumerate(layers)]

    def all_layers():
        for i, L in enumerate(layers):
            q, k, v = qkv[i]
            yb.fused_recurrent_gated_delta_rule(
                q, k, v, g=x['a'][i], beta=x['b'][i], initial_state=L['state'], output_final_state=True,
                use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=L['A_log'], dt_bias=L['dt_bias'],
                use_beta_sigmoid_in_kernel=True, z=x['z'][i], norm_weight=L['norm_w'], inplace=True)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        all_layers()
    g.replay()
    ms = time_events(torch, g.replay, reps, stream) / len(layers)
    del g
    return ms


def time_events(torch, fn, iters, stream):
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(iters):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


def decode_config(B, world):
    """The workload both arms report (the reference arm runs the same step on the host)."""
    return {
        'workload': 'decode hot path (config 3 shape): 24 GDN layers (short conv update, then the recurrence with '
                    'gates, L2 norm and gated RMSNorm) + 8 anchor-memory layers + greedy sampler, one token per '
                    'sequence per step, CUDA-graph replay',
        'conv': {'channels': CONV_C, 'kernel': CONV_KS, 'state': 'bf16, in place'},
        'batch_per_gpu': B, 'global_batch': B * world,
        'gdn': {'layers': L_GDN, 'H': H_K, 'HV': H_V, 'K': DK, 'V': DV, 'state': 'fp32, in place'},
        'memory': {'layers': L_MEM, 'G': MEM_G, 'H': MEM_H, 'D': MEM_D, 'CAP': MEM_CAP, 'chunk': MEM_CHUNK,
                   'steady_state': f'{MEM_CHUNK + 2} untimed steps fill every bank and pending chunk, then row b '
                                   f'starts at pending count b % {MEM_CHUNK}: each timed step merges 1 in '
                                   f'{MEM_CHUNK} rows of every memory layer'},
        'vocab': VOCAB, 'parallelism': f'sequence-sharded x{world}, no collective',
        'l2': 'no flush: 3.2 GB of GDN state per GPU streams through each step (> 126 MB L2)'}


def fill_and_stagger(torch, yb, layers, mems, inputs, active, ws, table):
    """Bring the anchor memory to a steady state before anything is timed:
    MEM_CHUNK + 2 eager steps fill every pending chunk and commit a bank,
    then row b's pending count is set to b % MEM_CHUNK (its pending slots
    hold the entries pushed by those steps).  From then on every step
    merges the rows whose chunk fills: 1 in MEM_CHUNK of the rows per step,
    as rows at different prompt lengths do."""
    for w in range(MEM_CHUNK + 2):
        decode_step(yb, layers, mems, inputs[w % len(inputs)], active, ws, table)
    B = active.shape[0]
    counts = torch.arange(B, device=active.device, dtype=torch.int64) % MEM_CHUNK
    for st in mems:
        st.count.copy_(counts)
    torch.cuda.synchronize()


def capture_steps(torch, yb, layers, mems, inputs, active, ws, table, device, extra=None):
    """One CUDA graph of the decode step per input set (plus `extra()` after
    the step, if given)."""
    stream = torch.cuda.current_stream(device)
    graphs, outs = [], []
    for x in inputs:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device)
        s.wait_stream(stream)
        with torch.cuda.stream(s):
            decode_step(yb, layers, mems, x, active, ws, table)   # pre-capture run on the side stream
            if extra is not None:
                extra()
        stream.wait_stream(s)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            outs.append(decode_step(yb, layers, mems, x, active, ws, table))
            if extra is not None:
                extra()
        graphs.append(g)
    return graphs, outs


def lockstep_merge_ms(torch, mems, graphs, stream, reps=3):
    """Time of one step in which every row of every memory layer merges its
    full pending chunk into its bank (counts set to MEM_CHUNK - 1 before
    each timed replay)."""
    total = 0.0
    for r in range(reps):
        for st in mems:
            st.count.fill_(MEM_CHUNK - 1)
        torch.cuda.synchronize()
        total += time_events(torch, graphs[r % len(graphs)].replay, 1, stream)
    return total / reps


def step_bytes(B, state_bytes=4):
    """Algorithmic HBM bytes of one decode step: per GDN layer the conv state
    read + write and the recurrence's bytes; per memory layer the bank read
    (2 CAP D 2 B per group), the push and, averaged over the chunk, the
    merge's bank rewrite; the logits once."""
    conv = B * CONV_C * CONV_KS * 2 * 2 + B * CONV_C * 2 * 2
    mem = B * MEM_G * (2 * MEM_CAP * MEM_D * 2 + 2 * MEM_D * 2 + 2 * MEM_CAP * MEM_D * 2 // MEM_CHUNK) \
        + B * MEM_H * MEM_D * 2 * 2
    return L_GDN * (conv + gdn_bytes_per_launch(B, state_bytes)) + L_MEM * mem + B * VOCAB * 2


def run_gpu(args, rank, world, local_rank, dist):
    import torch
    import yanchor_b200 as yb
    from yanchor_b200 import shard
    device = torch.device('cuda', local_rank)
    torch.cuda.set_device(device)
    B = args.batch
    layers, mems, inputs, active, ws, table = build_decode(torch, yb, B, device, seed=1234 + rank)
    stream = torch.cuda.current_stream(device)

    # memory in steady state (filled banks, staggered pending counts), then
    # eager warm-up (also loads the library and sets kernel attributes)
    fill_and_stagger(torch, yb, layers, mems, inputs, active, ws, table)
    for w in range(max(args.warmup, 3)):
        decode_step(yb, layers, mems, inputs[w % len(inputs)], active, ws, table)
    torch.cuda.synchronize()
    graphs, outs = capture_steps(torch, yb, layers, mems, inputs, active, ws, table, device)
    for w in range(args.warmup):
        graphs[w % len(graphs)].replay()
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident timed region ----
    barrier()
    with ClockSampler(local_rank) as clocks:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(args.steps):
            graphs[i % len(graphs)].replay()
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / args.steps
    if dist is not None:
        ms = shard.max_over_ranks(ms, device=device)
    value = world * B / (ms / 1e3)
    merge_ms = lockstep_merge_ms(torch, mems, graphs, stream)
    for st in mems:                                  # back to the staggered counts
        st.count.copy_(torch.arange(B, device=device, dtype=torch.int64) % MEM_CHUNK)
    torch.cuda.synchronize()

    # ---- dominant kernel alone: the recurrence, CUDA events on its stream ----
    gdn_ms = time_recurrences(torch, yb, layers, inputs[0], stream)
    hbm, tf_burst, tf_sust, peak_kind = peaks()
    gbytes = gdn_bytes_per_launch(B)
    achieved = gbytes / (gdn_ms / 1e3) / 1e9

    # ---- end to end: pinned host inputs -> step -> token ids back to host ----
    # Each request group's step inputs live in one device buffer (each tensor a view at a 256-byte
    # aligned offset) with a pinned host twin, so a step's inputs come in as one copy; the group's
    # graph is captured on those views.
    def flat_group(x):
        offs, off = {}, 0
        for k_, t in x.items():
            offs[k_] = off
            off += (t.numel() * t.element_size() + 255) // 256 * 256
        dev_buf = torch.empty(off, dtype=torch.uint8, device=device)
        views = {k_: dev_buf[offs[k_]:offs[k_] + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                 for k_, t in x.items()}
        for k_, t in x.items():
            views[k_].copy_(t)
        return dev_buf, views, dev_buf.cpu().pin_memory()

    def group_graph(layers_, mems_, x, ws_, table_):
        g_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_):
            o_ = decode_step(yb, layers_, mems_, x, active, ws_, table_)
        return g_, o_

    dev_a, views_a, host_a = flat_group(inputs[0])
    g_a, out_a = group_graph(layers, mems, views_a, ws, table)
    host_out = torch.empty((B, 1), dtype=torch.int64).pin_memory()
    h2d = host_a.numel()
    d2h = host_out.numel() * host_out.element_size()

    def e2e_step():
        dev_a.copy_(host_a, non_blocking=True)
        g_a.replay()
        host_out.copy_(out_a, non_blocking=True)
    for _ in range(2):
        e2e_step()
    barrier()
    e2e_serial_ms = time_events(torch, e2e_step, max(3, args.steps // 4), stream)

    # Pipelined: two independent request groups of B sequences (each with its
    # own state and graph) take turns; while one group's step runs, the other
    # group's inputs for its next step come in on a copy stream.  Every step
    # still copies its full inputs in and its token ids out inside the timed
    # region; no step's inputs depend on the other group.
    layers_b, mems_b, inputs_b, _, ws_b, table_b = build_decode(torch, yb, B, device, n_inputs=1, seed=4321 + rank)
    fill_and_stagger(torch, yb, layers_b, mems_b, inputs_b, active, ws_b, table_b)
    dev_b, views_b, host_b = flat_group(inputs_b[0])
    g_b, out_b = group_graph(layers_b, mems_b, views_b, ws_b, table_b)
    host_out_b = torch.empty((B, 1), dtype=torch.int64).pin_memory()
    groups = [(dev_a, g_a, out_a, host_a, host_out), (dev_b, g_b, out_b, host_b, host_out_b)]
    copy_stream = torch.cuda.Stream(device)
    copied = [torch.cuda.Event() for _ in groups]
    done = [torch.cuda.Event() for _ in groups]

    def e2e_run(n):
        for i in range(n):
            dbuf, g_, o, hin, hout = groups[i % 2]
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(done[i % 2])      # this group's previous step has read its inputs
                dbuf.copy_(hin, non_blocking=True)
                copied[i % 2].record(copy_stream)
            stream.wait_event(copied[i % 2])
            g_.replay()
            hout.copy_(o, non_blocking=True)
            done[i % 2].record(stream)
    e2e_run(4)
    barrier()
    n_e2e = max(4, args.steps // 2) // 2 * 2
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    copy_stream.wait_event(e0)
    e2e_run(n_e2e)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / n_e2e
    del g_a, g_b

    # ---- the host link alone: the same pinned copies with no step ----
    def h2d_only():
        dev_a.copy_(host_a, non_blocking=True)
    h2d_only()
    barrier()
    h2d_ms = time_events(torch, h2d_only, 5, stream)
    if dist is not None:
        e2e_ms = shard.max_over_ranks(e2e_ms, device=device)
        e2e_serial_ms = shard.max_over_ranks(e2e_serial_ms, device=device)
        h2d_ms = shard.max_over_ranks(h2d_ms, device=device)

    # ---- the reference's opt-in fp16 recurrent-state storage (install_inference(fp16_state=True)) ----
    layers16, mems16, inputs16, _, ws16, table16 = build_decode(torch, yb, B, device, n_inputs=1, seed=99 + rank,
                                                       state_dtype=torch.float16)
    fill_and_stagger(torch, yb, layers16, mems16, inputs16, active, ws16, table16)
    g16 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g16):
        decode_step(yb, layers16, mems16, inputs16[0], active, ws16, table16)
    for _ in range(3):
        g16.replay()
    ms16 = time_events(torch, g16.replay, max(3, args.steps // 2), stream)
    gdn16_ms = time_recurrences(torch, yb, layers16, inputs16[0], stream)
    gbytes16 = gdn_bytes_per_launch(B, state_bytes=2)
    del g16
    if dist is not None:
        ms16 = shard.max_over_ranks(ms16, device=device)

    # ---- sliding-window attention decode over the physical ring (the 8 SWA layers, an (f) row) ----
    bf = torch.bfloat16
    rings = [(torch.randn(B, SW_KVH, SW_W, SW_D, device=device).to(bf),
              torch.randn(B, SW_KVH, SW_W, SW_D, device=device).to(bf),
              torch.ones(B, SW_W, device=device, dtype=torch.bool),
              torch.zeros((), device=device, dtype=torch.int64)) for _ in range(L_MEM)]
    swq = torch.randn(L_MEM, B, 1, SW_QH, SW_D, device=device).to(bf)
    swk = torch.randn(L_MEM, B, SW_KVH, 1, SW_D, device=device).to(bf)
    sw_ws = torch.empty(yb.swa.workspace_bytes(B, SW_KVH, SW_QH, SW_W, SW_D), device=device, dtype=torch.uint8)

    def swa_layers():
        for i, (rk, rv, rval, ridx) in enumerate(rings):
            yb.physical_ring_update_(rk, rv, rval, ridx, swk[i], swk[i], active[:, None])
            yb.physical_ring_decode_attention(swq[i], rk, rv, rval, workspace=sw_ws)
    swa_layers()
    torch.cuda.synchronize()
    gsw = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gsw):
        swa_layers()
    gsw.replay()
    swa_ms = time_events(torch, gsw.replay, 20, stream) / L_MEM
    swa_bytes = B * SW_KVH * SW_W * SW_D * 2 * 2 + B * SW_QH * SW_D * 2 * 2
    del gsw
    # the whole decode step with the 8 SWA layers in it (ring write + attention after the hot path)
    gfull, _ = capture_steps(torch, yb, layers, mems, inputs[:1], active, ws, table, device, extra=swa_layers)
    for _ in range(3):
        gfull[0].replay()
    full_ms = time_events(torch, gfull[0].replay, max(5, args.steps // 2), stream)
    del gfull, rings
    if dist is not None:
        full_ms = shard.max_over_ranks(full_ms, device=device)

    result = {
        'metric': METRIC, 'value': round(value, 1), 'unit': 'tok/s', 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': round(ms, 4), 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'fp32 state, bf16 activations', 'data': 'synthetic (random init, seeded)',
        'config': decode_config(B, world),
        'roofline': {'bound': 'hbm', 'kernel': 'gdn_recurrent_sst_kernel', 'achieved': round(achieved, 1),
                     'peak': hbm, 'unit': 'GB/s', 'frac': round(achieved / hbm, 4), 'peak_kind': peak_kind,
                     'bytes_per_launch': gbytes, 'launch_ms': round(gdn_ms, 5), 'traffic': traffic_per_launch()},
        'step': {'bytes': step_bytes(B), 'achieved_gbs': round(step_bytes(B) / (ms / 1e3) / 1e9, 1),
                 'frac_of_hbm': round(step_bytes(B) / (ms / 1e3) / 1e9 / hbm, 4),
                 'lockstep_merge_ms': round(merge_ms, 4),
                 'how': 'algorithmic bytes of the whole step (conv, GDN state and activations, memory banks, '
                        'logits) over its CUDA-event time; lockstep_merge_ms: one step in which every row of '
                        'every memory layer merges its pending chunk'},
        'e2e': {'value': round(world * B / (e2e_ms / 1e3), 1), 'unit': 'tok/s', 'h2d_bytes_per_step': h2d,
                'd2h_bytes_per_step': d2h, 'ms_per_step': round(e2e_ms, 4),
                'h2d_gbs_per_rank': round(h2d / (e2e_ms / 1e3) / 1e9, 2),
                'h2d_gbs_aggregate': round(world * h2d / (e2e_ms / 1e3) / 1e9, 2),
                'h2d_only_ms': round(h2d_ms, 4), 'h2d_only_gbs_per_rank': round(h2d / (h2d_ms / 1e3) / 1e9, 2),
                'h2d_only_gbs_aggregate': round(world * h2d / (h2d_ms / 1e3) / 1e9, 2),
                'serial_ms_per_step': round(e2e_serial_ms, 4),
                'serial_value': round(world * B / (e2e_serial_ms / 1e3), 1),
                'how': 'two independent request groups of B sequences alternate; each step copies its pinned host '
                       'activations + logits in (one copy: the inputs are views of one buffer) on a copy stream '
                       '(overlapping the other group\'s step), replays '
                       'its graph and copies its token ids out; serial_*: one group, copy then step, one stream; '
                       'CUDA events on the compute stream'},
        'decode_fp16_state': {
            'value': round(world * B / (ms16 / 1e3), 1), 'unit': 'tok/s', 'ms_per_step': round(ms16, 4),
            'how': 'the same step with the GDN state stored as fp16 (the reference\'s opt-in fp16_non_anchor '
                   'storage): widened to fp32 per step, rounded to nearest on store',
            'gdn_kernel': {'achieved': round(gbytes16 / (gdn16_ms / 1e3) / 1e9, 1), 'peak': hbm, 'unit': 'GB/s',
                           'frac': round(gbytes16 / (gdn16_ms / 1e3) / 1e9 / hbm, 4), 'bytes_per_launch': gbytes16,
                           'launch_ms': round(gdn16_ms, 5)}},
        'swa_decode': {'layer_ms': round(swa_ms, 5), 'how': 'ring write + attention over W=1024 positions, '
                       '16 query heads over 4 KV heads, D=256, B per GPU, CUDA graph over 8 layers',
                       'achieved_gbs': round(swa_bytes / (swa_ms / 1e3) / 1e9, 1), 'peak': hbm,
                       'frac': round(swa_bytes / (swa_ms / 1e3) / 1e9 / hbm, 4), 'bytes_per_layer': swa_bytes},
        'decode_with_swa': {'value': round(world * B / (full_ms / 1e3), 1), 'unit': 'tok/s',
                            'ms_per_step': round(full_ms, 4),
                            'how': 'the same step with the 8 SWA layers (ring write + attention over W=1024) in '
                                   'its graph'},
        'gpu_launches': LAUNCHES_PER_STEP * args.steps,
        'clocks': clocks.summary(),
    }
    return result, (layers, mems, inputs)


def run_batch_decode(torch, yb, B, device, steps, warmup, hbm, seed):
    """The decode step at another batch (config 2: B=256), memory in steady
    state; returns its rate, the recurrence's HBM rate and the whole step's."""
    layers, mems, inputs, active, ws, table = build_decode(torch, yb, B, device, n_inputs=2, seed=seed)
    fill_and_stagger(torch, yb, layers, mems, inputs, active, ws, table)
    graphs, _ = capture_steps(torch, yb, layers, mems, inputs, active, ws, table, device)
    stream = torch.cuda.current_stream(device)
    for w in range(warmup):
        graphs[w % 2].replay()
    torch.cuda.synchronize()
    turn = [0]

    def replay():
        graphs[turn[0] % 2].replay()
        turn[0] += 1
    ms = time_events(torch, replay, steps, stream)
    gdn_ms = time_recurrences(torch, yb, layers, inputs[0], stream)
    gbytes = gdn_bytes_per_launch(B)
    del graphs, layers, mems, inputs, table
    torch.cuda.empty_cache()
    return {'batch': B, 'value': round(B / (ms / 1e3), 1), 'unit': 'tok/s', 'ms_per_step': round(ms, 4),
            'steps': steps,
            'step_gbs': round(step_bytes(B) / (ms / 1e3) / 1e9, 1), 'step_bytes': step_bytes(B),
            'gdn_kernel': {'achieved': round(gbytes / (gdn_ms / 1e3) / 1e9, 1), 'peak': hbm, 'unit': 'GB/s',
                           'frac': round(gbytes / (gdn_ms / 1e3) / 1e9 / hbm, 4), 'bytes_per_launch': gbytes,
                           'launch_ms': round(gdn_ms, 5)},
            'how': 'config 2: the decode step (24 GDN + 8 memory layers + greedy + bookkeeping) at B=256, '
                   'fp32 state 12.9 GB, memory in steady state, CUDA-graph replay, CUDA events; the GDN kernel '
                   'timed over the 24 layers\' own states'}


SERVE_REQUESTS, SERVE_MIN_LEN, SERVE_MAX_LEN = 512, 512, 16384
SERVE_GROUP_TOKENS = 1 << 19        # packed prompt tokens per prefill launch


def serve_lengths():
    """Config 4's prompt lengths: uniform over [512, 16384], seeded (the same on every rank)."""
    return np.random.default_rng(2024).integers(SERVE_MIN_LEN, SERVE_MAX_LEN + 1, SERVE_REQUESTS)


def run_serve(torch, yb, args, rank, world, device, dist):
    """Config 4 on this rank's share of the 512 requests (split by prompt
    length with shard.shard_requests, no collective on the data path):

    * prefill: the prompts packed by cu_seqlens in groups of at most
      SERVE_GROUP_TOKENS tokens, longest first; per group the chunked GDN
      prefill of all 24 layers (varlen, final states into the decode pool)
      and the anchor prefill of all 8 memory layers (the group left-padded to
      its longest prompt, states into the pool); the short convolution's
      prefill is not packed-varlen here and is left out;
    * decode: all of the rank's requests as one batch, starting from the
      states the prefill left (GDN states, banks, pending chunks and counts),
      `steps` timed steps of the CUDA-graph step.

    Times are CUDA events, max over ranks.  The 32K-token generation is
    reported as a projection: prefill time + 32768 x the measured step."""
    from yanchor_b200 import shard
    bf = torch.bfloat16
    lengths = serve_lengths()
    owned = shard.shard_requests(lengths, world)[rank]
    own = np.array(sorted(owned, key=lambda i: (-int(lengths[i]), i)), dtype=np.int64)   # pool row order
    own_len = lengths[own].astype(np.int64)
    groups, cur, tok = [], [], 0
    for r, n in enumerate(own_len):
        if cur and tok + n > SERVE_GROUP_TOKENS:
            groups.append(cur)
            cur, tok = [], 0
        cur.append(r)
        tok += int(n)
    groups.append(cur)
    Bd = len(own)
    layers, mems, inputs, active, ws, table = build_decode(torch, yb, Bd, device, n_inputs=1, seed=555 + rank)
    gen = torch.Generator(device=device).manual_seed(777 + rank)
    stream = torch.cuda.current_stream(device)

    def rnd(*shape, dtype=bf):
        return torch.randn(*shape, generator=gen, device=device).to(dtype)
    A_log = torch.empty(H_V, device=device).uniform_(1, 16, generator=gen).log()
    dt_bias = torch.ones(H_V, device=device)
    prefill_ms = 0.0
    for grp in groups:
        r0, r1 = grp[0], grp[-1] + 1
        lens = own_len[r0:r1]
        T = int(lens.sum())
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), device=device, dtype=torch.int64)
        q, k = rnd(1, T, H_K, DK), rnd(1, T, H_K, DK)
        v = rnd(1, T, H_V, DV)
        a, b_ = rnd(1, T, H_V, dtype=torch.float32), rnd(1, T, H_V)
        Tm = int(lens.max())
        valid = torch.arange(Tm, device=device)[None, :] >= torch.tensor(Tm - lens, device=device)[:, None]
        mq = rnd(r1 - r0, Tm, MEM_H, MEM_D)
        msc = (torch.randn(r1 - r0, Tm, MEM_G, generator=gen, device=device) * 2).round() / 2
        wk, wv = rnd((r1 - r0) * Tm, MEM_G, MEM_D), rnd((r1 - r0) * Tm, MEM_G, MEM_D)

        def writer(bi, ti):
            rows = bi * Tm + ti
            return wk.index_select(0, rows), wv.index_select(0, rows)

        def prefill_group():
            for L in layers:
                _, s = yb.chunk_gated_delta_rule(q, k, v, a, b_, output_final_state=True,
                                                 use_qk_l2norm_in_kernel=True, cu_seqlens=cu,
                                                 use_gate_in_kernel=True, A_log=A_log, dt_bias=dt_bias,
                                                 use_beta_sigmoid_in_kernel=True)
                L['state'][r0:r1].copy_(s)
            for st in mems:
                view = yb.MemoryState(*(getattr(st, f)[r0:r1] for f in MEMORY_FIELDS))
                yb.sequence(mq, msc, writer, valid, MEM_CHUNK, view)
        prefill_ms += time_events(torch, prefill_group, 1, stream)
        del q, k, v, a, b_, mq, msc, wk, wv
    torch.cuda.empty_cache()
    graphs, _ = capture_steps(torch, yb, layers, mems, inputs, active, ws, table, device)
    for _ in range(3):
        graphs[0].replay()
    steps = max(5, args.steps // 4)
    step_ms = time_events(torch, graphs[0].replay, steps, stream)
    del graphs, layers, mems, inputs, table
    torch.cuda.empty_cache()
    tokens = int(own_len.sum())
    if dist is not None:
        prefill_ms = shard.max_over_ranks(prefill_ms, device=device)
        step_ms = shard.max_over_ranks(step_ms, device=device)
    total_prompt = int(lengths.sum())
    job_s = prefill_ms / 1e3 + GEN_TOKENS * step_ms / 1e3
    return {'requests': SERVE_REQUESTS, 'requests_per_rank': Bd, 'prompt_tokens': total_prompt,
            'prompt_tokens_rank0': tokens, 'prefill_groups_rank0': len(groups),
            'prefill_ms': round(prefill_ms, 3),
            'prefill_tok_s': round(total_prompt / (prefill_ms / 1e3), 1),
            'prefill_tok_s_per_gpu': round(total_prompt / (prefill_ms / 1e3) / world, 1),
            'decode_ms_per_step': round(step_ms, 4), 'decode_steps_timed': steps,
            'decode_tok_s': round(SERVE_REQUESTS / (step_ms / 1e3), 1),
            'decode_tok_s_per_gpu': round(SERVE_REQUESTS / (step_ms / 1e3) / world, 1),
            'projected_job_s': round(job_s, 2),
            'projected_tok_s': round((total_prompt + SERVE_REQUESTS * GEN_TOKENS) / job_s, 1),
            'how': 'config 4: 512 requests, prompts U[512, 16384] (seeded), split over ranks by prompt tokens '
                   '(shard.shard_requests); prefill = 24 GDN layers (varlen chunked, cu_seqlens) + 8 anchor '
                   'prefills per packed group, the short conv left out; decode = all of the rank\'s requests in one '
                   'CUDA-graph step from the prefill\'s states; times max over ranks; the 32K-token generation '
                   'projected as prefill + 32768 x step'}


MEMORY_FIELDS = ('keys', 'values', 'scores', 'positions', 'pending_keys', 'pending_values', 'pending_scores', 'count',
                 'total')


def traffic_per_launch():
    """DRAM bytes (read + write) of one gdn_recurrent_sst_kernel launch from the
    committed ncu summary, or None when no capture has been summarised."""
    path = os.path.join(ROOT, 'profiles', 'gdn_recurrent_sst_decode_b64.json')
    try:
        with open(path) as f:
            return json.load(f).get('dram_bytes_per_launch')
    except Exception:  # noqa: BLE001
        return None


def run_prefill(torch, yb, device, hbm, tf_burst, peak_kind):
    """Config 1: chunked prefill B=8, T=8192, H=HV=32, K=V=128 (bf16 in, fp32
    state), and the anchor read over 64 slots per head at the memory shape."""
    gen = torch.Generator(device=device).manual_seed(7)
    bf = torch.bfloat16
    B, T, H, K = 8, 8192, 32, 128
    q = torch.randn(B, T, H, K, generator=gen, device=device).to(bf)
    k = torch.randn(B, T, H, K, generator=gen, device=device).to(bf)
    v = torch.randn(B, T, H, K, generator=gen, device=device).to(bf)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=gen, device=device))
    beta = torch.randn(B, T, H, generator=gen, device=device).sigmoid().to(bf)
    h0 = 0.02 * torch.randn(B, H, K, K, generator=gen, device=device)

    def chunk():
        yb.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True,
                                  use_qk_l2norm_in_kernel=True)
    for _ in range(2):
        chunk()
    stream = torch.cuda.current_stream(device)
    ms = time_events(torch, chunk, 3, stream)
    flops = B * T * H * (6 * K * K + 2 * 64 * (3 * K + 2 * K))
    # anchor read: blocks of 64 tokens, 16 query heads over 4 groups, D=256, 64 anchors
    blocks = T // 64
    mq = torch.randn(B, blocks, 64, MEM_H, MEM_D, generator=gen, device=device).to(bf)
    mk = torch.randn(1, 4096, MEM_G, MEM_D, generator=gen, device=device).to(bf)
    mv = torch.randn(1, 4096, MEM_G, MEM_D, generator=gen, device=device).to(bf)
    refs = torch.randint(0, 4096, (B, blocks, MEM_G, 64), generator=gen, device=device)
    for _ in range(2):
        yb.indexed_gqa(mq, mk, mv, refs)
    mem_ms = time_events(torch, lambda: yb.indexed_gqa(mq, mk, mv, refs), 3, stream)
    # prefix top-64 over the 128 blocks of each (row, group)
    psc = (torch.randn(B, blocks, MEM_G, 64, generator=gen, device=device) * 2).round() / 2
    ppos = torch.arange(T, device=device).reshape(1, blocks, 1, 64).expand(B, blocks, MEM_G, 64).contiguous()
    for _ in range(2):
        yb.exclusive_prefix_topk(psc, ppos, ppos, 64)
    topk_ms = time_events(torch, lambda: yb.exclusive_prefix_topk(psc, ppos, ppos, 64), 3, stream)
    # the whole prefill write + read of one memory layer on a fresh state; the
    # writer's rows come from per-token keys / values made beforehand (the
    # writer's projections are model GEMMs, outside this path)
    msc = (torch.randn(B, T, MEM_G, generator=gen, device=device) * 2).round() / 2
    mq2 = mq.reshape(B, T, MEM_H, MEM_D)
    wk = torch.randn(B, T, MEM_G, MEM_D, generator=gen, device=device).to(bf)
    wv = torch.randn(B, T, MEM_G, MEM_D, generator=gen, device=device).to(bf)

    def writer(b, t):            # stands in for the writer: N (token, group) rows
        rows = b * T + t
        return (wk.view(B * T, -1).index_select(0, rows).view(-1, MEM_G, MEM_D),
                wv.view(B * T, -1).index_select(0, rows).view(-1, MEM_G, MEM_D))

    def seq():
        st = yb.MemoryState.empty(B, MEM_G, 64, MEM_CHUNK, MEM_D, device, bf)
        yb.sequence(mq2, msc, writer, None, MEM_CHUNK, st)
    for _ in range(2):
        seq()
    seq_ms = time_events(torch, seq, 3, stream)
    # the same layer's prefill with no host synchronisation, captured once in a CUDA graph and replayed
    # (each replay continues the state the previous one left: same shapes, same work)
    st_g = yb.MemoryState.empty(B, MEM_G, 64, MEM_CHUNK, MEM_D, device, bf)
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        yb.sequence(mq2, msc, writer, None, MEM_CHUNK, st_g, capture_safe=True)
    stream.wait_stream(side)
    torch.cuda.synchronize()
    g_seq = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_seq):
        yb.sequence(mq2, msc, writer, None, MEM_CHUNK, st_g, capture_safe=True)
    g_seq.replay()
    seq_graph_ms = time_events(torch, g_seq.replay, 3, stream)
    del g_seq, st_g
    # sliding-window attention over the same prompts (an SWA layer: 16 query heads
    # over 4 KV heads, D=256, window 1024); free the GDN inputs first
    del q, k, v, mq, mq2, wk, wv
    sq = torch.randn(B, T, SW_QH, SW_D, generator=gen, device=device).to(bf)
    skv = torch.randn(2, B, T, SW_KVH, SW_D, generator=gen, device=device).to(bf)
    for _ in range(2):
        yb.reference_swa(sq, skv[0], skv[1], window=SW_W)
    swa_ms = time_events(torch, lambda: yb.reference_swa(sq, skv[0], skv[1], window=SW_W), 3, stream)
    swa_flops = B * SW_QH * sum(min(t + 1, SW_W) for t in range(T)) * 4 * SW_D
    del sq, skv
    achieved = flops / (ms / 1e3) / 1e12
    return {'workload': 'config 1: chunked prefill B=8 T=8192 H=HV=32 K=V=128 bf16, fp32 state; '
                        'plus the anchor prefill of one memory layer (64 slots, G=4 H=16 D=256, chunk 64)',
            'tok_s': round(B * T / (ms / 1e3), 1), 'gdn_ms': round(ms, 3), 'anchor_read_ms': round(mem_ms, 3),
            'anchor_prefix_topk_ms': round(topk_ms, 3), 'anchor_sequence_ms': round(seq_ms, 3),
            'anchor_sequence_graph_ms': round(seq_graph_ms, 3),
            'tok_s_with_anchor_read': round(B * T / ((ms + mem_ms) / 1e3), 1),
            'tok_s_with_anchor_prefill': round(B * T / ((ms + seq_ms) / 1e3), 1),
            'swa_prefill': {'ms': round(swa_ms, 3), 'how': f'reference_swa over the same prompts: {SW_QH} query heads '
                            f'over {SW_KVH} KV heads, D={SW_D}, window {SW_W}, tcgen05',
                            'tflops': round(swa_flops / (swa_ms / 1e3) / 1e12, 1),
                            'frac': round(swa_flops / (swa_ms / 1e3) / 1e12 / tf_burst, 4),
                            'flops_per_launch': swa_flops},
            'roofline': {'bound': 'tensor', 'kernel': 'gdn chunk', 'achieved': round(achieved, 2), 'peak': tf_burst,
                         'unit': 'TFLOP/s', 'frac': round(achieved / tf_burst, 4), 'peak_kind': peak_kind,
                         'flops_per_launch': flops}}


def run_only(args):
    """Run one kernel family `--steps` times at the bench shapes (for ncu
    captures of a small case); prints its mean CUDA-event time."""
    import torch
    import yanchor_b200 as yb
    dev = torch.device('cuda', 0)
    B = args.batch
    layers, mems, inputs, active, ws, table = build_decode(torch, yb, B, dev, n_inputs=1)
    x, L0, st = inputs[0], layers[0], mems[0]
    gen = torch.Generator(device=dev).manual_seed(3)
    bf = torch.bfloat16
    if args.only == 'gdn_chunk':
        Bp, T, H, K = args.prefill_batch, 8192, 32, 128
        q, k, v = (torch.randn(Bp, T, H, K, generator=gen, device=dev).to(bf) for _ in range(3))
        g = torch.nn.functional.logsigmoid(torch.randn(Bp, T, H, generator=gen, device=dev))
        beta = torch.randn(Bp, T, H, generator=gen, device=dev).sigmoid().to(bf)
        fn = lambda: yb.chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True,  # noqa: E731
                                               use_qk_l2norm_in_kernel=True)
    elif args.only == 'swa_prefill':
        Bp, T = args.prefill_batch, 8192
        sq = torch.randn(Bp, T, SW_QH, SW_D, generator=gen, device=dev).to(bf)
        skv = torch.randn(2, Bp, T, SW_KVH, SW_D, generator=gen, device=dev).to(bf)
        fn = lambda: yb.reference_swa(sq, skv[0], skv[1], window=SW_W)  # noqa: E731
    elif args.only == 'mem_indexed':
        blocks = 128
        mq = torch.randn(8, blocks, 64, MEM_H, MEM_D, generator=gen, device=dev).to(bf)
        mk = torch.randn(1, 4096, MEM_G, MEM_D, generator=gen, device=dev).to(bf)
        refs = torch.randint(0, 4096, (8, blocks, MEM_G, 64), generator=gen, device=dev)
        fn = lambda: yb.indexed_gqa(mq, mk, mk, refs)  # noqa: E731
    elif args.only in ('swa', 'swa_layer'):
        rk = torch.randn(B, 4, 1024, 256, generator=gen, device=dev).to(bf)
        rv = torch.randn(B, 4, 1024, 256, generator=gen, device=dev).to(bf)
        rval = torch.ones(B, 1024, device=dev, dtype=torch.bool)
        sq = torch.randn(B, 1, 16, 256, generator=gen, device=dev).to(bf)
        sw = torch.empty(yb.swa.workspace_bytes(B, 4, 16, 1024, 256), device=dev, dtype=torch.uint8)
        fn = lambda: yb.physical_ring_decode_attention(sq, rk, rv, rval, workspace=sw)  # noqa: E731
        if args.only == 'swa_layer':   # the whole SWA decode layer: ring write and advance, then attention
            ridx = torch.zeros((), device=dev, dtype=torch.int64)
            nk = torch.randn(B, 4, 1, 256, generator=gen, device=dev).to(bf)
            nval = torch.ones(B, 1, device=dev, dtype=torch.bool)

            def fn():
                yb.physical_ring_update_(rk, rv, rval, ridx, nk, nk, nval)
                yb.physical_ring_decode_attention(sq, rk, rv, rval, workspace=sw)
    elif args.only in ('mem_topk', 'mem_sequence', 'mem_sequence_graph'):
        blocks, T = 128, 8192
        psc = (torch.randn(8, blocks, MEM_G, 64, generator=gen, device=dev) * 2).round() / 2
        ppos = torch.arange(T, device=dev).reshape(1, blocks, 1, 64).expand(8, blocks, MEM_G, 64).contiguous()
        msc = (torch.randn(8, T, MEM_G, generator=gen, device=dev) * 2).round() / 2
        mq = torch.randn(8, T, MEM_H, MEM_D, generator=gen, device=dev).to(bf)
        wk = torch.randn(8, T, MEM_G, MEM_D, generator=gen, device=dev).to(bf)

        def writer(b, t):
            rows = wk.view(8 * T, -1).index_select(0, b * T + t).view(-1, MEM_G, MEM_D)
            return rows, rows

        def seq():
            st = yb.MemoryState.empty(8, MEM_G, MEM_CAP, MEM_CHUNK, MEM_D, dev, bf)
            yb.sequence(mq, msc, writer, None, MEM_CHUNK, st)
        fn = (lambda: yb.exclusive_prefix_topk(psc, ppos, ppos, 64)) if args.only == 'mem_topk' else seq
        if args.only == 'mem_sequence_graph':   # the capture-safe form, replayed from a CUDA graph
            st_g = yb.MemoryState.empty(8, MEM_G, MEM_CAP, MEM_CHUNK, MEM_D, dev, bf)
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                yb.sequence(mq, msc, writer, None, MEM_CHUNK, st_g, capture_safe=True)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize()
            g_seq = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_seq):
                yb.sequence(mq, msc, writer, None, MEM_CHUNK, st_g, capture_safe=True)
            fn = g_seq.replay
    elif args.only == 'mem_layers':
        # the 8 memory layers' decode step in one CUDA graph, three bank states: empty banks, full banks
        # with no row merging during the timed replays (counts restarted at 0), and full banks with pending
        # counts staggered over the chunk (1 in MEM_CHUNK rows merges per replay)
        mems8 = [yb.MemoryState.empty(B, MEM_G, MEM_CAP, MEM_CHUNK, MEM_D, dev, bf) for _ in range(L_MEM)]

        def layers8():
            for i, m in enumerate(mems8):
                yb.memory_decode_step(x['mq'][i], x['mk'][i], x['mv'][i], x['ms'][i], active, MEM_CHUNK, m)
        stream = torch.cuda.current_stream(dev)
        layers8()
        torch.cuda.synchronize()
        g8 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g8):
            layers8()
        res = {}
        for m in mems8:
            m.count.zero_()
        res['empty_banks_us'] = time_events(torch, g8.replay, 20, stream) * 1e3 / L_MEM
        for _ in range(MEM_CHUNK + 2):
            g8.replay()
        for m in mems8:
            m.count.zero_()
        res['full_banks_no_merge_us'] = time_events(torch, g8.replay, 20, stream) * 1e3 / L_MEM
        for m in mems8:
            m.count.copy_(torch.arange(B, device=dev) % MEM_CHUNK)
        res['full_banks_staggered_us'] = time_events(torch, g8.replay, 20, stream) * 1e3 / L_MEM
        for m in mems8:
            m.count.fill_(MEM_CHUNK - 1)
        res['all_rows_merge_us'] = time_events(torch, g8.replay, 1, stream) * 1e3 / L_MEM
        print(json.dumps({'only': 'mem_layers', 'batch': B, **{k: round(v, 2) for k, v in res.items()}}), flush=True)
        return
    elif args.only in ('mem_step', 'mem_step_merge'):
        # one memory layer's decode step (read + commit, one launch) on a full bank: pending counts
        # staggered over the chunk (1 in MEM_CHUNK rows merges per call), or every row merging
        for _ in range(MEM_CHUNK + 2):
            yb.memory_decode_step(x['mq'][0], x['mk'][0], x['mv'][0], x['ms'][0], active, MEM_CHUNK, st)
        st.count.copy_(torch.arange(B, device=dev) % MEM_CHUNK)
        torch.cuda.synchronize()

        def fn():
            if args.only == 'mem_step_merge':
                st.count.fill_(MEM_CHUNK - 1)
            yb.memory_decode_step(x['mq'][0], x['mk'][0], x['mv'][0], x['ms'][0], active, MEM_CHUNK, st)
    else:
        q0, k0, v0 = conv_qkv(yb, L0, x['mixed'][0])
        fns = {
            'conv_update': lambda: conv_qkv(yb, L0, x['mixed'][0]),
            'gdn_fused': lambda: yb.fused_gdn_decode(x['mixed'][0], x['z'][0], x['a'][0], x['b'][0], L0['conv_state'],
                                                     L0['conv_w'], None, L0['state'], L0['A_log'], L0['dt_bias'],
                                                     L0['norm_w'], num_k_heads=H_K),
            'gdn_decode': lambda: yb.fused_recurrent_gated_delta_rule(
                q0, k0, v0, g=x['a'][0], beta=x['b'][0], initial_state=L0['state'],
                output_final_state=True, use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True,
                A_log=L0['A_log'], dt_bias=L0['dt_bias'], use_beta_sigmoid_in_kernel=True, z=x['z'][0],
                norm_weight=L0['norm_w'], inplace=True),
            'mem_read': lambda: yb.committed_gqa(x['mq'][0], st),
            'mem_commit': lambda: yb.commit_decode(x['mk'][0], x['mv'][0], x['ms'][0], active, MEM_CHUNK, st),
            'greedy': lambda: yb.greedy(x['logits'], workspace=ws),
            'topk': lambda: yb.sample_top_k_top_p_counter(x['logits'], torch.arange(B, device=dev), 1, seed=0,
                                                          temperature=1.0, top_k=20, top_p=0.95),
        }
        fn = fns[args.only]
    for _ in range(args.warmup):
        fn()
    ms = time_events(torch, fn, args.steps, torch.cuda.current_stream(dev))
    print(json.dumps({'only': args.only, 'ms': round(ms, 5), 'steps': args.steps}), flush=True)


# ------------------------------------------------------------- CPU arm ------
def cpu_decode_sample(steps=2, B=64, seed=0, warmup=0):
    """Time the numpy restatement of the same decode step on the host
    (`warmup` untimed steps first)."""
    from oracle import conv as oconv, decode_state as ods, gdn as ogdn, memory as omem, sampling as osamp
    rng = np.random.default_rng(seed)
    i64 = np.int64
    table = dict(storage=np.zeros((2 * B, GEN_TOKENS + 1), np.int32), dense_seen=np.zeros((B, VOCAB), bool),
                 generated_lengths=np.zeros(2 * B, i64), finished_by_eos=np.zeros(2 * B, bool),
                 finished=np.zeros(B, bool), slot_rows=np.arange(B, dtype=i64), sink_rows=B + np.arange(B, dtype=i64),
                 slot_caps=np.full(B, GEN_TOKENS, i64), row_steps=np.ones(B, i64), row_positions=np.full(B, 1024, i64),
                 decode_ids=np.zeros((B, 1), i64), decode_useful_events=np.zeros((), i64))
    f32 = np.float32
    states = [(0.02 * rng.standard_normal((B, H_V, DK, DV))).astype(f32) for _ in range(L_GDN)]
    conv_states = [rng.standard_normal((B, CONV_C, CONV_KS)).astype(f32) for _ in range(L_GDN)]
    conv_w = (rng.standard_normal((CONV_C, CONV_KS)) * 0.5).astype(f32)
    A_log = np.log(rng.uniform(1, 16, H_V)).astype(f32)
    mem = [omem.empty_state(B, MEM_G, MEM_CAP, MEM_CHUNK, MEM_D) for _ in range(L_MEM)]
    t0 = time.perf_counter()
    for it in range(warmup + steps):
        if it == warmup:
            t0 = time.perf_counter()
        for i in range(L_GDN):
            mixed = rng.standard_normal((B, CONV_C, 1)).astype(f32)
            y, conv_states[i] = oconv.conv_update(mixed, conv_states[i], conv_w)
            y = y[:, :, 0].astype(f32)
            q = y[:, None, :H_K * DK].reshape(B, 1, H_K, DK)
            k = y[:, None, H_K * DK:2 * H_K * DK].reshape(B, 1, H_K, DK)
            v = y[:, None, 2 * H_K * DK:].reshape(B, 1, H_V, DV)
            a = rng.standard_normal((B, 1, H_V)).astype(f32)
            b = rng.standard_normal((B, 1, H_V)).astype(f32)
            z = rng.standard_normal((B, 1, H_V, DV)).astype(f32)
            g, beta = ogdn.gdn_gates(a, b, A_log, np.ones(H_V, f32))
            o, states[i] = ogdn.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=states[i],
                                                           use_qk_l2norm=True)
            ogdn.rmsnorm_gated(o, z, np.ones(DV, f32))
        for st in mem:
            mq = rng.standard_normal((B, 1, MEM_H, MEM_D)).astype(f32)
            omem.decode_read(mq, st['keys'], st['values'], st['positions'])
            omem.commit_decode(rng.standard_normal((B, 1, MEM_G, MEM_D)).astype(f32),
                               rng.standard_normal((B, 1, MEM_G, MEM_D)).astype(f32),
                               rng.standard_normal((B, 1, MEM_G)).astype(f32), np.ones(B, bool), MEM_CHUNK, st)
        tok = osamp.greedy(rng.standard_normal((B, VOCAB)).astype(f32))
        ods.update_decode_state(np.asarray(tok, i64).reshape(B, 1), *(table[k] for k in TABLE_FIELDS),
                                maximum_new_tokens=GEN_TOKENS, pad_token_id=PAD_ID, eos_token_ids=EOS_IDS)
    dt = time.perf_counter() - t0
    return B * steps / dt, dt


def cpu_model():
    """The host CPU's model name (Linux /proc/cpuinfo), for the baseline lines."""
    try:
        with open('/proc/cpuinfo') as f:
            for line in f:
                if line.startswith('model name'):
                    return line.split(':', 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or 'unknown'


REF_ROOT = os.path.join(ROOT, 'baseline', '_ref')


def reference_installed():
    return os.path.exists(os.path.join(REF_ROOT, 'modeling_yanchor.py'))


def reference_torch_decode(B, steps, warmup):
    """The reference's own CPU path for the same decode step, imported from the
    reference install (baseline/_ref), fp32, all host threads:

    * per GDN layer: ``torch_causal_conv1d_update`` (modeling_yanchor.py:349),
      the gate expressions of ``Qwen3_5GatedDeltaNet.forward`` (transformers
      qwen3_5 modeling_qwen3_5.py:500-502), q/k repeated for the 32 value
      heads, ``torch_recurrent_gated_delta_rule`` (same file :314-353) with
      the q/k L2 norm, and ``Qwen3_5RMSNormGated`` (:175-190);
    * per memory layer: ``IndependentGQAMemory._decode`` with the torch
      backend (modeling_yanchor.py:277-313), pending counts staggered as in
      the GPU arm;
    * ``sample_top_k_top_p_counter`` with top_k = 1 (greedy,
      runtime/model/inference_kernels.py:73-84).

    The per-step slot-table bookkeeping (a few small writes) is left out.
    Returns (tok/s, seconds for `steps` steps, threads)."""
    sys.path[:0] = [REF_ROOT, os.path.join(REF_ROOT, 'runtime')]
    import torch
    from types import SimpleNamespace
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    from transformers.models.qwen3_5 import modeling_qwen3_5 as qwen
    import modeling_yanchor as my
    import model.inference_kernels as ik
    F = torch.nn.functional
    gen = torch.Generator().manual_seed(5)
    rnd = lambda *shape: torch.randn(*shape, generator=gen)  # noqa: E731
    with torch.no_grad():
        states = [0.02 * rnd(B, H_V, DK, DV) for _ in range(L_GDN)]
        conv_states = [rnd(B, CONV_C, CONV_KS) for _ in range(L_GDN)]
        conv_w = 0.5 * rnd(CONV_C, CONV_KS)
        A_log = torch.empty(H_V).uniform_(1, 16, generator=gen).log()
        dt_bias = torch.ones(H_V)
        norm = qwen.Qwen3_5RMSNormGated(DV, eps=1e-6)
        mems = []
        for _ in range(L_MEM):
            st = my.IndependentMemoryState.empty(B, MEM_G, MEM_CAP, MEM_CHUNK, MEM_D, 'cpu', torch.float32)
            st.pending_keys.copy_(rnd(*st.pending_keys.shape))
            st.pending_values.copy_(rnd(*st.pending_values.shape))
            st.pending_scores.copy_(rnd(*st.pending_scores.shape))
            st.count.copy_(torch.arange(B) % MEM_CHUNK)
            st.total.copy_(torch.arange(B) % MEM_CHUNK)
            mems.append(st)
        ns = SimpleNamespace(backend='torch', capacity=MEM_CAP, groups=MEM_G, heads=MEM_H, dim=MEM_D)
        valid = torch.ones(B, 1, dtype=torch.bool)
        attempt = torch.arange(B)
        rep = H_V // H_K

        def inputs():
            return dict(mixed=rnd(L_GDN, B, CONV_C, 1), a=rnd(L_GDN, B, 1, H_V), b=rnd(L_GDN, B, 1, H_V),
                        z=rnd(L_GDN, B, 1, H_V, DV), mq=rnd(L_MEM, B, 1, MEM_H, MEM_D),
                        mk=rnd(L_MEM, B, 1, MEM_G, MEM_D), mv=rnd(L_MEM, B, 1, MEM_G, MEM_D),
                        ms=rnd(L_MEM, B, 1, MEM_G), logits=3 * rnd(B, VOCAB))
        xs = [inputs() for _ in range(warmup + steps)]
        t0 = time.perf_counter()
        for it, x in enumerate(xs):
            if it == warmup:
                t0 = time.perf_counter()
            for i in range(L_GDN):
                y = my.torch_causal_conv1d_update(x['mixed'][i], conv_states[i], conv_w, None, 'silu')[:, :, 0]
                q = y[:, None, :H_K * DK].reshape(B, 1, H_K, DK).repeat_interleave(rep, dim=2)
                k = y[:, None, H_K * DK:2 * H_K * DK].reshape(B, 1, H_K, DK).repeat_interleave(rep, dim=2)
                v = y[:, None, 2 * H_K * DK:].reshape(B, 1, H_V, DV)
                beta = x['b'][i].sigmoid()
                g = -A_log.float().exp() * F.softplus(x['a'][i].float() + dt_bias)
                o, states[i] = qwen.torch_recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=states[i],
                                                                     output_final_state=True,
                                                                     use_qk_l2norm_in_kernel=True)
                norm(o.reshape(-1, DV), x['z'][i].reshape(-1, DV))
            for j, st in enumerate(mems):
                my.IndependentGQAMemory._decode(ns, x['mq'][j], x['mk'][j], x['mv'][j], x['ms'][j], valid,
                                                MEM_CHUNK, st)
            ik.sample_top_k_top_p_counter(x['logits'], attempt, it, seed=0, temperature=1.0, top_k=1, top_p=1.0)
        dt = time.perf_counter() - t0
    return B * steps / dt, dt, threads


def cpu_sample_line(B, steps, warmup):
    """The CPU baseline sample as a dict: the reference's own torch path when
    the reference is installed here, else the numpy restatement (oracle/)."""
    if reference_installed():
        value, dt, threads = reference_torch_decode(B, steps, warmup)
        return {'value': round(value, 3), 'unit': 'tok/s', 'cores': threads, 'kind': 'reference',
                'cpu': cpu_model(),
                'sample': f'{steps} full decode steps (after {warmup} untimed) at B={B} through the reference\'s '
                          f'own torch path from baseline/_ref (conv update, gates, torch_recurrent_gated_delta_rule, '
                          f'Qwen3_5RMSNormGated, IndependentGQAMemory._decode torch backend, greedy sampler), fp32, '
                          f'{threads} torch threads, {dt:.1f} s'}, dt
    value, dt, cores = cpu_decode_parallel(steps=steps, B=B, warmup=warmup)
    return {'value': round(value, 3), 'unit': 'tok/s', 'cores': cores, 'kind': 'port', 'cpu': cpu_model(),
            'sample': f'{steps} full decode steps (after {warmup} untimed) at B={B} through the numpy restatement of '
                      f'the reference algorithm (oracle/), rows split over {cores} worker processes (one thread '
                      f'each), slowest worker {dt:.1f} s'}, dt


def cpu_sample_subprocess(B, steps, warmup):
    """cpu_sample_line in a fresh interpreter (no CUDA context, its own
    sys.path and thread settings)."""
    import subprocess
    res = subprocess.run([sys.executable, os.path.join(ROOT, 'bench.py'), '--cpu-sample', str(B), str(steps),
                          str(warmup)], capture_output=True, text=True, timeout=900)
    for line in res.stdout.splitlines()[::-1]:
        if line.startswith('{'):
            return json.loads(line)
    raise RuntimeError(f'CPU sample failed: {res.stderr[-2000:]}')


def _cpu_worker(job):
    steps, B, seed, warmup = job
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    return cpu_decode_sample(steps=steps, B=B, seed=seed, warmup=warmup)[1]


def cpu_decode_parallel(steps=2, B=64, warmup=0):
    """The numpy decode step over all host cores: the B sequences are
    independent, so each worker process (spawned, one BLAS thread each) runs
    its share of rows; the step time is the slowest worker's.  Returns
    (tok/s, seconds, workers)."""
    import concurrent.futures
    import multiprocessing
    workers = max(1, min(len(os.sched_getaffinity(0)), B))
    shares = [B // workers + (1 if i < B % workers else 0) for i in range(workers)]
    saved = {k: os.environ.get(k) for k in ('OMP_NUM_THREADS', 'OPENBLAS_NUM_THREADS', 'MKL_NUM_THREADS')}
    os.environ.update({k: '1' for k in saved})
    try:
        with concurrent.futures.ProcessPoolExecutor(workers, mp_context=multiprocessing.get_context('spawn')) as ex:
            dts = list(ex.map(_cpu_worker, [(steps, b, 17 + i, warmup) for i, b in enumerate(shares)]))
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    dt = max(dts)
    return B * steps / dt, dt, workers


def reference_gpu_decode_step(torch, yb, dev, ref_mem, fla_rec, B=64, reps=10):
    """The headline decode step at B=64 composed from the GPU kernels the reference's own stack runs for
    it, captured in one CUDA graph and replayed beside this library's graphed step on the same state:

    * per GDN layer: the graph-safe conv update and the fused gates (runtime/model/inference_kernels.py:
      358, :683), fla 0.5.1's fused_recurrent_gated_delta_rule (its native GQA indexing, no repeat of
      q/k; a new final-state buffer, so the same bytes as the in-place form), and the gated RMSNorm
      module modeling_yanchor.py:374 builds (transformers Qwen3_5RMSNormGated);
    * per memory layer: committed_gqa then commit_decode (runtime/model/independent_memory.py:177, :190);
    * greedy argmax (inference_kernels.py:83) and the decode loop's bookkeeping (:1206).

    Both graphs replay over the steady-state memory of `fill_and_stagger`."""
    spec = importlib.util.spec_from_file_location(
        'reference_inference_kernels', os.path.join(REF_ROOT, 'runtime', 'model', 'inference_kernels.py'))
    ik = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = ik            # its dataclasses look their module up by name
    spec.loader.exec_module(ik)
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5RMSNormGated
    stream = torch.cuda.current_stream(dev)
    layers, mems, inputs, active, ws, table = build_decode(torch, yb, B, dev, n_inputs=1, seed=3)
    x = inputs[0]
    norms = []
    for L in layers:
        n = Qwen3_5RMSNormGated(DV, eps=1e-6).to(dev)
        with torch.no_grad():
            n.weight.copy_(L['norm_w'].float())
        norms.append(n)
    fill_and_stagger(torch, yb, layers, mems, inputs, active, ws, table)

    def ref_step():
        for i, L in enumerate(layers):
            mix = ik.triton_graph_safe_causal_conv1d_update(x['mixed'][i].transpose(1, 2), L['conv_state'],
                                                            L['conv_w'], None, 'silu').transpose(1, 2)
            q = mix[..., :H_K * DK].unflatten(-1, (H_K, DK))
            k = mix[..., H_K * DK:2 * H_K * DK].unflatten(-1, (H_K, DK))
            v = mix[..., 2 * H_K * DK:].unflatten(-1, (H_V, DV))
            beta, g = ik.triton_qwen35_fused_gdn_gates(x['b'][i], x['a'][i], L['A_log'], L['dt_bias'])
            o, _ = fla_rec(q, k, v, g=g, beta=beta, initial_state=L['state'], output_final_state=True,
                           use_qk_l2norm_in_kernel=True)
            norms[i](o.reshape(-1, DV), x['z'][i].reshape(-1, DV))
        for i, m in enumerate(mems):
            ref_mem.committed_gqa(x['mq'][i], m, None)
            ref_mem.commit_decode(x['mk'][i], x['mv'][i], x['ms'][i], active, MEM_CHUNK, m, None)
        tok = x['logits'].argmax(dim=-1, keepdim=True)
        ik._update_fixed_decode_state_(tok, *(table[f] for f in TABLE_FIELDS), maximum_new_tokens=GEN_TOKENS,
                                       pad_token_id=PAD_ID, eos_token_ids=EOS_IDS)

    def graph_of(fn):
        s = torch.cuda.Stream(dev)
        s.wait_stream(stream)
        with torch.cuda.stream(s), torch.no_grad():
            fn()                                   # compiles the Triton kernels, then a pre-capture run
            fn()
        stream.wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g), torch.no_grad():
            fn()
        return g

    g_ref = graph_of(ref_step)
    g_ours = graph_of(lambda: decode_step(yb, layers, mems, x, active, ws, table))
    res = {}
    for name, g in (('reference_gpu_decode_step_ms', g_ref), ('yanchor_b200_decode_step_ms', g_ours)):
        g.replay()
        res[name] = round(time_events(torch, g.replay, reps, stream), 4)
    res['reference_gpu_decode_step_tok_s'] = round(B / res['reference_gpu_decode_step_ms'] * 1e3, 1)
    res['yanchor_b200_decode_step_tok_s'] = round(B / res['yanchor_b200_decode_step_ms'] * 1e3, 1)
    del g_ref, g_ours
    return res


def run_comparators(args):
    """Context only (not the reference arm): the GPU kernels the reference itself uses for this path,
    timed on the same B200 at the bench's shapes with CUDA events, beside this library's kernels.

    * fla 0.5.1 (the third-party package the reference pins, requirements.txt:20):
      chunk_gated_delta_rule at config 1 and fused_recurrent_gated_delta_rule for one decode layer at
      B=64, as modeling_yanchor.py:397-406 binds them;
    * the reference's Triton anchor-memory kernels from its install (runtime/model/independent_memory.py:
      committed_gqa then commit_decode, 8 layers at B=64 with full banks and staggered pending counts;
      indexed_gqa, the anchor prefill read, at config 1);
    * the whole B=64 decode step composed from those kernels (`reference_gpu_decode_step`), graphed.
    Each runs once to compile, then is timed; a failure is reported, not raised."""
    import torch
    import yanchor_b200 as yb
    dev = torch.device('cuda', 0)
    stream = torch.cuda.current_stream(dev)
    bf = torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(7)
    out = {}

    def timed(name, fn, iters=5):
        try:
            fn()
            torch.cuda.synchronize()
            out[name] = round(time_events(torch, fn, iters, stream), 4)
        except Exception as e:  # noqa: BLE001
            out[name] = f'failed: {type(e).__name__}: {str(e)[:200]}'

    B, T, H, K = 8, 8192, 32, 128
    q, k, v = (torch.randn(B, T, H, K, generator=gen, device=dev).to(bf) for _ in range(3))
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=gen, device=dev))
    beta = torch.randn(B, T, H, generator=gen, device=dev).sigmoid().to(bf)
    h0 = 0.02 * torch.randn(B, H, K, K, generator=gen, device=dev)
    timed('yanchor_b200_chunk_config1_ms', lambda: yb.chunk_gated_delta_rule(
        q, k, v, g, beta, initial_state=h0, output_final_state=True, use_qk_l2norm_in_kernel=True))
    try:
        from fla.ops.gated_delta_rule import chunk_gated_delta_rule as fla_chunk
        from fla.ops.gated_delta_rule import fused_recurrent_gated_delta_rule as fla_rec
        timed('fla_chunk_config1_ms', lambda: fla_chunk(q, k, v, g=g, beta=beta, initial_state=h0,
                                                           output_final_state=True, use_qk_l2norm_in_kernel=True))
    except Exception as e:  # noqa: BLE001
        out['fla_chunk_config1_ms'] = f'failed: {type(e).__name__}: {str(e)[:200]}'
        fla_rec = None
    del q, k, v, g, beta, h0
    Bd = 64
    qd = torch.randn(Bd, 1, H_K, DK, generator=gen, device=dev).to(bf)
    kd = torch.randn(Bd, 1, H_K, DK, generator=gen, device=dev).to(bf)
    vd = torch.randn(Bd, 1, H_V, DV, generator=gen, device=dev).to(bf)
    gd = torch.nn.functional.logsigmoid(torch.randn(Bd, 1, H_V, generator=gen, device=dev))
    bd = torch.randn(Bd, 1, H_V, generator=gen, device=dev).sigmoid().to(bf)
    sd = 0.02 * torch.randn(Bd, H_V, DK, DV, generator=gen, device=dev)
    timed('yanchor_b200_recurrent_b64_layer_ms', lambda: yb.fused_recurrent_gated_delta_rule(
        qd, kd, vd, g=gd, beta=bd, initial_state=sd, output_final_state=True, use_qk_l2norm_in_kernel=True,
        inplace=True), iters=20)
    if fla_rec is not None:
        qr, kr = qd.repeat_interleave(H_V // H_K, dim=2), kd.repeat_interleave(H_V // H_K, dim=2)
        timed('fla_recurrent_b64_layer_ms', lambda: fla_rec(qr, kr, vd, g=gd, beta=bd, initial_state=sd,
                                                            output_final_state=True, use_qk_l2norm_in_kernel=True),
              iters=20)
    # anchor memory decode, 8 layers
    mems = [yb.MemoryState.empty(Bd, MEM_G, MEM_CAP, MEM_CHUNK, MEM_D, dev, bf) for _ in range(L_MEM)]
    mq = torch.randn(L_MEM, Bd, 1, MEM_H, MEM_D, generator=gen, device=dev).to(bf)
    mk = torch.randn(L_MEM, Bd, 1, MEM_G, MEM_D, generator=gen, device=dev).to(bf)
    ms = torch.randn(L_MEM, Bd, 1, MEM_G, generator=gen, device=dev)
    act = torch.ones(Bd, device=dev, dtype=torch.bool)
    for _ in range(MEM_CHUNK + 2):
        for i, m in enumerate(mems):
            yb.memory_decode_step(mq[i], mk[i], mk[i], ms[i], act, MEM_CHUNK, m)
    for m in mems:
        m.count.copy_(torch.arange(Bd, device=dev) % MEM_CHUNK)
    timed('yanchor_b200_memory_8_layers_ms', lambda: [yb.memory_decode_step(mq[i], mk[i], mk[i], ms[i], act,
                                                                            MEM_CHUNK, m) for i, m in enumerate(mems)],
          iters=20)
    # anchor prefill read at config 1 (8 rows x 128 blocks x 4 groups, 64 referenced slots)
    iq = torch.randn(8, 128, MEM_CHUNK, MEM_H, MEM_D, generator=gen, device=dev).to(bf)
    ik = torch.randn(1, 4096, MEM_G, MEM_D, generator=gen, device=dev).to(bf)
    irefs = torch.randint(0, 4096, (8, 128, MEM_G, MEM_CAP), generator=gen, device=dev)
    timed('yanchor_b200_indexed_read_config1_ms', lambda: yb.indexed_gqa(iq, ik, ik, irefs), iters=20)
    if reference_installed():
        try:
            # the reference's module (it imports modeling_yanchor from the install root); loaded under
            # its own name so that this package's drop-in module of the same name is not picked up
            sys.path[:0] = [REF_ROOT, os.path.join(REF_ROOT, 'runtime')]
            spec = importlib.util.spec_from_file_location(
                'reference_independent_memory', os.path.join(REF_ROOT, 'runtime', 'model', 'independent_memory.py'))
            ref_mem = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(ref_mem)
            timed('reference_triton_indexed_read_config1_ms', lambda: ref_mem.indexed_gqa(iq, ik, ik, irefs),
                  iters=20)

            def ref_layers():
                for i, m in enumerate(mems):
                    ref_mem.committed_gqa(mq[i], m, None)
                    ref_mem.commit_decode(mk[i], mk[i], ms[i], act, MEM_CHUNK, m, None)
            timed('reference_triton_memory_8_layers_ms', ref_layers, iters=20)
        except Exception as e:  # noqa: BLE001
            out['reference_triton_memory_8_layers_ms'] = f'failed: {type(e).__name__}: {str(e)[:200]}'
            ref_mem = None
        del mems, iq, ik, irefs
        if ref_mem is not None and fla_rec is not None:
            try:
                out.update(reference_gpu_decode_step(torch, yb, dev, ref_mem, fla_rec))
            except Exception as e:  # noqa: BLE001
                out['reference_gpu_decode_step_ms'] = f'failed: {type(e).__name__}: {str(e)[:200]}'
    else:
        out['reference_triton'] = 'not installed'
    print(json.dumps({'comparators': out, 'how': 'CUDA events; eager launches (no CUDA graph) for every entry but '
                      'the two *_decode_step entries, which replay one CUDA graph of the whole step each, '
                      'same inputs per pair'}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=200)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--batch', type=int, default=64)
    ap.add_argument('--impl', default='yanchor_b200', choices=['yanchor_b200', 'reference'])
    ap.add_argument('--no-prefill', action='store_true')
    ap.add_argument('--no-cpu', action='store_true')
    ap.add_argument('--no-serve', action='store_true', help='skip the config-4 serving sweep')
    ap.add_argument('--no-b256', action='store_true', help='skip the config-2 batch (B=256)')
    ap.add_argument('--only', choices=['conv_update', 'gdn_decode', 'gdn_fused', 'gdn_chunk', 'mem_read', 'mem_commit',
                                       'mem_step', 'mem_step_merge', 'mem_layers', 'mem_indexed', 'mem_topk',
                                       'mem_sequence', 'mem_sequence_graph', 'swa', 'swa_layer', 'swa_prefill', 'greedy',
                                       'topk'], help='run one kernel family (small ncu captures)')
    ap.add_argument('--prefill-batch', type=int, default=8)
    ap.add_argument('--cpu-sample', nargs=3, type=int, metavar=('B', 'STEPS', 'WARMUP'), help=argparse.SUPPRESS)
    ap.add_argument('--comparators', action='store_true',
                    help='time the reference\'s own GPU kernels (fla, its Triton memory kernels) beside these')
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    sys.path.insert(0, ROOT)

    if args.cpu_sample:
        line, _ = cpu_sample_line(*args.cpu_sample)
        print(json.dumps(line), flush=True)
        return
    if args.comparators:
        run_comparators(args)
        return
    if args.only:
        run_only(args)
        return
    if args.impl == 'reference':
        if rank != 0:
            return
        steps = max(1, min(args.steps, 3))
        warm = min(args.warmup, 1)              # untimed steps first, bounded like the timed ones
        rows = args.batch                        # one GPU's batch: the host's rate on this step
        base, dt = cpu_sample_line(rows, steps, warm)
        line = {'metric': METRIC, 'value': base['value'], 'unit': 'tok/s', 'n_gpus': args.gpus, 'steps': steps,
                'warmup': warm, 'ms_per_step': round(dt / steps * 1e3, 1), 'higher_is_better': True,
                'scaling': 'weak', 'vs_baseline': None, 'dtype': 'fp32', 'data': 'synthetic (random init, seeded)',
                'impl': 'reference',
                'config': decode_config(args.batch, args.gpus),
                'cpu_baseline': base,
                'e2e': {'value': base['value'], 'unit': 'tok/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
        print(json.dumps(line), flush=True)
        return

    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device('cuda', local_rank))
        dist = tdist
    result, _ = run_gpu(args, rank, world, local_rank, dist)
    import torch
    import yanchor_b200 as yb
    hbm, tf_burst, tf_sust, peak_kind = peaks()
    device = torch.device('cuda', local_rank)
    if not args.no_serve:
        serve = run_serve(torch, yb, args, rank, world, device, dist)
        if rank == 0:
            result['serve'] = serve
    if rank == 0:
        if world == 1 and not args.no_b256:
            result['decode_b256'] = run_batch_decode(torch, yb, 256, device, max(10, args.steps // 4), args.warmup,
                                                     hbm, seed=256)
        if not args.no_prefill:
            result['prefill'] = run_prefill(torch, yb, device, hbm, tf_burst, peak_kind)
        if world == 1 and not args.no_cpu:
            result['cpu_baseline'], _ = cpu_sample_line(args.batch, 2, 1) if not reference_installed() else \
                (cpu_sample_subprocess(args.batch, 2, 1), None)
        print(json.dumps(result), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
