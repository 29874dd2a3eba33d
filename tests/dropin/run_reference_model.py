"""Runs the reference's own model code twice on one GPU and compares: a tiny
random-init ``YANchorForCausalLM`` (modeling_yanchor.py) with

  A. ``backend='torch'``: the reference's torch path (torch_chunk /
     torch_recurrent_gated_delta_rule, IndependentGQAMemory's torch
     _sequence / _decode, reference_swa);
  B. ``backend='cuda'`` after the maintainer's patch from INTEGRATION.md:
     ``bind_gdn_kernels`` through ``bind_native_qwen_gdn_kernels``,
     ``install_memory_module`` (``_cuda_module('independent_memory')``),
     ``bind_memory_prefill`` (``_sequence`` and the top-k helpers), and
     ``flash_swa`` / ``reference_swa`` — every hot-path op of B runs on this
     repository's CUDA library.

Same weights (B loads A's state dict), bf16, a 150-token prefill of two
prompts then 49 decode steps.  A third run, the same weights in fp32 on the
reference's torch path, is the yardstick: its greedy tokens feed all three
runs, and each bf16 path's logits are compared with it.  The model shape
(the smallest YANchorForCausalLM that has every layer kind: 4 layers, 3 GDN
+ 1 SWA layer with an IndependentGQAMemory of 16 slots, commit chunk 16,
window 32) uses the YANchor head shapes (GDN K = V = 128, memory / SWA head_dim 256).

fla is made unavailable in this process, so transformers builds the GDN
layers of both models with the same torch modules (its gated RMSNorm
included) and the only difference between A and B is the patch.  Prints
one JSON line with the largest logit differences and the greedy-id
comparison; run from the repository root as a child process (it imports the
reference's pinned transformers from baseline/_ref).
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(ROOT, 'baseline', '_ref')
sys.path[:0] = [REF, os.path.join(REF, 'runtime'), ROOT]


def main():
    import transformers.utils.import_utils as iu
    iu.is_flash_linear_attention_available = lambda: False     # same GDN modules in both runs
    import torch
    import modeling_yanchor as my
    import yanchor_b200

    def config(backend):
        return my.YANchorConfig(
            backend=backend, vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=4,
            num_attention_heads=4, num_key_value_heads=2, head_dim=256, linear_num_key_heads=2,
            linear_num_value_heads=4, linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
            layer_types=['linear_attention'] * 3 + ['full_attention'],
            fixed_memory_revision=my.INDEPENDENT_MEMORY_REVISION, fixed_memory_swa_layers=[3],
            fixed_memory_swa_window=32,
            independent_memory=dict(capacity=16, max_commit_chunk=16, admission_rank=16,
                                    writer_intermediate_size=256))

    dev = torch.device('cuda', 0)
    torch.manual_seed(0)
    ref_model = my.YANchorForCausalLM(config('torch')).to(dev, torch.bfloat16).eval()
    # the same weights in fp32 on the reference's torch path: the yardstick for both bf16 paths
    f32_model = my.YANchorForCausalLM(config('torch')).to(dev, torch.float32).eval()
    f32_model.load_state_dict({k: v.float() for k, v in ref_model.state_dict().items()}, strict=True)
    gen = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, 1024, (2, 150), generator=gen).to(dev)
    steps = 49

    def run(model, feed):
        cache = my.FixedMemoryHybridDynamicCache(model.config)
        with torch.no_grad():
            out = model(input_ids=prompt, past_key_values=cache, use_cache=True)
            logits = [out.logits.float()]
            ids = [out.logits[:, -1:].argmax(-1)] if feed is None else [feed[:, :1]]
            for t in range(steps):
                out = model(input_ids=ids[-1], past_key_values=cache, use_cache=True)
                logits.append(out.logits.float())
                ids.append(out.logits[:, -1:].argmax(-1) if feed is None else feed[:, t + 1:t + 2])
        torch.cuda.synchronize()
        return logits, torch.cat(ids, 1)

    # the two torch-path runs first: the patch below rebinds module-level functions for every model
    f32_logits, f32_ids = run(f32_model, None)          # the fp32 model's own greedy tokens
    ref_logits, _ = run(ref_model, f32_ids)             # both bf16 paths fed the same tokens
    # the maintainer's patch, applied to the imported reference modules
    yanchor_b200.install_memory_module()
    yanchor_b200.bind_memory_prefill(my)
    my.flash_swa = yanchor_b200.flash_swa
    my.reference_swa = yanchor_b200.reference_swa
    my.bind_native_qwen_gdn_kernels = lambda model: yanchor_b200.bind_gdn_kernels(model, inplace_decode=True)
    b200_model = my.YANchorForCausalLM(config('cuda')).to(dev, torch.bfloat16).eval()
    missing = b200_model.load_state_dict(ref_model.state_dict(), strict=True)
    bound = b200_model.bind_runtime_kernels()
    b200_logits, _ = run(b200_model, f32_ids)

    def worst(a, b, part):
        pairs = list(zip(a, b))
        pairs = pairs[:1] if part == 'prefill' else pairs[1:]
        return max((x - y).abs().max().item() for x, y in pairs)

    def ids_agree(test, truth, margin):
        compared = agree = 0
        for a, b in zip(truth, test):
            top2 = a.topk(2, -1).values
            sure = (top2[..., 0] - top2[..., 1]) > margin
            compared += int(sure.sum())
            agree += int(((a.argmax(-1) == b.argmax(-1)) & sure).sum())
        return compared, agree

    r = {'logit_scale': f32_logits[0].abs().max().item(),
         'b200_vs_ref_bf16': {'prefill': worst(b200_logits, ref_logits, 'prefill'),
                              'decode': worst(b200_logits, ref_logits, 'decode')},
         'b200_vs_fp32': {'prefill': worst(b200_logits, f32_logits, 'prefill'),
                          'decode': worst(b200_logits, f32_logits, 'decode')},
         'ref_bf16_vs_fp32': {'prefill': worst(ref_logits, f32_logits, 'prefill'),
                              'decode': worst(ref_logits, f32_logits, 'decode')},
         'bound_layers': bound.get('native_gdn_layers'),
         'state_dict_keys_ok': not missing.missing_keys and not missing.unexpected_keys}
    noise = max(max(r['b200_vs_fp32'].values()), max(r['ref_bf16_vs_fp32'].values()))
    r['id_margin'] = 2 * noise
    r['ids_b200'] = ids_agree(b200_logits, f32_logits, r['id_margin'])
    r['ids_ref_bf16'] = ids_agree(ref_logits, f32_logits, r['id_margin'])
    r['ids_b200_vs_ref_bf16_margin_1e-2'] = ids_agree(b200_logits, ref_logits, 1e-2)
    print(json.dumps(r), flush=True)


if __name__ == '__main__':
    main()
