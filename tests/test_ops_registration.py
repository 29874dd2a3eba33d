"""The torch custom-op registration (yanchor_b200/ops.py), no GPU: every op
is registered under torch.ops.yanchor_b200 with a schema that marks the
arguments it writes in place, and its fake implementation gives the output
shapes and dtypes on meta tensors (what a tracer such as torch.compile sees)."""
import torch

import yanchor_b200  # noqa: F401  (registers the ops)


def meta(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, device='meta', dtype=dtype)


def schema(name):
    return str(getattr(torch.ops.yanchor_b200, name).default._schema)


def test_schemas_mark_in_place_arguments():
    assert '(a' not in schema('chunk_gated_delta_rule')
    assert 'Tensor(a6!) state' in schema('fused_recurrent_gated_delta_rule_')
    assert 'conv_state' in schema('causal_conv1d_update_') and '!) conv_state' in schema('causal_conv1d_update_')
    for op in ('commit_decode_', 'memory_decode_step_'):
        s = schema(op)
        for field in ('keys', 'values', 'bank_scores', 'positions', 'pending_keys', 'pending_values',
                      'pending_scores', 'count', 'total'):
            assert f'!) {field}' in s, (op, field)
    for op in ('indexed_gqa', 'committed_gqa', 'greedy', 'sample_top_k_top_p_counter'):
        assert '!)' not in schema(op), op


def test_fake_shapes():
    ops = torch.ops.yanchor_b200
    q, v = meta(1, 300, 16, 128), meta(1, 300, 32, 128)
    g = meta(1, 300, 32, dtype=torch.float32)
    cu = torch.empty(4, device='meta', dtype=torch.int64)
    o, s = ops.chunk_gated_delta_rule(q, q, v, g, meta(1, 300, 32), 0.1, None, True, True, cu, True)
    assert o.shape == (1, 300, 32, 128) and o.dtype == torch.bfloat16
    assert s.shape == (3, 32, 128, 128) and s.dtype == torch.float32
    _, s0 = ops.chunk_gated_delta_rule(q, q, v, g, meta(1, 300, 32), 0.1, None, False, True, None, False)
    assert s0.numel() == 0
    st = meta(64, 32, 128, 128, dtype=torch.float32)
    o = ops.fused_recurrent_gated_delta_rule_(meta(64, 1, 16, 128), meta(64, 1, 16, 128), meta(64, 1, 32, 128),
                                              meta(64, 1, 32), meta(64, 1, 32), 0.1, st, True, True,
                                              meta(32, dtype=torch.float32), None, True, None, None, 1e-6)
    assert o.shape == (64, 1, 32, 128)
    y = ops.causal_conv1d_update_(meta(8, 10240, 1), meta(8, 10240, 4), meta(10240, 4, dtype=torch.float32), None,
                                  True)
    assert y.shape == (8, 10240, 1)
    B, G, CAP, PC, D = 8, 4, 64, 64, 256
    fields = (meta(B, G, CAP, D), meta(B, G, CAP, D), meta(B, G, CAP, dtype=torch.float32),
              meta(B, G, CAP, dtype=torch.int32), meta(B, G, PC, D), meta(B, G, PC, D),
              meta(B, G, PC, dtype=torch.float32), meta(B, dtype=torch.int64), meta(B, dtype=torch.int64))
    r = ops.committed_gqa(meta(B, 1, 16, D), *fields, None)
    assert r.shape == (B, 1, 16, D)
    r = ops.memory_decode_step_(meta(B, 1, 16, D), meta(B, 1, G, D), meta(B, 1, G, D),
                                meta(B, 1, G, dtype=torch.float32), meta(B, dtype=torch.bool), 64, *fields, None)
    assert r.shape == (B, 1, 16, D)
    assert ops.commit_decode_(meta(B, 1, G, D), meta(B, 1, G, D), meta(B, 1, G, dtype=torch.float32),
                              meta(B, dtype=torch.bool), 64, *fields, None) is None
    r = ops.indexed_gqa(meta(2, 5, 64, 16, D), meta(1, 300, G, D), meta(1, 300, G, D),
                        meta(2, 5, G, CAP, dtype=torch.int64))
    assert r.shape == (2, 5, 64, 16, D)
    ids = ops.greedy(meta(64, 248320))
    assert ids.shape == (64, 1) and ids.dtype == torch.int64
    ids = ops.sample_top_k_top_p_counter(meta(64, 248320, dtype=torch.float32), meta(64, dtype=torch.int64),
                                         meta(64, dtype=torch.int64), 0, 1.0, 20, 0.9, 0)
    assert ids.shape == (64, 1) and ids.dtype == torch.int64
