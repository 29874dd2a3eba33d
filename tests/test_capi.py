"""C-ABI library checks that need no GPU: the shared object loads, exports
every entry point declared in include/yanchor_b200.h, and rejects bad
arguments on the host (status codes, no launch)."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, 'include', 'yanchor_b200.h')


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return sorted(set(re.findall(r'\b(yb_[a-z0-9_]+)\s*\(', text)))


@pytest.fixture(scope='module')
def lib():
    from yanchor_b200 import _lib
    return _lib.lib()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ('yb_gdn_recurrent_fwd', 'yb_gdn_chunk_fwd', 'yb_mem_decode_read', 'yb_mem_decode_commit',
                 'yb_mem_indexed_read', 'yb_sample_greedy', 'yb_sample_top_k_top_p_counter'):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    from yanchor_b200 import _lib
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f'{name} has no ctypes signature'
    assert lib.yb_abi_version() == 1


def test_exports_are_c_symbols():
    """nm shows unmangled names (extern "C")."""
    import subprocess
    from yanchor_b200 import _lib
    out = subprocess.run(['nm', '-D', '--defined-only', _lib.LIB_PATH], capture_output=True, text=True).stdout
    names = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for name in declared_symbols():
        assert name in names, name


def _rec(lib, **over):
    args = dict(q=16, k=16, v=16, qs=512, ks=512, vs=512, g=16, beta=16, gs=4, bs=4, A_log=None, dt_bias=None,
                h0=None, ht=None, o=16, z=None, w=None, eps=1e-6, cu=None, B=1, T=1, H=4, HV=4, K=128, V=128, N=1,
                scale=0.1, io=2, gd=0, bd=2, flags=0, stream=None)
    args.update(over)
    return lib.yb_gdn_recurrent_fwd(*args.values())


def test_recurrent_rejects_bad_arguments_on_host(lib):
    from yanchor_b200 import _lib
    assert _rec(lib, HV=6) == _lib.YB_ERR_ARGUMENT          # HV % H != 0
    assert b'multiple of H' in lib.yb_last_error()
    assert _rec(lib, io=7) == _lib.YB_ERR_ARGUMENT           # dtype code
    assert _rec(lib, q=None) == _lib.YB_ERR_ARGUMENT         # null tensor
    assert _rec(lib, q=8) == _lib.YB_ERR_ARGUMENT            # misaligned
    assert _rec(lib, N=2) == _lib.YB_ERR_ARGUMENT            # N != B without cu_seqlens
    assert _rec(lib, cu=64, B=2, N=2) == _lib.YB_ERR_ARGUMENT  # cu_seqlens needs B == 1
    assert _rec(lib, qs=100) == _lib.YB_ERR_ARGUMENT         # token stride too small
    assert _rec(lib, flags=2) == _lib.YB_ERR_ARGUMENT        # gate in kernel without A_log
    assert _rec(lib, z=16) == _lib.YB_ERR_ARGUMENT           # z without norm weight


def test_chunk_and_memory_reject_bad_arguments(lib):
    from yanchor_b200 import _lib
    rc = lib.yb_mem_decode_read(16, 16, 16, 16, None, 16, 2, 4, 3, 16, 64, 4096, 64, 2, None)
    assert rc == _lib.YB_ERR_ARGUMENT                        # H % G != 0
    rc = lib.yb_mem_decode_commit(16, 16, 16, 16, 9, 16, 16, 16, 16, 16, 16, 16, 16, 16, None, 2, 4, 16, 8, 64,
                                  4096, 64, 2048, 32, 1, 2, None)
    assert rc == _lib.YB_ERR_ARGUMENT                        # chunk > PC
    rc = lib.yb_sample_greedy(16, 100, 4, 1000, 2, 16, None, 0, None)
    assert rc == _lib.YB_ERR_ARGUMENT                        # row stride < vocab
    rc = lib.yb_sample_greedy(16, 1000, 4, 1000, 2, 16, None, 0, None)
    assert rc == _lib.YB_ERR_WORKSPACE
    rc = lib.yb_sample_top_k_top_p_counter(16, 1000, 4, 1000, 2, 16, None, 0, 1, 0, 1.0, 0, 0.5, 16, 16, 16, None)
    assert rc == _lib.YB_ERR_WORKSPACE                       # the whole-vocabulary nucleus needs its row state
    rc = lib.yb_sample_top_k_top_p_counter(16, 1000, 4, 1000, 2, 16, None, 0, 1, 0, 1.0, 1001, 0.5, 16, 16, 1 << 20,
                                           None)
    assert rc == _lib.YB_ERR_ARGUMENT                        # top-k beyond the vocabulary
    assert lib.yb_sample_workspace_bytes(64, 248320, 20) > 0
    assert lib.yb_sample_workspace_bytes(64, 248320, 0) >= lib.yb_sample_workspace_bytes(64, 248320, 1000) > 0


def test_python_ops_refuse_cpu_tensors():
    import yanchor_b200 as yb
    q = torch.randn(1, 2, 2, 64)
    g = torch.zeros(1, 2, 2)
    with pytest.raises(ValueError, match='CUDA tensors only'):
        yb.chunk_gated_delta_rule(q, q, q, g, g)
    with pytest.raises(ValueError, match='CUDA tensors only'):
        yb.greedy(torch.randn(2, 10))


def test_greedy_noalloc_checks_out_and_stride_on_host():
    """The no-allocation greedy refuses an ``out`` the kernel would write past
    (wrong dtype, too short, non-contiguous) and scores it would have to copy,
    before anything touches a device."""
    import yanchor_b200 as yb
    scores = torch.randn(4, 10)
    with pytest.raises(ValueError, match='int64'):
        yb.greedy_noalloc(scores, out=torch.empty(4, dtype=torch.int32))
    with pytest.raises(ValueError, match='rows need one each'):
        yb.greedy_noalloc(scores, out=torch.empty(3, dtype=torch.int64))
    with pytest.raises(ValueError, match='contiguous'):
        yb.greedy_noalloc(scores, out=torch.empty(4, 2, dtype=torch.int64)[:, 0])
    with pytest.raises(ValueError, match='unit stride'):
        yb.greedy_noalloc(torch.randn(10, 4).t())
    with pytest.raises(ValueError, match='CUDA tensors only'):
        yb.greedy_noalloc(scores, out=torch.empty(4, dtype=torch.int64))


def test_python_ops_validate_shapes_first():
    """fla's head-count checks fire before anything touches a device."""
    import yanchor_b200.gated_delta_rule as gdr
    q = torch.randn(1, 2, 2, 64)
    v = torch.randn(1, 2, 3, 64)
    g = torch.zeros(1, 2, 3)
    with pytest.raises(ValueError, match='evenly divisible'):
        gdr._validate(q, q, v, g, g, None, None)
    with pytest.raises(ValueError, match='batch size is expected to be 1'):
        gdr._validate(torch.randn(2, 2, 3, 64), torch.randn(2, 2, 3, 64), torch.randn(2, 2, 3, 64),
                      torch.zeros(2, 2, 3), torch.zeros(2, 2, 3), None, torch.tensor([0, 2]))


def test_memory_module_install():
    import importlib
    import yanchor_b200
    mod = yanchor_b200.install_memory_module()
    assert importlib.import_module('model.independent_memory') is mod
    assert callable(mod.indexed_gqa) and callable(mod.committed_gqa) and callable(mod.commit_decode)


def test_bind_gdn_kernels():
    import yanchor_b200

    class Layer(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.chunk_gated_delta_rule = None
            self.recurrent_gated_delta_rule = None

    model = torch.nn.Sequential(Layer(), torch.nn.Linear(2, 2), Layer())
    info = yanchor_b200.bind_gdn_kernels(model)
    assert info['native_gdn_layers'] == ['0', '2']
    assert model[0].chunk_gated_delta_rule is yanchor_b200.chunk_gated_delta_rule
    assert model[2].recurrent_gated_delta_rule.keywords == {'inplace': True}
