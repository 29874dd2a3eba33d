"""The no-allocation greedy entry point (yb_sample_greedy_noalloc) against the
workspace entry point (yb_sample_greedy), both called through the C ABI.

yb_sample_greedy_noalloc exists for callers that cannot allocate device memory
when they sample (a host runtime binding the C ABI without a device allocator,
or a decode loop that must not allocate while its stream is captured); it keeps
its partial results in a fixed device array inside the library.  Token ids are
integers, so the two entry points must agree exactly, on two calls in a row
(the second call reuses the array the first one left behind).

This file is named so that pytest collects it last."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def lib():
    import yanchor_b200
    return yanchor_b200.lib()


def _workspace_greedy(lib, scores):
    B, V = scores.shape
    out = torch.full((B,), -1, device=scores.device, dtype=torch.int64)
    need = lib.yb_sample_workspace_bytes(B, V, 1)
    ws = torch.empty(need, device=scores.device, dtype=torch.uint8)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[scores.dtype]
    rc = lib.yb_sample_greedy(scores.data_ptr(), scores.stride(0), B, V, code, out.data_ptr(), ws.data_ptr(), need,
                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.yb_last_error()
    return out


def _noalloc_greedy(lib, scores):
    B, V = scores.shape
    out = torch.full((B,), -1, device=scores.device, dtype=torch.int64)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[scores.dtype]
    rc = lib.yb_sample_greedy_noalloc(scores.data_ptr(), scores.stride(0), B, V, code, out.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.yb_last_error()
    return out


@pytest.mark.parametrize('dtype,B,V', [(torch.bfloat16, 64, 248320), (torch.float32, 3, 50000),
                                       (torch.bfloat16, 4096, 3000)])
def test_noalloc_matches_workspace_entry_point_twice(lib, dtype, B, V):
    gen = torch.Generator(device='cuda').manual_seed(B)
    for call in range(2):
        scores = (torch.randn(B, V, generator=gen, device='cuda') * 3).to(dtype)
        scores[call % B, (17 * call + 5) % V] = 100.0
        ref = _workspace_greedy(lib, scores)
        got = _noalloc_greedy(lib, scores)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f'call {call}'
        assert int(got[call % B]) == (17 * call + 5) % V


def test_noalloc_rejects_batches_beyond_its_scratch(lib):
    scores = torch.zeros(5000, 100, device='cuda')
    out = torch.empty(5000, device='cuda', dtype=torch.int64)
    rc = lib.yb_sample_greedy_noalloc(scores.data_ptr(), 100, 5000, 100, 0, out.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 2  # YB_ERR_UNSUPPORTED
    assert b'built-in scratch' in lib.yb_last_error()
