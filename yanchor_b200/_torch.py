"""Small torch-side helpers shared by the operator modules (plumbing only)."""
from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.YB_F32, torch.float16: _lib.YB_F16, torch.bfloat16: _lib.YB_BF16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f'unsupported dtype {t.dtype}; expected float32, float16 or bfloat16') from None


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError('yanchor_b200 operators take CUDA tensors only (there is no CPU path)')


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def token_view(x: torch.Tensor, vector: bool = True) -> tuple[torch.Tensor, int]:
    """Return ``(x', stride)``: x' is ``x`` (or a contiguous copy of it) whose
    per-token trailing axes are contiguous and whose leading (batch, time) axes
    collapse to one token axis of ``stride`` elements.  With ``vector`` the
    base pointer and the token stride must also allow 16-byte vector access."""
    B, T = x.shape[0], x.shape[1]
    inner = 1
    for n in x.shape[2:]:
        inner *= n
    ok = x.stride(-1) == 1 and (x.dim() == 3 or x.stride(-2) == x.shape[-1])
    if B * T <= 1:
        ts = inner
    elif T == 1:
        ts = x.stride(0)
    elif B == 1:
        ts = x.stride(1)
    else:
        ts = x.stride(1) if x.stride(0) == T * x.stride(1) else None
    ok = ok and ts is not None
    if ok and vector:
        ok = (ts * x.element_size()) % 16 == 0 and x.data_ptr() % 16 == 0
    if not ok:
        x = x.contiguous()
        if vector and x.data_ptr() % 16:
            x = x.clone()
        ts = inner
    return x, ts


def scalar_token_view(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    """``token_view`` for ``[B, T, HV]`` per-head scalars (g, beta): no vector
    alignment needed."""
    return token_view(x, vector=False)
