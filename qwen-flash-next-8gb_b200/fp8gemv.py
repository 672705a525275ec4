"""Drop-in replacement for the reference's `fp8gemv` module on B200 (sm_100a).

gemv(q, s, x) keeps the signature and semantics of fp8gemv.gemv
(fp8gemv.py:20-26): y[n] = bf16(s[n] * sum_k q[n,k] * x[k]) with fp32
accumulation, computed by libqfn's HBM-streaming kernel (csrc/gemv.cu).
It allocates its output with torch's caching allocator on the current stream
and never synchronizes, so it can run inside CUDA-graph capture as the
reference's DeltaNet graphs require (qwen_delta_graph.py:55-57).
"""
import torch

from _lib import DTYPE_BF16, DTYPE_F32, check, lib, require_cuda, stream_of


def _gemv(q, s, x, out_dtype):
    require_cuda("q", q)
    if q.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise TypeError(f"q must be float8_e4m3fn (or its raw uint8 bytes), got {q.dtype}")
    require_cuda("s", s, torch.float32)
    require_cuda("x", x, torch.bfloat16)
    if q.dim() != 2:
        raise ValueError("q must be [N, K]")
    N, K = q.shape
    if s.numel() != N or x.numel() != K:
        raise ValueError(f"s must have {N} and x {K} elements; got {s.numel()}, {x.numel()}")
    y = torch.empty(N, dtype=out_dtype, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib().qfn_gemv_e4m3(q.data_ptr(), s.data_ptr(), x.data_ptr(), y.data_ptr(),
                                 DTYPE_F32 if out_dtype == torch.float32 else DTYPE_BF16, N, K, stream_of(y))
    check(rc, "qfn_gemv_e4m3")
    return y


def gemv(q, s, x):
    """q [N,K] float8_e4m3fn . s [N] fp32 . x [K] bf16 -> [N] bf16"""
    return _gemv(q, s, x, torch.bfloat16)


def gemv_f32(q, s, x):
    """As gemv, but returns the fp32 value before the bf16 rounding (for tight parity checks)."""
    return _gemv(q, s, x, torch.float32)
