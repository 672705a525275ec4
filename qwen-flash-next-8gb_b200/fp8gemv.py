"""Drop-in replacement for the reference's `fp8gemv` module on B200 (sm_100a).

gemv(q, s, x) keeps the signature and semantics of fp8gemv.gemv
(fp8gemv.py:20-26): y[n] = bf16(s[n] * sum_k q[n,k] * x[k]) with fp32
accumulation, computed by libqfn's HBM-streaming kernel (csrc/gemv.cu).
It allocates its output with torch's caching allocator on the current stream
and never synchronizes, so it can run inside CUDA-graph capture as the
reference's DeltaNet graphs require (qwen_delta_graph.py:55-57).

linear(x, q, s) is the engine's FP8 linear layer (Lin.__call__,
qwen_engine.py:79-83) for any number of tokens: the GEMV for one token, and
for T > 1 the reference's F.linear(x, (q.to(bf16) * s).to(bf16)) as one
libqfn GEMM that forms the bf16 weights on chip (csrc/linear.cu).
dequant_bf16(q, s) keeps the weight expression alone (bit-identical bf16
weights in memory).
"""
import torch

from _lib import DTYPE_BF16, DTYPE_F32, check, lib, ops, require_cuda, on_device, stream_of


def _gemv(q, s, x, out_dtype):
    """The torch operator qfn::gemv (libqfn_torch.so -> qfn_gemv_e4m3): checks
    the tensors, launches on torch's current stream."""
    return ops().gemv(q, s, x, out_dtype == torch.float32)


def gemv(q, s, x):
    """q [N,K] float8_e4m3fn . s [N] fp32 . x [K] bf16 -> [N] bf16"""
    return _gemv(q, s, x, torch.bfloat16)


def gemv_f32(q, s, x):
    """As gemv, but returns the fp32 value before the bf16 rounding (for tight parity checks)."""
    return _gemv(q, s, x, torch.float32)


def dequant_bf16(q, s):
    """(q.to(bf16) * s).to(bf16) of qwen_engine.py:83 -> bf16 [N, K], bit-identical.

    q [N,K] float8_e4m3fn (or its uint8 bytes) . s [N] or [N,1] fp32."""
    require_cuda("q", q)
    if q.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise TypeError(f"q must be float8_e4m3fn (or its raw uint8 bytes), got {q.dtype}")
    require_cuda("s", s, torch.float32)
    if q.dim() != 2:
        raise ValueError("q must be [N, K]")
    N, K = q.shape
    if s.numel() != N:
        raise ValueError(f"s must have {N} elements; got {s.numel()}")
    if s.device != q.device:
        raise ValueError(f"s is on {s.device}, q on {q.device}")
    q = q.contiguous()
    s = s.reshape(-1).contiguous()
    w = torch.empty(N, K, dtype=torch.bfloat16, device=q.device)
    with on_device(q.device):
        rc = lib().qfn_e4m3_rows_to_bf16(q.data_ptr(), s.data_ptr(), w.data_ptr(), N, K, stream_of(w))
    check(rc, "qfn_e4m3_rows_to_bf16")
    return w


def linear(x, q, s):
    """Lin.__call__ of an FP8 layer (qwen_engine.py:79-83): x [T,K] bf16 -> [T,N] bf16.

    T == 1: the GEMV (reads only the fp8 bytes).  T > 1: the torch operator
    qfn::linear (-> qfn_linear_e4m3), one tcgen05 GEMM that forms the
    reference's bf16 weights (q.to(bf16) * s).to(bf16) on chip from the fp8
    bytes and accumulates in fp32, as F.linear on those weights does."""
    if not isinstance(x, torch.Tensor) or x.dim() != 2:
        raise ValueError("x must be a [T, K] tensor")
    if x.shape[0] == 1:
        return gemv(q, s.reshape(-1), x[0].contiguous())[None]
    require_cuda("x", x, torch.bfloat16, contiguous=False)
    return ops().linear(x.contiguous(), q, s.reshape(-1).contiguous())
