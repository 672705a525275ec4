"""CPU oracle for the quantized matrix-product path -- TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl
reference legs import this module, as the checker and the CPU baseline.  The
product never imports it.

It wraps liboracle.so (qfn_oracle.c, a C restatement of the reference's torch
path; every function there cites the reference lines it follows) with numpy
in/out arrays.  Build with `python oracle/build.py` (or __graft_entry__.build()).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

HID, INTER, BLOCK = 2560, 640, 2764800
O_GW, O_UW, O_DW = 0, 819200, 1638400
O_GS, O_US, O_DS = 2457600, 2560000, 2662400

E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32)

_lib = None
_P = ctypes.c_void_p
_L = ctypes.c_long


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run `python oracle/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_threads.argtypes = [ctypes.c_int]
        L.oracle_threads.restype = ctypes.c_int
        L.oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.oracle_e4m3_to_f32.restype = ctypes.c_float
        L.oracle_f32_to_e4m3.argtypes = [ctypes.c_float]
        L.oracle_f32_to_e4m3.restype = ctypes.c_uint8
        L.oracle_deq.argtypes = [_P, _P, ctypes.c_float, _P, _L, _L, ctypes.c_int]
        L.oracle_block_deq.argtypes = [_P, _P, _P, _P, _P]
        L.oracle_moe_decode.argtypes = [_P, _P, _P, _P, _P, ctypes.c_int, _P, _P]
        L.oracle_to_fp8_rows.argtypes = [_P, _L, _L, _P, _P]
        L.oracle_gemv.argtypes = [_P, _P, _P, _L, _L, _P]
        L.oracle_moe_prefill.argtypes = [_P, _L, _P, _P, ctypes.c_int, _P, _L, _P, ctypes.c_int, _P]
        L.oracle_route.argtypes = [_P, _L, ctypes.c_int, ctypes.c_int, _P, _P]
        for f in ("oracle_deq", "oracle_block_deq", "oracle_moe_decode", "oracle_to_fp8_rows",
                  "oracle_gemv", "oracle_moe_prefill", "oracle_route"):
            getattr(L, f).restype = None
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def threads(n=0):
    """Set (n > 0) and return the OpenMP thread count the oracle uses."""
    return lib().oracle_threads(int(n))


def e4m3_to_f32(b):
    return lib().oracle_e4m3_to_f32(int(b))


def e4m3_decode_table():
    return np.array([e4m3_to_f32(b) for b in range(256)], dtype=np.float32)


def f32_to_e4m3(v):
    v = _c(v, np.float32).ravel()
    return np.array([lib().oracle_f32_to_e4m3(float(t)) for t in v], dtype=np.uint8)


def deq(w_u8, s_u8, ws2, swap=False):
    """qmoe.deq: u8[N,K/2], u8[N,K/16], float -> f32[N,K]."""
    w_u8, s_u8 = _c(w_u8, np.uint8), _c(s_u8, np.uint8)
    N, K = w_u8.shape[0], w_u8.shape[1] * 2
    out = np.empty((N, K), np.float32)
    lib().oracle_deq(_p(w_u8), _p(s_u8), float(ws2), _p(out), N, K, int(bool(swap)))
    return out


def block_deq(blk, s2):
    """qmoe.block_deq: u8[BLOCK], f32[3] -> gate f32[640,2560], up, down f32[2560,640]."""
    blk, s2 = _c(blk, np.uint8), _c(s2, np.float32)
    assert blk.size == BLOCK
    g = np.empty((INTER, HID), np.float32)
    u = np.empty((INTER, HID), np.float32)
    d = np.empty((HID, INTER), np.float32)
    lib().oracle_block_deq(_p(blk), _p(s2), _p(g), _p(u), _p(d))
    return g, u, d


def moe_decode(table, sidx, s2, coef, x, return_h=False):
    """tests/test_qmoe.py:24-28 reference: f32[2560] (and h f32[K,640])."""
    table = _c(table, np.uint8)
    sidx, s2, coef = _c(sidx, np.int32), _c(s2, np.float32), _c(coef, np.float32)
    x = _c(x, np.float32)
    K = sidx.size
    out = np.empty(HID, np.float32)
    h = np.empty((K, INTER), np.float32)
    lib().oracle_moe_decode(_p(table), _p(sidx), _p(s2), _p(coef), _p(x), K, _p(out), _p(h))
    return (out, h) if return_h else out


def to_fp8_rows(w):
    """qwen_engine.to_fp8_rows on fp32 input: (e4m3 bytes u8[N,K], f32[N])."""
    w = _c(w, np.float32)
    N, K = w.shape
    q = np.empty((N, K), np.uint8)
    s = np.empty(N, np.float32)
    lib().oracle_to_fp8_rows(_p(w), N, K, _p(q), _p(s))
    return q, s


def gemv(q, s, x):
    """tests/test_gemv.py:9: (q.float()*s) @ x.float() -> f32[N]."""
    q, s, x = _c(q, np.uint8), _c(s, np.float32), _c(x, np.float32)
    N, K = q.shape
    y = np.empty(N, np.float32)
    lib().oracle_gemv(_p(q), _p(s), _p(x), N, K, _p(y))
    return y


def moe_prefill(x, ti, tv, table, base, s2l):
    """qwen_engine.py:835-852 expert loop: f32[T,2560]."""
    x = _c(x, np.float32)
    ti, tv = _c(ti, np.int32), _c(tv, np.float32)
    table, s2l = _c(table, np.uint8), _c(s2l, np.float32)
    T, topk = ti.shape
    out = np.empty((T, HID), np.float32)
    lib().oracle_moe_prefill(_p(x), T, _p(ti), _p(tv), topk, _p(table), int(base), _p(s2l),
                             s2l.shape[0], _p(out))
    return out


def route(logits, topk=10):
    """qwen_engine.py:803-806 on fp32 logits: (ti int32[T,topk], coef f32[T,topk] = bf16 values)."""
    logits = _c(logits, np.float32)
    if logits.ndim == 1:
        logits = logits[None]
    T, E = logits.shape
    ti = np.empty((T, topk), np.int32)
    coef = np.empty((T, topk), np.float32)
    lib().oracle_route(_p(logits), T, E, topk, _p(ti), _p(coef))
    return ti, coef


def bf16_round(a):
    """fp32 -> nearest-even bf16, returned as fp32 (torch's .to(bfloat16))."""
    a = _c(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    nan = np.isnan(a)
    out = r.view(np.float32).copy()
    out[nan] = np.nan
    return out


def e4m3_rows_to_bf16(q, s):
    """qwen_engine.py:83 weight expression, (q.to(bf16) * s).to(bf16), as bf16
    bit patterns u16[N,K]: e4m3 -> fp32 (exact), one fp32 multiply by the row
    scale (round to nearest even), fp32 -> bf16 (round to nearest even)."""
    q, s = _c(q, np.uint8), _c(s, np.float32).reshape(-1)
    w = e4m3_decode_table()[q] * s[:, None]          # numpy float32 multiply: IEEE, nearest even
    return (bf16_round(w).view(np.uint32) >> 16).astype(np.uint16)


def fp8_linear(x, q, s):
    """Lin.__call__ for T > 1 (qwen_engine.py:83) in fp32: x [T,K] @ w_bf16.T -> f32[T,N]
    (the caller rounds to bf16; the GPU GEMM's accumulation order differs)."""
    w = (e4m3_rows_to_bf16(q, s).astype(np.uint32) << 16).view(np.float32)
    return _c(x, np.float32) @ w.T


def router_logits(x, w):
    """F.linear(x, Ld["router"]) of qwen_engine.py:803 in bf16: x [T, H], w [E, H]
    (bf16 values as fp32) -> fp32 [T, E] holding the bf16 rounding of the exact
    dot products (fp64 sums; the GPU's fp32 summation order can land one bf16
    step away when a sum lies next to a rounding boundary)."""
    return bf16_round((_c(x, np.float64) @ _c(w, np.float64).T).astype(np.float32))


def _silu(v):
    return (v / (np.float32(1.0) + np.exp(-v, dtype=np.float32))).astype(np.float32)


def shared_expert(x, wg, wu, wd, wsg, y=None):
    """The shared expert of qwen_engine.py:817-818 (and the combine of :829)
    with bf16 tensors, every step rounded to bf16 where the reference's bf16
    tensors round it; dot products exact (fp64) before their bf16 rounding.
      g = bf16(x.Wg), u = bf16(x.Wu), a = bf16(silu(g)), h = bf16(a * u),
      d = bf16(h.Wd), gt = bf16(sigmoid(bf16(x.wsg))), sh = bf16(gt * d),
      out = bf16(bf16(y) + sh) if y is given, else sh.
    All arguments hold bf16 values as fp32 (y: fp32)."""
    x = _c(x, np.float64)
    g = bf16_round((x @ _c(wg, np.float64).T).astype(np.float32))
    u = bf16_round((x @ _c(wu, np.float64).T).astype(np.float32))
    a = bf16_round(_silu(g))
    h = bf16_round(a * u)
    d = bf16_round((h.astype(np.float64) @ _c(wd, np.float64).T).astype(np.float32))
    z = bf16_round((x @ _c(wsg, np.float64).reshape(-1, 1)).astype(np.float32))
    gt = bf16_round((np.float32(1.0) / (np.float32(1.0) + np.exp(-z, dtype=np.float32))).astype(np.float32))
    sh = bf16_round(gt * d)
    if y is None:
        return sh
    return bf16_round(bf16_round(_c(y, np.float32)) + sh)


def deltanet_step(q, k, v, g, beta, S):
    """recurrent_gated_delta_rule at T == 1 (qwen_engine.py:158-174) in fp64,
    the state updated in place and the output rounded to bf16.
    q, k [Hk, dk]; v [H, dv]; g, beta [H]; S [H, dk, dv] float64 (in/out);
    value head h uses key head h // (H // Hk) (repeat_interleave, :717).
    Returns out [H, dv] (bf16 values as fp32)."""
    q, k = np.asarray(q, np.float64), np.asarray(k, np.float64)
    H, dk = S.shape[0], S.shape[1]
    r = H // q.shape[0]
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6) / np.sqrt(dk)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    out = np.empty((H, S.shape[2]), np.float64)
    for h in range(H):
        qh, kh = q[h // r], k[h // r]
        S[h] *= np.exp(np.float64(g[h]))
        delta = (np.asarray(v[h], np.float64) - kh @ S[h]) * np.float64(beta[h])
        S[h] += np.outer(kh, delta)
        out[h] = qh @ S[h]
    return bf16_round(out.astype(np.float32))
