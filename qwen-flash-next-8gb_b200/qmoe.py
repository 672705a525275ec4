"""Drop-in replacement for the reference's `qmoe` module on B200 (sm_100a).

Same names, constants and call signatures as qmoe.py of the reference, so
qwen_engine.py, its tests and tools import this module unchanged when this
directory comes first on sys.path.  All arithmetic runs in libqfn's CUDA
kernels (csrc/decode.cu, csrc/deq.cu); there is no Triton and no CPU path.

Layout of one repacked expert block (qmoe.py:9-14, repack_experts.py:12-19):
gate_w u8[640,1280] | up_w | down_w u8[2560,320] | gate_s e4m3[640,160] |
up_s | down_s e4m3[2560,40], 2,764,800 bytes.
"""
import ctypes

import torch

from _lib import DTYPE_BF16, DTYPE_F32, check, lib, ops, require_cuda, on_device, stream_of

HID, INTER = 2560, 640
BLOCK = 2764800
O_GW, O_UW, O_DW = 0, 819200, 1638400
O_GS, O_US, O_DS = 2457600, 2560000, 2662400
KB_UP, G_UP = HID // 2, HID // 16          # bytes and scale groups per gate/up row (1280, 160)
KB_DN, G_DN = INTER // 2, INTER // 16      # per down row (320, 40)
MAX_TOPK = 32

# e2m1 code -> value (qmoe.py:87); bit 3 is the sign.
E2M1 = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=torch.float32)

# The reference's nibble-order negative control (qmoe.py:90).  The CUDA path
# implements only the true order; the swapped order lives in the CPU oracle.
SWAP = False


def moe_decode(slots_u8, sidx, s2, coef, x, h_buf, out_buf):
    """bs=1 NVFP4 SwiGLU over K experts + weighted combine (qmoe.py:77-83).

    slots_u8 u8[S, BLOCK] (slot table or the HBM-resident expert table) . sidx
    int32[K] (block index of expert j) . s2 f32[K,3] (ws2 gate/up/down) .
    coef f32[K] (router weight) . x [2560] bf16/fp32 . h_buf f32[>=K,640]
    scratch (holds h on return) . out_buf f32[>=K,2560] (accepted for
    signature compatibility; the combine is fused so it is not written)
    -> new fp32 [2560] = sum_j coef_j * down_j(silu(gate_j x) * up_j x).
    Queued on torch's current stream; graph-capturable.
    """
    return _moe_decode(slots_u8, sidx, s2, coef, x, h_buf, 0)


# kernel paths of qfn_moe_decode_variant (1 and 3 were earlier paths, since removed)
VARIANT_AUTO, VARIANT_CUDA_CORE, VARIANT_SLICE = 0, 2, 4


def _moe_decode(slots_u8, sidx, s2, coef, x, h_buf, variant):
    """moe_decode with an explicit kernel path (tests / measurements): one call
    of the torch operator qfn::moe_decode (libqfn_torch.so -> qfn_moe_decode_variant),
    which checks the tensors and launches on torch's current stream."""
    return ops().moe_decode(slots_u8, sidx, s2, coef, x, h_buf, variant)


def moe_prefill(x, ti, tv, table, s2, L=0):
    """Batched-prefill MoE experts of one layer (the loop at qwen_engine.py:835-852).

    x bf16[T, 2560] . ti int64/int32[T, topk] expert ids of the layer . tv
    bf16/fp32[T, topk] routing weights . table u8[NB, BLOCK] (the HBM-resident
    expert table; expert e of layer L is block L * n_experts + e) . s2
    f32[n_experts, 3] ws2 of the layer's experts (store.s2[L]) -> new fp32
    [T, 2560] = sum_k tv[t,k] * down_e(silu(gate_e x_t) * up_e x_t), the
    reference's `out` before its cast to bf16.  One call replaces the whole
    per-expert loop (and its host syncs): grouped tcgen05 GEMMs on the GPU.
    Queued on torch's current stream; graph-capturable (the torch operator
    qfn::moe_prefill allocates its workspace from torch's caching allocator).
    """
    return ops().moe_prefill(x, ti, tv, table, s2, int(L))


def deq(w_u8, s_e4m3_u8, ws2):
    """w_u8 [N, K/2] . s [N, K/16] (E4M3 bytes) . ws2 -> fp32 [N, K] (qmoe.py:93-102), on the GPU."""
    if SWAP:
        raise NotImplementedError("qmoe.SWAP (nibble-order negative control) exists only in the CPU oracle")
    require_cuda("w_u8", w_u8, torch.uint8)
    require_cuda("s_e4m3_u8", s_e4m3_u8)
    if s_e4m3_u8.dtype not in (torch.uint8, torch.float8_e4m3fn):
        raise TypeError("s must hold E4M3 bytes (uint8 or float8_e4m3fn)")
    N, KB = w_u8.shape
    K = 2 * KB
    if tuple(s_e4m3_u8.shape) != (N, K // 16):
        raise ValueError(f"s must be [{N}, {K // 16}], got {tuple(s_e4m3_u8.shape)}")
    out = torch.empty(N, K, dtype=torch.float32, device=w_u8.device)
    with on_device(w_u8.device):
        rc = lib().qfn_deq(w_u8.data_ptr(), s_e4m3_u8.data_ptr(), float(ws2), out.data_ptr(), N, K,
                           stream_of(out))
    check(rc, "qfn_deq")
    return out


def block_deq(blk_u8, s2):
    """repacked block (u8 [BLOCK]) -> gate [640,2560], up [640,2560], down [2560,640] fp32 (qmoe.py:105-111)."""
    require_cuda("blk_u8", blk_u8, torch.uint8)
    if blk_u8.numel() != BLOCK:
        raise ValueError(f"blk_u8 must hold {BLOCK} bytes")
    vals = [float(v) for v in (s2.tolist() if isinstance(s2, torch.Tensor) else s2)][:3]
    dev = blk_u8.device
    g = torch.empty(INTER, HID, dtype=torch.float32, device=dev)
    u = torch.empty(INTER, HID, dtype=torch.float32, device=dev)
    d = torch.empty(HID, INTER, dtype=torch.float32, device=dev)
    s2c = (ctypes.c_float * 3)(*vals)
    with on_device(dev):
        rc = lib().qfn_block_deq(blk_u8.data_ptr(), ctypes.addressof(s2c), g.data_ptr(), u.data_ptr(),
                                 d.data_ptr(), stream_of(g))
    check(rc, "qfn_block_deq")
    return g, u, d
