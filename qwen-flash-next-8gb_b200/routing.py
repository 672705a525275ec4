"""Router of the MoE block (qwen_engine.py:803-806): softmax in fp32, top-k,
renormalise over the k, round the weights to the engine's activation dtype
(bf16).  The expert kernels consume (block index, fp32 coefficient) pairs;
`coef` is the bf16 weight as fp32, exactly what the engine passes to
moe_decode (qwen_engine.py:825).

route() is the reference's torch expression on given logits (used to make
benchmark inputs); route_fused() is libqfn's fused router (qfn_moe_route):
the router GEMV, softmax, top-k, renormalisation and the decode kernel's
arguments in two launches on the device, with no host synchronisation.
"""
import torch
import torch.nn.functional as F

from _lib import check, lib, on_device, require_cuda, stream_of


@torch.no_grad()
def route(logits, topk=10, weight_dtype=torch.bfloat16):
    """logits [T, E] -> (ti int64 [T, topk], tv weight_dtype [T, topk])."""
    probs = F.softmax(logits, dtype=torch.float, dim=-1)
    tv, ti = torch.topk(probs, topk, dim=-1)
    tv = (tv / tv.sum(-1, keepdim=True)).to(weight_dtype)
    return ti, tv


@torch.no_grad()
def decode_args(ti_row, tv_row, layer, n_experts, s2_table):
    """One token's routing -> (sidx int32[K], s2 f32[K,3], coef f32[K]) for
    moe_decode on the HBM-resident table, computed on the device (no host
    synchronisation): sidx = layer * n_experts + e."""
    sidx = (ti_row + layer * n_experts).to(torch.int32)
    return sidx, s2_table[layer, ti_row], tv_row.float()


def route_fused(x, w_router, topk=10, layer=0, s2_table=None, out=None):
    """x bf16 [T, 2560] . w_router bf16 [E, 2560] (Ld["router"]) -> dict of device tensors:
    ti int32 [T, topk], tv bf16 [T, topk], logits bf16 [T, E] (the reference's
    F.linear output), and the decode arguments sidx int32 [T, topk] = layer * E +
    ti, coef f32 [T, topk] = tv, s2 f32 [T, topk, 3] = s2_table[layer, ti] (with
    s2_table f32 [L, E, 3]).  `out` (a dict of preallocated tensors of those
    shapes) makes the call allocation-free, e.g. inside a captured CUDA graph."""
    require_cuda("x", x, torch.bfloat16)
    require_cuda("w_router", w_router, torch.bfloat16)
    if x.dim() == 1:
        x = x[None]
    if x.dim() != 2 or x.shape[1] != 2560 or w_router.dim() != 2 or w_router.shape[1] != 2560:
        raise ValueError(f"x must be [T, 2560] and w_router [E, 2560]; got {tuple(x.shape)}, {tuple(w_router.shape)}")
    if w_router.device != x.device:
        raise ValueError(f"w_router is on {w_router.device}, x on {x.device}")
    T, E = x.shape[0], w_router.shape[0]
    dev = x.device
    o = out if out is not None else {
        "ti": torch.empty(T, topk, dtype=torch.int32, device=dev),
        "tv": torch.empty(T, topk, dtype=torch.bfloat16, device=dev),
        "logits": torch.empty(T, E, dtype=torch.bfloat16, device=dev),
        "sidx": torch.empty(T, topk, dtype=torch.int32, device=dev),
        "coef": torch.empty(T, topk, dtype=torch.float32, device=dev),
    }
    s2l = None
    if s2_table is not None:
        require_cuda("s2_table", s2_table, torch.float32)
        if s2_table.dim() != 3 or s2_table.shape[1] != E or s2_table.shape[2] != 3:
            raise ValueError(f"s2_table must be f32[L, {E}, 3]")
        s2l = s2_table[layer]
        if "s2" not in o:
            o["s2"] = torch.empty(T, topk, 3, dtype=torch.float32, device=dev)
    with on_device(dev):
        rc = lib().qfn_moe_route(x.data_ptr(), w_router.data_ptr(), T, E, topk, int(layer) * E,
                                 None if s2l is None else s2l.data_ptr(), o["ti"].data_ptr(), o["tv"].data_ptr(),
                                 o["sidx"].data_ptr(), o["coef"].data_ptr(),
                                 None if s2l is None else o["s2"].data_ptr(), o["logits"].data_ptr(), stream_of(x))
    check(rc, "qfn_moe_route")
    return o
