"""Router of the MoE block (qwen_engine.py:803-806), in torch ops on the
caller's device: softmax in fp32, top-k, renormalise over the k, round the
weights to the engine's activation dtype (bf16).  The expert kernels consume
(block index, fp32 coefficient) pairs; `coef` is the bf16 weight as fp32,
exactly what the engine passes to moe_decode (qwen_engine.py:825).
"""
import torch
import torch.nn.functional as F


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
