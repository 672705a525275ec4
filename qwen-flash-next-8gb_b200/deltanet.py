"""One-token gated delta rule of the DeltaNet layers on B200 (libqfn's
qfn_deltanet_step): a drop-in for qwen_engine.recurrent_gated_delta_rule at
T == 1 (qwen_engine.py:158-174), the call QwenEngine.deltanet makes for every
linear-attention layer of every decoded token (qwen_engine.py:718-719).
"""
import torch

from _lib import check, lib, on_device, require_cuda, stream_of


def recurrent_gated_delta_rule(query, key, value, g, beta, initial_state):
    """query, key [1, 1, Hq, dk] bf16 (Hq = H, the engine's repeated heads, or the
    H / r key heads) . value [1, 1, H, dv] bf16 . g [1, 1, H] fp32 . beta [1, 1, H]
    bf16 . initial_state [1, H, dk, dv] fp32 -> (out [1, 1, H, dv] bf16, S).

    S is initial_state updated in place (the engine stores the returned state,
    st["S"] = S, so the in-place update is what it keeps)."""
    for name, t, dt in (("query", query, torch.bfloat16), ("key", key, torch.bfloat16),
                        ("value", value, torch.bfloat16), ("beta", beta, torch.bfloat16),
                        ("g", g, torch.float32), ("initial_state", initial_state, torch.float32)):
        require_cuda(name, t, dt)
    if query.dim() != 4 or query.shape[0] != 1 or query.shape[1] != 1:
        raise ValueError(f"query must be [1, 1, heads, dk] (one token), got {tuple(query.shape)}")
    Hq, dk = query.shape[2], query.shape[3]
    H, dv = value.shape[2], value.shape[3]
    if tuple(key.shape) != tuple(query.shape) or value.shape[:2] != (1, 1) or H % Hq:
        raise ValueError("key must match query; value [1, 1, H, dv] with H a multiple of query's heads")
    if g.numel() != H or beta.numel() != H or tuple(initial_state.shape) != (1, H, dk, dv):
        raise ValueError(f"g, beta [1, 1, {H}] and initial_state [1, {H}, {dk}, {dv}] expected")
    out = torch.empty(1, 1, H, dv, dtype=torch.bfloat16, device=query.device)
    with on_device(query.device):
        rc = lib().qfn_deltanet_step(query.data_ptr(), key.data_ptr(), value.data_ptr(), g.data_ptr(),
                                     beta.data_ptr(), initial_state.data_ptr(), out.data_ptr(), H, Hq, dk, dv,
                                     stream_of(out))
    check(rc, "qfn_deltanet_step")
    return out, initial_state
