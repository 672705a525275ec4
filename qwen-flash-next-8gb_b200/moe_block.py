"""The decode MoE block of QwenEngine.moe (qwen_engine.py:801-831) on the device
with no host synchronisation:

    router (qfn_moe_route) -> routed experts (qfn_moe_decode)
    -> shared expert down + combine (qfn_shared_expert_down)
    with the shared expert's gate/up (qfn_shared_expert_gate_up) on a side stream

The reference runs the router as torch ops, reads the chosen experts back
to the host (ti[0].tolist(), qwen_engine.py:812/815) to drive its expert
cache, computes the shared expert with bf16 F.linear calls and adds the two
in bf16.  With every expert resident in HBM the expert indices never need
to leave the GPU: the fused router writes the decode kernel's arguments
directly, so a whole 48-layer MoE step can be one CUDA graph.
"""
import torch

import qmoe
import routing
from _lib import check, lib, on_device, require_cuda, stream_of


def shared_expert(x, w_gate, w_up, w_down, w_sg, y=None, out=None, h=None, gt=None):
    """sigmoid(x . w_sg) * w_down(silu(w_gate x) * w_up x) [+ bf16(y)] -> bf16 [T, 2560].

    x bf16 [T, 2560] . w_gate, w_up bf16 [I, 2560] . w_down bf16 [2560, I] .
    w_sg bf16 [1, 2560] (Ld["sh_g"]) . y fp32 [T, 2560] (the routed experts'
    output) or None.  h / gt / out: optional preallocated scratch and output."""
    for name, t in (("x", x), ("w_gate", w_gate), ("w_up", w_up), ("w_down", w_down), ("w_sg", w_sg)):
        require_cuda(name, t, torch.bfloat16)
    if x.dim() == 1:
        x = x[None]
    T, I = x.shape[0], w_gate.shape[0]
    if x.shape[1] != 2560 or tuple(w_gate.shape) != (I, 2560) or tuple(w_up.shape) != (I, 2560) \
            or tuple(w_down.shape) != (2560, I) or w_sg.numel() != 2560:
        raise ValueError("shapes: x [T, 2560], w_gate/w_up [I, 2560], w_down [2560, I], w_sg [1, 2560]")
    if y is not None:
        require_cuda("y", y, torch.float32)
        if y.numel() != T * 2560:
            raise ValueError(f"y must hold {T} x 2560 values")
    dev = x.device
    h = torch.empty(T, I, dtype=torch.bfloat16, device=dev) if h is None else h
    gt = torch.empty(T, dtype=torch.bfloat16, device=dev) if gt is None else gt
    out = torch.empty(T, 2560, dtype=torch.bfloat16, device=dev) if out is None else out
    with on_device(dev):
        rc = lib().qfn_shared_expert(x.data_ptr(), T, w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(),
                                     w_sg.data_ptr(), I, None if y is None else y.data_ptr(), h.data_ptr(),
                                     gt.data_ptr(), out.data_ptr(), stream_of(x))
    check(rc, "qfn_shared_expert")
    return out


class DecodeMoE:
    """One decode MoE block per call, on preallocated buffers (graph-capturable).

    layer weights: router bf16 [E, 2560]; shared expert (w_gate, w_up, w_down,
    w_sg) bf16; the HBM-resident expert table (expert_table.ExpertTable)."""

    def __init__(self, table, topk=10, max_tokens=1):
        self.table, self.topk = table, topk
        dev, E = table.slots.device, table.n_experts
        T = max_tokens
        self.route_buf = {
            "ti": torch.empty(T, topk, dtype=torch.int32, device=dev),
            "tv": torch.empty(T, topk, dtype=torch.bfloat16, device=dev),
            "logits": torch.empty(T, E, dtype=torch.bfloat16, device=dev),
            "sidx": torch.empty(T, topk, dtype=torch.int32, device=dev),
            "coef": torch.empty(T, topk, dtype=torch.float32, device=dev),
            "s2": torch.empty(T, topk, 3, dtype=torch.float32, device=dev),
        }
        self.side = None
        self.h_buf = torch.empty(topk, 640, dtype=torch.float32, device=dev)
        self.o_buf = torch.empty(topk, 2560, dtype=torch.float32, device=dev)
        self.sh_gt = torch.empty(T, dtype=torch.bfloat16, device=dev)
        self.sh_h = {}

    def __call__(self, x, layer, router, w_gate, w_up, w_down, w_sg, out=None):
        """x bf16 [1, 2560] (the MoE input of one token) -> bf16 [1, 2560] =
        moe_decode(routed experts).to(bf16) + shared expert (qwen_engine.py:801-829).

        The shared expert's gate/up half does not depend on the routing: it
        runs on a side stream while the router and the routed experts run on
        the caller's stream.  Its down half follows the routed experts on the
        caller's stream and applies the reference's combine,
        y.to(bf16) + sh (qwen_engine.py:829), in the same kernel."""
        if x.dim() != 2 or x.shape[0] != 1:
            raise ValueError("DecodeMoE takes one token: x [1, 2560]")
        for name, t in (("x", x), ("w_gate", w_gate), ("w_up", w_up), ("w_down", w_down), ("w_sg", w_sg)):
            require_cuda(name, t, torch.bfloat16)
        I = w_gate.shape[0]
        if tuple(w_gate.shape) != (I, 2560) or tuple(w_up.shape) != (I, 2560) or tuple(w_down.shape) != (2560, I) \
                or w_sg.numel() != 2560:
            raise ValueError("shapes: w_gate/w_up [I, 2560], w_down [2560, I], w_sg [1, 2560]")
        dev = x.device
        h = self.sh_h.get(I)
        if h is None:
            h = self.sh_h[I] = torch.empty(1, I, dtype=torch.bfloat16, device=dev)
        out = torch.empty(1, 2560, dtype=torch.bfloat16, device=dev) if out is None else out
        cur = torch.cuda.current_stream(dev)
        if self.side is None:
            self.side = torch.cuda.Stream(dev)
        self.side.wait_stream(cur)
        with on_device(dev):
            check(lib().qfn_shared_expert_gate_up(x.data_ptr(), 1, w_gate.data_ptr(), w_up.data_ptr(),
                                                  w_sg.data_ptr(), I, h.data_ptr(), self.sh_gt.data_ptr(),
                                                  self.side.cuda_stream), "qfn_shared_expert_gate_up")
            r = routing.route_fused(x, router, self.topk, layer, self.table.s2, out=self.route_buf)
            y = qmoe.moe_decode(self.table.slots, r["sidx"][0], r["s2"][0], r["coef"][0], x[0], self.h_buf,
                                self.o_buf)
            cur.wait_stream(self.side)
            check(lib().qfn_shared_expert_down(w_down.data_ptr(), I, 1, h.data_ptr(), self.sh_gt.data_ptr(),
                                               y.data_ptr(), out.data_ptr(), cur.cuda_stream),
                  "qfn_shared_expert_down")
        return out
