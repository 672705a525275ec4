"""Generate the golden vectors in tests/golden/ by running the reference itself.

Run in a container where the reference project is importable (its root given
by QFN_REFERENCE); the fixtures are committed so the tests never need it:

    QFN_REFERENCE=/path/to/reference python tests/golden/make_golden.py

Inputs come from the package's seeded generators (synthetic.py), so the tests
regenerate the same inputs and compare against the recorded outputs.
Outputs of pure elementwise reference code (e4m3 decode, deq, block_deq,
to_fp8_rows) are recorded as SHA-256 of their bytes and checked bit-exactly;
outputs that go through torch's CPU matmul (whose summation order is its own)
are stored as arrays and checked with a tolerance.
"""
import hashlib
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("QFN_REFERENCE")
if not REF or not os.path.exists(os.path.join(REF, "qmoe.py")):
    sys.exit("set QFN_REFERENCE to the reference project root")
sys.path.insert(0, REF)
import qmoe  # noqa: E402  (the reference's module)
from qwen_engine import recurrent_gated_delta_rule, to_fp8_rows  # noqa: E402

spec = importlib.util.spec_from_file_location("synthetic", os.path.join(REPO, "qwen-flash-next-8gb_b200",
                                                                      "synthetic.py"))
synthetic = importlib.util.module_from_spec(spec)
spec.loader.exec_module(synthetic)

torch.set_num_threads(os.cpu_count())


def canon(a):
    a = np.array(a, dtype=np.float32, copy=True)
    a[np.isnan(a)] = np.float32("nan")
    return a


def sha(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float32:
        a = canon(a)
    return hashlib.sha256(a.tobytes()).hexdigest()


def save(name, a):
    np.save(os.path.join(HERE, name + ".npy"), a)


def ref_route(logits, topk=10):
    """qwen_engine.py:803-806 with the weights rounded to bf16 as the engine's bf16 logits imply."""
    probs = torch.nn.functional.softmax(logits, dtype=torch.float, dim=-1)
    tv, ti = torch.topk(probs, topk, dim=-1)
    tv = (tv / tv.sum(-1, keepdim=True)).to(torch.bfloat16)
    return ti, tv


def deltanet_golden(C):
    steps, H, Hk, dk, dv, seed = 8, 4, 2, 128, 128, 71
    q, k, v, g, beta, S = synthetic.deltanet_inputs(steps, H, Hk, dk, dv, seed)
    S = S[None].clone()
    outs = []
    for t in range(steps):
        qr = q[t].repeat_interleave(H // Hk, dim=0)[None, None]
        kr = k[t].repeat_interleave(H // Hk, dim=0)[None, None]
        o, S = recurrent_gated_delta_rule(qr, kr, v[t][None, None], g[t][None, None], beta[t][None, None], S)
        outs.append(o[0, 0].float().numpy())
    save("deltanet_out", np.stack(outs))
    save("deltanet_state", S[0].numpy())
    C["deltanet"] = {"steps": steps, "heads": H, "key_heads": Hk, "dk": dk, "dv": dv, "seed": seed}


def main():
    meta = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__, "cases": {}}
    C = meta["cases"]

    # 1. e4m3 decode of all 256 bytes (torch.float8_e4m3fn view, qmoe.py:101)
    tab = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    save("e4m3_table", tab)
    C["e4m3_table"] = {"sha256": sha(tab)}

    # 2. to_fp8_rows (qwen_engine.py:59-64) on N(0,.02) bf16 rows plus edge rows
    w = synthetic.gemv_weights(64, 512, seed=11).float()
    edge = torch.zeros(8, 512)
    grid = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    finite = grid[torch.isfinite(grid) & (grid >= 0)].sort().values      # 0 .. 448
    mids = (finite[1:] + finite[:-1]) / 2                                  # exact ties
    edge[0, : mids.numel()] = mids; edge[0, -1] = 448.0                     # s = 1 -> ties to even
    edge[1, : mids.numel()] = -mids; edge[1, -1] = -448.0
    edge[2, : finite.numel()] = finite * 0.37; edge[2, -1] = 448.0 * 0.37   # non power-of-two scale
    edge[3] = torch.linspace(-1e-3, 1e-3, 512); edge[3, 0] = 3.0            # many subnormal q
    # row 4 stays zero: amax = 0 -> s = 1e-12
    edge[5] = torch.from_numpy(np.random.Generator(np.random.PCG64(12)).standard_normal(512).astype(np.float32))
    edge[6, ::2] = 1e-30; edge[6, 1] = 1.0
    edge[7] = mids[-8:].repeat(64)                                          # near the top of the range
    wq = torch.cat([w, edge])
    q, s = to_fp8_rows(wq)
    save("fp8rows_w", wq.numpy())
    C["to_fp8_rows"] = {"q_sha256": sha(q.view(torch.uint8).numpy()), "s_sha256": sha(s.view(-1).numpy())}

    # 3. deq over every (weight byte, scale byte) pair, and the SWAP control (qmoe.py:90-102)
    wb = np.tile(np.arange(256, dtype=np.uint8), (256, 1))                 # [256, 256] -> K = 512
    sb = np.repeat(np.arange(256, dtype=np.uint8)[:, None], 32, axis=1)      # row n uses scale byte n
    ws2 = 0.37
    d = qmoe.deq(torch.from_numpy(wb), torch.from_numpy(sb), ws2).numpy()
    qmoe.SWAP = True
    d_swap = qmoe.deq(torch.from_numpy(wb), torch.from_numpy(sb), ws2).numpy()
    qmoe.SWAP = False
    C["deq_all"] = {"ws2": ws2, "sha256": sha(d), "swap_sha256": sha(d_swap)}

    # 4. block_deq of one synthetic block (qmoe.py:105-111)
    blk = synthetic.make_blocks(1, seed=21)[0]
    s2 = synthetic.make_s2(1, seed=22, spread=True)[0]
    g, u, dd = qmoe.block_deq(torch.from_numpy(blk), torch.from_numpy(s2))
    C["block_deq"] = {"block_seed": 21, "s2_seed": 22, "gate_sha256": sha(g.numpy()),
                      "up_sha256": sha(u.numpy()), "down_sha256": sha(dd.numpy())}

    # 5. moe_decode reference of tests/test_qmoe.py:21-28 (fp32, torch CPU)
    def moe_ref(slots, sidx, s2k, coef, x):
        ref = torch.zeros(2560)
        hs = []
        for j in range(len(sidx)):
            g, u, d = qmoe.block_deq(slots[sidx[j]], s2k[j])
            h = torch.nn.functional.silu(g @ x.float()) * (u @ x.float())
            hs.append(h)
            ref += coef[j] * (d @ h)
        return ref.numpy(), torch.stack(hs).numpy()

    slots = torch.from_numpy(synthetic.make_blocks(12, seed=31))
    for name, K, xdt, xseed in (("moe_decode_k10_bf16", 10, torch.bfloat16, 33),
                                ("moe_decode_k3_f32", 3, torch.float32, 34)):
        sidx = list(range(2, 2 + K)) if K == 10 else [11, 0, 5]
        s2k = torch.from_numpy(synthetic.make_s2(K, seed=32 + K, spread=True))
        coef = torch.from_numpy(np.random.Generator(np.random.PCG64(35 + K)).random(K).astype(np.float32))
        x = synthetic.make_x(2560, seed=xseed, std=0.5, dtype=xdt)
        out, h = moe_ref(slots, sidx, s2k, coef, x)
        save(name + "_out", out)
        save(name + "_h", h)
        C[name] = {"table_seed": 31, "n_blocks": 12, "sidx": sidx, "s2_seed": 32 + K, "coef_seed": 35 + K,
                   "x_seed": xseed, "x_dtype": str(xdt).replace("torch.", ""), "x_std": 0.5}

    # 6. gemv reference of tests/test_gemv.py:6-9 on small and benchmark shapes
    for N, K, seed in ((256, 512, 61), (12288, 2560, 62), (2560, 4096, 63)):
        wg = synthetic.gemv_weights(N, K, seed)
        q, s = to_fp8_rows(wg)
        s = s.view(-1)
        x = synthetic.make_x(K, seed=seed + 100)
        y = ((q.float() * s[:, None]) @ x.float()).numpy()
        name = f"gemv_{N}x{K}"
        save(name + "_y", y)
        C[name] = {"N": N, "K": K, "w_seed": seed, "x_seed": seed + 100,
                   "q_sha256": sha(q.view(torch.uint8).numpy()), "s_sha256": sha(s.numpy())}

    # 7. routing (qwen_engine.py:803-806) on fp32 logits
    for name, logits in (("route_zipf", synthetic.zipf_logits(64, seed=41)),
                         ("route_normal", synthetic.normal_logits(64, seed=42))):
        ti, tv = ref_route(torch.from_numpy(logits))
        save(name + "_ti", ti.numpy().astype(np.int32))
        save(name + "_coef", tv.float().numpy())
        C[name] = {"seed": 41 if name == "route_zipf" else 42, "rows": 64, "experts": 512, "topk": 10}

    # 8. prefill expert loop of qwen_engine.py:835-852 (16-expert table, top-4, T=8)
    T, E, k = 8, 16, 4
    pt = torch.from_numpy(synthetic.make_blocks(E, seed=51))
    s2l = torch.from_numpy(synthetic.make_s2(E, seed=52, spread=True))
    x = synthetic.make_x(T * 2560, seed=53).view(T, 2560)
    ti, tv = ref_route(torch.from_numpy(synthetic.zipf_logits(T, seed=54, n_experts=E)), k)
    out = torch.zeros(T, 2560, dtype=torch.float32)
    ti_c, tv_c = ti.cpu(), tv.float()
    for e in sorted(set(ti_c.flatten().tolist())):
        tok, slot = torch.where(ti_c == e)
        gw, uw, dw = qmoe.block_deq(pt[e], s2l[e])
        xs = x[tok].float()
        h = torch.nn.functional.silu(xs @ gw.T) * (xs @ uw.T)
        out.index_add_(0, tok, (h @ dw.T) * tv_c[tok, slot, None])
    save("prefill_t8_out", out.numpy())
    save("prefill_t8_ti", ti.numpy().astype(np.int32))
    save("prefill_t8_coef", tv.float().numpy())
    C["prefill_t8"] = {"T": T, "experts": E, "topk": k, "table_seed": 51, "s2_seed": 52, "x_seed": 53,
                       "logit_seed": 54}

    # 9. the one-token gated delta rule (qwen_engine.py:158-174) over 8 steps, the
    #    state carried from step to step; q, k repeated over the value heads as the
    #    engine does (qwen_engine.py:717)
    deltanet_golden(C)

    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", len(C), "cases")


if __name__ == "__main__" and sys.argv[1:] == ["deltanet"]:
    # add only the delta-rule case to an existing golden.json
    with open(os.path.join(HERE, "golden.json")) as f:
        meta = json.load(f)
    deltanet_golden(meta["cases"])
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("added deltanet")
elif __name__ == "__main__":
    main()
