"""Pin the CPU oracle against golden vectors recorded from the reference
itself (tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest
import torch

import oracle
import synthetic
from conftest import bf16_steps, rel_err, sha


def test_e4m3_decode_table_bit_exact(golden):
    ref = golden.load("e4m3_table")
    got = oracle.e4m3_decode_table()
    assert sha(got) == golden.cases["e4m3_table"]["sha256"] == sha(ref)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert np.array_equal(got[fin].view(np.uint32), ref[fin].view(np.uint32))   # incl. -0


def test_to_fp8_rows_bit_exact(golden):
    w = golden.load("fp8rows_w")
    q, s = oracle.to_fp8_rows(w)
    assert sha(q) == golden.cases["to_fp8_rows"]["q_sha256"]
    assert sha(s) == golden.cases["to_fp8_rows"]["s_sha256"]


def _deq_all_inputs():
    wb = np.tile(np.arange(256, dtype=np.uint8), (256, 1))
    sb = np.repeat(np.arange(256, dtype=np.uint8)[:, None], 32, axis=1)
    return wb, sb


def test_deq_every_byte_and_scale_bit_exact(golden):
    c = golden.cases["deq_all"]
    wb, sb = _deq_all_inputs()
    assert sha(oracle.deq(wb, sb, c["ws2"])) == c["sha256"]


def test_deq_swapped_nibbles_negative_control(golden):
    """The reference's SWAP control (qmoe.py:90): swapping the nibble order must
    change the result, and the oracle's swapped path must equal the reference's."""
    c = golden.cases["deq_all"]
    wb, sb = _deq_all_inputs()
    swapped = oracle.deq(wb, sb, c["ws2"], swap=True)
    assert sha(swapped) == c["swap_sha256"]
    assert sha(swapped) != c["sha256"]


def test_block_deq_bit_exact(golden):
    c = golden.cases["block_deq"]
    blk = synthetic.make_blocks(1, seed=c["block_seed"])[0]
    s2 = synthetic.make_s2(1, seed=c["s2_seed"], spread=True)[0]
    g, u, d = oracle.block_deq(blk, s2)
    assert (sha(g), sha(u), sha(d)) == (c["gate_sha256"], c["up_sha256"], c["down_sha256"])


def decode_case(golden, name):
    c = golden.cases[name]
    table = synthetic.make_blocks(c["n_blocks"], seed=c["table_seed"])
    K = len(c["sidx"])
    sidx = np.array(c["sidx"], np.int32)
    s2 = synthetic.make_s2(K, seed=c["s2_seed"], spread=True)
    coef = np.random.Generator(np.random.PCG64(c["coef_seed"])).random(K).astype(np.float32)
    x = synthetic.make_x(2560, seed=c["x_seed"], std=c["x_std"], dtype=getattr(torch, c["x_dtype"]))
    return table, sidx, s2, coef, x


@pytest.mark.parametrize("name", ["moe_decode_k10_bf16", "moe_decode_k3_f32"])
def test_moe_decode_oracle_matches_reference(golden, name):
    table, sidx, s2, coef, x = decode_case(golden, name)
    out, h = oracle.moe_decode(table, sidx, s2, coef, x.float().numpy(), return_h=True)
    assert rel_err(out, golden.load(name + "_out")) < 1e-5
    assert rel_err(h, golden.load(name + "_h")) < 1e-5


@pytest.mark.parametrize("N,K", [(256, 512), (12288, 2560), (2560, 4096)])
def test_gemv_oracle_matches_reference(golden, N, K):
    c = golden.cases[f"gemv_{N}x{K}"]
    w = synthetic.gemv_weights(N, K, c["w_seed"]).float().numpy()
    q, s = oracle.to_fp8_rows(w)
    assert sha(q) == c["q_sha256"] and sha(s) == c["s_sha256"]
    x = synthetic.make_x(K, seed=c["x_seed"]).float().numpy()
    assert rel_err(oracle.gemv(q, s, x), golden.load(f"gemv_{N}x{K}_y")) < 1e-5


@pytest.mark.parametrize("name,gen", [("route_zipf", "zipf"), ("route_normal", "normal")])
def test_route_oracle_matches_reference(golden, name, gen):
    c = golden.cases[name]
    logits = (synthetic.zipf_logits(c["rows"], seed=c["seed"]) if gen == "zipf"
              else synthetic.normal_logits(c["rows"], seed=c["seed"]))
    ti, coef = oracle.route(logits, c["topk"])
    assert np.array_equal(ti, golden.load(name + "_ti"))
    ref = golden.load(name + "_coef")
    # bf16 weights: identical except where fp32 summation order moves a value across a rounding boundary
    ulp = np.abs(ref) * 2.0 ** -7
    assert np.all(np.abs(coef - ref) <= ulp)
    assert np.mean(coef == ref) > 0.99


def test_prefill_oracle_matches_reference(golden):
    c = golden.cases["prefill_t8"]
    table = synthetic.make_blocks(c["experts"], seed=c["table_seed"])
    s2l = synthetic.make_s2(c["experts"], seed=c["s2_seed"], spread=True)
    x = synthetic.make_x(c["T"] * 2560, seed=c["x_seed"]).view(c["T"], 2560).float().numpy()
    ti, coef = oracle.route(synthetic.zipf_logits(c["T"], seed=c["logit_seed"], n_experts=c["experts"]),
                            c["topk"])
    assert np.array_equal(ti, golden.load("prefill_t8_ti"))
    assert np.array_equal(coef, golden.load("prefill_t8_coef"))
    out = oracle.moe_prefill(x, ti, coef, table, 0, s2l)
    assert rel_err(out, golden.load("prefill_t8_out")) < 1e-5


def test_e4m3_rows_to_bf16_matches_reference_expression():
    """oracle.e4m3_rows_to_bf16 against qwen_engine.py:83 itself, executed by
    torch on the CPU: (q.to(bf16) * s).to(bf16), every e4m3 byte, scales from
    the engine's quantizer and extreme ones."""
    g = np.random.default_rng(7)
    q = np.tile(np.arange(256, dtype=np.uint8), (6, 4))                 # every byte, 6 rows x 1024
    w = g.standard_normal((6, 1024)).astype(np.float32) * 0.02
    s = np.concatenate([oracle.to_fp8_rows(w[:3])[1], np.float32([1e-12, 3.7e4, 0.3333333])])
    ref = (torch.from_numpy(q).view(torch.float8_e4m3fn).to(torch.bfloat16)
           * torch.from_numpy(s)[:, None]).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = oracle.e4m3_rows_to_bf16(q, s)
    nan_ref = (ref & 0x7FFF) > 0x7F80
    nan_got = (got & 0x7FFF) > 0x7F80
    assert np.array_equal(nan_ref, nan_got)
    assert np.array_equal(got[~nan_ref], ref[~nan_ref])            # incl. signed zeros and bf16 subnormals


def test_shared_expert_oracle_matches_reference_expression():
    """oracle.shared_expert against the reference's own expression run by torch
    on the CPU with bf16 tensors: sigmoid(F.linear(x, sh_g)) * sh_down(silu(
    sh_gate(x)) * sh_up(x)) (qwen_engine.py:817-818, Lin = F.linear on bf16
    weights, :84) and y.to(bf16) + sh (:829).  torch's CPU GEMMs sum in fp32,
    the oracle exactly, so an element may sit one bf16 step apart; at most a
    few in a thousand do."""
    import torch.nn.functional as F
    rng = np.random.Generator(np.random.PCG64(5))
    T, I = 3, 256
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)
    x, wg, wu = bf(rng.standard_normal((T, 2560))), bf(rng.standard_normal((I, 2560)) * .02), bf(rng.standard_normal((I, 2560)) * .02)
    wd, wsg = bf(rng.standard_normal((2560, I)) * .02), bf(rng.standard_normal((1, 2560)) * .02)
    y = torch.from_numpy(rng.standard_normal((T, 2560)).astype(np.float32))
    sh = F.linear(F.silu(F.linear(x, wg)) * F.linear(x, wu), wd)
    sh = torch.sigmoid(F.linear(x, wsg)) * sh
    ref = (y.to(torch.bfloat16) + sh).float().numpy()
    got = oracle.shared_expert(*(t.float().numpy() for t in (x, wg, wu, wd, wsg)), y.numpy())
    ulp = bf16_steps(got, ref)
    assert ulp.max() <= 2 and (ulp > 0).mean() < 0.01, (ulp.max(), (ulp > 0).mean())


def test_router_logits_oracle_matches_reference_expression():
    """oracle.router_logits against F.linear(x, W_router) in bf16 on the CPU
    (qwen_engine.py:803): equal to within one bf16 step, rarely apart."""
    import torch.nn.functional as F
    rng = np.random.Generator(np.random.PCG64(6))
    x = torch.from_numpy(rng.standard_normal((4, 2560)).astype(np.float32)).to(torch.bfloat16)
    w = torch.from_numpy((rng.standard_normal((512, 2560)) * .02).astype(np.float32)).to(torch.bfloat16)
    ref = F.linear(x, w).float().numpy()
    got = oracle.router_logits(x.float().numpy(), w.float().numpy())
    ulp = bf16_steps(got, ref)
    assert ulp.max() <= 1 and (ulp > 0).mean() < 0.02


def test_deltanet_oracle_matches_reference(golden):
    """oracle.deltanet_step (fp64) against the reference's recurrent_gated_delta_rule
    (torch fp32 on the CPU, qwen_engine.py:158-174) over 8 carried steps: the
    bf16 outputs agree to one bf16 step, the fp32 state to fp32 rounding."""
    c = golden.cases["deltanet"]
    q, k, v, g, beta, S0 = synthetic.deltanet_inputs(c["steps"], c["heads"], c["key_heads"], c["dk"], c["dv"], c["seed"])
    S = S0.double().numpy().copy()
    ref_out = golden.load("deltanet_out")
    for t in range(c["steps"]):
        o = oracle.deltanet_step(q[t].float().numpy(), k[t].float().numpy(), v[t].float().numpy(), g[t].numpy(),
                                 beta[t].float().numpy(), S)
        steps = bf16_steps(o, ref_out[t])
        assert steps.max() <= 1 and (steps > 0).mean() < 0.02
    ref_S = golden.load("deltanet_state")
    assert np.abs(S - ref_S).max() / np.sqrt(np.mean(ref_S.astype(np.float64) ** 2)) < 1e-5
