"""GPU parity of the decode MoE block's prologue and epilogue (router, shared expert):
the fused router (routing.route_fused, the C ABI's qfn_moe_route), the bf16
shared expert with the combine (moe_block.shared_expert, qfn_shared_expert)
and the whole device-side block (moe_block.DecodeMoE) against the CPU oracle.

Router: the logits are the bf16 rounding of fp32 dot products, so they may sit
one bf16 step from the exact value (oracle.router_logits) when a sum lies next
to a rounding boundary.  From the kernel's logits, the chosen experts must
equal the oracle's router (oracle.route, the reference's softmax / topk /
renormalisation) exactly, and the bf16 weights must equal them to within one
bf16 step: the softmax's exp and sums are fp32 with their own rounding order
(the reference's torch CPU and CUDA softmaxes differ from each other the
same way), so a weight next to a bf16 rounding boundary may round either way.
"""
import numpy as np
import pytest
import torch

import moe_block
import oracle
import qmoe
import routing
import synthetic
from conftest import bf16_steps, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).to(DEV)


def assert_weights_close(a, b):
    """Router weights within one bf16 step of the oracle's, and rarely off at
    all: the fp32 sum of the exponentials is summed in another order than the
    oracle's (as torch's own CUDA softmax is), so a weight whose fp32 value
    lies next to a bf16 rounding boundary can round the other way."""
    st = bf16_steps(a, b)
    assert st.max() <= 1 and (st > 0).sum() <= max(1, 0.05 * st.size), (st.max(), (st > 0).mean())


def router_case(T, E, seed, dup_rows=0):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = bf16(rng.standard_normal((T, 2560)))
    w = rng.standard_normal((E, 2560)) * 0.02
    if dup_rows:   # identical rows: equal logits, the tie goes to the lower expert id
        w[E - dup_rows:] = w[:dup_rows]
    return x, bf16(w)


@pytest.mark.parametrize("T,E,topk,seed", [(1, 512, 10, 1), (7, 512, 10, 2), (64, 512, 10, 3), (3, 128, 4, 4),
                                           (2, 1024, 32, 5), (1, 128, 4, 6), (1, 1024, 32, 7), (1, 4, 4, 8)])
def test_route_fused_matches_oracle(T, E, topk, seed):
    x, w = router_case(T, E, seed)
    s2_table = torch.from_numpy(synthetic.make_s2(3 * E, seed=seed, spread=True).reshape(3, E, 3)).to(DEV)
    layer = 2
    r = routing.route_fused(x, w, topk, layer, s2_table)
    torch.cuda.synchronize()
    logits = r["logits"].float().cpu().numpy()
    exact = oracle.router_logits(x.float().cpu().numpy(), w.float().cpu().numpy())
    steps = bf16_steps(logits, exact)
    assert steps.max() <= 1 and (steps > 0).mean() < 0.02
    ti_ref, coef_ref = oracle.route(logits, topk)
    ti = r["ti"].cpu().numpy()
    assert np.array_equal(ti, ti_ref)
    assert_weights_close(r["tv"].float().cpu().numpy(), coef_ref)
    # the reference's torch expression on the same logits: the same experts and weights
    # (torch.topk on CUDA may list experts of equal probability in either order)
    ti_t, tv_t = routing.route(r["logits"], topk)
    o_t, o = np.argsort(ti_t.cpu().numpy(), 1), np.argsort(ti, 1)
    assert np.array_equal(np.take_along_axis(ti_t.cpu().numpy(), o_t, 1), np.take_along_axis(ti, o, 1))
    assert_weights_close(np.take_along_axis(tv_t.float().cpu().numpy(), o_t, 1),
                         np.take_along_axis(r["tv"].float().cpu().numpy(), o, 1))
    assert np.array_equal(r["sidx"].cpu().numpy(), ti + layer * E)
    assert np.array_equal(r["coef"].cpu().numpy(), r["tv"].float().cpu().numpy())
    assert torch.equal(r["s2"], s2_table[layer][r["ti"].long()])


@pytest.mark.parametrize("T", [1, 5])
def test_route_fused_ties_go_to_the_lower_expert(T):
    x, w = router_case(T, 512, 11, dup_rows=256)         # experts e and e + 256 have equal logits
    r = routing.route_fused(x, w, 10)
    logits = r["logits"].float().cpu().numpy()
    ti_ref, coef_ref = oracle.route(logits, 10)
    assert np.array_equal(r["ti"].cpu().numpy(), ti_ref)
    assert_weights_close(r["tv"].float().cpu().numpy(), coef_ref)
    # both copies of a duplicated row tie; the lower id is ranked first
    for row in r["ti"].cpu().numpy():
        pos = {int(e): i for i, e in enumerate(row)}
        for e, i in pos.items():
            if e >= 256:
                assert e - 256 in pos and pos[e - 256] < i, row


def shared_case(T, I, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = bf16(rng.standard_normal((T, 2560)))
    wg, wu = bf16(rng.standard_normal((I, 2560)) * .02), bf16(rng.standard_normal((I, 2560)) * .02)
    wd, wsg = bf16(rng.standard_normal((2560, I)) * .02), bf16(rng.standard_normal((1, 2560)) * .02)
    y = torch.from_numpy(rng.standard_normal((T, 2560)).astype(np.float32)).to(DEV)
    return x, wg, wu, wd, wsg, y


@pytest.mark.parametrize("T,I,seed,with_y", [(1, 512, 1, True), (1, 640, 2, False), (9, 256, 3, True),
                                             (4, 1536, 4, True), (2, 4096, 5, False), (3, 40, 6, True)])
def test_shared_expert_matches_oracle(T, I, seed, with_y):
    """bf16 results equal the oracle's (each step rounded to bf16 as the
    reference rounds it) but for rare one-step differences where an fp32 sum
    lies next to a bf16 rounding boundary."""
    x, wg, wu, wd, wsg, y = shared_case(T, I, seed)
    out = moe_block.shared_expert(x, wg, wu, wd, wsg, y if with_y else None)
    torch.cuda.synchronize()
    ref = oracle.shared_expert(*(t.float().cpu().numpy() for t in (x, wg, wu, wd, wsg)),
                               y.cpu().numpy() if with_y else None)
    got = out.float().cpu().numpy()
    steps = bf16_steps(got, ref)
    assert np.isfinite(got).all()
    assert rel_err(got, ref) <= 1e-2      # a few bf16 steps at most, relative to RMS
    assert (steps > 0).mean() < 0.02


def test_decode_moe_block_device_only_in_a_graph():
    """The decode MoE block (router -> routed experts -> shared expert + combine)
    on the device, captured in one CUDA graph: replayed on new inputs it equals
    the oracle's block on the same routing; nothing leaves the GPU."""
    from expert_table import ExpertTable
    E, L = 64, 2
    table = ExpertTable(K=10, dev=DEV, n_layers=L, n_experts=E)
    table.fill_synthetic(seed=3)
    table.s2.copy_(torch.from_numpy(synthetic.make_s2(L * E, seed=4, spread=True).reshape(L, E, 3)))
    _, router = router_case(1, E, 21)
    _, wg, wu, wd, wsg, _ = shared_case(1, 512, 22)
    blk = moe_block.DecodeMoE(table, topk=10)
    x = bf16(synthetic.make_x(2560, seed=23).float().numpy()[None])
    out = torch.empty(1, 2560, dtype=torch.bfloat16, device=DEV)
    blk(x, 1, router, wg, wu, wd, wsg, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        blk(x, 1, router, wg, wu, wd, wsg, out=out)
    x.copy_(bf16(synthetic.make_x(2560, seed=24).float().numpy()[None]))
    g.replay()
    torch.cuda.synchronize()
    # the oracle's block on the kernel's routing (which the router test pins)
    ti = blk.route_buf["ti"][0].cpu().numpy()
    coef = blk.route_buf["tv"][0].float().cpu().numpy()
    logits = blk.route_buf["logits"].float().cpu().numpy()
    ti_ref, coef_ref = oracle.route(logits, 10)
    assert np.array_equal(ti, ti_ref[0])
    assert_weights_close(coef, coef_ref[0])
    blocks = table.slots[torch.from_numpy(ti + E).long().to(DEV)].cpu().numpy()
    y = oracle.moe_decode(blocks, np.arange(10, dtype=np.int32), table.s2[1][torch.from_numpy(ti).long()].cpu().numpy(),
                          coef, x.float().cpu().numpy()[0])
    ref = oracle.shared_expert(*(t.float().cpu().numpy() for t in (x, wg, wu, wd, wsg)), y[None])
    got = out.float().cpu().numpy()
    assert rel_err(got, ref) <= 1e-2
    assert int(np.argmax(got)) == int(np.argmax(ref))
    del g
