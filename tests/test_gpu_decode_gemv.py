"""GPU parity of the CUDA path against the reference's golden vectors and the
CPU oracle, through the drop-in Python API (which calls the C ABI).

Tolerances: the contract is max|cand - ref| <= 1e-3 * RMS(ref) for fp32
results (TOL); fp32-accumulating kernels are expected to land far inside it,
checked at FP32_GRADE.  A bf16 output is checked in two exact steps: it must
equal the round-to-nearest-even of the kernel's own fp32 result (the fp32
variant of the same kernel), and that fp32 result must be within FP32_GRADE
of the oracle.  (A direct bf16-vs-bf16(oracle) comparison cannot have a
relative bound: outputs near zero lose all relative precision to
cancellation, and a value on a rounding boundary may round either way.)
"""
import numpy as np
import pytest
import torch

import _lib
import fp8gemv
import oracle
import qmoe
import routing
import synthetic
from conftest import rel_err, sha
from test_oracle_golden import _deq_all_inputs, decode_case

pytestmark = pytest.mark.gpu

TOL = 1e-3
FP32_GRADE = 5e-5
DEV = "cuda"


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def check_bf16(y_bf16, y_f32, ref_f32):
    got = y_bf16.float().cpu().numpy()
    y32 = y_f32.cpu().numpy()
    assert np.array_equal(got, oracle.bf16_round(y32)), "bf16 output is not RNE of the fp32 result"
    assert rel_err(y32, ref_f32) <= FP32_GRADE
    # bf16 rounding error is at most half an ulp of the largest output
    assert np.abs(got - ref_f32).max() <= 2.0 ** -8 * np.abs(ref_f32).max()
    assert (got != oracle.bf16_round(ref_f32)).mean() < 0.01


# ---------------------------------------------------------------- dequantization
def test_deq_every_byte_and_scale_bit_exact(golden):
    c = golden.cases["deq_all"]
    wb, sb = _deq_all_inputs()
    out = qmoe.deq(cuda(wb), cuda(sb), c["ws2"]).cpu().numpy()
    assert sha(out) == c["sha256"]


def test_block_deq_bit_exact(golden):
    c = golden.cases["block_deq"]
    blk = synthetic.make_blocks(1, seed=c["block_seed"])[0]
    s2 = synthetic.make_s2(1, seed=c["s2_seed"], spread=True)[0]
    g, u, d = qmoe.block_deq(cuda(blk), torch.from_numpy(s2))
    assert sha(g.cpu().numpy()) == c["gate_sha256"]
    assert sha(u.cpu().numpy()) == c["up_sha256"]
    assert sha(d.cpu().numpy()) == c["down_sha256"]


# ---------------------------------------------------------------- decode expert layer
VARIANTS = [qmoe.VARIANT_CUDA_CORE, qmoe.VARIANT_SLICE]
SMALL_K_VARIANTS = (qmoe.VARIANT_SLICE,)   # K <= 10
# The slice path (the default for K <= 10) sums its per-CTA partials with fp32
# atomics: repeated calls agree to fp32 rounding of the summation order.
REPEAT_GRADE = 1e-5


def run_decode(table, sidx, s2, coef, x, variant=qmoe.VARIANT_AUTO):
    K = len(sidx)
    hb = torch.full((K, 640), float("nan"), device=DEV)
    y = qmoe._moe_decode(table, cuda(np.asarray(sidx, np.int32)), cuda(np.asarray(s2, np.float32)),
                         cuda(np.asarray(coef, np.float32)), x.to(DEV), hb, variant)
    torch.cuda.synchronize()
    return y.cpu().numpy(), hb.cpu().numpy()


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    import _lib
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0, "a kernel's bounded wait timed out"


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("name", ["moe_decode_k10_bf16", "moe_decode_k3_f32"])
def test_moe_decode_matches_reference_golden(golden, name, variant):
    table, sidx, s2, coef, x = decode_case(golden, name)
    y, h = run_decode(cuda(table), sidx, s2, coef, x, variant)
    ref = golden.load(name + "_out")
    assert rel_err(y, ref) <= TOL
    assert rel_err(y, ref) <= FP32_GRADE
    assert rel_err(h, golden.load(name + "_h")) <= FP32_GRADE
    assert np.argmax(y) == np.argmax(ref)


@pytest.fixture(scope="module")
def table24():
    blocks = synthetic.make_blocks(24, seed=7)
    return blocks, cuda(blocks)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("K,xdtype,seed", [(10, torch.bfloat16, 1), (10, torch.float32, 2), (1, torch.bfloat16, 3),
                                           (7, torch.float32, 4), (32, torch.bfloat16, 5), (16, torch.float32, 6)])
def test_moe_decode_matches_oracle(table24, K, xdtype, seed, variant):
    if K > 10 and variant in SMALL_K_VARIANTS:
        pytest.skip("this path takes K <= 10")
    blocks, table = table24
    rng = np.random.Generator(np.random.PCG64(100 + seed))
    sidx = rng.choice(24, size=K, replace=K > 24).astype(np.int32)
    s2 = synthetic.make_s2(K, seed=200 + seed, spread=True)
    coef = rng.random(K).astype(np.float32)
    x = synthetic.make_x(2560, seed=300 + seed, dtype=xdtype)
    y, h = run_decode(table, sidx, s2, coef, x, variant)
    ref, href = oracle.moe_decode(blocks, sidx, s2, coef, x.float().numpy(), return_h=True)
    assert rel_err(y, ref) <= FP32_GRADE
    assert rel_err(h[:K], href) <= FP32_GRADE
    assert np.argmax(y) == np.argmax(ref)


@pytest.mark.parametrize("variant", VARIANTS)
def test_moe_decode_out_of_range_block_gives_nan_without_reading(table24, variant):
    _, table = table24
    sidx = np.array([0, 1, 24, 3], np.int32)           # 24 == n_blocks: out of range
    y, h = run_decode(table, sidx, synthetic.make_s2(4), np.ones(4, np.float32), synthetic.make_x(2560, 9), variant)
    assert np.isnan(y).all()
    assert np.isnan(h[2]).all() and np.isfinite(h[[0, 1, 3]]).all()
    sidx[2] = -5
    y, _ = run_decode(table, sidx, synthetic.make_s2(4), np.ones(4, np.float32), synthetic.make_x(2560, 9), variant)
    assert np.isnan(y).all()


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("K,seed", [(10, 11), (10, 12), (7, 13), (3, 14), (1, 15)])
def test_moe_decode_repeated_calls_identical(table24, variant, K, seed):
    """Repeated calls agree: bit for bit on the CUDA-core path; on the slice
    path (fp32 atomics in no fixed order) to fp32 rounding, argmax included."""
    _, table = table24
    rng = np.random.Generator(np.random.PCG64(seed))
    args = (rng.permutation(24)[:K].astype(np.int32), synthetic.make_s2(K, seed=seed, spread=True),
            rng.random(K).astype(np.float32), synthetic.make_x(2560, seed))
    a, _ = run_decode(table, *args, variant=variant)
    b, _ = run_decode(table, *args, variant=variant)
    if variant in SMALL_K_VARIANTS:
        assert rel_err(a, b) <= REPEAT_GRADE and np.argmax(a) == np.argmax(b)
    else:
        assert np.array_equal(a, b)      # fixed reduction order: bit-reproducible


def test_moe_decode_paths_agree(table24):
    """The slice and CUDA-core paths compute the same layer to fp32 grade."""
    blocks, table = table24
    args = (np.array([23, 0, 5, 17, 9, 2, 11, 8, 20, 14], np.int32), synthetic.make_s2(10, seed=3, spread=True),
            np.linspace(0.02, 0.3, 10).astype(np.float32), synthetic.make_x(2560, 21))
    b, hb = run_decode(table, *args, variant=qmoe.VARIANT_CUDA_CORE)
    for v in SMALL_K_VARIANTS:
        a, ha = run_decode(table, *args, variant=v)
        assert rel_err(a, b) <= FP32_GRADE and rel_err(ha, hb) <= FP32_GRADE


@pytest.mark.parametrize("variant", SMALL_K_VARIANTS)
def test_moe_decode_large_and_tiny_x(table24, variant):
    """Per-call power-of-two prescale of x: results scale exactly with x."""
    _, table = table24
    sidx = np.arange(10, dtype=np.int32)
    s2, coef = synthetic.make_s2(10), np.full(10, .1, np.float32)
    x = synthetic.make_x(2560, 31, dtype=torch.float32)
    for f in (2.0 ** 40, 2.0 ** -40):
        y, _ = run_decode(table, sidx, s2, coef, x * f, variant)
        ref = oracle.moe_decode(table24[0], sidx, s2, coef, (x * f).numpy())
        assert rel_err(y, ref) <= FP32_GRADE


def test_moe_decode_graph_capture(table24):
    _, table = table24
    K = 10
    sidx = cuda(np.arange(K, dtype=np.int32) + 3)
    s2 = cuda(synthetic.make_s2(K, seed=1, spread=True))
    coef = cuda(np.linspace(0.05, 0.2, K).astype(np.float32))
    x = synthetic.make_x(2560, 12).to(DEV)
    hb = torch.empty(K, 640, device=DEV)
    ob = torch.empty(K, 2560, device=DEV)
    eager = qmoe.moe_decode(table, sidx, s2, coef, x, hb, ob).clone()
    g = torch.cuda.CUDAGraph()
    qmoe.moe_decode(table, sidx, s2, coef, x, hb, ob)
    torch.cuda.synchronize()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        y = qmoe.moe_decode(table, sidx, s2, coef, x, hb, ob)
    x.copy_(synthetic.make_x(2560, 13).to(DEV))
    g.replay()
    torch.cuda.synchronize()
    want = qmoe.moe_decode(table, sidx, s2, coef, x, hb, ob)
    assert rel_err(y.cpu().numpy(), want.cpu().numpy()) <= REPEAT_GRADE
    assert rel_err(y.cpu().numpy(), eager.cpu().numpy()) > 1e-2


# ---------------------------------------------------------------- FP8 GEMV
def gemv_inputs(N, K, wseed, xseed):
    w = synthetic.gemv_weights(N, K, wseed).float().numpy()
    q, s = oracle.to_fp8_rows(w)
    x = synthetic.make_x(K, seed=xseed)
    return q, s, x


@pytest.mark.parametrize("N,K", [(256, 512), (12288, 2560), (2560, 4096)])
def test_gemv_matches_reference_golden(golden, N, K):
    c = golden.cases[f"gemv_{N}x{K}"]
    q, s, x = gemv_inputs(N, K, c["w_seed"], c["x_seed"])
    qd = cuda(q).view(torch.float8_e4m3fn)
    ref = golden.load(f"gemv_{N}x{K}_y")
    y32 = fp8gemv.gemv_f32(qd, cuda(s), x.to(DEV))
    assert rel_err(y32.cpu().numpy(), ref) <= FP32_GRADE
    check_bf16(fp8gemv.gemv(qd, cuda(s), x.to(DEV)), y32, oracle.gemv(q, s, x.float().numpy()))


@pytest.mark.parametrize("N,K", [(13, 48), (1, 16), (10240, 2560), (6144, 2560), (2560, 6144), (33, 32768),
                                 (3, 64), (100, 1024), (150, 2560), (20480, 4096)])
def test_gemv_matches_oracle_odd_shapes(N, K):
    q, s, x = gemv_inputs(N, K, N + K, K)
    qd = cuda(q).view(torch.float8_e4m3fn)
    ref = oracle.gemv(q, s, x.float().numpy())
    y32 = fp8gemv.gemv_f32(qd, cuda(s), x.to(DEV))
    check_bf16(fp8gemv.gemv(qd, cuda(s), x.to(DEV)), y32, ref)


def test_gemv_graph_capture():
    q, s, x = gemv_inputs(2560, 4096, 1, 2)
    qd, sd, xd = cuda(q).view(torch.float8_e4m3fn), cuda(s), x.to(DEV)
    fp8gemv.gemv(qd, sd, xd)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        y = fp8gemv.gemv(qd, sd, xd)
    xd.copy_(synthetic.make_x(4096, 3).to(DEV))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, fp8gemv.gemv(qd, sd, xd))


def test_gemv_accepts_engine_quantizer_output():
    """The engine's own producer (to_fp8_rows on the device) feeds gemv unchanged (qwen_engine.py:71-82)."""
    w = synthetic.gemv_weights(512, 2560, 5).to(DEV)
    q, s = synthetic.to_fp8_rows(w)
    x = synthetic.make_x(2560, 6).to(DEV)
    s1 = s.view(-1).contiguous()
    ref = oracle.gemv(q.view(torch.uint8).cpu().numpy(), s1.cpu().numpy(), x.float().cpu().numpy())
    check_bf16(fp8gemv.gemv(q, s1, x), fp8gemv.gemv_f32(q, s1, x), ref)


# ---------------------------------------------------------------- routing on the device
def test_route_on_device_matches_oracle():
    logits = synthetic.zipf_logits(64, seed=77)
    ti, tv = routing.route(cuda(logits))
    oti, ocoef = oracle.route(logits)
    assert np.array_equal(ti.cpu().numpy(), oti)
    got = tv.float().cpu().numpy()
    assert np.all(np.abs(got - ocoef) <= np.abs(ocoef) * 2.0 ** -7)


# ---------------------------------------------------------------- FP8 linear, T > 1
def _bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("N,K", [(1, 16), (7, 48), (333, 1040), (2560, 4096), (12288, 2560)])
def test_e4m3_rows_to_bf16_bit_exact(N, K):
    """The weight expression of qwen_engine.py:83, bit for bit: against the
    reference's own torch expression on the GPU and against the oracle; every
    e4m3 byte value occurs (NaN codes included: NaN stays NaN)."""
    g = torch.Generator().manual_seed(N + K)
    qb = torch.randint(0, 256, (N, K), dtype=torch.uint8, generator=g)
    s = torch.rand(N, generator=g) * 1e-3 + 1e-6
    qd = qb.to(DEV).view(torch.float8_e4m3fn)
    got = _bits(fp8gemv.dequant_bf16(qd, s.to(DEV)[:, None]))
    ref = _bits((qd.to(torch.bfloat16) * s.to(DEV)[:, None]).to(torch.bfloat16))
    orc = oracle.e4m3_rows_to_bf16(qb.numpy(), s.numpy())
    nan = (ref & 0x7FFF) > 0x7F80
    assert np.array_equal(nan, (got & 0x7FFF) > 0x7F80)
    assert np.array_equal(got[~nan], ref[~nan])
    assert np.array_equal(got[~nan], orc[~nan])


def _bf16_steps_off(y, exact):
    """Per output: how many bf16 steps y lies from the exact value (fp64 sums of
    the same bf16 weights), in units of the bf16 step at |exact|, less an
    allowance of 1e-5 x RMS(exact) for the fp32 accumulation (it matters only
    for sums that cancel to near zero, where a bf16 step is tiny)."""
    y = np.asarray(y, np.float64)
    exact = np.asarray(exact, np.float64)
    mag = np.maximum(np.abs(exact), 1e-30)
    step = np.exp2(np.floor(np.log2(mag)) - 7)
    return np.maximum(np.abs(y - exact) - 1e-5 * np.sqrt(np.mean(exact ** 2)), 0.0) / step


@pytest.mark.parametrize("T,N,K", [(1, 2560, 4096), (2, 2560, 4096), (17, 2560, 4096), (256, 2560, 4096),
                                   (300, 333, 1040), (129, 128, 16), (3, 1, 32), (1000, 12288, 2560)])
def test_fp8_linear_matches_reference(T, N, K):
    """Lin.__call__ (qwen_engine.py:79-83) for T tokens.  T > 1: the tcgen05
    GEMM against the exact products of the reference's bf16 weights
    (q.to(bf16) * s).to(bf16) (fp64 sums; all rows, or 64 sampled rows of the
    largest case): every output within one bf16 step of the exact value and
    fewer than 1 % not equal to its rounding to bf16 (fp32 summation order).
    Against the reference expression F.linear(x, w) as run on the same GPU:
    max |y - ref| <= 2^-7 max |ref| (that GEMM may itself be a step away:
    torch lets cuBLAS reduce bf16 GEMMs in reduced precision).  Ragged shapes:
    a token tile of 44 of 256 tokens, 333 rows (a row tile of 77), K = 1040 (a
    K-block of 16 of 64), 129 tokens (one beyond an accumulator half).
    T == 1: the GEMV."""
    q, s, _ = gemv_inputs(N, K, 11, 12)
    x = torch.randn(T, K, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16)
    qd, sd, xd = cuda(q).view(torch.float8_e4m3fn), cuda(s)[:, None], x.to(DEV)
    y = fp8gemv.linear(xd, qd, sd)
    assert y.shape == (T, N) and y.dtype == torch.bfloat16
    if T == 1:
        assert torch.equal(y[0], fp8gemv.gemv(qd, sd.view(-1), xd[0]))
        return
    assert _lib.device_status() == 0
    ref = torch.nn.functional.linear(xd, (qd.to(torch.bfloat16) * sd).to(torch.bfloat16)).float()
    assert (y.float() - ref).abs().max().item() <= 2.0 ** -7 * ref.abs().max().item()
    rows = np.arange(T) if T <= 300 else np.random.default_rng(T).choice(T, 64, replace=False)
    got = y[torch.from_numpy(rows).to(DEV)].float().cpu().numpy()
    w = (oracle.e4m3_rows_to_bf16(q, s).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    exact = x[rows].double().numpy() @ w.T
    assert _bf16_steps_off(got, exact).max() <= 1.0
    assert (got != oracle.bf16_round(exact.astype(np.float32))).mean() < 0.01


def test_fp8_linear_nan_weight_codes():
    """An e4m3 NaN code (S.1111.111) in a weight row makes that output column
    NaN for every token, as F.linear on the reference's bf16 weights does; the
    other columns are unaffected."""
    N, K, T = 256, 512, 40
    q, s, _ = gemv_inputs(N, K, 31, 32)
    q = q.copy()
    q[3, 100] = 0x7F
    q[200, 7] = 0xFF
    x = torch.randn(T, K, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    qd, sd, xd = cuda(q).view(torch.float8_e4m3fn), cuda(s)[:, None], x.to(DEV)
    y = fp8gemv.linear(xd, qd, sd).float().cpu()
    ref = torch.nn.functional.linear(xd, (qd.to(torch.bfloat16) * sd).to(torch.bfloat16)).float().cpu()
    nan = torch.isnan(ref)
    assert nan[:, 3].all() and nan[:, 200].all() and nan.sum() == 2 * T
    assert torch.equal(torch.isnan(y), nan)
    ok = ~nan
    assert (y[ok] - ref[ok]).abs().max().item() <= 2.0 ** -7 * ref[ok].abs().max().item()


def test_fp8_linear_repeated_calls_and_graph():
    """The GEMM in a CUDA graph and called back to back on one stream gives
    the eager result bit for bit (a fixed summation order per output)."""
    N, K, T = 2560, 4096, 512
    q, s, _ = gemv_inputs(N, K, 21, 22)
    qd, sd = cuda(q).view(torch.float8_e4m3fn), cuda(s)[:, None]
    xd = torch.randn(T, K, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(DEV)
    y0 = fp8gemv.linear(xd, qd, sd)
    for _ in range(3):
        assert torch.equal(fp8gemv.linear(xd, qd, sd), y0)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        fp8gemv.linear(xd, qd, sd)   # warm-up outside capture
    torch.cuda.current_stream().wait_stream(st)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = fp8gemv.linear(xd, qd, sd)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, y0)
    assert _lib.device_status() == 0
