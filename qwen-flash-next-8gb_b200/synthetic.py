"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (there are no real weights in this environment).

  * expert blocks: e2m1 weight bytes uniform over 0..255 (uniformly random
    nibbles); E4M3 scale bytes = e4m3(2**U(-4, 2)); ws2 = 1/448 per projection.
  * GEMV weights: W ~ N(0, 0.02) rounded to bf16, quantized by to_fp8_rows.
  * routing: fp32 logits, N(0,1) (uniform popularity) or log p + Gumbel with
    p_r ~ r**-1.1 over a seeded permutation (Zipf popularity, top-k without
    replacement).
CPU generators use numpy PCG64 (bit-reproducible); the *_gpu generators fill
large HBM tensors in place with torch's CUDA generator.
"""
import numpy as np
import torch

HID, INTER, BLOCK = 2560, 640, 2764800
O_GS = 2457600
N_EXPERTS = 512
WS2 = 1.0 / 448.0


def _e4m3_bytes(v):
    """fp32 array -> float8_e4m3fn bytes (torch's round-to-nearest-even)."""
    t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def make_blocks(n, seed, scale_lo=-4.0, scale_hi=2.0):
    """u8[n, BLOCK]: n expert blocks in the repacked layout."""
    rng = np.random.Generator(np.random.PCG64(seed))
    blocks = rng.integers(0, 256, size=(n, BLOCK), dtype=np.uint8)
    u = rng.uniform(scale_lo, scale_hi, size=(n, BLOCK - O_GS)).astype(np.float32)
    blocks[:, O_GS:] = _e4m3_bytes(np.exp2(u))
    return blocks


def make_s2(n, seed=None, spread=False):
    """f32[n, 3] global scales: 1/448 (the benchmark value), or with spread=True
    distinct values in [0.5/448, 2/448] per expert and projection (so that a
    mixed-up gate/up/down scale cannot pass a parity test)."""
    if not spread:
        return np.full((n, 3), WS2, np.float32)
    rng = np.random.Generator(np.random.PCG64(seed))
    return (WS2 * np.exp2(rng.uniform(-1, 1, size=(n, 3)))).astype(np.float32)


def make_x(n, seed, std=1.0, dtype=torch.bfloat16):
    """x ~ N(0, std) rounded to `dtype`; returns a CPU torch tensor [n]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    v = (rng.standard_normal(n) * std).astype(np.float32)
    return torch.from_numpy(v).to(dtype)


def gemv_weights(N, K, seed):
    """W ~ N(0, 0.02) as bf16 (tests/test_gemv.py:6), CPU torch tensor [N, K]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    v = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    return torch.from_numpy(v).to(torch.bfloat16)


@torch.no_grad()
def to_fp8_rows(w):
    """The engine's weight quantizer (qwen_engine.py:59-64), the producer of
    the GEMV's inputs: bf16/fp32 [N,K] -> (float8_e4m3fn [N,K], fp32 [N,1])."""
    w = w.float()
    s = (w.abs().amax(1, keepdim=True) / 448.0).clamp_min(1e-12)
    return (w / s).to(torch.float8_e4m3fn), s


def zipf_logits(n_rows, seed, n_experts=N_EXPERTS, s=1.1, rows_per_perm=None):
    """fp32 [n_rows, n_experts] = log p[perm] + Gumbel noise, p_r ~ r**-s.
    One popularity permutation per `rows_per_perm` rows (default: one for all)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    logp = -s * np.log(np.arange(1, n_experts + 1, dtype=np.float64))
    logp -= np.log(np.exp(logp).sum())
    rows_per_perm = rows_per_perm or n_rows
    out = np.empty((n_rows, n_experts), np.float32)
    for r0 in range(0, n_rows, rows_per_perm):
        perm = rng.permutation(n_experts)
        r1 = min(n_rows, r0 + rows_per_perm)
        g = rng.gumbel(size=(r1 - r0, n_experts))
        out[r0:r1] = (logp[perm][None, :] + g).astype(np.float32)
    return out


def normal_logits(n_rows, seed, n_experts=N_EXPERTS):
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((n_rows, n_experts)).astype(np.float32)


@torch.no_grad()
def fill_blocks_gpu(table, seed, chunk=256):
    """Fill a CUDA u8[n, BLOCK] table in place with the make_blocks
    distributions (torch CUDA generator; not bit-identical to make_blocks)."""
    g = torch.Generator(device=table.device)
    g.manual_seed(seed)
    n = table.shape[0]
    for b0 in range(0, n, chunk):
        b1 = min(n, b0 + chunk)
        view = table[b0:b1]
        view[:, :O_GS] = torch.randint(0, 256, (b1 - b0, O_GS), dtype=torch.uint8, device=table.device,
                                       generator=g)
        u = torch.empty((b1 - b0, BLOCK - O_GS), dtype=torch.float32, device=table.device)
        u.uniform_(-4.0, 2.0, generator=g)
        view[:, O_GS:] = torch.exp2(u).to(torch.float8_e4m3fn).view(torch.uint8)
        del u
    return table


def block_seed(seed, layer, expert):
    """Seed of the synthetic block of (layer, global expert id): every process
    can regenerate any expert's bytes, whichever rank's table holds it."""
    return (int(seed) * 1000003 + int(layer) * 4099 + int(expert)) % (2 ** 62)


@torch.no_grad()
def fill_block_gpu(dst, seed):
    """Fill one CUDA u8[BLOCK] block with the make_blocks distributions from
    its own seed (torch's CUDA generator: the same bytes on every device)."""
    g = torch.Generator(device=dst.device)
    g.manual_seed(seed)
    dst[:O_GS] = torch.randint(0, 256, (O_GS,), dtype=torch.uint8, device=dst.device, generator=g)
    u = torch.empty(BLOCK - O_GS, dtype=torch.float32, device=dst.device)
    u.uniform_(-4.0, 2.0, generator=g)
    dst[O_GS:] = torch.exp2(u).to(torch.float8_e4m3fn).view(torch.uint8)
    return dst


@torch.no_grad()
def fill_table_gpu(table, n_layers, experts, seed):
    """Fill a CUDA table u8[n_layers * len(experts), BLOCK]: row L * len(experts)
    + i holds the block of (L, experts[i]), seeded by block_seed."""
    n = len(experts)
    for L in range(n_layers):
        for i, e in enumerate(experts):
            fill_block_gpu(table[L * n + i], block_seed(seed, L, e))
    return table


@torch.no_grad()
def expert_block(layer, expert, seed, dev):
    """The synthetic block of (layer, expert) as a new CUDA u8[BLOCK] tensor
    (what fill_table_gpu wrote into whichever table holds it)."""
    return fill_block_gpu(torch.empty(BLOCK, dtype=torch.uint8, device=dev), block_seed(seed, layer, expert))


def deltanet_inputs(steps, heads, key_heads, dk, dv, seed):
    """Seeded inputs of `steps` one-token delta-rule steps (qwen_engine.py:696-719
    at T == 1): q, k bf16 [steps, key_heads, dk] and v bf16 [steps, heads, dv]
    ~ silu(N(0, 1)) (the conv output's activation); g fp32 [steps, heads] =
    -exp(A_log) * softplus(a + dt_bias) with A_log ~ U(-2, 1), a + dt_bias ~
    N(0, 1); beta bf16 [steps, heads] = sigmoid(N(0, 1)); S0 fp32 [heads, dk, dv]
    ~ N(0, 0.05).  CPU torch tensors."""
    rng = np.random.Generator(np.random.PCG64(seed))

    def silu_bf16(shape):
        z = rng.standard_normal(shape).astype(np.float32)
        return torch.from_numpy(z / (1 + np.exp(-z))).to(torch.bfloat16)

    q, k, v = silu_bf16((steps, key_heads, dk)), silu_bf16((steps, key_heads, dk)), silu_bf16((steps, heads, dv))
    a_log = rng.uniform(-2, 1, size=heads).astype(np.float32)
    a = rng.standard_normal((steps, heads)).astype(np.float32)
    g = torch.from_numpy((-np.exp(a_log) * np.log1p(np.exp(a))).astype(np.float32))
    beta = torch.from_numpy(1 / (1 + np.exp(-rng.standard_normal((steps, heads))))).float().to(torch.bfloat16)
    S0 = torch.from_numpy((rng.standard_normal((heads, dk, dv)) * 0.05).astype(np.float32))
    return q, k, v, g, beta, S0
