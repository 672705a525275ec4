// Slice path of the bs=1 decode layer (K <= 10 on a 148-SM part): one
// cooperative launch per layer with NO grid-wide barrier.
//
// Restates qmoe.moe_decode (qmoe.py:77-83): h_j = silu(ws2_g * G_j x) * (ws2_u * U_j x)
// (the _gate_up kernel, qmoe.py:24-51), out = sum_j coef_j * ws2_d * D_j h_j
// (_down, qmoe.py:54-74, and out_buf[:K].sum(0), qmoe.py:83).
//
// Work split.  The layer's K x 640 output features of the gate/up
// projections come in blocks of 16 (one E4M3 scale group of the down rows).
// Every CTA owns one expert and 2-3 consecutive blocks of it (K = 10 on 148
// SMs: 14-15 CTAs per expert, 40 blocks per expert).  Because the down
// projection's K dimension IS the feature dimension, a CTA can finish its
// features on its own: it computes h for its <= 48 features (gate and up
// rows x x), then multiplies them into the matching 24-byte column slice of
// all 2,560 down rows.  Nothing crosses CTAs except the final sum over the
// CTAs' partial output vectors, done with fp32 vector atomics into `out`.
//
// Copies: per block four contiguous bulk copies (its 16 gate rows, 16 up
// rows, 20 KB each, and their two 2.5 KB scale runs; 4-D tensor boxes of the
// same bytes streamed measurably slower); the down column slice as two 4-D
// TMA boxes of 1,280 rows x 32 bytes (the 16-byte aligned cover of the 16-24
// needed bytes).  The down scales (1-3 bytes of each 40-byte row) are
// gathered with 32-bit loads once block 0 has landed.  Copies go out in two waves: blocks 0 and 1 at entry,
// the rest once block 0 has landed.  Issued all at once, every copy would
// complete near the end of the layer's whole stream (HBM serves the queued
// requests in no particular order) and the arithmetic could not overlap it.
//
// `out` starts at zero for the atomics: each CTA zeroes 1/grid of it after
// the programmatic-dependency wait and counts itself on a monotonic counter
// (one slot per call site, 64-bit, grows by grid per call); before its
// atomics a CTA waits until the counter reaches the end of this call's
// range.  Every CTA zeroes at entry and adds at exit, so the wait is normally
// already satisfied when it is checked.  Calls that share a slot must not
// overlap on the device (the host hands each call a different slot out of
// 1,024, so only a captured graph replayed concurrently on two streams could).
//
// Dot products: mma.sync m16n8k16 with f16 operands as in the stream path
// (A = e2m1 x E4M3 scale, exact in f16; B = activation as an f16 hi/lo pair
// after a power-of-two prescale).  Phase 1: warp w owns K-slice [128w,
// 128w+128) of every 8-feature octet (A rows 0-7 gate, 8-15 up); the 20
// warps' partials meet in shared memory through fp32 atomic adds.  Phase 2:
// A = 16 down rows x 16 features (one block: one scale per row), the k order
// permuted inside the block so that lane t reads bytes 2t, 2t+1 of the
// block's 8 bytes per row (B permuted to match).  The summation order of the
// atomics varies from call to call: results are reproducible to fp32
// rounding, not bit for bit (the stream path is the bit-reproducible one).
#pragma once

namespace qfn {

constexpr int kLThreads = 640;
constexpr int kLWarps = kLThreads / 32;
constexpr int kLBlocksPerExpert = kInter / 16;   // 40 scale groups of a down row
constexpr int kLMaxBlk = 3;                      // blocks per CTA (checked on the host)
constexpr int kLGuBytes = 2 * 16 * (kHid / 2);   // 40,960: 16 gate rows | 16 up rows
constexpr int kLGsBytes = 2 * 16 * (kHid / 16);  // 5,120: their scale rows
constexpr int kLDnRow = 32;                      // bytes of a down row held in shared memory
constexpr int kLDnHalf = (kHid / 2) * kLDnRow;   // 40,960: 1,280 rows
constexpr int kLSlots = 1024;

// byte offsets from the 128-aligned base of one CTA's dynamic shared memory
constexpr int kLSmGu = 0;
constexpr int kLSmGs = kLSmGu + kLMaxBlk * kLGuBytes;  // 122,880
constexpr int kLSmDn = kLSmGs + kLMaxBlk * kLGsBytes;  // 138,240
constexpr int kLSmDs = kLSmDn + kHid * kLDnRow;        // 220,160: down scales, one u32 per row
constexpr int kLSmMisc = kLSmDs + kHid * 4;            // 230,400
constexpr int kLSmTotal = kLSmMisc + 1024 + 128;       // + alignment slack for the base

// Per-call-site counters of the zeroing protocol (zero at module load).
__device__ unsigned long long g_slice_ctr[kLSlots];

// The call-site slot of the next decode call on a device (round robin over
// kLSlots, shared by the slice and row paths, which share the counters).
inline int next_decode_slot(int device) {
  static std::atomic<unsigned int> next_slot[64];
  return static_cast<int>(next_slot[device].fetch_add(1u) % kLSlots);
}

struct SliceSplit {
  int grid, K;
  __host__ __device__ int expert_of(int c) const { return static_cast<int>(static_cast<long long>(c) * K / grid); }
  __host__ __device__ int first_cta(int j) const {
    return static_cast<int>((static_cast<long long>(j) * grid + K - 1) / K);
  }
  // CTA c: expert j, blocks [b0, b1) of it; it is CTA i of the expert's n
  __host__ __device__ void blocks(int c, int& j, int& b0, int& b1, int& i, int& n) const {
    j = expert_of(c);
    const int f = first_cta(j);
    n = first_cta(j + 1) - f;
    i = c - f;
    b0 = kLBlocksPerExpert * i / n;
    b1 = kLBlocksPerExpert * (i + 1) / n;
  }
};

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <bool kXF32>
__global__ void __launch_bounds__(kLThreads, 1)
    moe_decode_slice(const __grid_constant__ CUtensorMap dn_map, const uint8_t* __restrict__ table, int64_t n_blocks,
                     const int32_t* __restrict__ sidx, const float* __restrict__ s2, const float* __restrict__ coef,
                     const void* __restrict__ x, float* __restrict__ h, float* __restrict__ out, int K, int slot) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
  uint8_t* misc = smem + kLSmMisc;
  uint64_t* bar = reinterpret_cast<uint64_t*>(misc);      // [0, 3): gate/up blocks; 3, 4: down halves
  __half* hhi = reinterpret_cast<__half*>(misc + 448);    // [48] h hi, then [48] h lo
  __half* hlo = hhi + 48;
  uint32_t* dsc = reinterpret_cast<uint32_t*>(smem + kLSmDs);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = static_cast<int>(gridDim.x);

  int j, b0, b1, ci, cn;
  SliceSplit{G, K}.blocks(blockIdx.x, j, b0, b1, ci, cn);
  const int nb = b1 - b0, nf = 16 * nb;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&dn_map);
  }
  __syncthreads();
  // Everything below reads this call's inputs or writes h / out.
  pdl_wait();
  pdl_launch_dependents();

  const int64_t blk = nb > 0 ? static_cast<int64_t>(sidx[j]) : -1;
  const bool ok = nb > 0 && blk >= 0 && blk < n_blocks;
  const int nbl = ok ? nb : 0;  // blocks whose bytes are loaded

  // Copies go out in two waves so that the first blocks land early (HBM
  // serves queued requests in no particular order: a copy issued together
  // with the whole layer completes near the end of the whole stream).  At
  // entry: the gate/up rows of blocks 0 and 1 and an L2 prefetch of this
  // CTA's contiguous 1/n share of the expert's down scales.  Once block 0
  // has landed: block 2, an L2 prefetch of this CTA's 1/n share of the
  // expert's down rows (all of the expert's CTAs read those in narrow column
  // slices; the prefetches make HBM read them sequentially), then the down
  // column slice.
  const uint8_t* eb = table + (ok ? blk : 0) * kBlock;
  const int ra = kHid * ci / cn, rb = kHid * (ci + 1) / cn;  // this CTA's 1/n of the expert's down rows
  auto issue_gu = [&](int b) {
    const int f0 = 16 * (b0 + b);
    mbar_arrive_expect_tx(&bar[b], kLGuBytes + kLGsBytes);
    uint8_t* gu = smem + kLSmGu + b * kLGuBytes;
    uint8_t* gs = smem + kLSmGs + b * kLGsBytes;
    bulk_g2s(gu, eb + kOGW + f0 * (kHid / 2), kLGuBytes / 2, &bar[b]);
    bulk_g2s(gu + kLGuBytes / 2, eb + kOUW + f0 * (kHid / 2), kLGuBytes / 2, &bar[b]);
    bulk_g2s(gs, eb + kOGS + f0 * (kHid / 16), kLGsBytes / 2, &bar[b]);
    bulk_g2s(gs + kLGsBytes / 2, eb + kOUS + f0 * (kHid / 16), kLGsBytes / 2, &bar[b]);
  };
  auto issue_wave_b = [&]() {
    if (nb > 2) issue_gu(2);
    bulk_prefetch_l2(eb + kODW + 320 * ra, 320 * (rb - ra));
    for (int half = 0; half < 2; ++half) {
      mbar_arrive_expect_tx(&bar[3 + half], kLDnHalf);
      tma_load_4d(smem + kLSmDn + half * kLDnHalf, &dn_map, 16 * (b0 >> 1), 0, 5 * half, static_cast<int>(blk),
                  &bar[3 + half]);
    }
  };
  unsigned long long ticket = 0, seen = 0;  // used by warp 1 lane 0
  if (warp == 0) {
    if (ok && lane < (nb < 2 ? nb : 2)) issue_gu(lane);
    if (ok && nb == 1 && lane == 0) issue_wave_b();
  } else if (warp == 1) {
    if (ok && lane == 0) {
      const int sa = (40 * ra) & ~15, sb = ci + 1 == cn ? 40 * kHid : (40 * rb) & ~15;
      if (sb > sa) bulk_prefetch_l2(eb + kODS + sa, sb - sa);
    }
    // zero this CTA's share of out, then count it on the call's counter
    const int r0 = static_cast<int>(static_cast<long long>(blockIdx.x) * kHid / G);
    const int r1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * kHid / G);
    for (int r = r0 + lane; r < r1; r += 32) out[r] = 0.f;
    __syncwarp();
    if (lane == 0) {
      __threadfence();
      ticket = atomicAdd(&g_slice_ctr[slot], 1ull);
    }
    __syncwarp();
  }

  // B fragments of x for this warp's K-slice [128 warp, +128): lane (g, t), g < 2,
  // holds x[128 warp + 32 t, +32) times 2^ex as f16 hi (g = 0) or lo (g = 1).
  uint4 bq[4];
  int ex;
  {
    float xv[32];
    const int k0 = 128 * warp + 32 * t;
    if (g < 2) {
      if (kXF32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + k0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 a = p[q];
          xv[4 * q] = a.x; xv[4 * q + 1] = a.y; xv[4 * q + 2] = a.z; xv[4 * q + 3] = a.w;
        }
      } else {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + k0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 a = p[q];
          const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            xv[8 * q + 2 * i] = bf16_bits_to_f32(w[i] & 0xffffu);
            xv[8 * q + 2 * i + 1] = bf16_bits_to_f32(w[i] >> 16);
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) xv[i] = 0.f;
    }
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) mx = nanmax(mx, fabsf(xv[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = nanmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    ex = f16_prescale_exp(mx);
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      __half h0, l0, h1, l1;
      split_f16(scale_pow2(xv[2 * i], ex), h0, l0);
      split_f16(scale_pow2(xv[2 * i + 1], ex), h1, l1);
      const __half a0 = g == 0 ? h0 : l0, a1 = g == 0 ? h1 : l1;
      w[i] = g < 2 ? (static_cast<uint32_t>(__half_as_ushort(a0)) | (static_cast<uint32_t>(__half_as_ushort(a1)) << 16))
                   : 0u;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) bq[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
  const float ws_g = s2[3 * j], ws_u = s2[3 * j + 1];
  const float cw = ok ? coef[j] * s2[3 * j + 2] : __int_as_float(0x7fc00000);
  if (warp == 1 && lane == 0) seen = ld_relaxed_u64(&g_slice_ctr[slot]);  // usually final by the time it is checked

  // The down scales of this CTA's blocks: bytes [b0, b1) of every 40-byte row,
  // gathered by warps 2-19 as one or two aligned words per row.  The loads go
  // out once block 0 has landed (by then the L2 prefetch of the expert's
  // down scales issued at entry has brought them in; issued at entry they
  // queue behind the layer's stream) and are stored after phase 1.
  constexpr int kGN = kLThreads - 64, kGIt = (kHid + kGN - 1) / kGN;
  uint32_t wa[kGIt], wb[kGIt];
  auto gather_scales = [&]() {
    const uint8_t* ds = eb + kODS + (b0 & ~3);
    const bool two = (b0 & 3) + nb > 4;
#pragma unroll
    for (int i = 0; i < kGIt; ++i) {
      const int r = threadIdx.x - 64 + i * kGN;
      const uint32_t* q = reinterpret_cast<const uint32_t*>(ds + 40 * (r < kHid ? r : 0));
      wa[i] = __ldg(q);
      wb[i] = two ? __ldg(q + 1) : 0u;
    }
  };

  // Wait (bounded, warp 1 lane 0) until every CTA of this call has zeroed its
  // share of out; the caller follows with a block barrier.
  auto wait_zeroed = [&]() {
    if (warp == 1 && lane == 0) {
      const unsigned long long target = (ticket / static_cast<unsigned long long>(G) + 1ull) * G;
      const unsigned long long t0 = global_ns();
      for (uint32_t i = 1; seen < target && !wait_expired(i, t0); ++i) seen = ld_relaxed_u64(&g_slice_ctr[slot]);
      if (seen < target) note_timeout();
      __threadfence();
    }
    // lanes 1-31 must not reach the caller's block barrier before lane 0:
    // a barrier reached by a diverged warp completes without its lagging lanes
    if (warp == 1) __syncwarp();
  };
  if (nbl == 0) {  // no features, or an expert out of range: that one poisons out (NaN), as the other paths do
    if (nf == 0) return;  // (its zeroing is counted)
    if (threadIdx.x < nf) h[j * kInter + 16 * b0 + threadIdx.x] = __int_as_float(0x7fc00000);
    wait_zeroed();
    __syncthreads();
    atomicAdd(reinterpret_cast<float4*>(out) + threadIdx.x, make_float4(cw, cw, cw, cw));
    return;
  }

  // ---- phase 1: gate/up rows of each block as they land.  Lane (g, 0) keeps
  // its warp's partial sums of gate row g and up row g of every octet.
  float pg[2 * kLMaxBlk], pu[2 * kLMaxBlk];
#pragma unroll
  for (int b = 0; b < kLMaxBlk; ++b) {
    pg[2 * b] = pg[2 * b + 1] = pu[2 * b] = pu[2 * b + 1] = 0.f;
    if (b < nbl) {
      if (!mbar_wait(&bar[b], 0)) note_timeout();
      if (warp == 0 && b == 0 && nb > 1 && lane == 0) issue_wave_b();
      // re-read the zeroing counter once block 0 is in (the read at entry may
      // precede the last CTA's count; under the layer's stream a load takes
      // microseconds, so it is issued long before its use)
      if (warp == 1 && b == 0 && lane == 0) seen = ld_relaxed_u64(&g_slice_ctr[slot]);
      if (warp >= 2 && b == 0) gather_scales();
      const uint8_t* gu = smem + kLSmGu + b * kLGuBytes;
      const uint8_t* gs = smem + kLSmGs + b * kLGsBytes;
#pragma unroll
      for (int o = 0; o < 2; ++o) {
        const int row = 8 * o + g;
        const uint4 ra4 = lds128(gu + row * (kHid / 2) + 64 * warp + 16 * t);
        const uint4 rb4 = lds128(gu + (16 + row) * (kHid / 2) + 64 * warp + 16 * t);
        const uint32_t sa = lds16(gs + row * (kHid / 16) + 8 * warp + 2 * t);
        const uint32_t sb = lds16(gs + (16 + row) * (kHid / 16) + 8 * warp + 2 * t);
        float d[4][4] = {};
        mma_chunk(d, ra4, rb4, sa, sb, bq);
        const float2 r = unit_rows(d);
        pg[2 * b + o] = scale_pow2(r.x, -ex);
        pu[2 * b + o] = scale_pow2(r.y, -ex);
      }
    }
  }
  // one more read if that one was early too
  if (warp == 1 && lane == 0 && seen < (ticket / static_cast<unsigned long long>(G) + 1ull) * G)
    seen = ld_relaxed_u64(&g_slice_ctr[slot]);
  __syncthreads();  // every warp is done with the gate/up rows: that region now takes the partials
  float* part = reinterpret_cast<float*>(smem + kLSmGu);  // [warp][feature][gate, up]
  if (t == 0) {
#pragma unroll
    for (int b = 0; b < kLMaxBlk; ++b)
#pragma unroll
      for (int o = 0; o < 2; ++o)
        if (b < nbl) {
          const int f = 16 * b + 8 * o + g;
          part[(warp * 48 + f) * 2] = pg[2 * b + o];
          part[(warp * 48 + f) * 2 + 1] = pu[2 * b + o];
        }
  }
  __syncthreads();

  // h of this CTA's features (the reference's formula; the warps' partials
  // summed in a fixed order), kept in h_buf like the reference, and as f16
  // hi/lo after a power-of-two prescale for phase 2.
  float hv = 0.f;
  if (threadIdx.x < nf) {
    float gs[4] = {0.f, 0.f, 0.f, 0.f}, us[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kLWarps; ++w) {
      gs[w & 3] += part[(w * 48 + threadIdx.x) * 2];
      us[w & 3] += part[(w * 48 + threadIdx.x) * 2 + 1];
    }
    const float gg = ((gs[0] + gs[1]) + (gs[2] + gs[3])) * ws_g, uu = ((us[0] + us[1]) + (us[2] + us[3])) * ws_u;
    hv = gg / (1.0f + expf(-gg)) * uu;
  }
  float* wred = reinterpret_cast<float*>(misc + 640);  // [2] warp maxima of |h|
  if (warp < 2) {
    float m = fabsf(hv);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wred[warp] = m;
  }
  wait_zeroed();  // phase 2 adds into out tile by tile
  __syncthreads();
  // After the wait: its fence would otherwise wait for this store (warp 1
  // holds features 32-47), and the scale stores wait for their gathers.
  if (threadIdx.x < nf) h[j * kInter + 16 * b0 + threadIdx.x] = hv;
  if (warp >= 2) {
#pragma unroll
    for (int i = 0; i < kGIt; ++i) {
      const int r = threadIdx.x - 64 + i * kGN;
      if (r < kHid) dsc[r] = __funnelshift_r(wa[i], wb[i], 8 * (b0 & 3));
    }
  }
  const int eh = f16_prescale_exp(nanmax(wred[0], wred[1]));
  if (threadIdx.x < nf) split_f16(scale_pow2(hv, eh), hhi[threadIdx.x], hlo[threadIdx.x]);
  __syncthreads();

  // ---- phase 2: the down column slice.  Tile T = 16 rows; warp w takes tiles
  // w, w + 20, ..., w + 140.  Each tile's 16 sums are gathered by shuffles
  // into lanes 0, 4, 8, 12 (4 consecutive rows each) and added into out as
  // soon as the tile is done, so the atomics spread over the phase.
  uint32_t hb0[kLMaxBlk], hb1[kLMaxBlk];
#pragma unroll
  for (int b = 0; b < kLMaxBlk; ++b) {
    hb0[b] = hb1[b] = 0u;
    if (g < 2 && b < nbl) {
      const __half* src = (g == 0 ? hhi : hlo) + 16 * b + 4 * t;
      hb0[b] = *reinterpret_cast<const uint32_t*>(src);
      hb1[b] = *reinterpret_cast<const uint32_t*>(src + 2);
    }
  }
  const float fo = scale_pow2(cw, -eh);
  const uint8_t* dn = smem + kLSmDn + 8 * (b0 & 1) + 2 * t;
  if (!mbar_wait(&bar[3], 0)) note_timeout();
  if (!mbar_wait(&bar[4], 0)) note_timeout();
  const int kq = lane >> 2;  // lanes 0, 4, 8, 12: which 4 rows of a tile they add into out
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int T = warp + kLWarps * i;
    const int r0 = 16 * T + g, r1 = r0 + 8;
    const uint32_t sc0 = dsc[r0], sc1 = dsc[r1];
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int b = 0; b < kLMaxBlk; ++b) {
      if (b < nbl) {
        const uint32_t w0 = lds16(dn + r0 * kLDnRow + 8 * b);
        const uint32_t w1 = lds16(dn + r1 * kLDnRow + 8 * b);
        uint32_t s0, s1, e[4];
        e4m3x2_to_bcast(((sc0 >> (8 * b)) & 0xffu) | (((sc1 >> (8 * b)) & 0xffu) << 8), s0, s1);
        e2m1x8_to_f16x2(w0 | (w1 << 16), e);  // e[0], e[1]: row r0 bytes 2t, 2t+1; e[2], e[3]: row r1
        const uint32_t a[4] = {hmul2_u32(e[0], s0), hmul2_u32(e[2], s1), hmul2_u32(e[1], s0), hmul2_u32(e[3], s1)};
        mma_16816(d, a, hb0[b], hb1[b]);
      }
    }
    // rows r0 (v0) and r1 (v1) live in lane 4g
    const float v0 = d[0] + d[1], v1 = d[2] + d[3];
    float q[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int src = 4 * (4 * (kq & 1) + k);
      const float a0 = __shfl_sync(0xffffffffu, v0, src), a1 = __shfl_sync(0xffffffffu, v1, src);
      q[k] = (kq < 2 ? a0 : a1) * fo;
    }
    if (t == 0 && kq < 4)
      atomicAdd(reinterpret_cast<float4*>(out + 16 * T + 4 * kq), make_float4(q[0], q[1], q[2], q[3]));
  }
}

// Whether the slice split fits this device: every CTA <= kLMaxBlk blocks.
inline bool slice_fits(int K, const DeviceInfo* dev) {
  if (K < 1 || K > 10 || static_cast<size_t>(kLSmTotal) > dev->smem_optin) return false;
  const SliceSplit sp{dev->sm_count, K};
  for (int c = 0; c < sp.grid; ++c) {
    int j, b0, b1, ci, cn;
    sp.blocks(c, j, b0, b1, ci, cn);
    if (b1 - b0 > kLMaxBlk) return false;
  }
  return kHid == 4 * kLThreads;
}

inline int launch_moe_decode_slice(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                                   const float* coef, const void* x, int x_dtype, float* h_buf, float* out, int K,
                                   cudaStream_t st, const DeviceInfo* dev) {
  CUtensorMap dn_map;
  const uint64_t nbk = static_cast<uint64_t>(n_blocks);
  {  // down rows as bytes: [block][10 row groups][256 rows][320 B]
    const uint64_t dims[4] = {320, 256, 10, nbk}, strides[3] = {320, 81920, static_cast<uint64_t>(kBlock)};
    const uint32_t box[4] = {32, 256, 5, 1};
    int rc = tensor_map_nd(table + kODW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, dims, strides, box, dev->device, &dn_map,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (rc) return rc;
  }
  auto fn = x_dtype == QFN_DTYPE_F32 ? moe_decode_slice<true> : moe_decode_slice<false>;
  static bool attr_set[64][2] = {};
  const int ti = x_dtype == QFN_DTYPE_F32 ? 1 : 0;
  if (!attr_set[dev->device][ti]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kLSmTotal);
    if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "slice decode smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev->device][ti] = true;
  }
  const int slot = next_decode_slot(dev->device);
  // Cooperative (every CTA resident: a CTA waits for the others' zeroing) and a
  // programmatic dependent of the previous kernel in the stream.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(dev->sm_count);
  cfg.blockDim = dim3(kLThreads);
  cfg.dynamicSmemBytes = kLSmTotal;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, dn_map, table, n_blocks, sidx, s2, coef, x, h_buf,
                                     out, K, slot);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "moe_decode_slice launch: %s", cudaGetErrorString(e));
  return check_launch("moe_decode_slice");
}

}  // namespace qfn
