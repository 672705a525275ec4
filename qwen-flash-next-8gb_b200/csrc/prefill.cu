// Batched-prefill NVFP4 SwiGLU MoE layer: the grouped expert GEMM.
//
// Restates the expert loop of QwenEngine.moe (qwen_engine.py:835-852):
//   for each expert e with routed tokens:
//     h = silu(x[tok] @ Wg_e^T) * (x[tok] @ Wu_e^T)           (fp32)
//     out.index_add_(tok, (h @ Wd_e^T) * tv[tok, slot])        (fp32)
// with the weights of qmoe.block_deq (qmoe.py:93-111): e2m1 code x E4M3 block
// scale (one per 16 k) x per-tensor ws2.
//
// Pipeline (one stream, six launches):
//  1. pf_route: (token, slot) pairs grouped by expert (counting sort), and
//     tiles of up to 128 pairs of one expert.
//  2. pf_gather_x: the x row of every pair in pair order, as f16 scaled by a
//     power of two per token (max |x| in [2^14, 2^15)): exact for bf16 x.
//  3. pf_gemm<GATEUP>: per (tile, 64 features): D[128 rows][pairs] = A x B^T
//     on tcgen05 (kind::f16, fp32 accumulators in TMEM).  A = 64 gate rows +
//     64 up rows of the expert, dequantised from NVFP4 to f16 in shared memory
//     (e2m1 x E4M3 is exact in f16), B = the tile's x rows (TMA, 128-byte
//     swizzle).  Epilogue: h = silu(ws2_g g) * (ws2_u u) in fp32.
//  4. pf_hpack: h rows -> f16 hi + lo (h * 2^e = hi + lo, one e per pair).
//  5. out = 0.
//  6. pf_gemm<DOWN>: per (tile, 128 output rows): A = down rows, B = h hi
//     and h lo (two MMAs into one accumulator: ~22-bit h), epilogue adds
//     coef * ws2_d * D into out with fp32 atomics (as index_add_ on CUDA).
//
// pf_gemm is persistent (one CTA per SM) and warp-specialised: warp 0 issues
// TMA loads (activation tiles, raw e2m1 rows, scale rows) into a ring of
// stages; warps 4-7 dequantise the raw rows of each stage into the f16 A
// tile; one thread of warp 1 issues the MMAs; warps 8-11 drain the TMEM
// accumulators (two, so the epilogue of one job overlaps the next job's
// MMAs).  Every wait is bounded; a wait that runs out sets a status bit.
#include <cuda_fp16.h>

#include "common.cuh"
#include "host.cuh"

namespace qfn {

constexpr int kPfRows = 128;           // pairs per tile (MMA N <= 128) and A rows (MMA M)
constexpr int kPfThreads = 384;
constexpr int kPfMaxExperts = 1024;
constexpr unsigned kPfStatusTimeout = 1u, kPfStatusBadExpert = 4u;

__device__ unsigned int g_prefill_status = 0;
__device__ __forceinline__ void pf_flag(unsigned bit) { atomicOr(&g_prefill_status, bit); }

static __device__ __forceinline__ float nanmax_f(float a, float b) { return (isnan(b) || b > a) ? b : a; }

// v * 2^e, exact for |e| <= 252 (two normal power-of-two factors).
static __device__ __forceinline__ float pow2_mul(float v, int e) {
  const int a = e / 2, b = e - a;
  return v * __int_as_float((a + 127) << 23) * __int_as_float((b + 127) << 23);
}

// ---------------------------------------------------------------------------
// 1. routing: counting sort of the pairs by expert, tiles of <= 128 pairs

__device__ __forceinline__ int block_exclusive_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    tmp[lane] = w;
  }
  __syncthreads();
  const int incl = x + (warp ? tmp[warp - 1] : 0);
  *total = tmp[nw - 1];
  __syncthreads();
  return incl - v;
}

// One CTA of 1024 threads.  ti: [T][topk] expert ids (int32 or int64), tv:
// [T][topk] routing weights (bf16 or f32).  Outputs (workspace): hdr[0] =
// number of tiles, hdr[1] = number of valid pairs; offs[E + 1]; pair_tok[P],
// pair_w[P] (grouped by expert); tile_e/tile_p0/tile_n.
template <typename TI, bool kTvBf16>
__global__ void __launch_bounds__(1024) pf_route_kernel(const TI* __restrict__ ti, const void* __restrict__ tv,
                                                        int64_t T, int topk, int E, int* hdr, int* offs,
                                                        int* tile_e, int* tile_p0, int* tile_n, int* pair_tok,
                                                        float* pair_w) {
  __shared__ int cnt[kPfMaxExperts], cur[kPfMaxExperts], tmp[32];
  const int tid = threadIdx.x;
  const int64_t P = T * topk;
  for (int i = tid; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int64_t p = tid; p < P; p += blockDim.x) {
    const int64_t e = static_cast<int64_t>(ti[p]);
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    else pf_flag(kPfStatusBadExpert);
  }
  __syncthreads();
  const int c = tid < E ? cnt[tid] : 0;
  int np, nt;
  const int o = block_exclusive_scan(c, tmp, &np);
  const int ntile = (c + kPfRows - 1) / kPfRows;
  const int tb = block_exclusive_scan(ntile, tmp, &nt);
  if (tid < E) {
    offs[tid] = o;
    cur[tid] = o;
    for (int k = 0; k < ntile; ++k) {
      tile_e[tb + k] = tid;
      tile_p0[tb + k] = o + k * kPfRows;
      tile_n[tb + k] = min(kPfRows, c - k * kPfRows);
    }
  }
  if (tid == 0) {
    offs[E] = np;
    hdr[0] = nt;
    hdr[1] = np;
  }
  __syncthreads();
  for (int64_t p = tid; p < P; p += blockDim.x) {
    const int64_t e = static_cast<int64_t>(ti[p]);
    if (e < 0 || e >= E) continue;
    const int pos = atomicAdd(&cur[e], 1);
    pair_tok[pos] = static_cast<int>(p / topk);
    float w;
    if (kTvBf16) w = bf16_bits_to_f32(static_cast<const uint16_t*>(tv)[p]);
    else w = static_cast<const float*>(tv)[p];
    pair_w[pos] = w;
  }
}

// ---------------------------------------------------------------------------
// 2. x rows in pair order as f16 * 2^e (one CTA of 320 threads per pair)

__device__ __forceinline__ float pf_block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = (isnan(u) || u > v) ? u : v;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m = (isnan(red[w]) || red[w] > m) ? red[w] : m;
  return m;
}

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(320) pf_gather_x_kernel(const uint16_t* __restrict__ x, const int* __restrict__ hdr,
                                                          const int* __restrict__ pair_tok, __half* x16,
                                                          int* pair_ex) {
  __shared__ float red[10];
  const int p = blockIdx.x;
  if (p >= hdr[1]) return;
  const int t = pair_tok[p];
  const uint4 r = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * kHid)[threadIdx.x];
  float v[8];
  v[0] = bf16_bits_to_f32(r.x & 0xffffu); v[1] = bf16_bits_to_f32(r.x >> 16);
  v[2] = bf16_bits_to_f32(r.y & 0xffffu); v[3] = bf16_bits_to_f32(r.y >> 16);
  v[4] = bf16_bits_to_f32(r.z & 0xffffu); v[5] = bf16_bits_to_f32(r.z >> 16);
  v[6] = bf16_bits_to_f32(r.w & 0xffffu); v[7] = bf16_bits_to_f32(r.w >> 16);
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = fabsf(v[i]);
    m = (isnan(a) || a > m) ? a : m;
  }
  const int e = f16_prescale_exp(pf_block_max(m, red));
  uint4 o;
  o.x = pack_f16x2(pow2_mul(v[0], e), pow2_mul(v[1], e));
  o.y = pack_f16x2(pow2_mul(v[2], e), pow2_mul(v[3], e));
  o.z = pack_f16x2(pow2_mul(v[4], e), pow2_mul(v[5], e));
  o.w = pack_f16x2(pow2_mul(v[6], e), pow2_mul(v[7], e));
  reinterpret_cast<uint4*>(x16 + static_cast<int64_t>(p) * kHid)[threadIdx.x] = o;
  if (threadIdx.x == 0) pair_ex[p] = e;
}

// ---------------------------------------------------------------------------
// 4. h rows -> f16 hi / lo with one power-of-two scale per pair (160 threads)

__global__ void __launch_bounds__(160) pf_hpack_kernel(const float* __restrict__ h32, const int* __restrict__ hdr,
                                                       __half* hhi, __half* hlo, int* pair_eh) {
  __shared__ float red[5];
  const int p = blockIdx.x;
  if (p >= hdr[1]) return;
  const float4 v = reinterpret_cast<const float4*>(h32 + static_cast<int64_t>(p) * kInter)[threadIdx.x];
  float m = nanmax_f(nanmax_f(fabsf(v.x), fabsf(v.y)), nanmax_f(fabsf(v.z), fabsf(v.w)));
  const int e = f16_prescale_exp(pf_block_max(m, red));
  __half h[4], l[4];
  split_f16(pow2_mul(v.x, e), h[0], l[0]);
  split_f16(pow2_mul(v.y, e), h[1], l[1]);
  split_f16(pow2_mul(v.z, e), h[2], l[2]);
  split_f16(pow2_mul(v.w, e), h[3], l[3]);
  reinterpret_cast<uint2*>(hhi + static_cast<int64_t>(p) * kInter)[threadIdx.x] = *reinterpret_cast<const uint2*>(h);
  reinterpret_cast<uint2*>(hlo + static_cast<int64_t>(p) * kInter)[threadIdx.x] = *reinterpret_cast<const uint2*>(l);
  if (threadIdx.x == 0) pair_eh[p] = e;
}

// ---------------------------------------------------------------------------
// 3 / 6. the grouped GEMM

enum { kGateUp = 0, kDown = 1 };

template <int MODE>
struct PfCfg;
template <>
struct PfCfg<kGateUp> {
  static constexpr int kStages = 4;
  static constexpr int kKBlocks = kHid / 64;   // 40 K-blocks of 64
  static constexpr int kSub = kInter / 64;     // 10 jobs (64 features each) per tile
  static constexpr int kBBytes = 16384;        // x tile: 128 rows x 64 f16
  static constexpr int kScBytes = 2 * 64 * 160;  // gate + up scale rows of 64 features
};
template <>
struct PfCfg<kDown> {
  static constexpr int kStages = 3;
  static constexpr int kKBlocks = kInter / 64;  // 10
  static constexpr int kSub = kHid / 128;       // 20 jobs (128 output rows each) per tile
  static constexpr int kBBytes = 32768;         // h hi and h lo tiles
  static constexpr int kScBytes = 128 * 40;     // scale rows of 128 down rows
};

template <int MODE>
struct PfSmem {
  static constexpr int kB = 0;
  static constexpr int kA = kB + PfCfg<MODE>::kStages * PfCfg<MODE>::kBBytes;
  static constexpr int kRaw = kA + PfCfg<MODE>::kStages * 16384;
  static constexpr int kSc = kRaw + PfCfg<MODE>::kStages * 4096;
  static constexpr int kBar = kSc + 2 * PfCfg<MODE>::kScBytes;
  static constexpr int kCols = kBar + 256;     // per-column epilogue data: 2 x 3 x 128 words
  static constexpr int kTotal = kCols + 2 * 3 * 128 * 4 + 1024;  // + alignment slack
};

struct PfArgs {
  const int* hdr;
  const int* tile_e;
  const int* tile_p0;
  const int* tile_n;
  const int* pair_tok;
  const float* pair_w;
  const int* pair_ex;  // x exponent (GATEUP) or h exponent (DOWN) per pair
  int64_t base;        // table block of expert 0
  const float* s2l;    // [E][3]
  float* h32;          // GATEUP output [P][640]
  float* out;          // DOWN output [T][2560] (accumulated)
};

// Bounded wait.  After the first wait of a CTA runs out (`abort`, a word in
// the CTA's shared memory), every later wait returns at once, so a CTA whose
// pipeline broke drains in one time-out rather than one per wait.
__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*abort) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort = 1u;
  pf_flag(kPfStatusTimeout);
  return false;
}

template <int MODE>
__global__ void __launch_bounds__(kPfThreads, 1)
    pf_gemm_kernel(const __grid_constant__ CUtensorMap map_b0, const __grid_constant__ CUtensorMap map_b1,
                   const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_s,
                   const PfArgs args) {
  using C = PfCfg<MODE>;
  using L = PfSmem<MODE>;
  constexpr int S = C::kStages, KB = C::kKBlocks;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* a_ready = full + S;
  uint64_t* empty = a_ready + S;
  uint64_t* sc_full = empty + S;
  uint64_t* sc_empty = sc_full + 2;
  uint64_t* tm_full = sc_empty + 2;
  uint64_t* tm_empty = tm_full + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tm_empty + 2);
  volatile uint32_t* abort = tslot + 1;
  int* cols = reinterpret_cast<int*>(smem + L::kCols);  // [2][3][128]: token, weight bits, exponent
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort = 0u;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&a_ready[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sc_full[b], 1);
      mbar_init(&sc_empty[b], 4);
      mbar_init(&tm_full[b], 1);
      mbar_init(&tm_empty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tslot, 256);
  if (threadIdx.x == 32) {
    prefetch_tensormap(&map_b0);
    prefetch_tensormap(&map_w);
    prefetch_tensormap(&map_s);
    if (MODE == kDown) prefetch_tensormap(&map_b1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const int n_jobs = args.hdr[0] * C::kSub;

  if (warp == 0 && lane == 0) {
    // ---------------- producer
    int it = 0, jj = 0;
    for (int u = blockIdx.x; u < n_jobs; u += gridDim.x, ++jj) {
      const int t = u / C::kSub, sub = u % C::kSub;
      const int e = args.tile_e[t], p0 = args.tile_p0[t];
      const int64_t blk = args.base + e;
      const int sb = jj & 1;
      pf_wait(&sc_empty[sb], ((jj >> 1) & 1) ^ 1, abort);
      uint8_t* sc = smem + L::kSc + sb * C::kScBytes;
      mbar_arrive_expect_tx(&sc_full[sb], C::kScBytes);
      if (MODE == kGateUp) {
        const int f0 = 64 * sub;
        tma_load_2d(sc, &map_s, 0, static_cast<int>(blk * 17280 + 15360 + f0), &sc_full[sb]);
        tma_load_2d(sc + 64 * 160, &map_s, 0, static_cast<int>(blk * 17280 + 16000 + f0), &sc_full[sb]);
      } else {
        const int r0 = 128 * sub;
        tma_load_2d(sc, &map_s, 0, static_cast<int>(blk * 34560 + 33280 + r0 / 2), &sc_full[sb]);
      }
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        pf_wait(&empty[s], ((it / S) & 1) ^ 1, abort);
        mbar_arrive_expect_tx(&full[s], C::kBBytes + 4096);
        uint8_t* bt = smem + L::kB + s * C::kBBytes;
        uint8_t* raw = smem + L::kRaw + s * 4096;
        tma_load_2d(bt, &map_b0, 64 * kb, p0, &full[s]);
        if (MODE == kGateUp) {
          const int f0 = 64 * sub;
          tma_load_2d(raw, &map_w, 32 * kb, static_cast<int>(blk * 2160 + f0), &full[s]);
          tma_load_2d(raw + 2048, &map_w, 32 * kb, static_cast<int>(blk * 2160 + 640 + f0), &full[s]);
        } else {
          tma_load_2d(bt + 16384, &map_b1, 64 * kb, p0, &full[s]);
          tma_load_2d(raw, &map_w, 32 * kb, static_cast<int>(blk * 8640 + 5120 + 128 * sub), &full[s]);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    int it = 0, jj = 0;
    for (int u = blockIdx.x; u < n_jobs; u += gridDim.x, ++jj) {
      const int t = u / C::kSub;
      const int n = args.tile_n[t];
      const int N = n <= 16 ? 16 : (n + 15) & ~15;
      const uint32_t idesc = idesc_f16(128, N);
      const int ab = jj & 1;
      const uint32_t d = tmem + 128 * ab;
      pf_wait(&tm_empty[ab], ((jj >> 1) & 1) ^ 1, abort);
      tc_fence_after();
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        pf_wait(&a_ready[s], (it / S) & 1, abort);
        pf_wait(&full[s], (it / S) & 1, abort);
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + L::kA + s * 16384);
        const uint32_t b0 = smem_u32(smem + L::kB + s * C::kBBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          mma_f16(d, umma_desc_sw128(a0 + 32 * k, 1024), umma_desc_sw128(b0 + 32 * k, 1024), idesc, kb > 0 || k > 0);
          if (MODE == kDown)
            mma_f16(d, umma_desc_sw128(a0 + 32 * k, 1024), umma_desc_sw128(b0 + 16384 + 32 * k, 1024), idesc, true);
        }
        mma_commit(&empty[s]);
      }
      mma_commit(&tm_full[ab]);
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------- dequantisers: thread r builds A row r of every stage
    const int r = threadIdx.x - 128;
    int src_raw, src_sc;  // byte offsets of this row in the raw stage / scale buffer
    if (MODE == kGateUp) {
      const int q = r >> 5, i = r & 31;
      const int f = 16 * q + (i & 15);     // feature within the job's 64
      src_raw = (i < 16 ? 0 : 2048) + f * 32;
      src_sc = (i < 16 ? 0 : 64 * 160) + f * 160;
    } else {
      src_raw = r * 32;
      src_sc = r * 40;
    }
    const uint32_t a_row = (r >> 3) * 1024 + (r & 7) * 128;
    int it = 0, jj = 0;
    for (int u = blockIdx.x; u < n_jobs; u += gridDim.x, ++jj) {
      const int sb = jj & 1;
      pf_wait(&sc_full[sb], (jj >> 1) & 1, abort);
      const uint8_t* sc = smem + L::kSc + sb * C::kScBytes + src_sc;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        pf_wait(&full[s], (it / S) & 1, abort);
        const uint8_t* raw = smem + L::kRaw + s * 4096 + src_raw;
        const uint4 w0 = *reinterpret_cast<const uint4*>(raw);
        const uint4 w1 = *reinterpret_cast<const uint4*>(raw + 16);
        const uint32_t sw = *reinterpret_cast<const uint32_t*>(sc + 4 * kb);
        uint32_t sa0, sa1, sa2, sa3;
        e4m3x2_to_bcast(sw & 0xffffu, sa0, sa1);
        e4m3x2_to_bcast(sw >> 16, sa2, sa3);
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint8_t* a = smem + L::kA + s * 16384 + a_row;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t h[4];
          e2m1x8_to_f16x2(words[j], h);
          const uint32_t sc2 = j < 2 ? sa0 : (j < 4 ? sa1 : (j < 6 ? sa2 : sa3));
          const uint4 o = make_uint4(hmul2_u32(h[0], sc2), hmul2_u32(h[1], sc2), hmul2_u32(h[2], sc2),
                                     hmul2_u32(h[3], sc2));
          *reinterpret_cast<uint4*>(a + ((j ^ (r & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_ready[s]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sc_empty[sb]);
    }
  } else if (warp >= 8) {
    // ---------------- epilogue: warp 8 + q reads TMEM lanes 32q .. 32q + 31
    const int q = warp - 8;
    const int et = threadIdx.x - 256;  // 0..127
    int jj = 0;
    for (int u = blockIdx.x; u < n_jobs; u += gridDim.x, ++jj) {
      const int t = u / C::kSub, sub = u % C::kSub;
      const int e = args.tile_e[t], p0 = args.tile_p0[t], n = args.tile_n[t];
      const int ab = jj & 1;
      int* ccol = cols + ab * 3 * 128;
      // per-column data of this job (all four epilogue warps, then a named barrier)
      if (et < n) {
        ccol[et] = args.pair_tok[p0 + et];
        ccol[128 + et] = __float_as_int(args.pair_w[p0 + et]);
        ccol[256 + et] = args.pair_ex[p0 + et];
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      pf_wait(&tm_full[ab], (jj >> 1) & 1, abort);
      tc_fence_after();
      const uint32_t taddr = tmem + 128 * ab + (static_cast<uint32_t>(32 * q) << 16);
      if (MODE == kGateUp) {
        const float ws_g = args.s2l[3 * e + 0], ws_u = args.s2l[3 * e + 1];
        const int feat = 64 * sub + 16 * q + (lane & 15);
        for (int c0 = 0; c0 < n; c0 += 32) {
          uint32_t v[32];
          tmem_ld_x32(taddr + c0, v);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float mine = __uint_as_float(v[c]);
            const float up = __shfl_down_sync(0xffffffffu, mine, 16);
            const int col = c0 + c;
            if (lane < 16 && col < n) {
              const int ex = ccol[256 + col];
              const float g = pow2_mul(mine, -ex) * ws_g;
              const float uu = pow2_mul(up, -ex) * ws_u;
              args.h32[static_cast<int64_t>(p0 + col) * kInter + feat] = g / (1.0f + expf(-g)) * uu;
            }
          }
        }
      } else {
        const float ws_d = args.s2l[3 * e + 2];
        const int row = 128 * sub + 32 * q + lane;
        for (int c0 = 0; c0 < n; c0 += 32) {
          uint32_t v[32];
          tmem_ld_x32(taddr + c0, v);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int col = c0 + c;
            if (col < n) {
              const int tok = ccol[col];
              const float w = __int_as_float(ccol[128 + col]);
              const int eh = ccol[256 + col];
              const float val = pow2_mul(__uint_as_float(v[c]), -eh) * ws_d * w;
              atomicAdd(args.out + static_cast<int64_t>(tok) * kHid + row, val);
            }
          }
        }
      }
      tc_fence_before();
      asm volatile("bar.sync 1, 128;" ::: "memory");  // per-column data is reused two jobs later
      if (lane == 0) mbar_arrive(&tm_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------
// host side

struct PfWs {  // byte offsets in the workspace
  size_t hdr, offs, tile_e, tile_p0, tile_n, pair_tok, pair_w, pair_ex, pair_eh, x16, h32, hhi, hlo, total;
};

static inline size_t pf_align(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static PfWs pf_ws_map(int64_t T, int topk, int E) {
  const int64_t P = T * topk;
  const int64_t NT = E + (P + kPfRows - 1) / kPfRows + 1;
  PfWs w;
  size_t o = 0;
  w.hdr = o; o = pf_align(o + 16);
  w.offs = o; o = pf_align(o + 4 * (E + 1));
  w.tile_e = o; o = pf_align(o + 4 * NT);
  w.tile_p0 = o; o = pf_align(o + 4 * NT);
  w.tile_n = o; o = pf_align(o + 4 * NT);
  w.pair_tok = o; o = pf_align(o + 4 * P);
  w.pair_w = o; o = pf_align(o + 4 * P);
  w.pair_ex = o; o = pf_align(o + 4 * P);
  w.pair_eh = o; o = pf_align(o + 4 * P);
  w.x16 = o; o = pf_align(o + static_cast<size_t>(P) * kHid * 2);
  w.h32 = o; o = pf_align(o + static_cast<size_t>(P) * kInter * 4);
  w.hhi = o; o = pf_align(o + static_cast<size_t>(P) * kInter * 2);
  w.hlo = o; o = pf_align(o + static_cast<size_t>(P) * kInter * 2);
  w.total = o;
  return w;
}

template <int MODE>
static int pf_launch_gemm(const CUtensorMap& b0, const CUtensorMap& b1, const CUtensorMap& w, const CUtensorMap& s,
                          const PfArgs& a, const DeviceInfo* dev, cudaStream_t st) {
  constexpr int smem = PfSmem<MODE>::kTotal;
  static bool attr_set[64] = {};
  if (!attr_set[dev->device]) {
    cudaError_t e = cudaFuncSetAttribute(pf_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "prefill gemm smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev->device] = true;
  }
  pf_gemm_kernel<MODE><<<dev->sm_count, kPfThreads, smem, st>>>(b0, b1, w, s, a);
  return check_launch(MODE == kGateUp ? "pf_gemm<gate/up>" : "pf_gemm<down>");
}

}  // namespace qfn

using namespace qfn;

extern "C" size_t qfn_moe_prefill_workspace(int64_t T, int topk, int n_experts) {
  if (T <= 0 || topk <= 0 || n_experts <= 0) return 0;
  return pf_ws_map(T, topk, n_experts).total;
}

extern "C" int qfn_moe_prefill(const void* x, int64_t T, const void* ti, int ti_is_int64, const void* tv,
                               int tv_dtype, int topk, const uint8_t* table, int64_t n_blocks, int64_t base,
                               const float* s2l, int n_experts, float* out, void* workspace,
                               size_t workspace_bytes, qfn_stream_t stream) {
  QFN_REQUIRE(T >= 0 && topk >= 1 && topk <= QFN_MAX_TOPK, QFN_ERR_INVALID_ARG,
              "qfn_moe_prefill: T=%lld topk=%d", (long long)T, topk);
  QFN_REQUIRE(n_experts >= 1 && n_experts <= kPfMaxExperts, QFN_ERR_UNSUPPORTED,
              "qfn_moe_prefill: n_experts=%d outside [1, %d]", n_experts, kPfMaxExperts);
  QFN_REQUIRE(tv_dtype == QFN_DTYPE_F32 || tv_dtype == QFN_DTYPE_BF16, QFN_ERR_INVALID_ARG,
              "qfn_moe_prefill: bad tv dtype %d", tv_dtype);
  if (T == 0) return QFN_OK;
  QFN_REQUIRE(x && ti && tv && table && s2l && out && workspace, QFN_ERR_INVALID_ARG, "qfn_moe_prefill: null pointer");
  QFN_REQUIRE(base >= 0 && n_blocks > 0 && base + n_experts <= n_blocks, QFN_ERR_INVALID_ARG,
              "qfn_moe_prefill: experts [%lld, %lld) outside the table of %lld blocks", (long long)base,
              (long long)(base + n_experts), (long long)n_blocks);
  QFN_REQUIRE(T * topk <= (int64_t(1) << 30), QFN_ERR_UNSUPPORTED, "qfn_moe_prefill: too many pairs");
  QFN_REQUIRE(aligned(x, 16) && aligned(table, 16) && aligned(workspace, 256) && aligned(out, 16), QFN_ERR_ALIGNMENT,
              "qfn_moe_prefill: x, table, out must be 16-byte and workspace 256-byte aligned");
  const PfWs W = pf_ws_map(T, topk, n_experts);
  QFN_REQUIRE(workspace_bytes >= W.total, QFN_ERR_WORKSPACE, "qfn_moe_prefill: workspace %zu < %zu bytes",
              workspace_bytes, W.total);
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* hdr = reinterpret_cast<int*>(ws + W.hdr);
  int* offs = reinterpret_cast<int*>(ws + W.offs);
  int* tile_e = reinterpret_cast<int*>(ws + W.tile_e);
  int* tile_p0 = reinterpret_cast<int*>(ws + W.tile_p0);
  int* tile_n = reinterpret_cast<int*>(ws + W.tile_n);
  int* pair_tok = reinterpret_cast<int*>(ws + W.pair_tok);
  float* pair_w = reinterpret_cast<float*>(ws + W.pair_w);
  int* pair_ex = reinterpret_cast<int*>(ws + W.pair_ex);
  int* pair_eh = reinterpret_cast<int*>(ws + W.pair_eh);
  __half* x16 = reinterpret_cast<__half*>(ws + W.x16);
  float* h32 = reinterpret_cast<float*>(ws + W.h32);
  __half* hhi = reinterpret_cast<__half*>(ws + W.hhi);
  __half* hlo = reinterpret_cast<__half*>(ws + W.hlo);
  const int64_t P = T * topk;

  // 1. routing
  if (ti_is_int64) {
    if (tv_dtype == QFN_DTYPE_BF16)
      pf_route_kernel<int64_t, true><<<1, 1024, 0, st>>>(static_cast<const int64_t*>(ti), tv, T, topk, n_experts,
                                                         hdr, offs, tile_e, tile_p0, tile_n, pair_tok, pair_w);
    else
      pf_route_kernel<int64_t, false><<<1, 1024, 0, st>>>(static_cast<const int64_t*>(ti), tv, T, topk, n_experts,
                                                          hdr, offs, tile_e, tile_p0, tile_n, pair_tok, pair_w);
  } else {
    if (tv_dtype == QFN_DTYPE_BF16)
      pf_route_kernel<int32_t, true><<<1, 1024, 0, st>>>(static_cast<const int32_t*>(ti), tv, T, topk, n_experts,
                                                         hdr, offs, tile_e, tile_p0, tile_n, pair_tok, pair_w);
    else
      pf_route_kernel<int32_t, false><<<1, 1024, 0, st>>>(static_cast<const int32_t*>(ti), tv, T, topk, n_experts,
                                                          hdr, offs, tile_e, tile_p0, tile_n, pair_tok, pair_w);
  }
  if ((rc = check_launch("pf_route"))) return rc;
  // 2. x rows in pair order
  pf_gather_x_kernel<<<static_cast<unsigned>(P), 320, 0, st>>>(static_cast<const uint16_t*>(x), hdr, pair_tok, x16,
                                                                pair_ex);
  if ((rc = check_launch("pf_gather_x"))) return rc;

  // tensor maps
  CUtensorMap m_x, m_gw, m_gs, m_dw, m_ds, m_hhi, m_hlo;
  if ((rc = tensor_map_2d(x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kHid, P, kHid * 2, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B, dev->device, &m_x)))
    return rc;
  if ((rc = tensor_map_2d(table, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1280, n_blocks * 2160, 1280, 32, 64,
                          CU_TENSOR_MAP_SWIZZLE_NONE, dev->device, &m_gw)))
    return rc;
  if ((rc = tensor_map_2d(table, CU_TENSOR_MAP_DATA_TYPE_UINT8, 160, n_blocks * 17280, 160, 160, 64,
                          CU_TENSOR_MAP_SWIZZLE_NONE, dev->device, &m_gs)))
    return rc;
  if ((rc = tensor_map_2d(table, CU_TENSOR_MAP_DATA_TYPE_UINT8, 320, n_blocks * 8640, 320, 32, 128,
                          CU_TENSOR_MAP_SWIZZLE_NONE, dev->device, &m_dw)))
    return rc;
  if ((rc = tensor_map_2d(table, CU_TENSOR_MAP_DATA_TYPE_UINT8, 80, n_blocks * 34560, 80, 80, 64,
                          CU_TENSOR_MAP_SWIZZLE_NONE, dev->device, &m_ds)))
    return rc;
  if ((rc = tensor_map_2d(hhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kInter, P, kInter * 2, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B, dev->device, &m_hhi)))
    return rc;
  if ((rc = tensor_map_2d(hlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kInter, P, kInter * 2, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B, dev->device, &m_hlo)))
    return rc;

  // 3. gate/up
  PfArgs a{hdr, tile_e, tile_p0, tile_n, pair_tok, pair_w, pair_ex, base, s2l, h32, out};
  if ((rc = pf_launch_gemm<kGateUp>(m_x, m_x, m_gw, m_gs, a, dev, st))) return rc;
  // 4. h -> f16 hi/lo
  pf_hpack_kernel<<<static_cast<unsigned>(P), 160, 0, st>>>(h32, hdr, hhi, hlo, pair_eh);
  if ((rc = check_launch("pf_hpack"))) return rc;
  // 5. out = 0, 6. down + combine
  cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(T) * kHid * sizeof(float), st);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "qfn_moe_prefill: memset: %s", cudaGetErrorString(e));
  a.pair_ex = pair_eh;
  return pf_launch_gemm<kDown>(m_hhi, m_hlo, m_dw, m_ds, a, dev, st);
}

extern "C" int qfn_prefill_status(unsigned int* status, int clear) {
  QFN_REQUIRE(status, QFN_ERR_INVALID_ARG, "qfn_prefill_status: null pointer");
  cudaError_t e = cudaMemcpyFromSymbol(status, g_prefill_status, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_prefill_status, &zero, sizeof(unsigned int));
  }
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "qfn_prefill_status: %s", cudaGetErrorString(e));
  return QFN_OK;
}
