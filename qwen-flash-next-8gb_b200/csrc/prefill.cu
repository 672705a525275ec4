// Batched-prefill NVFP4 SwiGLU MoE layer: the grouped expert GEMM.
//
// Restates the expert loop of QwenEngine.moe (qwen_engine.py:835-852):
//   for each expert e with routed tokens:
//     h = silu(x[tok] @ Wg_e^T) * (x[tok] @ Wu_e^T)           (fp32)
//     out.index_add_(tok, (h @ Wd_e^T) * tv[tok, slot])        (fp32)
// with the weights of qmoe.block_deq (qmoe.py:93-111): e2m1 code x E4M3 block
// scale (one per 16 k) x per-tensor ws2.
//
// Pipeline (one stream: a memset of out, then seven launches, each a
// programmatic dependent of the one before):
//  1. pf_count / pf_plan / pf_scatter: (token, slot) pairs grouped by expert
//     (a counting sort over 64 slices of the pairs), and tiles of up to 128
//     pairs of one expert.
//  2. pf_gather_x: the x row of every pair in pair order, as f16 scaled by a
//     power of two per token (max |x| in [2^14, 2^15)): exact for bf16 x.
//  3. pf_gemm<GATEUP>: per (tile, 128 features): D[128 rows][pairs] = A x B^T
//     twice (gate rows, up rows) on tcgen05 (kind::f16, fp32 accumulators in
//     TMEM).  A = the expert's rows dequantised from NVFP4 to f16 in shared
//     memory (e2m1 x E4M3 is exact in f16), B = the tile's x rows (TMA,
//     128-byte swizzle).  Epilogue: h = silu(ws2_g g) * (ws2_u u) in fp32.
//  4. pf_hpack: h rows -> f16 hi + lo (h * 2^e = hi + lo, one e per pair).
//  5. pf_gemm<DOWN>: per (tile, 128 output rows): A = down rows, B = the
//     tile's h hi rows followed by its h lo rows (one MMA computes both;
//     the epilogue sums the two column blocks: ~22-bit h), and adds
//     coef * ws2_d * D into out with fp32 atomics (as index_add_ on CUDA).
//
// pf_gemm is persistent (one CTA per SM) and warp-specialised: warp 0 loads
// the activation tiles (TMA) into a ring of stages and hands out the jobs;
// warp 3 loads the raw e2m1 rows and their scales; warps 4-19 dequantise the
// raw rows of each stage into the f16 A operand in TMEM; one thread of warp 1
// issues the MMAs; warps 20-23 drain the TMEM accumulators (two halves, so the
// epilogue of one job overlaps the next job's MMAs).  Every wait is bounded;
// a wait that runs out sets a status bit.
#include <cuda_fp16.h>

#include <utility>

#include "common.cuh"
#include "host.cuh"

namespace qfn {

constexpr int kPfRows = 128;           // pairs per tile (MMA N <= 128) and A rows (MMA M)
#ifndef PF_DEQ_WARPS
#define PF_DEQ_WARPS 16
#endif
// Warps: 0 activation producer, 1 MMA issuer, 2 spare, 3 weight producer,
// 4 .. 4 + kPfDeq - 1 dequantisers, the last 4 the epilogue.  The dequantisers
// come in groups of 8 (4 lane quarters x 2 matrices or K halves); with 16 the
// two groups take alternate K-blocks of a stage (twice the warps to hide the
// latency of the conversion chains: it is latency-, not issue-bound).
constexpr int kPfDeq = PF_DEQ_WARPS;
constexpr int kPfDeqSplit = kPfDeq / 8;
constexpr int kPfEpi0 = 4 + kPfDeq;                 // first epilogue warp
constexpr int kPfThreads = 32 * (kPfEpi0 + 4);
constexpr int kPfMaxExperts = 1024;
constexpr int kPfJobQ = 8;                           // job-queue slots (jobs handed to the roles ahead of use)
constexpr int kPfJobAhead = 2;                       // jobs warp 0 publishes beyond the one it works on
constexpr uint32_t kPfJobReaders = 2 + kPfDeq + 4;   // warps that read each job: MMA, weights, dequantisers, epilogue
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

// Three launches.  ti: [T][topk] expert ids (int32 or int64), tv: [T][topk]
// routing weights (bf16 or f32).  Outputs (workspace): hdr[0] = number of
// tiles, hdr[1] = number of valid pairs; offs[E + 1]; pair_tok[P], pair_w[P]
// (grouped by expert: by slice, then in shared-atomic order within a slice);
// tile_e/tile_p0/tile_n.  Scratch: hist/base [kPfRouteCtas][E].
// Launches of the prefill pipeline: each a programmatic dependent of the
// previous kernel in the stream (its launch and prologue overlap that
// kernel's tail; it waits with griddepcontrol.wait before touching memory).
template <typename... KArgs, typename... Args>
static cudaError_t pf_launch(void (*k)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                             Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

constexpr int kPfRouteCtas = 64;  // CTAs of the count and scatter passes, each a contiguous slice of the pairs

// (a) per-slice expert counts
template <typename TI>
__global__ void __launch_bounds__(1024) pf_count_kernel(const TI* __restrict__ ti, int64_t P, int E, int* hist) {
  pdl_wait();   // inputs come from the previous kernel in the stream
  pdl_launch_dependents();
  __shared__ int cnt[kPfMaxExperts];
  const int tid = threadIdx.x;
  for (int i = tid; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int64_t p0 = P * blockIdx.x / gridDim.x, p1 = P * (blockIdx.x + 1) / gridDim.x;
  for (int64_t p = p0 + tid; p < p1; p += blockDim.x) {
    const int64_t e = static_cast<int64_t>(ti[p]);
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    else if (e != -1) pf_flag(kPfStatusBadExpert);  // -1 marks a pair to skip (expert-parallel padding)
  }
  __syncthreads();
  for (int i = tid; i < E; i += blockDim.x) hist[blockIdx.x * E + i] = cnt[i];
}

// (b) one CTA (thread = expert): offsets, tiles, and each slice's first slot per expert
__global__ void __launch_bounds__(1024) pf_plan_kernel(const int* __restrict__ hist, int G, int E, int* hdr, int* offs,
                                                       int* tile_e, int* tile_p0, int* tile_n, int* base) {
  pdl_wait();   // inputs come from the previous kernel in the stream
  pdl_launch_dependents();
  __shared__ int tmp[32];
  const int tid = threadIdx.x;
  int c = 0;
  if (tid < E)
    for (int g = 0; g < G; ++g) c += hist[g * E + tid];
  int np, nt;
  const int o = block_exclusive_scan(c, tmp, &np);
  const int ntile = (c + kPfRows - 1) / kPfRows;
  const int tb = block_exclusive_scan(ntile, tmp, &nt);
  if (tid < E) {
    offs[tid] = o;
    for (int k = 0; k < ntile; ++k) {
      tile_e[tb + k] = tid;
      tile_p0[tb + k] = o + k * kPfRows;
      tile_n[tb + k] = min(kPfRows, c - k * kPfRows);
    }
    int b = o;
    for (int g = 0; g < G; ++g) {
      base[g * E + tid] = b;
      b += hist[g * E + tid];
    }
  }
  if (tid == 0) {
    offs[E] = np;
    hdr[0] = nt;
    hdr[1] = np;
    hdr[2] = 0;   // the job counters of the two GEMMs
    hdr[3] = 0;
  }
}

// (c) per-slice scatter of the pairs to their slots
template <typename TI, bool kTvBf16>
__global__ void __launch_bounds__(1024) pf_scatter_kernel(const TI* __restrict__ ti, const void* __restrict__ tv,
                                                          int64_t P, int topk, int E, const int* __restrict__ base,
                                                          int* pair_tok, float* pair_w) {
  pdl_wait();   // inputs come from the previous kernel in the stream
  pdl_launch_dependents();
  __shared__ int cur[kPfMaxExperts];
  const int tid = threadIdx.x;
  for (int i = tid; i < E; i += blockDim.x) cur[i] = base[blockIdx.x * E + i];
  __syncthreads();
  const int64_t p0 = P * blockIdx.x / gridDim.x, p1 = P * (blockIdx.x + 1) / gridDim.x;
  for (int64_t p = p0 + tid; p < p1; p += blockDim.x) {
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

template <typename TI>
static int pf_route(const TI* ti, const void* tv, bool tv_bf16, int64_t P, int topk, int E, int* hist, int* base,
                    int* hdr, int* offs, int* tile_e, int* tile_p0, int* tile_n, int* pair_tok, float* pair_w,
                    cudaStream_t st) {
  cudaError_t e = pf_launch(pf_count_kernel<TI>, kPfRouteCtas, 1024, 0, st, ti, P, E, hist);
  if (e == cudaSuccess)
    e = pf_launch(pf_plan_kernel, 1, 1024, 0, st, static_cast<const int*>(hist), kPfRouteCtas, E, hdr, offs, tile_e,
                  tile_p0, tile_n, base);
  if (e == cudaSuccess)
    e = tv_bf16 ? pf_launch(pf_scatter_kernel<TI, true>, kPfRouteCtas, 1024, 0, st, ti, tv, P, topk, E,
                            static_cast<const int*>(base), pair_tok, pair_w)
                : pf_launch(pf_scatter_kernel<TI, false>, kPfRouteCtas, 1024, 0, st, ti, tv, P, topk, E,
                            static_cast<const int*>(base), pair_tok, pair_w);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "pf_route launch: %s", cudaGetErrorString(e));
  return check_launch("pf_route");
}

// ---------------------------------------------------------------------------
// 2. x rows in pair order as f16 * 2^e (one warp per pair)

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One warp per pair (8 per CTA of 256): a lane loads 10 of the row's 320
// 16-byte chunks, the row maximum of |x| (NaN wins, as the block version it
// replaced) meets in a warp shuffle, and no block barrier is needed.
constexpr int kPfRowWarps = 8;

__device__ __forceinline__ float pf_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = nanmax_f(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void __launch_bounds__(32 * kPfRowWarps) pf_gather_x_kernel(const uint16_t* __restrict__ x,
                                                                      const int* __restrict__ hdr,
                                                                      const int* __restrict__ pair_tok,
                                                                      __half* x16, int* pair_ex) {
  pdl_wait();   // inputs come from the previous kernel in the stream
  pdl_launch_dependents();
  constexpr int kChunks = kHid / 8 / 32;  // 16-byte chunks per lane: 10
  const int lane = threadIdx.x & 31;
  const int p = blockIdx.x * kPfRowWarps + (threadIdx.x >> 5);
  if (p >= hdr[1]) return;  // warp-uniform
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(pair_tok[p]) * kHid);
  uint4 r[kChunks];
#pragma unroll
  for (int i = 0; i < kChunks; ++i) r[i] = src[lane + 32 * i];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const uint32_t w[4] = {r[i].x, r[i].y, r[i].z, r[i].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      m = nanmax_f(m, fabsf(bf16_bits_to_f32(w[k] & 0xffffu)));
      m = nanmax_f(m, fabsf(bf16_bits_to_f32(w[k] >> 16)));
    }
  }
  const int e = f16_prescale_exp(pf_warp_max(m));
  uint4* dst = reinterpret_cast<uint4*>(x16 + static_cast<int64_t>(p) * kHid);
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const uint32_t w[4] = {r[i].x, r[i].y, r[i].z, r[i].w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      o[k] = pack_f16x2(pow2_mul(bf16_bits_to_f32(w[k] & 0xffffu), e), pow2_mul(bf16_bits_to_f32(w[k] >> 16), e));
    dst[lane + 32 * i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (lane == 0) pair_ex[p] = e;
}

// ---------------------------------------------------------------------------
// 4. h rows -> f16 hi / lo with one power-of-two scale per pair (one warp per pair)

// One warp per pair (8 per CTA): a lane takes 5 of the row's 160 float4.
__global__ void __launch_bounds__(32 * kPfRowWarps) pf_hpack_kernel(const float* __restrict__ h32,
                                                                   const int* __restrict__ hdr, __half* hhi,
                                                                   __half* hlo, int* pair_eh) {
  pdl_wait();   // inputs come from the previous kernel in the stream
  pdl_launch_dependents();
  constexpr int kChunks = kInter / 4 / 32;  // float4 per lane: 5
  const int lane = threadIdx.x & 31;
  const int p = blockIdx.x * kPfRowWarps + (threadIdx.x >> 5);
  if (p >= hdr[1]) return;  // warp-uniform
  const float4* src = reinterpret_cast<const float4*>(h32 + static_cast<int64_t>(p) * kInter);
  float4 v[kChunks];
#pragma unroll
  for (int i = 0; i < kChunks; ++i) v[i] = src[lane + 32 * i];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kChunks; ++i)
    m = nanmax_f(m, nanmax_f(nanmax_f(fabsf(v[i].x), fabsf(v[i].y)), nanmax_f(fabsf(v[i].z), fabsf(v[i].w))));
  const int e = f16_prescale_exp(pf_warp_max(m));
  uint2* dh = reinterpret_cast<uint2*>(hhi + static_cast<int64_t>(p) * kInter);
  uint2* dl = reinterpret_cast<uint2*>(hlo + static_cast<int64_t>(p) * kInter);
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    __half h[4], l[4];
    split_f16(pow2_mul(v[i].x, e), h[0], l[0]);
    split_f16(pow2_mul(v[i].y, e), h[1], l[1]);
    split_f16(pow2_mul(v[i].z, e), h[2], l[2]);
    split_f16(pow2_mul(v[i].w, e), h[3], l[3]);
    dh[lane + 32 * i] = *reinterpret_cast<const uint2*>(h);
    dl[lane + 32 * i] = *reinterpret_cast<const uint2*>(l);
  }
  if (lane == 0) pair_eh[p] = e;
}

// ---------------------------------------------------------------------------
// 3 / 6. the grouped GEMM

enum { kGateUp = 0, kDown = 1 };

#ifndef PF_GU_SK
#define PF_GU_SK 2
#endif
#ifndef PF_DN_SK
#define PF_DN_SK 2
#endif

// A job is (tile of <= 128 pairs, 128 weight rows): gate/up jobs take 128
// features (their 128 gate rows and 128 up rows: two M = 128 accumulators
// that hold g and u of the same feature in the same TMEM lane); down jobs
// take 128 output rows.  The K loop runs in stages of two K-blocks of 64.
template <int MODE>
struct PfCfg;
template <>
struct PfCfg<kGateUp> {
  static constexpr int kRStages = 4;            // raw weight rows + scales (freed by the dequantisers)
  static constexpr int kRawKB = 4;              // K-blocks per raw stage: [gate|up][128 rows][128 B], 128-byte swizzle
  static constexpr int kKBlocks = kHid / 64;    // 40 K-blocks of 64
  static constexpr int kSub = kInter / 128;     // 5 jobs (128 features) per tile
  static constexpr int kStageKB = PF_GU_SK;     // K-blocks per stage
  static constexpr int kKStages = 4 / PF_GU_SK;  // stages in flight (A slots: 256 TMEM columns)
  static constexpr int kBMax = kStageKB * 16384;  // x tile per K-block: <= 128 rows x 64 f16
  static constexpr int kRawBytes = 32768;
  static constexpr int kRaw = kRawBytes + 4096;  // + [gate|up][128 rows][16 B] scales of the stage's 4 K-blocks
  static constexpr int kJobScales = 0;
  static constexpr uint32_t kASlot = 64 * kStageKB;  // TMEM columns per A slot: per K-block gate 32 + up 32
};
template <>
struct PfCfg<kDown> {
  static constexpr int kRStages = 6;
  static constexpr int kRawKB = 2;              // [128 rows][64 B], 64-byte swizzle
  static constexpr int kKBlocks = kInter / 64;  // 10
  static constexpr int kSub = kHid / 128;       // 20 jobs (128 output rows) per tile
  static constexpr int kStageKB = PF_DN_SK;
  static constexpr int kKStages = 4 / PF_DN_SK;
  static constexpr int kBMax = kStageKB * 2 * 16384;  // per K-block: h hi rows, then h lo rows
  static constexpr int kRawBytes = 8192;
  static constexpr int kRaw = kRawBytes;
  static constexpr int kJobScales = 128 * (kInter / 16);  // a job's 128 scale rows of 40 B, loaded once per job
  static constexpr uint32_t kASlot = 32 * kStageKB;  // per K-block 32 columns
};
// Stages: activation tiles in shared memory and A slots in TMEM, two K-blocks each.
// TMEM: columns [0, 256) hold the accumulators as two halves of 128 columns.
// Down jobs always take one half (a tile of <= 64 pairs: N = hi rows + lo
// rows of the box; larger tiles: hi and lo MMAs into the same N = 128
// accumulator); gate/up jobs of <= 64 pairs take one half (g in 64
// columns, u in the next 64), larger ones both.  A job in one half has its
// epilogue overlapped with the next job's MMAs.  Columns [256, 512) hold the
// dequantised A slots.
constexpr uint32_t kPfTmemA = 256;

template <int MODE>
struct PfSmem {
  using C = PfCfg<MODE>;
  static constexpr int kB = 0;
  static constexpr int kRaw = kB + C::kKStages * C::kBMax;
  static constexpr int kJs = kRaw + C::kRStages * C::kRaw;  // down: two per-job scale buffers
  static constexpr int kBar = kJs + 2 * C::kJobScales;
  static constexpr int kCols = kBar + 512;     // per-column epilogue data: 2 x 2 x 128 words
  static constexpr int kTotal = kCols + 2 * 2 * 128 * 4 + 1024;  // + alignment slack
};

// Activation tensor maps with boxes of 16, 32, 64 and 128 rows (a job loads
// the smallest box that holds its tile), the raw weight rows and the scale
// rows.
struct PfMaps {
  CUtensorMap b[4];
  CUtensorMap b_lo[4];  // down: h lo (gate/up: unused)
  CUtensorMap w;
  CUtensorMap s;
};

struct PfArgs {
  const int* hdr;
  const int* tile_e;
  const int* tile_p0;
  const int* tile_n;
  const int* pair_tok;
  const float* pair_w;
  const int* pair_ex;    // x exponent (GATEUP) or h exponent (DOWN) per pair
  const uint8_t* table;  // expert blocks
  int64_t base;          // table block of expert 0
  const float* s2l;      // [E][3]
  float* h32;            // GATEUP output [P][640]
  float* out;            // DOWN output [T][2560] (accumulated)
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

// Accumulator halves in use: the MMA issuers and the epilogue walk the same
// job sequence and keep identical copies of this state.
template <int MODE>
struct PfHalves {
  uint32_t u0 = 0u, u1 = 0u;  // jobs that used half 0 / half 1 so far
  int next = 0;
  // the half a job of n pairs takes (2 = both)
  __device__ __forceinline__ int pick(int n) const { return (MODE == kGateUp && n > 64) ? 2 : next; }
  __device__ __forceinline__ void done(int h) {
    if (h != 1) ++u0;
    if (h != 0) ++u1;
    next = h == 0 ? 1 : 0;
  }
};

__device__ __forceinline__ int pf_box(int n) { return n <= 16 ? 0 : (n <= 32 ? 1 : (n <= 64 ? 2 : 3)); }

template <int MODE>
__global__ void __launch_bounds__(kPfThreads, 1)
    pf_gemm_kernel(const __grid_constant__ PfMaps maps, const PfArgs args) {
  using C = PfCfg<MODE>;
  using L = PfSmem<MODE>;
  constexpr int KS = C::kKStages, SK = C::kStageKB, RS = C::kRStages, KB = C::kKBlocks, NST = KB / SK;
  constexpr int NI = 1;  // MMA issuers: one warp (a second issuing warp halves each one's MMA rate)
  static_assert(KB % SK == 0 && C::kRawKB % SK == 0 || SK % C::kRawKB == 0, "stage / raw stage sizes");
  static_assert(SK % kPfDeqSplit == 0 && C::kRawKB % kPfDeqSplit == 0, "dequantiser groups share a stage's K-blocks");
  static_assert(SK <= C::kRawKB, "a stage ends at most one raw stage");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  // stage s: activation tile s in shared memory + A slot s in TMEM.
  uint64_t* k_full = reinterpret_cast<uint64_t*>(smem + L::kBar);  // producer (tx) + the dequant warps
  uint64_t* k_empty = k_full + KS;   // NI MMA issuers (commit)
  uint64_t* r_full = k_empty + KS;
  uint64_t* r_empty = r_full + RS;   // the dequant warps
  uint64_t* tm_full = r_empty + RS;  // [2] accumulator halves: NI MMA issuers -> epilogue
  uint64_t* tm_empty = tm_full + 2;  // [2] 4 epilogue warps
  uint64_t* js_full = tm_empty + 2;  // [2] down: per-job scale rows
  uint64_t* js_empty = js_full + 2;  // [2] the dequant warps
  uint32_t* tslot = reinterpret_cast<uint32_t*>(js_empty + 2);
  volatile uint32_t* abort = tslot + 1;
  // job queue: warp 0 takes job indices from the call's counter and hands
  // them to the other roles through a ring of kPfJobQ slots
  uint64_t* jq_full = reinterpret_cast<uint64_t*>(tslot + 2);
  uint64_t* jq_empty = jq_full + kPfJobQ;
  int* jq_ids = reinterpret_cast<int*>(jq_empty + kPfJobQ);
  int* cols = reinterpret_cast<int*>(smem + L::kCols);  // [2][2][128]: per-column factors (epilogue)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort = 0u;
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 2);   // the activation producer (tx) + one arrival for all dequantisers
      mbar_init(&k_empty[s], NI);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 1);  // one arrival for all dequantisers
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&tm_full[h], NI);
      mbar_init(&tm_empty[h], 4);
      mbar_init(&js_full[h], 1);
      mbar_init(&js_empty[h], 1);
    }
    for (int q = 0; q < kPfJobQ; ++q) {
      mbar_init(&jq_full[q], 1);
      mbar_init(&jq_empty[q], kPfJobReaders);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tslot, 512);
  if (threadIdx.x == 32) {
    for (int h = 0; h < 4; ++h) {
      prefetch_tensormap(&maps.b[h]);
      if (MODE == kDown) prefetch_tensormap(&maps.b_lo[h]);
    }
    prefetch_tensormap(&maps.w);
    prefetch_tensormap(&maps.s);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // (the prologue above overlaps the previous kernel's tail; the tile lists,
  // activations and out come from earlier kernels in the stream)
  pdl_wait();
  pdl_launch_dependents();
  const int n_jobs = args.hdr[0] * C::kSub;
  // Gate/up jobs are handed out dynamically (an atomic counter in the
  // workspace header, zeroed by the plan kernel): a CTA whose jobs ran fast
  // takes more, so the CTAs finish together instead of each running a fixed
  // 1/grid of the jobs (measured: the slowest CTA ended 327 us after the
  // start against 309 us); every role walks the same sequence from the ring.
  // Down jobs are dealt statically (job blockIdx.x + q * grid), which measured
  // faster for them (286 against 301 us).
  int* const job_ctr = const_cast<int*>(args.hdr) + 2 + MODE;
  auto publish_job = [&](int q) -> int {   // warp 0, all lanes: the q-th job of this CTA (-1: none left)
    if (MODE == kDown) {   // down jobs (a few us each) measured faster dealt statically: 1/grid of the jobs per CTA
      const int u = static_cast<int>(blockIdx.x) + q * static_cast<int>(gridDim.x);
      if (lane == 0) jq_ids[q % kPfJobQ] = u < n_jobs ? u : -1;
      return u < n_jobs ? u : -1;
    }
    const int slot = q % kPfJobQ;
    if (!pf_wait(&jq_empty[slot], ((q / kPfJobQ) & 1) ^ 1, abort)) return -1;
    int u = -1;
    if (lane == 0) {
      u = atomicAdd(job_ctr, 1);
      if (u >= n_jobs) u = -1;
      jq_ids[slot] = u;
      mbar_arrive(&jq_full[slot]);
    }
    return __shfl_sync(0xffffffffu, u, 0);
  };
  auto next_job = [&](int q) -> int {      // a reading warp, all lanes
    if (MODE == kDown) {
      const int u = static_cast<int>(blockIdx.x) + q * static_cast<int>(gridDim.x);
      return u < n_jobs && !*abort ? u : -1;
    }
    const int slot = q % kPfJobQ;
    if (!pf_wait(&jq_full[slot], (q / kPfJobQ) & 1, abort)) return -1;
    const int u = *reinterpret_cast<volatile int*>(&jq_ids[slot]);
    __syncwarp();
    if (lane == 0) mbar_arrive(&jq_empty[slot]);
    return u;
  };

  if (warp == 0) {
    // ---------------- activation producer (warp 0; one elected lane issues):
    // per stage the tile's activation rows of two K-blocks (down: h hi and
    // h lo per K-block) in the smallest box that holds them, completing on
    // the stage's k_full barrier.
    int st = 0, pub = 0;
    bool fin = false;
    for (int jq = 0;; ++jq) {
      // keep kPfJobAhead jobs published beyond this one (the counter's atomic
      // round trip then stays off the path between two jobs)
      while (!fin && pub <= jq + kPfJobAhead) fin = publish_job(pub++) < 0;
      __syncwarp();
      const int u = *reinterpret_cast<volatile int*>(&jq_ids[jq % kPfJobQ]);
      if (u < 0 || *abort) break;
      const int t = u / C::kSub;
      const int p0 = args.tile_p0[t], hb = pf_box(args.tile_n[t]);
      const uint32_t bbytes = (16u << hb) * 128u;
      for (int q = 0; q < NST; ++q, ++st) {
        const int s = st % KS;
        pf_wait(&k_empty[s], ((st / KS) & 1) ^ 1, abort);
        if (elect_one()) {
          mbar_arrive_expect_tx(&k_full[s], (MODE == kDown ? 2 : 1) * SK * bbytes);
          uint8_t* bt = smem + L::kB + s * C::kBMax;
#pragma unroll
          for (int j = 0; j < SK; ++j) {
            const int kb = SK * q + j;
            if (MODE == kGateUp) {
              tma_load_2d(bt + j * bbytes, &maps.b[hb], 64 * kb, p0, &k_full[s]);
            } else {  // [hi rows][lo rows] per K-block
              tma_load_2d(bt + 2 * j * bbytes, &maps.b[hb], 64 * kb, p0, &k_full[s]);
              tma_load_2d(bt + (2 * j + 1) * bbytes, &maps.b_lo[hb], 64 * kb, p0, &k_full[s]);
            }
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == 3) {
    // ---------------- weight producer (warp 3; one elected lane issues): per raw stage the job's raw rows of
    // kRawKB K-blocks (gate/up: with their scale bytes); per down job its
    // 128 scale rows.  (An L2 prefetch of the next job's rows measured
    // slower: with the activation rows it overflows L2 and doubles DRAM reads.)
    int rt = 0, jj = 0;
    for (int jq = 0;; ++jq, ++jj) {
      const int u = next_job(jq);
      if (u < 0) break;
      const int t = u / C::kSub, sub = u % C::kSub;
      const int blk = static_cast<int>(args.base + args.tile_e[t]);
      if (MODE == kDown) {  // the job's scale rows: [64 row pairs][80 B]
        const int js = jj & 1;
        pf_wait(&js_empty[js], ((jj >> 1) & 1) ^ 1, abort);
        if (elect_one()) {
          mbar_arrive_expect_tx(&js_full[js], C::kJobScales);
          tma_load_3d(smem + L::kJs + js * C::kJobScales, &maps.s, 0, 64 * sub, blk, &js_full[js]);
        }
        __syncwarp();
      }
      for (int kb = 0; kb < KB; kb += C::kRawKB, ++rt) {
        const int sr = rt % RS;
        pf_wait(&r_empty[sr], ((rt / RS) & 1) ^ 1, abort);
        if (elect_one()) {
          mbar_arrive_expect_tx(&r_full[sr], C::kRaw);
          uint8_t* raw = smem + L::kRaw + sr * C::kRaw;
          if (MODE == kGateUp) {  // [gate|up][128 rows][128 B] + [gate|up][128 rows][16 B of scales]
            tma_load_4d(raw, &maps.w, 32 * kb, 128 * sub, 0, blk, &r_full[sr]);
            tma_load_4d(raw + C::kRawBytes, &maps.s, 4 * kb, 128 * sub, 0, blk, &r_full[sr]);
          } else {  // [128 rows][64 B]
            tma_load_2d(raw, &maps.w, 32 * kb, blk * 8640 + 5120 + 128 * sub, &r_full[sr]);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (one elected lane of warp 1 issues).  Gate/up:
    // the gate and the up accumulators, interleaved per k-step.  A single
    // issuing warp: measured on this part (M = 128, K = 16, A in TMEM), one
    // warp issues an MMA every 24 (N = 16) to 32 (N = 64) cycles, while two
    // warps issuing into separate accumulators take ~56 cycles per MMA.  Commits
    // once per stage (k_empty) and once per job (tm_full).
    constexpr int NG = MODE == kGateUp ? 2 : 1;
    int st = 0;
    PfHalves<MODE> hv;
    for (int jq = 0;; ++jq) {
      const int u = next_job(jq);
      if (u < 0) break;
      const int n = args.tile_n[u / C::kSub];
      const int hb = pf_box(n), rows = 16 << hb;
      const uint32_t bbytes = static_cast<uint32_t>(rows) * 128u;
      // gate/up: the tile's pairs (rounded up to 16); down: hi rows then lo rows
      // of the box in one MMA, or (128-row box) hi and lo in two MMAs
      const bool split = MODE == kDown && rows == 128;
      const int N = MODE == kDown ? (split ? 128 : 2 * rows) : (n <= 16 ? 16 : (n + 15) & ~15);
      const uint32_t idesc = idesc_f16(128, N);
      const int h = hv.pick(n);
      if (h != 1) pf_wait(&tm_empty[0], (hv.u0 & 1) ^ 1, abort);
      if (h != 0) pf_wait(&tm_empty[1], (hv.u1 & 1) ^ 1, abort);
      tc_fence_after();
      const uint32_t d0 = tmem + (h == 1 ? 128u : 0u);
      const uint32_t d1 = d0 + (h == 2 ? 128u : 64u);   // gate/up: the up accumulator
      // B descriptors differ only in the start address field (address / 16):
      // +2 per k-step of 16, +jstep per K-block, +lostep for the h lo rows.
      const uint64_t bdesc0 = umma_desc_sw128(smem_u32(smem + L::kB), 1024);
      const uint32_t jstep = ((MODE == kDown ? 2u : 1u) * bbytes) >> 4, lostep = bbytes >> 4;
      for (int q = 0; q < NST; ++q, ++st) {
        const int s = st % KS;
        pf_wait(&k_full[s], (st / KS) & 1, abort);
        tc_fence_after();
        if (elect_one()) {
          const uint32_t a = tmem + kPfTmemA + C::kASlot * s;
          const uint64_t bd = bdesc0 + static_cast<uint32_t>((s * C::kBMax) >> 4);
#pragma unroll
          for (int j = 0; j < SK; ++j) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint64_t bk = bd + (j * jstep + 2 * k);
              const bool acc = (j | k) != 0 || q > 0;
#pragma unroll
              for (int g = 0; g < NG; ++g) {
                const uint32_t ak = a + (MODE == kGateUp ? 64u : 32u) * j + 32 * g + 8 * k;
                mma_f16_ta(g ? d1 : d0, ak, bk, idesc, acc);
                if (split) mma_f16_ta(d0, ak, bk + lostep, idesc, true);
              }
            }
          }
          mma_commit(&k_empty[s]);
        }
        __syncwarp();
      }
      if (elect_one()) {
        if (h != 1) mma_commit(&tm_full[0]);
        if (h != 0) mma_commit(&tm_full[1]);
      }
      __syncwarp();
      hv.done(h);
    }
  } else if (warp >= 4 && warp < kPfEpi0) {
    // ---------------- dequantisers: warp 4 + w writes TMEM lanes 32 (w % 4) ..
    // + 31 of the A slot, K-blocks kbs, kbs + kPfDeqSplit, ... of each stage
    // (group kbs = w / 8).  Gate/up: matrix i = (w / 4) % 2 (gate / up rows of
    // the job's 128 features), 64 k per K-block; down: K half i (32 k) of the
    // job's 128 output rows.  A warp converts its K-blocks of the stage into
    // registers before it waits for the A slot, so the conversion overlaps the
    // MMAs of the previous stage.
    constexpr int SKT = SK / kPfDeqSplit;  // K-blocks of a stage per thread
    const int w = warp - 4;
    const int kbs = w >> 3;
    const int i = (w >> 2) & 1;
    const int r = 32 * (w & 3) + lane;    // A row = TMEM lane
    const int d = 128 * i + r;            // gate/up: row of the raw stage ([gate|up][128])
    // raw row of this thread in a raw stage (gate/up: 128-byte rows, 128-byte
    // swizzle; down: 64-byte rows, 64-byte swizzle)
    const int raw_row = MODE == kGateUp ? d * 128 : r * 64;
    const int swz = MODE == kGateUp ? (d & 7) : ((r >> 1) & 3);
    const uint32_t lane_base = static_cast<uint32_t>(32 * (w & 3)) << 16;
    constexpr int NV = MODE == kGateUp ? 32 : 16;  // f16x2 words per K-block and thread
    int st = 0, jj = 0;
    uint4 sc = make_uint4(0, 0, 0, 0);
    for (int jq = 0;; ++jq, ++jj) {
      const int u = next_job(jq);
      if (u < 0) break;
      const uint8_t* jsc = smem + L::kJs + (jj & 1) * C::kJobScales + r * (kInter / 16);
      if (MODE == kDown) pf_wait(&js_full[jj & 1], (jj >> 1) & 1, abort);
      for (int q = 0; q < NST; ++q, ++st) {
        const int s = st % KS;
        uint32_t v[SKT][NV];
#pragma unroll
        for (int jt = 0; jt < SKT; ++jt) {
          const int kb = SK * q + kbs + kPfDeqSplit * jt;
          const int gkb = jj * KB + kb;  // K-blocks of this CTA so far
          const int rt = gkb / C::kRawKB, sr = rt % RS;
          const int kr = kb % C::kRawKB;  // K-block within the raw stage
          const uint8_t* stage = smem + L::kRaw + sr * C::kRaw;
          if (kr < kPfDeqSplit) {   // this thread's first K-block of the raw stage
            pf_wait(&r_full[sr], (rt / RS) & 1, abort);
            if (MODE == kGateUp) sc = *reinterpret_cast<const uint4*>(stage + C::kRawBytes + 16 * d);
          }
          const uint32_t sw = MODE == kGateUp ? (kr == 0 ? sc.x : (kr == 1 ? sc.y : (kr == 2 ? sc.z : sc.w)))
                                              : *reinterpret_cast<const uint32_t*>(jsc + 4 * kb);
          const uint8_t* raw = stage + raw_row;
          uint32_t sa0, sa1, sa2, sa3;
          e4m3x2_to_bcast(sw & 0xffffu, sa0, sa1);
          e4m3x2_to_bcast(sw >> 16, sa2, sa3);
          if (MODE == kGateUp) {
            const uint4 w0 = *reinterpret_cast<const uint4*>(raw + (((2 * kr) ^ swz) << 4));
            const uint4 w1 = *reinterpret_cast<const uint4*>(raw + (((2 * kr + 1) ^ swz) << 4));
            const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int jq = 0; jq < 8; ++jq) {
              uint32_t hf[4];
              e2m1x8_to_f16x2(words[jq], hf);
              const uint32_t sc2 = jq < 2 ? sa0 : (jq < 4 ? sa1 : (jq < 6 ? sa2 : sa3));
#pragma unroll
              for (int e = 0; e < 4; ++e) v[jt][(4 * jq + e) % NV] = hmul2_u32(hf[e], sc2);
            }
          } else {
            const uint4 w0 = *reinterpret_cast<const uint4*>(raw + (((2 * kr + i) ^ swz) << 4));
            const uint32_t words[4] = {w0.x, w0.y, w0.z, w0.w};
            const uint32_t s0 = i ? sa2 : sa0, s1 = i ? sa3 : sa1;
#pragma unroll
            for (int jq = 0; jq < 4; ++jq) {
              uint32_t hf[4];
              e2m1x8_to_f16x2(words[jq], hf);
              const uint32_t sc2 = jq < 2 ? s0 : s1;
#pragma unroll
              for (int e = 0; e < 4; ++e) v[jt][4 * jq + e] = hmul2_u32(hf[e], sc2);
            }
          }
        }
        pf_wait(&k_empty[s], ((st / KS) & 1) ^ 1, abort);
        tc_fence_after();
        const uint32_t aslot = tmem + kPfTmemA + C::kASlot * s + lane_base;
#pragma unroll
        for (int jt = 0; jt < SKT; ++jt) {
          const int j = kbs + kPfDeqSplit * jt;
          if (MODE == kGateUp) tmem_st_x32(aslot + 64 * j + 32 * i, *reinterpret_cast<uint32_t(*)[32]>(v[jt]));
          else tmem_st_x16(aslot + 32 * j + 16 * i, *reinterpret_cast<uint32_t(*)[16]>(v[jt]));
        }
        tmem_st_wait();
        tc_fence_before();
        // All dequantiser warps meet on a named barrier and one thread signals
        // the MMA issuer (and releases the raw stage and the job's scale rows
        // when this stage used their last K-block): one mbarrier arrival per
        // handoff instead of one per warp (arrivals on one mbarrier serialise).
        asm volatile("bar.sync 2, %0;" ::"n"(32 * kPfDeq) : "memory");
        if (w == 0 && lane == 0) {
          mbar_arrive(&k_full[s]);
          const int last_kb = SK * q + SK - 1;
          if (last_kb % C::kRawKB == C::kRawKB - 1)
            mbar_arrive(&r_empty[((jj * KB + last_kb) / C::kRawKB) % RS]);
          if (MODE == kDown && q == NST - 1) mbar_arrive(&js_empty[jj & 1]);
        }
      }
    }
  } else if (warp >= kPfEpi0) {
    // ---------------- epilogue: warp kPfEpi0 + q reads TMEM lanes 32q .. 32q + 31
    const int q = warp - kPfEpi0;
    const int et = threadIdx.x - 32 * kPfEpi0;  // 0..127
    int jj = 0;
    PfHalves<MODE> hv;
    for (int jq = 0;; ++jq, ++jj) {
      const int u = next_job(jq);
      if (u < 0) break;
      const int t = u / C::kSub, sub = u % C::kSub;
      const int e = args.tile_e[t], p0 = args.tile_p0[t], n = args.tile_n[t];
      // per-column factors of the job: gate/up: ws2_g 2^-ex, ws2_u 2^-ex;
      // down: coef ws2_d 2^-eh and the token's output row offset
      float* cf = reinterpret_cast<float*>(cols) + (jj & 1) * 2 * 128;
      int* ci = reinterpret_cast<int*>(cf + 128);
      if (et < n) {
        const int ex = args.pair_ex[p0 + et];
        if (MODE == kGateUp) {
          cf[et] = pow2_mul(args.s2l[3 * e + 0], -ex);
          reinterpret_cast<float*>(ci)[et] = pow2_mul(args.s2l[3 * e + 1], -ex);
        } else {
          cf[et] = pow2_mul(args.pair_w[p0 + et] * args.s2l[3 * e + 2], -ex);
          ci[et] = args.pair_tok[p0 + et];
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int h = hv.pick(n);
      if (h != 1) pf_wait(&tm_full[0], hv.u0 & 1, abort);
      if (h != 0) pf_wait(&tm_full[1], hv.u1 & 1, abort);
      tc_fence_after();
      const uint32_t t0 = tmem + (static_cast<uint32_t>(32 * q) << 16) + (h == 1 ? 128u : 0u);
      if (MODE == kGateUp) {
        const uint32_t t1 = t0 + (h == 2 ? 128u : 64u);
        const float* fu = reinterpret_cast<const float*>(ci);
        float* hrow = args.h32 + static_cast<int64_t>(p0) * kInter + 128 * sub + 32 * q + lane;
        for (int c0 = 0; c0 < n; c0 += 16) {
          uint32_t vg[16], vu[16];
          tmem_ld_x16(t0 + c0, vg);
          tmem_ld_x16(t1 + c0, vu);
          const int lim = n - c0;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (c < lim) {
              const float gg = __uint_as_float(vg[c]) * cf[c0 + c];
              const float uu = __uint_as_float(vu[c]) * fu[c0 + c];
              hrow[(c0 + c) * kInter] = __fdividef(gg, 1.0f + __expf(-gg)) * uu;
            }
          }
        }
      } else {
        const int rows = 16 << pf_box(n);
        float* orow = args.out + 128 * sub + 32 * q + lane;
        for (int c0 = 0; c0 < n; c0 += 16) {
          uint32_t vh[16], vl[16];
          tmem_ld_x16(t0 + c0, vh);
          if (rows < 128) tmem_ld_x16(t0 + rows + c0, vl);  // lo columns (128-row boxes: summed by the MMA)
          const int lim = n - c0;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (c < lim) {
              const float v = rows < 128 ? __uint_as_float(vh[c]) + __uint_as_float(vl[c]) : __uint_as_float(vh[c]);
              atomicAdd(orow + static_cast<int64_t>(ci[c0 + c]) * kHid, v * cf[c0 + c]);
            }
          }
        }
      }
      tc_fence_before();
      asm volatile("bar.sync 1, 128;" ::: "memory");  // per-column data is reused two jobs later
      if (lane == 0) {
        if (h != 1) mbar_arrive(&tm_empty[0]);
        if (h != 0) mbar_arrive(&tm_empty[1]);
      }
      hv.done(h);
    }
  }
  __syncwarp();   // the role loops end with diverged lanes (elected issuers): reconverge before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// host side

struct PfWs {  // byte offsets in the workspace
  size_t hdr, offs, rhist, rbase, tile_e, tile_p0, tile_n, pair_tok, pair_w, pair_ex, pair_eh, x16, h32, hhi, hlo, total;
};

static inline size_t pf_align(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static PfWs pf_ws_map(int64_t T, int topk, int E) {
  const int64_t P = T * topk;
  const int64_t NT = E + (P + kPfRows - 1) / kPfRows + 1;
  PfWs w;
  size_t o = 0;
  w.hdr = o; o = pf_align(o + 16);
  w.offs = o; o = pf_align(o + 4 * (E + 1));
  w.rhist = o; o = pf_align(o + 4 * static_cast<size_t>(kPfRouteCtas) * E);
  w.rbase = o; o = pf_align(o + 4 * static_cast<size_t>(kPfRouteCtas) * E);
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
static int pf_launch_gemm(const PfMaps& maps, const PfArgs& a, const DeviceInfo* dev, cudaStream_t st) {
  constexpr int smem = PfSmem<MODE>::kTotal;
  static bool attr_set[64] = {};
  if (!attr_set[dev->device]) {
    cudaError_t e = cudaFuncSetAttribute(pf_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "prefill gemm smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev->device] = true;
  }
  const int grid = dev->pf_ctas > 0 && dev->pf_ctas < dev->sm_count ? dev->pf_ctas : dev->sm_count;
  cudaError_t e = pf_launch(pf_gemm_kernel<MODE>, grid, kPfThreads, smem, st, maps, a);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "pf_gemm launch: %s", cudaGetErrorString(e));
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

  // 0. out = 0 (the down GEMM adds into it; zeroed first so that the kernels
  // after it follow one another as programmatic dependents)
  {
    cudaError_t e0 = cudaMemsetAsync(out, 0, static_cast<size_t>(T) * kHid * sizeof(float), st);
    if (e0 != cudaSuccess) return set_error(QFN_ERR_CUDA, "qfn_moe_prefill: memset: %s", cudaGetErrorString(e0));
  }
  // 1. routing
  int* rhist = reinterpret_cast<int*>(ws + W.rhist);
  int* rbase = reinterpret_cast<int*>(ws + W.rbase);
  rc = ti_is_int64 ? pf_route(static_cast<const int64_t*>(ti), tv, tv_dtype == QFN_DTYPE_BF16, P, topk, n_experts,
                              rhist, rbase, hdr, offs, tile_e, tile_p0, tile_n, pair_tok, pair_w, st)
                   : pf_route(static_cast<const int32_t*>(ti), tv, tv_dtype == QFN_DTYPE_BF16, P, topk, n_experts,
                              rhist, rbase, hdr, offs, tile_e, tile_p0, tile_n, pair_tok, pair_w, st);
  if (rc) return rc;
  // 2. x rows in pair order
  const unsigned row_ctas = static_cast<unsigned>((P + kPfRowWarps - 1) / kPfRowWarps);
  cudaError_t e = pf_launch(pf_gather_x_kernel, row_ctas, 32 * kPfRowWarps, 0, st, static_cast<const uint16_t*>(x),
                            static_cast<const int*>(hdr), static_cast<const int*>(pair_tok), x16, pair_ex);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "pf_gather_x launch: %s", cudaGetErrorString(e));
  if ((rc = check_launch("pf_gather_x"))) return rc;

  // tensor maps
  PfMaps gu_maps, dn_maps;
  for (int hb = 0; hb < 4; ++hb) {
    const uint32_t rows = 16u << hb;
    if ((rc = tensor_map_2d(x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kHid, P, kHid * 2, 64, rows,
                            CU_TENSOR_MAP_SWIZZLE_128B, dev->device, &gu_maps.b[hb])))
      return rc;
    gu_maps.b_lo[hb] = gu_maps.b[hb];
    if ((rc = tensor_map_2d(hhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kInter, P, kInter * 2, 64, rows,
                            CU_TENSOR_MAP_SWIZZLE_128B, dev->device, &dn_maps.b[hb])))
      return rc;
    if ((rc = tensor_map_2d(hlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kInter, P, kInter * 2, 64, rows,
                            CU_TENSOR_MAP_SWIZZLE_128B, dev->device, &dn_maps.b_lo[hb])))
      return rc;
  }
  {  // gate and up rows of a block: [block][gate|up][640 rows][1280 B]
    const uint64_t dims[4] = {1280, 640, 2, static_cast<uint64_t>(n_blocks)};
    const uint64_t strides[3] = {1280, 819200, static_cast<uint64_t>(kBlock)};
    const uint32_t box[4] = {128, 128, 2, 1};
    if ((rc = tensor_map_nd(table, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, dims, strides, box, dev->device, &gu_maps.w,
                            CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  if ((rc = tensor_map_2d(table, CU_TENSOR_MAP_DATA_TYPE_UINT8, 320, n_blocks * 8640, 320, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_64B, dev->device, &dn_maps.w)))
    return rc;
  {  // gate and up scale rows: [block][gate|up][640 rows][160 B]; a box is 16 B (4 K-blocks) of 128 rows of both
    const uint64_t dims[4] = {160, 640, 2, static_cast<uint64_t>(n_blocks)};
    const uint64_t strides[3] = {160, static_cast<uint64_t>(kOUS - kOGS), static_cast<uint64_t>(kBlock)};
    const uint32_t box[4] = {16, 128, 2, 1};
    if ((rc = tensor_map_nd(table + kOGS, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, dims, strides, box, dev->device,
                            &gu_maps.s)))
      return rc;
  }
  {  // down scale rows as row pairs: [block][1280 pairs][80 B]; a box is a job's 128 rows
    const uint64_t dims[3] = {80, 1280, static_cast<uint64_t>(n_blocks)};
    const uint64_t strides[2] = {80, static_cast<uint64_t>(kBlock)};
    const uint32_t box[3] = {80, 64, 1};
    if ((rc = tensor_map_nd(table + kODS, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, dims, strides, box, dev->device,
                            &dn_maps.s)))
      return rc;
  }

  // 3. gate/up
  PfArgs a{hdr, tile_e, tile_p0, tile_n, pair_tok, pair_w, pair_ex, table, base, s2l, h32, out};
  if ((rc = pf_launch_gemm<kGateUp>(gu_maps, a, dev, st))) return rc;
  // 4. h -> f16 hi/lo
  e = pf_launch(pf_hpack_kernel, row_ctas, 32 * kPfRowWarps, 0, st, static_cast<const float*>(h32),
                static_cast<const int*>(hdr), hhi, hlo, pair_eh);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "pf_hpack launch: %s", cudaGetErrorString(e));
  if ((rc = check_launch("pf_hpack"))) return rc;
  // 5. down + combine (into out, zeroed at entry)
  a.pair_ex = pair_eh;
  return pf_launch_gemm<kDown>(dn_maps, a, dev, st);
}

extern "C" int qfn_set_prefill_sm_budget(int n_sms) {
  QFN_REQUIRE(n_sms >= 0, QFN_ERR_INVALID_ARG, "qfn_set_prefill_sm_budget: n_sms=%d", n_sms);
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  dev->pf_ctas = n_sms;
  return QFN_OK;
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
