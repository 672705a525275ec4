// bs=1 NVFP4 SwiGLU expert layer over K experts + weighted combine.
//
// Restates qmoe.moe_decode (qmoe.py:77-83) and its two Triton kernels
// _gate_up (qmoe.py:24-51) and _down (qmoe.py:54-74), plus the torch
// reduction out_buf[:K].sum(0) (qmoe.py:83), in two launches:
//
//  gate_up: grid (640/16, K).  Each warp owns 2 output features of one expert
//    and streams the matching gate and up rows (1280 B each + 160 B of
//    scales) with 64-bit non-allocating loads issued before x is staged in
//    shared memory; it writes h[j][n] = silu(ws2_g*g) * (ws2_u*u) to h_buf.
//  down: grid (2560/16).  Each warp owns 2 output rows and walks all K
//    experts' down rows for them, so the weighted combine happens in
//    registers and `out` is written once, deterministically (no atomics).
//    It is launched as a programmatic dependent of gate_up: its CTAs start
//    while gate_up runs, issue their first weight loads (the table and sidx
//    were complete before gate_up started), then wait for gate_up's h.
#include <cooperative_groups.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "host.cuh"

namespace qfn {

constexpr int kGuThreads = 256;
constexpr int kGuFeatPerWarp = 2;
constexpr int kGuFeatPerCta = (kGuThreads / 32) * kGuFeatPerWarp;  // 16
constexpr int kGuGroups = kHid / 16;                                // 160 scale groups per row
constexpr int kGuPerLane = kGuGroups / 32;                          // 5

constexpr int kDnThreads = 256;
constexpr int kDnRowsPerWarp = 2;
constexpr int kDnRowsPerCta = (kDnThreads / 32) * kDnRowsPerWarp;  // 16
constexpr int kDnGroups = kInter / 16;                             // 40 scale groups per row
constexpr int kDnBatch = 8;                                        // items per lane per row per batch

__device__ __forceinline__ bool block_ok(int64_t b, int64_t n_blocks) { return b >= 0 && b < n_blocks; }

template <bool kXF32>
__global__ void __launch_bounds__(kGuThreads) moe_gate_up_generic_kernel(const uint8_t* __restrict__ table,
                                                                  int64_t n_blocks,
                                                                  const int32_t* __restrict__ sidx,
                                                                  const float* __restrict__ s2,
                                                                  const void* __restrict__ x,
                                                                  float* __restrict__ h) {
  __shared__ float4 xs[4 * kGuGroups];  // xs[q*160 + g] = x[16g + 4q .. 16g + 4q + 3]
  const int j = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * kGuFeatPerCta + warp * kGuFeatPerWarp;
  const int64_t b = sidx[j];
  const bool ok = block_ok(b, n_blocks);
  pdl_launch_dependents();

  const uint8_t* blk = table + (ok ? b : 0) * kBlock;
  uint2 wg[kGuFeatPerWarp][kGuPerLane], wu[kGuFeatPerWarp][kGuPerLane];
  uint32_t sg[kGuFeatPerWarp][kGuPerLane], su[kGuFeatPerWarp][kGuPerLane];
#pragma unroll
  for (int f = 0; f < kGuFeatPerWarp; ++f) {
#pragma unroll
    for (int u = 0; u < kGuPerLane; ++u) {
      const int g = lane + 32 * u;
      const int64_t row = f0 + f;
      if (ok) {
        wg[f][u] = ldg_stream_v2(blk + kOGW + row * (kHid / 2) + 8 * g);
        wu[f][u] = ldg_stream_v2(blk + kOUW + row * (kHid / 2) + 8 * g);
        sg[f][u] = ldg_stream_u8(blk + kOGS + row * kGuGroups + g);
        su[f][u] = ldg_stream_u8(blk + kOUS + row * kGuGroups + g);
      } else {
        wg[f][u] = wu[f][u] = make_uint2(0, 0);
        sg[f][u] = su[f][u] = 0;
      }
    }
  }

  for (int i = threadIdx.x; i < 4 * kGuGroups; i += kGuThreads) {
    const int g = i >> 2, q = i & 3;
    float4 v;
    if (kXF32) {
      v = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + 16 * g + 4 * q);
    } else {
      const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + 16 * g + 4 * q);
      v.x = bf16_bits_to_f32(r.x & 0xffffu);
      v.y = bf16_bits_to_f32(r.x >> 16);
      v.z = bf16_bits_to_f32(r.y & 0xffffu);
      v.w = bf16_bits_to_f32(r.y >> 16);
    }
    xs[q * kGuGroups + g] = v;
  }
  __syncthreads();

  const float ws_g = s2[3 * j + 0];
  const float ws_u = s2[3 * j + 1];
#pragma unroll
  for (int f = 0; f < kGuFeatPerWarp; ++f) {
    float ag = 0.f, au = 0.f;
#pragma unroll
    for (int u = 0; u < kGuPerLane; ++u) {
      const int g = lane + 32 * u;
      const float4 x0 = xs[g], x1 = xs[kGuGroups + g], x2 = xs[2 * kGuGroups + g], x3 = xs[3 * kGuGroups + g];
      ag = fmaf(dot16_e2m1(wg[f][u], x0, x1, x2, x3), e4m3_to_f32(sg[f][u]), ag);
      au = fmaf(dot16_e2m1(wu[f][u], x0, x1, x2, x3), e4m3_to_f32(su[f][u]), au);
    }
    ag = warp_sum(ag);
    au = warp_sum(au);
    if (lane == 0) {
      const float gg = ag * ws_g;
      const float uu = au * ws_u;
      const float hv = gg / (1.0f + expf(-gg)) * uu;
      h[j * kInter + f0 + f] = ok ? hv : __int_as_float(0x7fc00000);
    }
  }
}

__global__ void __launch_bounds__(kDnThreads) moe_down_generic_kernel(const uint8_t* __restrict__ table, int64_t n_blocks,
                                                              const int32_t* __restrict__ sidx,
                                                              const float* __restrict__ s2,
                                                              const float* __restrict__ coef,
                                                              const float* __restrict__ h,
                                                              float* __restrict__ out, int K) {
  extern __shared__ float4 hs[];  // hs[j*160 + q*40 + g] = h[j][16g + 4q .. +3]
  __shared__ const uint8_t* bases[QFN_MAX_TOPK];
  __shared__ float cw[QFN_MAX_TOPK];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < K) {
    const int64_t b = sidx[threadIdx.x];
    const bool ok = block_ok(b, n_blocks);
    bases[threadIdx.x] = table + (ok ? b : 0) * kBlock;
    cw[threadIdx.x] = ok ? coef[threadIdx.x] * s2[3 * threadIdx.x + 2] : __int_as_float(0x7fc00000);
  }
  __syncthreads();

  const int r0 = blockIdx.x * kDnRowsPerCta + warp * kDnRowsPerWarp;
  const int items = K * kDnGroups;
  uint2 w[kDnRowsPerWarp][kDnBatch];
  uint32_t sc[kDnRowsPerWarp][kDnBatch];
  auto load_batch = [&](int it0) {
#pragma unroll
    for (int u = 0; u < kDnBatch; ++u) {
      const int it = it0 + lane + 32 * u;
      if (it < items) {
        const int jj = it / kDnGroups;
        const int g = it - jj * kDnGroups;
        const uint8_t* base = bases[jj];
#pragma unroll
        for (int f = 0; f < kDnRowsPerWarp; ++f) {
          const int64_t r = r0 + f;
          w[f][u] = ldg_stream_v2(base + kODW + r * (kInter / 2) + 8 * g);
          sc[f][u] = ldg_stream_u8(base + kODS + r * kDnGroups + g);
        }
      }
    }
  };
  load_batch(0);

  // h is produced by the gate_up grid this launch depends on.
  pdl_wait();
  for (int i = threadIdx.x; i < K * 4 * kDnGroups; i += kDnThreads) {
    const int jj = i / (4 * kDnGroups);
    const int rem = i - jj * 4 * kDnGroups;
    const int g = rem >> 2, q = rem & 3;
    hs[jj * 4 * kDnGroups + q * kDnGroups + g] =
        *reinterpret_cast<const float4*>(h + jj * kInter + 16 * g + 4 * q);
  }
  __syncthreads();

  float acc[kDnRowsPerWarp] = {};
  for (int it0 = 0; it0 < items; it0 += 32 * kDnBatch) {
    if (it0 > 0) load_batch(it0);
#pragma unroll
    for (int u = 0; u < kDnBatch; ++u) {
      const int it = it0 + lane + 32 * u;
      if (it < items) {
        const int jj = it / kDnGroups;
        const int g = it - jj * kDnGroups;
        const float4* hj = hs + jj * 4 * kDnGroups;
        const float4 h0 = hj[g], h1 = hj[kDnGroups + g], h2 = hj[2 * kDnGroups + g], h3 = hj[3 * kDnGroups + g];
        const float c = cw[jj];
#pragma unroll
        for (int f = 0; f < kDnRowsPerWarp; ++f)
          acc[f] = fmaf(dot16_e2m1(w[f][u], h0, h1, h2, h3), c * e4m3_to_f32(sc[f][u]), acc[f]);
      }
    }
  }
#pragma unroll
  for (int f = 0; f < kDnRowsPerWarp; ++f) {
    const float v = warp_sum(acc[f]);
    if (lane == 0) out[r0 + f] = v;
  }
}

static int launch_moe_decode_generic(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                             const float* coef, const void* x, int x_dtype, float* h_buf, float* out, int K,
                             cudaStream_t st) {
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  const dim3 gu_grid(kInter / kGuFeatPerCta, K);
  if (x_dtype == QFN_DTYPE_F32)
    moe_gate_up_generic_kernel<true><<<gu_grid, kGuThreads, 0, st>>>(table, n_blocks, sidx, s2, x, h_buf);
  else
    moe_gate_up_generic_kernel<false><<<gu_grid, kGuThreads, 0, st>>>(table, n_blocks, sidx, s2, x, h_buf);
  rc = check_launch("moe_gate_up_generic_kernel");
  if (rc) return rc;

  const size_t smem = static_cast<size_t>(K) * kInter * sizeof(float);
  static bool attr_set[64] = {};
  if (smem > 48 * 1024 && !attr_set[dev->device]) {
    cudaError_t e = cudaFuncSetAttribute(moe_down_generic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         QFN_MAX_TOPK * kInter * static_cast<int>(sizeof(float)));
    if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "down smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev->device] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kHid / kDnRowsPerCta);
  cfg.blockDim = dim3(kDnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, moe_down_generic_kernel, table, n_blocks, sidx, s2, coef,
                                     static_cast<const float*>(h_buf), out, K);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "moe_down_generic_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("moe_down_generic_kernel");
}

// ============================================================================
// Persistent path (K <= kFastMaxK): one cooperative launch, one CTA per SM.
//
// Work: the gate/up phase has K*80 "gate tiles" (8 output features = their 8
// gate rows + 8 up rows + 16 scale rows of one expert: four contiguous pieces,
// 23,040 B); the down phase has 160 "down tiles" (16 output rows x all K
// experts: 2K contiguous pieces, K*5,760 B).  Down tile d belongs to CTA
// d % grid; gate tiles are split into contiguous ranges weighted so that
// every CTA streams about the same number of bytes (a down tile costs K/4
// gate tiles).  At entry the lanes of warp 0 issue one bulk TMA copy per
// piece of every tile the CTA owns, gate tiles first, each tile completing
// its own mbarrier: the CTA's whole share of the layer is in flight at once
// and the down rows land while the gate/up phase computes.
//
// Both phases reduce 16-row x 64-byte units with mma.sync m16n8k16 (tensor
// cores as the dot-product engine): the A operand is the e2m1 codes converted
// to f16 and multiplied by their E4M3 block scale (<= 6 significant bits:
// exact in f16); the B operand holds x (phase 1) or coef_j * ws2_d_j * h_j
// (phase 2) as an f16 hi/lo pair (v * 2^e = hi + lo, one power-of-two e per
// phase) in columns 0 and 1, so every tensor-core product is exact and the
// fp32 sums keep ~22 bits of the activations.  Folding coef_j * ws2_d_j into
// B lets one accumulator sum all experts: the weighted combine is part of the
// MMA.  Per-unit partials are summed in a fixed order, so results are
// bit-reproducible.  A grid-wide barrier (cooperative groups) separates
// writing h from reading it.
// ============================================================================

constexpr int kFastMaxK = 10;
constexpr int kPWarps = 20;
constexpr int kPThreads = kPWarps * 32;              // 640
constexpr int kMaxGateTiles = 6;
constexpr int kMaxDownTiles = 2;
constexpr int kTileBytes = 16 * 1280 + 2 * 1280;     // 23040: gate rows | up rows | gate scales | up scales
constexpr int kTilesPerExpert = kInter / 8;          // 80
constexpr int kDownTiles = kHid / 16;                // 160
constexpr int kDnWBytes = 16 * (kInter / 2);         // 5120 per expert per down tile
constexpr int kDnSBytes = 16 * (kInter / 16);        // 640
constexpr int kXUnits = (kHid / 128) * 16;           // 320 16-byte units per hi (or lo) array
constexpr int kHUnitsMax = kFastMaxK * (kInter / 128) * 16;  // 800

__device__ unsigned int g_decode_status = 0;

__device__ __forceinline__ void note_timeout() { atomicOr(&g_decode_status, kStatusTimeout); }
constexpr unsigned kStatusNegativeScale = 2u;

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

// Exact v * 2^e for |e| <= 252 (two power-of-two factors, each a normal float).
__device__ __forceinline__ float scale_pow2(float v, int e) {
  const int a = e / 2, b = e - a;
  return v * __int_as_float((a + 127) << 23) * __int_as_float((b + 127) << 23);
}

// Block-wide max of non-negative values (NaN-propagating); all threads get it.
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = (isnan(u) || u > v) ? u : v;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m = (isnan(red[w]) || red[w] > m) ? red[w] : m;
    red[32] = m;
  }
  __syncthreads();
  return red[32];
}

// One 16-row x 64-byte unit through 8 tensor-core MMAs.
//   ra/rb: this thread's 16 bytes of rows g and g+8; sa/sb: the two E4M3
//   scales (groups 2t, 2t+1 of the chunk) of those rows; bq: the B operand
//   (f16 pairs for this thread's 32 k, or zero).  Word i of the 16 bytes
//   feeds accumulator set d[i] (four independent MMA chains).
__device__ __forceinline__ void mma_chunk(float (&d)[4][4], uint4 ra, uint4 rb, uint32_t sa, uint32_t sb,
                                          const uint4 (&bq)[4]) {
  uint32_t sa0, sa1, sb0, sb1;
  e4m3x2_to_bcast(sa, sa0, sa1);
  e4m3x2_to_bcast(sb, sb0, sb1);
  const uint32_t wa[4] = {ra.x, ra.y, ra.z, ra.w};
  const uint32_t wb[4] = {rb.x, rb.y, rb.z, rb.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t ha[4], hb[4];
    e2m1x8_to_f16x2(wa[i], ha);
    e2m1x8_to_f16x2(wb[i], hb);
    const uint32_t sA = i < 2 ? sa0 : sa1;
    const uint32_t sB = i < 2 ? sb0 : sb1;
    const uint32_t a0[4] = {hmul2_u32(ha[0], sA), hmul2_u32(hb[0], sB), hmul2_u32(ha[1], sA), hmul2_u32(hb[1], sB)};
    mma_16816(d[i], a0, bq[i].x, bq[i].y);
    const uint32_t a1[4] = {hmul2_u32(ha[2], sA), hmul2_u32(hb[2], sB), hmul2_u32(ha[3], sA), hmul2_u32(hb[3], sB)};
    mma_16816(d[i], a1, bq[i].z, bq[i].w);
  }
}

// Row sums (B columns 0 + 1) of the four accumulator sets: (row g, row g+8).
__device__ __forceinline__ float2 unit_rows(const float (&d)[4][4]) {
  return make_float2(((d[0][0] + d[0][1]) + (d[1][0] + d[1][1])) + ((d[2][0] + d[2][1]) + (d[3][0] + d[3][1])),
                     ((d[0][2] + d[0][3]) + (d[1][2] + d[1][3])) + ((d[2][2] + d[2][3]) + (d[3][2] + d[3][3])));
}

// Pack 8 fp32 values (already scaled by 2^e) into f16 hi and lo 16-byte units.
__device__ __forceinline__ void pack_hi_lo(const float (&v)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half h0, l0, h1, l1;
    split_f16(v[2 * i], h0, l0);
    split_f16(v[2 * i + 1], h1, l1);
    h[i] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
    l[i] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Work split shared by host and device (see the header comment).
struct DecodeSplit {
  int grid, K;
  __host__ __device__ int n_gate() const { return K * kTilesPerExpert; }
  __host__ __device__ int down_tiles_of(int c) const {  // down tiles c, c+grid, ... < 160
    return kDownTiles / grid + (c < kDownTiles % grid ? 1 : 0);
  }
  __host__ __device__ int down_before(int c) const {  // down tiles owned by CTAs < c (closed form)
    const int r = kDownTiles % grid;
    return (kDownTiles / grid) * c + (c < r ? c : r);
  }
  __host__ __device__ int gate_start(int c) const {  // 4*x in units of quarter gate tiles
    if (c >= grid) return n_gate();
    const long long tot4 = 4LL * n_gate() + static_cast<long long>(kDownTiles) * K;
    long long s4 = tot4 * c / grid - static_cast<long long>(down_before(c)) * K;
    long long s = s4 / 4;
    if (s < 0) s = 0;
    if (s > n_gate()) s = n_gate();
    return static_cast<int>(s);
  }
};

struct PSmem {  // byte offsets (from the 1024-aligned base) of the dynamic shared-memory map of one CTA
  int a, b, gsc, tsc, gu, down, hst, part, bar, eoff, red, cw, slot, total;
};

constexpr int kTerms = 8;              // e2m1 terms of an activation vector (B rows)
constexpr int kARowGroupBytes = 10240; // 8 rows x 10 K-chunks x 128 B (SWIZZLE_128B atoms)
constexpr int kAReach = 16 * kARowGroupBytes;  // bytes an M=128 MMA operand spans from its base
constexpr int kKSteps = kHid / 64;     // 40 MMA K-steps (K = 64 e2m1 each)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmD = 0, kTmSfa = 32, kTmSfb = 32 + 4 * kKSteps;

__host__ __device__ inline PSmem psmem_map(int n_gate_tiles, int n_down_tiles, int K) {
  PSmem m;
  m.a = 0;                                         // A: 2 row groups (gate, up) per gate tile
  m.b = 2 * n_gate_tiles * kARowGroupBytes;        // B: x terms, one 8-row group (1024-aligned)
  m.gsc = m.b + kARowGroupBytes;                   // gate-tile scales, natural [tile][gate|up][8][160]
  m.tsc = m.gsc + n_gate_tiles * 2 * 8 * (kHid / 16);  // term scales, natural [8][160]
  m.gu = m.tsc + kTerms * (kHid / 16);             // 128 gate/up row values
  m.down = m.gu + 128 * 4;
  int end = m.down + n_down_tiles * K * (kDnWBytes + kDnSBytes);
  // Phase 2 stages h (hi/lo) in the gate-tile region, which is free by then,
  // or after the down rows when that region is too small.
  const int hneed = 2 * kHUnitsMax * 16 + 64;
  m.hst = m.down >= hneed ? 0 : end;
  if (end < m.hst + hneed) end = m.hst + hneed;
  m.part = (end + 15) / 16 * 16;
  m.bar = m.part + kMaxDownTiles * kFastMaxK * 5 * 16 * 4;
  m.eoff = m.bar + (kMaxGateTiles + kMaxDownTiles + 1) * 8;
  m.red = m.eoff + kFastMaxK * 8;
  m.cw = m.red + 64 * 4;
  m.slot = m.cw + 4 * kFastMaxK * 4;  // cw, ws_g, ws_u (floats) and block indices (ints)
  end = m.slot + 16;
  // the M = 128 A operand reads 16 row groups from its base (rows past 2 * n_gate_tiles * 8 are
  // never used, but must lie inside the allocation)
  m.total = (end > kAReach ? end : kAReach) + 1024;  // + alignment slack for the 1024-byte base
  return m;
}

template <bool kXF32>
__global__ void __launch_bounds__(kPThreads, 1)
    moe_decode_persistent(const __grid_constant__ CUtensorMap gate_map, const uint8_t* __restrict__ table,
                          int64_t n_blocks, const int32_t* __restrict__ sidx, const float* __restrict__ s2,
                          const float* __restrict__ coef, const void* __restrict__ x, float* h,
                          float* __restrict__ out, int K) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const DecodeSplit sp{static_cast<int>(gridDim.x), K};
  const int c = blockIdx.x;
  const int g0 = sp.gate_start(c);
  const int ng = sp.gate_start(c + 1) - g0;
  const int nd = sp.down_tiles_of(c);
  const PSmem M = psmem_map(ng, nd, K);
  float* part = reinterpret_cast<float*>(smem + M.part);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + M.bar);  // [0,ng) gate, [6,6+nd) down, [8] MMA done
  uint64_t* mma_bar = bar + kMaxGateTiles + kMaxDownTiles;
  float* red = reinterpret_cast<float*>(smem + M.red);
  float* cw = reinterpret_cast<float*>(smem + M.cw);
  float* gu = reinterpret_cast<float*>(smem + M.gu);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + M.slot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  // x loads first (they depend on nothing), so their latency overlaps the
  // parameter loads below.  Thread u owns k in [4u, 4u + 4).
  const int u = threadIdx.x;
  float xv[4];
  if (kXF32) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + 4 * u);
    xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
  } else {
    const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + 4 * u);
    xv[0] = bf16_bits_to_f32(r.x & 0xffffu); xv[1] = bf16_bits_to_f32(r.x >> 16);
    xv[2] = bf16_bits_to_f32(r.y & 0xffffu); xv[3] = bf16_bits_to_f32(r.y >> 16);
  }
  if (threadIdx.x == 32) prefetch_tensormap(&gate_map);

  // Per-expert parameters, loaded once by K threads in parallel: block
  // offset (-1 if out of range), ws2 gate/up, coef * ws2_down (NaN if invalid).
  int64_t* eoff = reinterpret_cast<int64_t*>(smem + M.eoff);
  float* ws_g = cw + kFastMaxK;
  float* ws_u = cw + 2 * kFastMaxK;
  int* eblk = reinterpret_cast<int*>(cw + 3 * kFastMaxK);
  if (threadIdx.x < K) {
    const int j = threadIdx.x;
    const int64_t b = sidx[j];
    const bool ok = block_ok(b, n_blocks);
    eoff[j] = ok ? b * kBlock : -1;
    eblk[j] = ok ? static_cast<int>(b) : 0;
    ws_g[j] = s2[3 * j + 0];
    ws_u[j] = s2[3 * j + 1];
    cw[j] = ok ? coef[j] * s2[3 * j + 2] : __int_as_float(0x7fc00000);
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < ng; ++i) mbar_init(&bar[i], 1);
    for (int i = 0; i < nd; ++i) mbar_init(&bar[kMaxGateTiles + i], 1);
    mbar_init(mma_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // Arm the barriers (lane i < ng: gate tile i; lane ng + i: down tile i).
    if (lane < ng) {
      mbar_arrive_expect_tx(&bar[lane], eoff[(g0 + lane) / kTilesPerExpert] >= 0 ? kTileBytes : 0);
    } else if (lane < ng + nd) {
      uint32_t tx = 0;
      for (int j = 0; j < K; ++j) tx += eoff[j] >= 0 ? kDnWBytes + kDnSBytes : 0;
      mbar_arrive_expect_tx(&bar[kMaxGateTiles + lane - ng], tx);
    }
    __syncwarp();
    // Copies: 4 per gate tile (gate rows, up rows: 3-D tensor boxes into the
    // SWIZZLE_128B operand layout; gate and up scales: bulk), then 2 per
    // (down tile, expert); lane q issues copies q, q+32, ...
    const int n_copies = 4 * ng + 2 * K * nd;
    for (int q = lane; q < n_copies; q += 32) {
      if (q < 4 * ng) {
        const int i = q >> 2, piece = q & 3;
        const int T = g0 + i;
        const int j = T / kTilesPerExpert;
        const int64_t off = eoff[j];
        if (off < 0) continue;
        const int f0 = (T % kTilesPerExpert) * 8;
        const int row0 = eblk[j] * 2160 + f0;  // table row of gate row f0 (2160 rows of 1280 B per block)
        if (piece == 0) tma_load_3d(smem + M.a + (2 * i) * kARowGroupBytes, &gate_map, 0, row0, 0, &bar[i]);
        else if (piece == 1) tma_load_3d(smem + M.a + (2 * i + 1) * kARowGroupBytes, &gate_map, 0, row0 + kInter, 0, &bar[i]);
        else if (piece == 2) bulk_g2s(smem + M.gsc + i * 2560, table + off + kOGS + f0 * 160, 1280, &bar[i]);
        else bulk_g2s(smem + M.gsc + i * 2560 + 1280, table + off + kOUS + f0 * 160, 1280, &bar[i]);
      } else {
        const int r = q - 4 * ng;
        const int i = r / (2 * K), j = (r / 2) % K, piece = r & 1;
        const int64_t off = eoff[j];
        if (off < 0) continue;
        const int64_t r0 = static_cast<int64_t>(c + i * sp.grid) * 16;
        const uint8_t* blk = table + off;
        uint8_t* dst = smem + M.down + (i * K + j) * (kDnWBytes + kDnSBytes);
        if (piece == 0) bulk_g2s(dst, blk + kODW + r0 * (kInter / 2), kDnWBytes, &bar[kMaxGateTiles + i]);
        else bulk_g2s(dst + kDnWBytes, blk + kODS + r0 * (kInter / 16), kDnSBytes, &bar[kMaxGateTiles + i]);
      }
    }
  } else if (warp == 1) {
    tmem_alloc(tslot, kTmemCols);
  }

  // ---- phase 1: x -> kTerms e2m1 terms with ue4m3 scales per 16 k (the B
  // operand).  Term t carries the column factor 2^(ex - 2t); block scales are
  // rounded up so |residual / scale| <= 6.  Four threads share a 16-block.
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = fabsf(xv[i]);
    mx = (isnan(a) || a > mx) ? a : mx;
  }
  const float xmax = block_max(mx, red);
  int ex = 0;  // 2^ex >= xmax / (6 * 448): term 0's block scales stay <= 448
  if (xmax > 0.f && isfinite(xmax)) frexpf(xmax * (1.0f / 2688.0f), &ex);
  {
    uint8_t* bt = smem + M.b;
    uint8_t* tsc = smem + M.tsc;
    const int cch = u >> 6, jj = (u & 63) >> 3, wb = 2 * (u & 7);  // K-chunk, 16-B chunk, byte in it
#pragma unroll 1
    for (int tt = 0; tt < kTerms; ++tt) {
      const float F = scale_pow2(1.0f, ex - 2 * tt);
      float a = fmaxf(fmaxf(fabsf(xv[0]), fabsf(xv[1])), fmaxf(fabsf(xv[2]), fabsf(xv[3])));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
      uint32_t sb = 0;
      float sF = 0.f;
      if (a > 0.f) {
        const float y = fmaxf(a / (6.0f * F), 1.0f / 512.0f);
        sb = f32_to_e4m3_rn(y);
        if (e4m3_to_f32(sb) < y && sb < 0x7eu) sb += 1;
        sF = e4m3_to_f32(sb) * F;
      }
      const float inv = sF > 0.f ? 1.0f / sF : 0.f;
      const uint32_t b0 = f32x2_to_e2m1(xv[0] * inv, xv[1] * inv);
      const uint32_t b1 = f32x2_to_e2m1(xv[2] * inv, xv[3] * inv);
      uint32_t hq[4];
      e2m1x8_to_f16x2(b0 | (b1 << 8), hq);
      const float2 q0 = f16x2_to_f32x2(hq[0]), q1 = f16x2_to_f32x2(hq[1]);
      xv[0] = fmaf(-q0.x, sF, xv[0]);
      xv[1] = fmaf(-q0.y, sF, xv[1]);
      xv[2] = fmaf(-q1.x, sF, xv[2]);
      xv[3] = fmaf(-q1.y, sF, xv[3]);
      *reinterpret_cast<uint16_t*>(bt + cch * 1024 + tt * 128 + ((jj ^ tt) << 4) + wb) =
          static_cast<uint16_t>(b0 | (b1 << 8));
      if ((u & 3) == 0) tsc[tt * (kHid / 16) + (u >> 2)] = static_cast<uint8_t>(sb);
    }
  }

  // ---- phase 1: wait for the gate tiles, scale factors -> TMEM, 40 MMAs
  for (int i = 0; i < ng; ++i)
    if (!mbar_wait(&bar[i], 0)) note_timeout();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  uint32_t neg = 0;
  if (warp < 16) {
    // TMEM lane l (of every 32-lane quadrant), column base + 4s + m1 holds the
    // 4 scales of K-step s of operand row l + 32*m1.  Warp w writes quadrant
    // w % 4, K-steps [10 (w / 4), +10).
    const uint32_t lane_off = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const int ks0 = 10 * (warp >> 2);
    const uint8_t* gsc = smem + M.gsc;
    const uint8_t* tsc = smem + M.tsc;
    uint32_t va[40], vb[40];
#pragma unroll
    for (int m1 = 0; m1 < 4; ++m1) {
      const int m = lane + 32 * m1;  // A row: row group m/8 = (tile, gate|up), row m%8
      const int rg = m >> 3;
      const bool live = rg < 2 * ng && eoff[(g0 + (rg >> 1)) / kTilesPerExpert] >= 0;
      const uint8_t* ra = gsc + (rg >> 1) * 2560 + (rg & 1) * 1280 + (m & 7) * 160 + 4 * ks0;
      const uint8_t* rb = tsc + m * 160 + 4 * ks0;
#pragma unroll
      for (int k = 0; k < 10; ++k) {
        va[4 * k + m1] = live ? *reinterpret_cast<const uint32_t*>(ra + 4 * k) : 0x38383838u;  // 1.0 if not loaded
        vb[4 * k + m1] = m < kTerms ? *reinterpret_cast<const uint32_t*>(rb + 4 * k) : 0u;
        neg |= va[4 * k + m1];
      }
    }
    const uint32_t ca = tbase + lane_off + kTmSfa + 4 * ks0, cb = tbase + lane_off + kTmSfb + 4 * ks0;
    tmem_st_x32(ca, *reinterpret_cast<const uint32_t(*)[32]>(&va[0]));
    tmem_st_x8(ca + 32, *reinterpret_cast<const uint32_t(*)[8]>(&va[32]));
    tmem_st_x32(cb, *reinterpret_cast<const uint32_t(*)[32]>(&vb[0]));
    tmem_st_x8(cb + 32, *reinterpret_cast<const uint32_t(*)[8]>(&vb[32]));
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && ng > 0) {
    const uint32_t idesc = idesc_mxf4nvf4(128, 16);
    const uint32_t a0 = smem_u32(smem + M.a), b0 = smem_u32(smem + M.b);
#pragma unroll 1
    for (int ks = 0; ks < kKSteps; ++ks) {
      const uint32_t koff = (ks >> 2) * 1024 + 32 * (ks & 3);
      mma_mxf4nvf4(tbase + kTmD, umma_desc_sw128(a0 + koff, kARowGroupBytes), umma_desc_sw128(b0 + koff, 0), idesc,
                   ks > 0, tbase + kTmSfa + 4 * ks, tbase + kTmSfb + 4 * ks);
    }
    mma_commit(mma_bar);
  }
  // A scale with its sign bit set is outside the ue4m3 range the tensor core reads.
  const bool bad_scale = __syncthreads_or((neg & 0x80808080u) != 0);
  if (ng > 0) {
    if (!mbar_wait(mma_bar, 0)) note_timeout();
    tc_fence_after();
    if (warp < 4) {
      uint32_t d[8];
      tmem_ld_x8(tbase + (static_cast<uint32_t>(32 * warp) << 16) + kTmD, d);
      float v = 0.f;
#pragma unroll
      for (int tt = 0; tt < kTerms; ++tt) v = fmaf(__uint_as_float(d[tt]), scale_pow2(1.0f, ex - 2 * tt), v);
      gu[32 * warp + lane] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < ng * 8) {
    const int i = threadIdx.x >> 3, f = threadIdx.x & 7;
    const int T = g0 + i;
    const int j = T / kTilesPerExpert;
    const float gg = gu[16 * i + f] * ws_g[j];
    const float uu = gu[16 * i + 8 + f] * ws_u[j];
    const float hv = gg / (1.0f + expf(-gg)) * uu;
    const bool ok = eoff[j] >= 0 && isfinite(xmax) && !bad_scale;
    h[j * kInter + (T % kTilesPerExpert) * 8 + f] = ok ? hv : __int_as_float(0x7fc00000);
  }
  if (bad_scale && threadIdx.x == 0) atomicOr(&g_decode_status, kStatusNegativeScale);

  cooperative_groups::this_grid().sync();  // every h row is written

  // ---- phase 2: B = coef_j * ws2_d_j * h_j as f16 hi/lo units (unit u = j*80 + (c, q, t))
  uint4* hh = reinterpret_cast<uint4*>(smem + M.hst);
  uint4* hl = reinterpret_cast<uint4*>(smem + M.hst + kHUnitsMax * 16 + 64);
  const int n_units = K * (kInter / 8);
  constexpr int kMaxUnitsPerThread = (kHUnitsMax + kPThreads - 1) / kPThreads;  // 2
  float hv[kMaxUnitsPerThread][8];
  mx = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxUnitsPerThread; ++k) {
    const int uu = threadIdx.x + k * kPThreads;
    if (uu < n_units) {
      const int j = uu / 80, rem = uu % 80;
      const int n0 = (rem >> 4) * 128 + (rem & 3) * 32 + ((rem >> 2) & 3) * 8;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(h + j * kInter + n0));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(h + j * kInter + n0 + 4));
      const float m = cw[j];
      hv[k][0] = a.x * m; hv[k][1] = a.y * m; hv[k][2] = a.z * m; hv[k][3] = a.w * m;
      hv[k][4] = b.x * m; hv[k][5] = b.y * m; hv[k][6] = b.z * m; hv[k][7] = b.w * m;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float aa = fabsf(hv[k][i]);
        mx = (isnan(aa) || aa > mx) ? aa : mx;
      }
    }
  }
  const float hmax = block_max(mx, red);
  const int eh = f16_prescale_exp(hmax);
#pragma unroll
  for (int k = 0; k < kMaxUnitsPerThread; ++k) {
    const int uu = threadIdx.x + k * kPThreads;
    if (uu < n_units) {
#pragma unroll
      for (int i = 0; i < 8; ++i) hv[k][i] = scale_pow2(hv[k][i], eh);
      pack_hi_lo(hv[k], hh[uu], hl[uu]);
    }
  }
  __syncthreads();

  // ---- phase 2: (down tile, expert, 64-byte chunk) units, 5K per down tile (mma.sync)
  const int per_tile = 5 * K;
  for (int uu = warp; uu < nd * per_tile; uu += kPWarps) {
    const int i = uu / per_tile, p = uu % per_tile;
    const int j = p / 5, ch = p % 5;
    if (!mbar_wait(&bar[kMaxGateTiles + i], 0)) note_timeout();
    const uint8_t* wj = smem + M.down + (i * K + j) * (kDnWBytes + kDnSBytes);
    const uint4 ra = lds128(wj + g * (kInter / 2) + 64 * ch + 16 * t);
    const uint4 rb = lds128(wj + (g + 8) * (kInter / 2) + 64 * ch + 16 * t);
    const uint32_t sa = lds16(wj + kDnWBytes + g * (kInter / 16) + 8 * ch + 2 * t);
    const uint32_t sb = lds16(wj + kDnWBytes + (g + 8) * (kInter / 16) + 8 * ch + 2 * t);
    uint4 bq[4];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const int un = (j * 5 + ch) * 16 + qq * 4 + t;
      bq[qq] = g == 0 ? hh[un] : (g == 1 ? hl[un] : make_uint4(0, 0, 0, 0));
    }
    float d[4][4] = {};
    mma_chunk(d, ra, rb, sa, sb, bq);
    if (t == 0) {
      const float2 r = unit_rows(d);
      part[uu * 16 + g] = r.x;
      part[uu * 16 + 8 + g] = r.y;
    }
  }
  __syncthreads();
  if (threadIdx.x < nd * 16) {
    const int i = threadIdx.x >> 4, row = threadIdx.x & 15;
    float acc = 0.f;
    for (int p = 0; p < per_tile; ++p) acc += part[(i * per_tile + p) * 16 + row];
    out[(c + i * sp.grid) * 16 + row] = isnan(hmax) ? hmax : scale_pow2(acc, -eh);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, kTmemCols);
}

static int launch_moe_decode_fast(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                                  const float* coef, const void* x, int x_dtype, float* h_buf, float* out, int K,
                                  cudaStream_t st, const DeviceInfo* dev, int grid) {
  CUtensorMap gate_map;
  int rc = gate_rows_tensor_map(table, n_blocks, dev->device, &gate_map);
  if (rc) return rc;
  // shared memory: the largest per-CTA map of this split
  const DecodeSplit sp{grid, K};
  int smem = 0;
  for (int c = 0; c < grid; ++c) {
    const PSmem m = psmem_map(sp.gate_start(c + 1) - sp.gate_start(c), sp.down_tiles_of(c), K);
    if (m.total > smem) smem = m.total;
  }
  auto fn = x_dtype == QFN_DTYPE_F32 ? moe_decode_persistent<true> : moe_decode_persistent<false>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "decode smem attribute (%d B): %s", smem, cudaGetErrorString(e));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, fn, gate_map, table, n_blocks, sidx, s2, coef, x, h_buf, out, K);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "moe_decode_persistent launch: %s", cudaGetErrorString(e));
  return check_launch("moe_decode_persistent");
}

// Whether the persistent path fits this device: per-CTA tile counts within the
// static bounds and the shared-memory map within the opt-in limit.
static bool persistent_fits(int K, const DeviceInfo* dev) {
  if (K > kFastMaxK) return false;
  const int grid = dev->sm_count;
  const DecodeSplit sp{grid, K};
  for (int c = 0; c < grid; ++c) {
    const int ng = sp.gate_start(c + 1) - sp.gate_start(c), nd = sp.down_tiles_of(c);
    if (ng > kMaxGateTiles || nd > kMaxDownTiles || ng + nd > 32) return false;
    if (static_cast<size_t>(psmem_map(ng, nd, K).total) > dev->smem_optin) return false;
  }
  return true;
}

// ============================================================================
// Stream path (K <= 10): one cooperative launch, one CTA per SM, the CTA's
// whole share of the layer requested from HBM at entry.
//
// Work items are 8-row "octets": a gate/up octet is 8 output features of one
// expert (8 gate rows + 8 up rows + their scale rows, 23,040 B); a down octet
// is 8 output rows of every expert (K x (2,560 B rows + 320 B scales)).  Down
// octets are dealt evenly (320 of them: 2 or 3 per CTA on 148 SMs); gate/up
// octets fill each CTA's remaining byte budget, so every SM streams about
// 1/148 of the layer.  After the routing loads, warps 0 and 1 issue every
// bulk copy of the CTA's share at once (gate/up runs in chunks of two octets
// with one mbarrier each; the down rows and scales of each expert as one copy
// each, on one more mbarrier), so HBM sees the whole layer's requests at once
// and the down rows land while the gate/up rows are reduced.
//
// Dot products run on mma.sync m16n8k16 with f16 operands: A = e2m1 codes
// times their E4M3 block scale (exact in f16), B = the activation as an f16
// hi/lo pair (v * 2^e = hi + lo, one power-of-two e per vector) in B columns
// 0/1, so every product is exact and the fp32 sums keep ~22 bits of x and h.
// Phase 1: warp w owns K-slice [128w, 128w + 128) of every gate/up octet (its
// B fragment of x stays in registers); A rows 0-7 are the gate rows and 8-15
// the up rows, so one MMA chain yields both projections.  The 20 per-warp
// partials are summed in a fixed order into h (global h_buf).  A grid-wide
// barrier separates writing h from reading it.  Phase 2: A rows 0-7 are down
// rows of expert j, rows 8-15 the same rows of expert j+1, B columns 0/1 hold
// h_j and 2/3 h_(j+1); the per-(expert, K-slice) partials are combined with
// coef_j * ws2_d_j in a fixed order, so results are bit-reproducible.
// ============================================================================

constexpr int kSMaxK = 10;
constexpr int kSMaxGu = 8;               // gate/up octets per CTA (checked on the host)
constexpr int kSChunk = 2;               // gate/up octets per copy / mbarrier
constexpr int kGuOctBytes = 23040;       // gate rows | up rows | gate scales | up scales
constexpr int kDnOctBytes = 2880;        // 8 down rows of one expert (2,560 B) + their scales (320 B)
constexpr int kDnOctets = kHid / 8;      // 320
constexpr int kSMiscBytes = 1024;

struct StreamSplit {
  int grid, K;
  __host__ __device__ int dn0(int c) const { return c * kDnOctets / grid; }
  // First gate/up octet of CTA c.  Bytes are counted in units of 2,880 B (a
  // gate/up octet is 8 units, a down octet K units); CTA c's byte range starts
  // at c/grid of the layer, minus what its down octets take before it.
  __host__ __device__ int gu0(int c) const {
    const int n = K * kTilesPerExpert;
    if (c >= grid) return n;
    const long long P = static_cast<long long>(c) * 960 * K / grid;
    const long long s = (P - static_cast<long long>(K) * dn0(c) + 4) / 8;
    return static_cast<int>(s < 0 ? 0 : (s > n ? n : s));
  }
};

struct SSmem {  // byte offsets from the aligned base of one CTA's dynamic shared memory
  int gu, dn, hs, scratch, misc, total;
};

__host__ __device__ inline SSmem ssmem_map(int ng, int nd, int K) {
  SSmem m;
  m.gu = 0;
  m.dn = ng * kGuOctBytes;
  int end = m.dn + nd * K * kDnOctBytes;
  // Phase 2 keeps h as f16 hi + lo rows (K x 640 x 4 B) in the gate/up region,
  // which is free by then, or after the down octets when that region is smaller.
  const int hneed = K * kInter * 4;
  m.hs = m.dn >= hneed ? 0 : end;
  if (m.hs) end += hneed;
  m.scratch = (end + 15) & ~15;  // x hi/lo, then the gate/up partials, then the down partials
  int scratch = 2 * kHid * 2;
  const int red = ng * kPWarps * 16 * 4, part = nd * K * 5 * 8 * 4;
  if (red > scratch) scratch = red;
  if (part > scratch) scratch = part;
  m.misc = m.scratch + scratch;
  m.total = m.misc + kSMiscBytes + 1024;  // + slack for aligning the base to 1,024 B
  return m;
}

__device__ __forceinline__ float nanmax(float a, float b) { return (isnan(b) || b > a) ? b : a; }

template <bool kXF32>
__global__ void __launch_bounds__(kPThreads, 1)
    moe_decode_stream(const uint8_t* __restrict__ table, int64_t n_blocks, const int32_t* __restrict__ sidx,
                      const float* __restrict__ s2, const float* __restrict__ coef, const void* __restrict__ x,
                      float* h, float* __restrict__ out, int K) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const StreamSplit sp{static_cast<int>(gridDim.x), K};
  const int c = blockIdx.x;
  const int g0 = sp.gu0(c), ng = sp.gu0(c + 1) - g0;
  const int d0 = sp.dn0(c), nd = sp.dn0(c + 1) - d0;
  const SSmem M = ssmem_map(ng, nd, K);
  uint8_t* misc = smem + M.misc;
  uint64_t* bar = reinterpret_cast<uint64_t*>(misc);           // [0, chunks): gate/up; [kSMaxGu]: down
  int64_t* eoff = reinterpret_cast<int64_t*>(misc + 128);      // block byte offset, -1 if out of range
  float* ws_g = reinterpret_cast<float*>(misc + 256);
  float* ws_u = ws_g + kSMaxK;
  float* cw = ws_u + kSMaxK;                                   // coef * ws2_down (NaN if invalid)
  int* hexp = reinterpret_cast<int*>(cw + kSMaxK);             // phase-2 prescale exponent per expert
  float* wred = reinterpret_cast<float*>(hexp + kSMaxK);       // per-warp maxima
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ng; ++i) mbar_init(&bar[i], 1);
    mbar_init(&bar[kSMaxGu], 1);
    fence_mbar_init();
  }
  // Warm the address translations of h_buf and out (a prefetch reads nothing
  // the previous kernel may still be writing into this SM's caches).
  if (threadIdx.x == 64) asm volatile("prefetch.global.L2 [%0];" ::"l"(h) : "memory");
  if (threadIdx.x == 96) asm volatile("prefetch.global.L2 [%0];" ::"l"(out) : "memory");
  // Everything below reads this call's inputs or writes h_buf / out.
  pdl_wait();
  pdl_launch_dependents();

  // x (thread u owns k in [4u, 4u + 4)) and the per-expert parameters.
  const int u = threadIdx.x;
  float xv[4];
  if (kXF32) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + 4 * u);
    xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
  } else {
    const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + 4 * u);
    xv[0] = bf16_bits_to_f32(r.x & 0xffffu); xv[1] = bf16_bits_to_f32(r.x >> 16);
    xv[2] = bf16_bits_to_f32(r.y & 0xffffu); xv[3] = bf16_bits_to_f32(r.y >> 16);
  }
  if (threadIdx.x < K) {
    const int j = threadIdx.x;
    const int64_t b = sidx[j];
    const bool ok = block_ok(b, n_blocks);
    eoff[j] = ok ? b * kBlock : -1;
    ws_g[j] = s2[3 * j + 0];
    ws_u[j] = s2[3 * j + 1];
    cw[j] = ok ? coef[j] * s2[3 * j + 2] : __int_as_float(0x7fc00000);
  }
  float mx = nanmax(nanmax(fabsf(xv[0]), fabsf(xv[1])), nanmax(fabsf(xv[2]), fabsf(xv[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = nanmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) wred[warp] = mx;
  __syncthreads();

  // Gate/up octets come in runs of one expert (at most two runs); each run is
  // cut into chunks of kSChunk octets, one mbarrier per chunk.  Warp 0 issues
  // 4 copies per chunk (gate rows, up rows, gate scales, up scales), warp 1
  // 2 per expert for the down octets (all nd octets' rows, then scales: both
  // contiguous in the block): few large copies, since the TMA unit spends a
  // roughly fixed time per copy.
  const int nA = ng < kTilesPerExpert - g0 % kTilesPerExpert ? ng : kTilesPerExpert - g0 % kTilesPerExpert;
  const int ncA = (nA + kSChunk - 1) / kSChunk;
  const int nc = ncA + (ng - nA + kSChunk - 1) / kSChunk;
  if (warp == 0) {
    if (lane < nc) {
      const int i0 = lane < ncA ? lane * kSChunk : nA + (lane - ncA) * kSChunk;
      const int n = min(kSChunk, (lane < ncA ? nA : ng) - i0);
      mbar_arrive_expect_tx(&bar[lane], eoff[(g0 + i0) / kTilesPerExpert] >= 0 ? n * kGuOctBytes : 0);
    }
    if (lane == 31) {
      uint32_t tx = 0;
      for (int j = 0; j < K; ++j) tx += eoff[j] >= 0 ? nd * kDnOctBytes : 0;
      mbar_arrive_expect_tx(&bar[kSMaxGu], tx);
    }
    __syncwarp();
    if (lane < 4 * nc) {
      const int ch = lane >> 2, piece = lane & 3;
      const int i0 = ch < ncA ? ch * kSChunk : nA + (ch - ncA) * kSChunk;
      const int n = min(kSChunk, (ch < ncA ? nA : ng) - i0);
      const int T = g0 + i0, j = T / kTilesPerExpert;
      const int64_t off = eoff[j];
      if (off >= 0) {
        const int f0 = (T % kTilesPerExpert) * 8;
        const uint8_t* blk = table + off;
        if (piece == 0) bulk_g2s(smem + M.gu + i0 * 10240, blk + kOGW + f0 * (kHid / 2), n * 10240, &bar[ch]);
        else if (piece == 1) bulk_g2s(smem + M.gu + (ng + i0) * 10240, blk + kOUW + f0 * (kHid / 2), n * 10240, &bar[ch]);
        else if (piece == 2) bulk_g2s(smem + M.gu + 2 * ng * 10240 + i0 * 1280, blk + kOGS + f0 * (kHid / 16), n * 1280, &bar[ch]);
        else bulk_g2s(smem + M.gu + 2 * ng * 10240 + (ng + i0) * 1280, blk + kOUS + f0 * (kHid / 16), n * 1280, &bar[ch]);
      }
    }
  } else if (warp == 1 && nd > 0) {
    if (lane < 2 * K) {
      const int j = lane >> 1;
      const int64_t off = eoff[j];
      if (off >= 0) {
        const int64_t row0 = static_cast<int64_t>(d0) * 8;
        const uint8_t* blk = table + off;
        if ((lane & 1) == 0)
          bulk_g2s(smem + M.dn + j * nd * 2560, blk + kODW + row0 * (kInter / 2), nd * 2560, &bar[kSMaxGu]);
        else
          bulk_g2s(smem + M.dn + K * nd * 2560 + j * nd * 320, blk + kODS + row0 * (kInter / 16), nd * 320,
                   &bar[kSMaxGu]);
      }
    }
  }

  // x * 2^ex as f16 hi/lo rows, then each warp's B fragments for its K-slice.
  float xmax = 0.f;
  for (int w = 0; w < kPWarps; ++w) xmax = nanmax(xmax, wred[w]);
  const int ex = f16_prescale_exp(xmax);
  uint8_t* xs = smem + M.scratch;  // hi: 2,560 f16, then lo
  {
    uint32_t hw[2], lw[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      __half h0, l0, h1, l1;
      split_f16(scale_pow2(xv[2 * i], ex), h0, l0);
      split_f16(scale_pow2(xv[2 * i + 1], ex), h1, l1);
      hw[i] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
      lw[i] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
    }
    *reinterpret_cast<uint2*>(xs + 8 * u) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(xs + 2 * kHid + 8 * u) = make_uint2(lw[0], lw[1]);
  }
  __syncthreads();
  uint4 bq[4];
  {
    const uint8_t* src = xs + (g == 1 ? 2 * kHid : 0) + 2 * (128 * warp + 32 * t);
#pragma unroll
    for (int q = 0; q < 4; ++q) bq[q] = g < 2 ? lds128(src + 16 * q) : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();  // the scratch region now takes the gate/up partials

  // ---- phase 1: gate/up octets in arrival order
  float* red = reinterpret_cast<float*>(smem + M.scratch);  // [octet][warp][16]
  for (int i = 0; i < ng; ++i) {
    if (!mbar_wait(&bar[i < nA ? i / kSChunk : ncA + (i - nA) / kSChunk], 0)) note_timeout();
    const uint8_t* gate = smem + M.gu + i * 10240;
    const uint8_t* up = smem + M.gu + (ng + i) * 10240;
    const uint8_t* gsc = smem + M.gu + 2 * ng * 10240 + i * 1280;
    const uint8_t* usc = smem + M.gu + 2 * ng * 10240 + (ng + i) * 1280;
    const uint4 ra = lds128(gate + g * (kHid / 2) + 64 * warp + 16 * t);
    const uint4 rb = lds128(up + g * (kHid / 2) + 64 * warp + 16 * t);
    const uint32_t sa = lds16(gsc + g * (kHid / 16) + 8 * warp + 2 * t);
    const uint32_t sb = lds16(usc + g * (kHid / 16) + 8 * warp + 2 * t);
    float d[4][4] = {};
    mma_chunk(d, ra, rb, sa, sb, bq);
    if (t == 0) {
      const float2 r = unit_rows(d);
      red[(i * kPWarps + warp) * 16 + g] = r.x;
      red[(i * kPWarps + warp) * 16 + 8 + g] = r.y;
    }
  }
  __syncthreads();
  if (threadIdx.x < 8 * ng) {
    const int i = threadIdx.x >> 3, f = threadIdx.x & 7;
    const int T = g0 + i, j = T / kTilesPerExpert;
    float gs = 0.f, us = 0.f;
    for (int w = 0; w < kPWarps; ++w) {
      gs += red[(i * kPWarps + w) * 16 + f];
      us += red[(i * kPWarps + w) * 16 + 8 + f];
    }
    const float gg = scale_pow2(gs, -ex) * ws_g[j];
    const float uu = scale_pow2(us, -ex) * ws_u[j];
    const float hv = gg / (1.0f + expf(-gg)) * uu;
    h[j * kInter + (T % kTilesPerExpert) * 8 + f] = eoff[j] >= 0 ? hv : __int_as_float(0x7fc00000);
  }

  cooperative_groups::this_grid().sync();  // every h row is written

  // ---- phase 2: h -> f16 hi/lo rows.  Thread i loads 16-byte units i,
  // i + 640, i + 1280 of h (unit v = expert v / 160, features 4 (v % 160) ..);
  // warp w's r-th load covers 32 units of expert (w + 20 r) / 5.
  uint8_t* hs = smem + M.hs;  // hi row j at 1,280 j; lo row j at 1,280 (K + j)
  const int n_units = K * (kInter / 4);
  float4 hv[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int v = threadIdx.x + r * kPThreads;
    hv[r] = v < n_units ? __ldcg(reinterpret_cast<const float4*>(h) + v) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    float hm = nanmax(nanmax(fabsf(hv[r].x), fabsf(hv[r].y)), nanmax(fabsf(hv[r].z), fabsf(hv[r].w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) hm = nanmax(hm, __shfl_xor_sync(0xffffffffu, hm, o));
    if (lane == 0) wred[32 + r * kPWarps + warp] = hm;
  }
  __syncthreads();
  if (threadIdx.x < K) {
    const int j = threadIdx.x;
    float m = 0.f;
    for (int q = 0; q < 5; ++q) m = nanmax(m, wred[32 + 5 * j + q]);  // warps 5j .. 5j + 4 of load (5j) / 20
    hexp[j] = f16_prescale_exp(m);
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int v = threadIdx.x + r * kPThreads;
    if (v < n_units) {
      const int j = v / 160, f = 4 * (v % 160), e = hexp[j];
      __half h0[4], l0[4];
      split_f16(scale_pow2(hv[r].x, e), h0[0], l0[0]);
      split_f16(scale_pow2(hv[r].y, e), h0[1], l0[1]);
      split_f16(scale_pow2(hv[r].z, e), h0[2], l0[2]);
      split_f16(scale_pow2(hv[r].w, e), h0[3], l0[3]);
      *reinterpret_cast<uint2*>(hs + j * 1280 + 2 * f) = *reinterpret_cast<const uint2*>(h0);
      *reinterpret_cast<uint2*>(hs + (K + j) * 1280 + 2 * f) = *reinterpret_cast<const uint2*>(l0);
    }
  }
  if (nd > 0 && !mbar_wait(&bar[kSMaxGu], 0)) note_timeout();
  __syncthreads();

  // ---- phase 2: (down octet, expert pair, 128-k slice) items, one per warp
  float* part = reinterpret_cast<float*>(smem + M.scratch);  // [octet][expert][slice][8 rows]
  const int P = (K + 1) >> 1;
  const int n_items = nd * P * 5;
  for (int it = warp; it < n_items; it += kPWarps) {
    const int i = it / (P * 5), rem = it - i * (P * 5);
    const int p = rem / 5, s = rem - p * 5;
    const int j0 = 2 * p, j1 = 2 * p + 1;
    const bool has1 = j1 < K;
    const int jb = has1 ? j1 : j0;
    const uint8_t* w0 = smem + M.dn + (j0 * nd + i) * 2560;
    const uint8_t* w1 = smem + M.dn + (jb * nd + i) * 2560;
    const uint8_t* s0 = smem + M.dn + K * nd * 2560 + (j0 * nd + i) * 320;
    const uint8_t* s1 = smem + M.dn + K * nd * 2560 + (jb * nd + i) * 320;
    const uint4 ra = lds128(w0 + g * (kInter / 2) + 64 * s + 16 * t);
    const uint4 rb = lds128(w1 + g * (kInter / 2) + 64 * s + 16 * t);
    const uint32_t sa = lds16(s0 + g * (kInter / 16) + 8 * s + 2 * t);
    const uint32_t sb = lds16(s1 + g * (kInter / 16) + 8 * s + 2 * t);
    // B columns: 0/1 = h_j0 hi/lo, 2/3 = h_j1 hi/lo, 4-7 = 0
    const int jj = g < 2 ? j0 : j1;
    const bool live = g < 2 || (g < 4 && has1);
    const uint8_t* src = hs + ((g & 1) ? K + jj : jj) * 1280 + 2 * (128 * s + 32 * t);
    uint4 hq[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) hq[q] = live ? lds128(src + 16 * q) : make_uint4(0, 0, 0, 0);
    float d[4][4] = {};
    mma_chunk(d, ra, rb, sa, sb, hq);
    if (t == 0)
      part[((i * K + j0) * 5 + s) * 8 + g] = ((d[0][0] + d[0][1]) + (d[1][0] + d[1][1])) + ((d[2][0] + d[2][1]) + (d[3][0] + d[3][1]));
    if (t == 1 && has1)
      part[((i * K + j1) * 5 + s) * 8 + g] = ((d[0][2] + d[0][3]) + (d[1][2] + d[1][3])) + ((d[2][2] + d[2][3]) + (d[3][2] + d[3][3]));
  }
  __syncthreads();
  if (threadIdx.x < 8 * nd) {
    const int i = threadIdx.x >> 3, r = threadIdx.x & 7;
    float acc = 0.f;
    for (int j = 0; j < K; ++j) {
      const float* pj = part + (i * K + j) * 40 + r;
      const float sj = (((pj[0] + pj[8]) + (pj[16] + pj[24])) + pj[32]);
      acc = fmaf(scale_pow2(sj, -hexp[j]), cw[j], acc);
    }
    out[8 * (d0 + i) + r] = acc;
  }
}

// Shared memory of the stream path for (K, grid), or 0 when it does not fit.
static int stream_smem(int K, const DeviceInfo* dev) {
  if (K > kSMaxK) return 0;
  const StreamSplit sp{dev->sm_count, K};
  int smem = 0;
  for (int c = 0; c < sp.grid; ++c) {
    const int ng = sp.gu0(c + 1) - sp.gu0(c), nd = sp.dn0(c + 1) - sp.dn0(c);
    if (ng > kSMaxGu) return 0;
    const SSmem m = ssmem_map(ng, nd, K);
    if (m.total > smem) smem = m.total;
  }
  return static_cast<size_t>(smem) <= dev->smem_optin ? smem : 0;
}

static int launch_moe_decode_stream(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                                    const float* coef, const void* x, int x_dtype, float* h_buf, float* out, int K,
                                    cudaStream_t st, const DeviceInfo* dev, int smem) {
  auto fn = x_dtype == QFN_DTYPE_F32 ? moe_decode_stream<true> : moe_decode_stream<false>;
  static bool attr_set[64][2] = {};
  const int ti = x_dtype == QFN_DTYPE_F32 ? 1 : 0;
  if (!attr_set[dev->device][ti]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(dev->smem_optin));
    if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "stream decode smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev->device][ti] = true;
  }
  // Cooperative (the grid barrier needs every CTA resident) and a programmatic
  // dependent of the previous kernel in the stream (its launch overlaps that
  // kernel's tail; the kernel waits for it before touching any input).
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(dev->sm_count);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, table, n_blocks, sidx, s2, coef, x, h_buf, out, K);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "moe_decode_stream launch: %s", cudaGetErrorString(e));
  return check_launch("moe_decode_stream");
}

}  // namespace qfn

#include "decode_slice.cuh"

namespace qfn {

static int launch_moe_decode(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                             const float* coef, const void* x, int x_dtype, float* h_buf, float* out, int K,
                             cudaStream_t st, int variant) {
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  if (variant == 0 || variant == 4) {
    // The slice path adds 16-byte vectors into out.
    if (slice_fits(K, dev) && aligned(out, 16))
      return launch_moe_decode_slice(table, n_blocks, sidx, s2, coef, x, x_dtype, h_buf, out, K, st, dev);
    if (variant == 4)
      return set_error(QFN_ERR_UNSUPPORTED,
                       "slice decode path needs K <= 10, a 148-SM-class device and a 16-byte aligned out");
  }
  if (variant == 1) {
    // The persistent path keeps a CTA's whole share of the layer in shared memory.
    if (!persistent_fits(K, dev))
      return set_error(QFN_ERR_UNSUPPORTED, "tensor-core decode path needs K <= %d (and a 148-SM-class device)",
                       kFastMaxK);
    return launch_moe_decode_fast(table, n_blocks, sidx, s2, coef, x, x_dtype, h_buf, out, K, st, dev,
                                  dev->sm_count);
  }
  if (variant == 0 || variant == 3) {
    const int smem = stream_smem(K, dev);
    if (smem > 0)
      return launch_moe_decode_stream(table, n_blocks, sidx, s2, coef, x, x_dtype, h_buf, out, K, st, dev, smem);
    if (variant == 3)
      return set_error(QFN_ERR_UNSUPPORTED, "stream decode path needs K <= %d (and a 148-SM-class device)", kSMaxK);
  }
  return launch_moe_decode_generic(table, n_blocks, sidx, s2, coef, x, x_dtype, h_buf, out, K, st);
}

}  // namespace qfn

using namespace qfn;

static int check_decode_args(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                             const float* coef, const void* x, int x_dtype, float* h_buf, float* out, int K) {
  QFN_REQUIRE(table && sidx && s2 && coef && x && h_buf && out, QFN_ERR_INVALID_ARG,
              "qfn_moe_decode: null pointer");
  QFN_REQUIRE(n_blocks > 0, QFN_ERR_INVALID_ARG, "qfn_moe_decode: n_blocks=%lld", (long long)n_blocks);
  QFN_REQUIRE(K >= 1 && K <= QFN_MAX_TOPK, QFN_ERR_UNSUPPORTED, "qfn_moe_decode: K=%d outside [1, %d]", K,
              QFN_MAX_TOPK);
  QFN_REQUIRE(x_dtype == QFN_DTYPE_F32 || x_dtype == QFN_DTYPE_BF16, QFN_ERR_INVALID_ARG,
              "qfn_moe_decode: bad x_dtype %d", x_dtype);
  QFN_REQUIRE(aligned(table, 16) && aligned(h_buf, 16) && aligned(x, 16), QFN_ERR_ALIGNMENT,
              "qfn_moe_decode: table, h_buf and x must be 16-byte aligned");
  return QFN_OK;
}

extern "C" int qfn_moe_decode(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                              const float* coef, const void* x, int x_dtype, float* h_buf, float* out, int K,
                              qfn_stream_t stream) {
  int rc = check_decode_args(table, n_blocks, sidx, s2, coef, x, x_dtype, h_buf, out, K);
  if (rc) return rc;
  return launch_moe_decode(table, n_blocks, sidx, s2, coef, x, x_dtype, h_buf, out, K, as_stream(stream), 0);
}

extern "C" int qfn_moe_decode_variant(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                                      const float* coef, const void* x, int x_dtype, float* h_buf, float* out,
                                      int K, int variant, qfn_stream_t stream) {
  int rc = check_decode_args(table, n_blocks, sidx, s2, coef, x, x_dtype, h_buf, out, K);
  if (rc) return rc;
  QFN_REQUIRE(variant >= 0 && variant <= 4, QFN_ERR_INVALID_ARG, "qfn_moe_decode_variant: variant %d", variant);
  QFN_REQUIRE(variant != 1 || K <= kFastMaxK, QFN_ERR_UNSUPPORTED,
              "qfn_moe_decode_variant: the tensor-core path takes K <= %d", kFastMaxK);
  QFN_REQUIRE(variant != 3 || K <= kSMaxK, QFN_ERR_UNSUPPORTED,
              "qfn_moe_decode_variant: the stream path takes K <= %d", kSMaxK);
  QFN_REQUIRE(variant != 4 || K <= 10, QFN_ERR_UNSUPPORTED, "qfn_moe_decode_variant: the slice path takes K <= 10");
  return launch_moe_decode(table, n_blocks, sidx, s2, coef, x, x_dtype, h_buf, out, K, as_stream(stream), variant);
}

extern "C" int qfn_device_status(unsigned int* status, int clear) {
  QFN_REQUIRE(status, QFN_ERR_INVALID_ARG, "qfn_device_status: null pointer");
  cudaError_t e = cudaMemcpyFromSymbol(status, g_decode_status, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_decode_status, &zero, sizeof(unsigned int));
  }
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "qfn_device_status: %s", cudaGetErrorString(e));
  return QFN_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free entry point.  Some callers cannot allocate device memory at
// the point where they run a decode step: a runtime whose device memory is
// planned once up front (an 8 GB card running a 63 GiB model has no slack),
// an embedding through a foreign-language FFI that has no binding to a device
// allocator, or a real-time loop that forbids allocator calls.  For them the
// h scratch lives in this file-scope device array instead of a caller buffer.
// ---------------------------------------------------------------------------
namespace {
constexpr int kNoAllocMaxK = QFN_MAX_TOPK;  // 32 experts x 640 floats = 80 KB per device
__device__ __align__(256) float g_noalloc_h[kNoAllocMaxK * qfn::kInter];
float* g_noalloc_ptr[64] = {};
std::mutex g_noalloc_mu;
}  // namespace

extern "C" int qfn_moe_decode_noalloc(const uint8_t* table, int64_t n_blocks, const int32_t* sidx, const float* s2,
                                      const float* coef, const void* x, int x_dtype, float* out, int K,
                                      qfn_stream_t stream) {
  QFN_REQUIRE(K >= 1 && K <= kNoAllocMaxK, QFN_ERR_UNSUPPORTED,
              "qfn_moe_decode_noalloc: K=%d outside [1, %d] (the static scratch holds %d experts)", K, kNoAllocMaxK,
              kNoAllocMaxK);
  QFN_REQUIRE(table && sidx && s2 && coef && x && out, QFN_ERR_INVALID_ARG, "qfn_moe_decode_noalloc: null pointer");
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  float* h = nullptr;
  {
    // First call on a device: resolve the device address of the scratch array
    // (host code must not use the symbol itself: that is a host-side stand-in).
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev->device]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_h);
      if (e != cudaSuccess)
        return set_error(QFN_ERR_CUDA, "qfn_moe_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      g_noalloc_ptr[dev->device] = static_cast<float*>(p);
    }
    h = g_noalloc_ptr[dev->device];
  }
  rc = check_decode_args(table, n_blocks, sidx, s2, coef, x, x_dtype, h, out, K);
  if (rc) return rc;
  return launch_moe_decode(table, n_blocks, sidx, s2, coef, x, x_dtype, h, out, K, as_stream(stream), 0);
}
