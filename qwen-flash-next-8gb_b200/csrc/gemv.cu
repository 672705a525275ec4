// FP8 E4M3 row-scaled matrix x vector (the DeltaNet projections at T == 1).
//
// Restates fp8gemv._gemv (fp8gemv.py:5-17): y[n] = bf16(s[n] * sum_k q[n,k] x[k])
// with fp32 accumulation.  A pure HBM stream: every weight byte is read once
// with 128-bit non-allocating loads issued before the x vector is staged, x
// sits in shared memory as fp32 in a [4][K/16] float4 layout (conflict-free
// for the lane -> 16-byte-chunk mapping), each warp owns two rows and
// reduces its K partial sums with shuffles.
#include "common.cuh"
#include "host.cuh"

namespace qfn {

__device__ unsigned int g_gemv_status = 0;

__device__ __forceinline__ float warp_sum_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

constexpr int kGemvThreads = 256;
constexpr int kGemvRowsPerWarp = 2;
constexpr int kGemvRowsPerCta = (kGemvThreads / 32) * kGemvRowsPerWarp;
constexpr int kGemvBatch = 8;              // 16-byte chunks per lane per row per batch
constexpr int64_t kGemvMaxK = 32768;       // x staged in <= 128 KB of shared memory

__device__ __forceinline__ float dot16_e4m3(uint4 w, const float4* __restrict__ xs, int c, int nchunk) {
  const float4 xa = xs[c];
  const float4 xb = xs[nchunk + c];
  const float4 xc = xs[2 * nchunk + c];
  const float4 xd = xs[3 * nchunk + c];
  uint32_t lo, hi;
  float2 a, b;
  float s;
  e4m3x4_to_f16x2(w.x, lo, hi);
  a = f16x2_to_f32x2(lo); b = f16x2_to_f32x2(hi);
  s = a.x * xa.x; s = fmaf(a.y, xa.y, s); s = fmaf(b.x, xa.z, s); s = fmaf(b.y, xa.w, s);
  e4m3x4_to_f16x2(w.y, lo, hi);
  a = f16x2_to_f32x2(lo); b = f16x2_to_f32x2(hi);
  s = fmaf(a.x, xb.x, s); s = fmaf(a.y, xb.y, s); s = fmaf(b.x, xb.z, s); s = fmaf(b.y, xb.w, s);
  e4m3x4_to_f16x2(w.z, lo, hi);
  a = f16x2_to_f32x2(lo); b = f16x2_to_f32x2(hi);
  s = fmaf(a.x, xc.x, s); s = fmaf(a.y, xc.y, s); s = fmaf(b.x, xc.z, s); s = fmaf(b.y, xc.w, s);
  e4m3x4_to_f16x2(w.w, lo, hi);
  a = f16x2_to_f32x2(lo); b = f16x2_to_f32x2(hi);
  s = fmaf(a.x, xd.x, s); s = fmaf(a.y, xd.y, s); s = fmaf(b.x, xd.z, s); s = fmaf(b.y, xd.w, s);
  return s;
}

template <bool kOutF32>
__global__ void __launch_bounds__(kGemvThreads) gemv_e4m3_kernel(const uint8_t* __restrict__ q,
                                                                  const float* __restrict__ s,
                                                                  const uint16_t* __restrict__ x,
                                                                  void* __restrict__ y, int64_t N, int K) {
  extern __shared__ float4 xs[];
  const int nchunk = K >> 4;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kGemvRowsPerCta + warp * kGemvRowsPerWarp;
  const bool v0 = r0 < N;
  const bool v1 = r0 + 1 < N;
  const uint4* q0 = reinterpret_cast<const uint4*>(q + r0 * K);
  const uint4* q1 = q0 + nchunk;

  uint4 w0[kGemvBatch], w1[kGemvBatch];
  auto load_batch = [&](int c0) {
#pragma unroll
    for (int u = 0; u < kGemvBatch; ++u) {
      const int c = c0 + lane + 32 * u;
      w0[u] = (v0 && c < nchunk) ? ldg_stream_v4(q0 + c) : make_uint4(0, 0, 0, 0);
      w1[u] = (v1 && c < nchunk) ? ldg_stream_v4(q1 + c) : make_uint4(0, 0, 0, 0);
    }
  };
  load_batch(0);

  // Stage x (bf16) as fp32 while the first weight loads are in flight.
  for (int i = threadIdx.x; i < nchunk * 4; i += kGemvThreads) {
    const int c = i >> 2, qq = i & 3;
    const uint2 v = *reinterpret_cast<const uint2*>(x + 16 * c + 4 * qq);
    float4 f;
    f.x = bf16_bits_to_f32(v.x & 0xffffu);
    f.y = bf16_bits_to_f32(v.x >> 16);
    f.z = bf16_bits_to_f32(v.y & 0xffffu);
    f.w = bf16_bits_to_f32(v.y >> 16);
    xs[qq * nchunk + c] = f;
  }
  __syncthreads();

  float a0 = 0.f, a1 = 0.f;
  for (int c0 = 0; c0 < nchunk; c0 += 32 * kGemvBatch) {
    if (c0 > 0) load_batch(c0);
#pragma unroll
    for (int u = 0; u < kGemvBatch; ++u) {
      const int c = c0 + lane + 32 * u;
      if (c < nchunk) {
        a0 += dot16_e4m3(w0[u], xs, c, nchunk);
        a1 += dot16_e4m3(w1[u], xs, c, nchunk);
      }
    }
  }
  a0 = warp_sum(a0);
  a1 = warp_sum(a1);
  if (lane == 0) {
    if (v0) {
      const float r = a0 * s[r0];
      if (kOutF32) static_cast<float*>(y)[r0] = r;
      else static_cast<__nv_bfloat16*>(y)[r0] = __float2bfloat16_rn(r);
    }
    if (v1) {
      const float r = a1 * s[r0 + 1];
      if (kOutF32) static_cast<float*>(y)[r0 + 1] = r;
      else static_cast<__nv_bfloat16*>(y)[r0 + 1] = __float2bfloat16_rn(r);
    }
  }
}

// ---------------------------------------------------------------------------
// Stream path (K % 64 == 0, K <= 8192): one CTA of 512 threads per SM owns a
// contiguous range of 16-row tiles.  Tiles are bulk-copied (TMA, non-tensor:
// a tile is 16 x K contiguous bytes) into a ring of shared-memory slots, all
// slots requested at entry, refilled as tiles are consumed.  x is staged once
// as an f16 hi/lo pair after one power-of-two prescale.  Dot products run on
// mma.sync.m16n8k16: A = 16 weight rows (E4M3 -> f16 is exact; the row scale
// is applied to the fp32 result), B = x hi / x lo in columns 0 / 1.  Warp w
// owns a K-range of 64-element spans of every tile; lane t takes bytes
// [16t, 16t + 16) of a span's 64 bytes, so one 128-bit load per row feeds
// four MMAs (the K order inside a span is permuted identically in A and B).
// Per-warp partial sums meet in shared memory and are added in a fixed order.

constexpr int kGsThreads = 512;
constexpr int kGsWarps = kGsThreads / 32;
constexpr int kGsMaxTilesPerCta = 16;
#ifndef QFN_GEMV_SMEM_KB
#define QFN_GEMV_SMEM_KB 225
#endif
constexpr int kGsSmemBudget = QFN_GEMV_SMEM_KB * 1024;

struct GsLayout {
  int slots, ring, xs, xraw, red, bar, sc, total;
};

// Shared memory of the stream path for K and up to `tiles` tiles per CTA:
// the ring of 16 x K weight slots, x hi/lo (f16), x as loaded (bf16; dead
// after staging, so it shares its bytes with the per-tile partial sums), the
// CTA's row scales.
__host__ __device__ inline GsLayout gs_layout(int K, int tiles) {
  GsLayout L;
  const int tile = 16 * K;
  const int red = tiles * kGsWarps * 16 * 4;
  const int scratch = red > 2 * K ? red : 2 * K;
  const int fixed = 4 * K + scratch + 256 + 64 * tiles + 128;
  int slots = (kGsSmemBudget - fixed) / tile;
  slots = slots < 1 ? 1 : (slots > 8 ? 8 : (slots > tiles ? tiles : slots));
  L.slots = slots;
  L.ring = 0;
  L.xs = slots * tile;        // x hi [K] f16, then x lo [K] f16
  L.xraw = L.xs + 4 * K;      // x as loaded (bf16)
  L.red = L.xraw;             // [tile][warp][16] fp32 partials (after x is staged)
  L.bar = L.xraw + scratch;
  L.sc = L.bar + 256;           // [16 x tiles] fp32 row scales
  L.total = L.sc + 64 * tiles + 128;  // + alignment slack
  return L;
}

template <bool kOutF32>
__global__ void __launch_bounds__(kGsThreads, 1)
    gemv_stream_kernel(const uint8_t* __restrict__ q, const float* __restrict__ s, const uint16_t* __restrict__ x,
                       void* __restrict__ y, int64_t N, int K, int max_tiles) {
  extern __shared__ __align__(128) uint8_t gsm_raw[];
  uint8_t* sm = gsm_raw + ((128 - (smem_u32(gsm_raw) & 127)) & 127);
  const GsLayout L = gs_layout(K, max_tiles);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint64_t* empty = full + 9;
  __shared__ float wmax[kGsWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t n_tiles = (N + 15) / 16;
  const int64_t t0 = n_tiles * blockIdx.x / gridDim.x, t1 = n_tiles * (blockIdx.x + 1) / gridDim.x;
  const int nt = static_cast<int>(t1 - t0);
  const int S = L.slots;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGsWarps);
    }
    mbar_init(&full[8], 1);  // x
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i) {  // tile i of this CTA into slot i % S
    const int64_t row0 = (t0 + i) * 16;
    const int64_t rows = N - row0 < 16 ? N - row0 : 16;
    const uint32_t bytes = static_cast<uint32_t>(rows * K);
    mbar_arrive_expect_tx(&full[i % S], bytes);
    bulk_g2s(sm + L.ring + (i % S) * 16 * K, q + row0 * K, bytes, &full[i % S]);
  };
  // Inputs may come from the previous kernel in the stream: wait for it (the
  // launch and the prologue above overlap its tail).  Requesting the weight
  // tiles before the wait measured no faster: at 225 KB of shared memory the
  // next call's CTAs become resident only as this call's leave.
  pdl_wait();
  pdl_launch_dependents();
  // x and the CTA's row scales first (ordinary loads would queue behind the
  // weight stream; the scales would otherwise be read at the very end), then
  // the tiles, one per lane of warp 0 (a single thread issuing bulk copies
  // back to back takes ~0.2 us per copy).
  const int64_t nrows = N - 16 * t0 < 16 * nt ? N - 16 * t0 : 16 * nt;
  const bool sbulk = (reinterpret_cast<uintptr_t>(s) & 15u) == 0 && nrows % 4 == 0;
  float* sc = reinterpret_cast<float*>(sm + L.sc);
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&full[8], 2 * K + (sbulk ? static_cast<uint32_t>(4 * nrows) : 0u));
    bulk_g2s(sm + L.xraw, x, 2 * K, &full[8]);
    if (sbulk) bulk_g2s(sc, s + 16 * t0, static_cast<uint32_t>(4 * nrows), &full[8]);
  }
  if (warp == 0 && lane < S && lane < nt) issue(lane);

  // x -> f16 hi/lo * 2^ex (thread u owns k = u, u + 512, ...)
  if (!mbar_wait(&full[8], 0)) atomicOr(&g_gemv_status, kStatusTimeout);
  const uint16_t* xr = reinterpret_cast<const uint16_t*>(sm + L.xraw);
  constexpr int kMaxPer = 8192 / kGsThreads;
  float xv[kMaxPer];
  float mx = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int k = threadIdx.x + j * kGsThreads;
    xv[j] = k < K ? bf16_bits_to_f32(xr[k]) : 0.f;
    mx = fmaxf(mx, fabsf(xv[j]));
  }
  mx = warp_sum_max(mx);
  if (lane == 0) wmax[warp] = mx;
  __syncthreads();
  float xm = 0.f;
  for (int w = 0; w < kGsWarps; ++w) xm = fmaxf(xm, wmax[w]);
  const int ex = f16_prescale_exp(xm);
  __half* xh = reinterpret_cast<__half*>(sm + L.xs);
  __half* xl = xh + K;
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int k = threadIdx.x + j * kGsThreads;
    if (k < K) {
      __half hi, lo;
      split_f16(ldexpf(xv[j], ex), hi, lo);
      xh[k] = hi;
      xl[k] = lo;
    }
  }
  __syncthreads();

  const int spans = K >> 6;
  const int sp0 = spans * warp / kGsWarps, sp1 = spans * (warp + 1) / kGsWarps;
  const __half* xsrc = g == 0 ? xh : xl;
  float* red = reinterpret_cast<float*>(sm + L.red);
  for (int i = 0; i < nt; ++i) {
    const int slot = i % S;
    if (!mbar_wait(&full[slot], (i / S) & 1)) atomicOr(&g_gemv_status, kStatusTimeout);
    const uint8_t* tile = sm + L.ring + slot * 16 * K;
    float d4[4][4] = {};  // four independent MMA chains (one per 16-k step of a span)
    for (int sp = sp0; sp < sp1; ++sp) {
      const uint4 ra = *reinterpret_cast<const uint4*>(tile + g * K + 64 * sp + 16 * t);
      const uint4 rb = *reinterpret_cast<const uint4*>(tile + (g + 8) * K + 64 * sp + 16 * t);
      const uint32_t wa[4] = {ra.x, ra.y, ra.z, ra.w};
      const uint32_t wb[4] = {rb.x, rb.y, rb.z, rb.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t alo, ahi, blo, bhi;
        e4m3x4_to_f16x2(wa[j], alo, ahi);
        e4m3x4_to_f16x2(wb[j], blo, bhi);
        const uint32_t a[4] = {alo, blo, ahi, bhi};
        uint2 bq = make_uint2(0, 0);
        if (g < 2) bq = *reinterpret_cast<const uint2*>(xsrc + 64 * sp + 16 * t + 4 * j);
        mma_16816(d4[j], a, bq.x, bq.y);
      }
    }
    if (t == 0) {
      red[(i * kGsWarps + warp) * 16 + g] =
          ((d4[0][0] + d4[0][1]) + (d4[1][0] + d4[1][1])) + ((d4[2][0] + d4[2][1]) + (d4[3][0] + d4[3][1]));
      red[(i * kGsWarps + warp) * 16 + 8 + g] =
          ((d4[0][2] + d4[0][3]) + (d4[1][2] + d4[1][3])) + ((d4[2][2] + d4[2][3]) + (d4[3][2] + d4[3][3]));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (threadIdx.x == 0 && i + S < nt) {
      if (!mbar_wait(&empty[slot], (i / S) & 1)) atomicOr(&g_gemv_status, kStatusTimeout);
      issue(i + S);
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < 16 * nt; r += kGsThreads) {
    const int i = r >> 4, rr = r & 15;
    const int64_t row = (t0 + i) * 16 + rr;
    if (row >= N) continue;
    float acc = 0.f;
    for (int w = 0; w < kGsWarps; ++w) acc += red[(i * kGsWarps + w) * 16 + rr];
    const float v = ldexpf(acc, -ex) * (sbulk ? sc[r] : s[row]);
    if (kOutF32) static_cast<float*>(y)[row] = v;
    else static_cast<__nv_bfloat16*>(y)[row] = __float2bfloat16_rn(v);
  }
}

static int launch_gemv(const uint8_t* q, const float* s, const uint16_t* x, void* y, int y_dtype, int64_t N,
                       int64_t K, cudaStream_t st) {
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  if (K % 64 == 0 && K <= 8192 && aligned(x, 16)) {
    const int64_t n_tiles = (N + 15) / 16;
    int64_t grid = dev->sm_count;
    if (n_tiles > grid * kGsMaxTilesPerCta) grid = (n_tiles + kGsMaxTilesPerCta - 1) / kGsMaxTilesPerCta;
    if (grid > n_tiles) grid = n_tiles;
    const int max_tiles = static_cast<int>((n_tiles + grid - 1) / grid);
    const GsLayout L = gs_layout(static_cast<int>(K), max_tiles);
    if (static_cast<size_t>(L.total) + 1024 <= dev->smem_optin && grid <= 65535) {
      static int attr_set[64][2] = {};  // largest dynamic shared memory enabled so far
      const int ti = y_dtype == QFN_DTYPE_F32 ? 1 : 0;
      auto fn = y_dtype == QFN_DTYPE_F32 ? gemv_stream_kernel<true> : gemv_stream_kernel<false>;
      if (attr_set[dev->device][ti] < L.total) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
        if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "gemv smem attribute: %s", cudaGetErrorString(e));
        attr_set[dev->device][ti] = L.total;
      }
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(grid));
      cfg.blockDim = dim3(kGsThreads);
      cfg.dynamicSmemBytes = L.total;
      cfg.stream = st;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cudaError_t e = cudaLaunchKernelEx(&cfg, fn, q, s, x, y, N, static_cast<int>(K), max_tiles);
      if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "gemv_stream_kernel launch: %s", cudaGetErrorString(e));
      return check_launch("gemv_stream_kernel");
    }
  }
  const size_t smem = static_cast<size_t>(K) * 4;
  const unsigned grid = static_cast<unsigned>((N + kGemvRowsPerCta - 1) / kGemvRowsPerCta);
  if (y_dtype == QFN_DTYPE_F32) {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(gemv_e4m3_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "gemv smem attribute: %s", cudaGetErrorString(e));
    }
    gemv_e4m3_kernel<true><<<grid, kGemvThreads, smem, st>>>(q, s, x, y, N, static_cast<int>(K));
  } else {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(gemv_e4m3_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "gemv smem attribute: %s", cudaGetErrorString(e));
    }
    gemv_e4m3_kernel<false><<<grid, kGemvThreads, smem, st>>>(q, s, x, y, N, static_cast<int>(K));
  }
  return check_launch("gemv_e4m3_kernel");
}

// ---------------------------------------------------------------------------
// E4M3 rows -> bf16 weights for the T > 1 path of the engine's FP8 linear
// layer (qwen_engine.py:79-83): F.linear(x, (q.to(bf16) * s).to(bf16)).
// w[n][k] = bf16_rn(f32(q[n][k]) * s[n]): e4m3 -> bf16 is exact, the product
// is one fp32 multiply rounded to nearest even, then rounded to bf16 -- the
// same two roundings as the reference's torch expression, in one pass that
// reads 1 byte and writes 2 per weight (the torch chain writes a bf16 and an
// fp32 temporary and reads both back).  A thread takes up to four 16-weight
// chunks a grid stride apart and issues their loads before any store, so
// each SM keeps ~128 KB of reads in flight.
__device__ __forceinline__ void e4m3x16_rows_to_bf16(uint4 v, float sc, uint16_t* __restrict__ w, int64_t c) {
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t lo, hi;
    e4m3x4_to_f16x2(in[i], lo, hi);
    const float2 a = f16x2_to_f32x2(lo), b = f16x2_to_f32x2(hi);
    const __nv_bfloat162 ra = __floats2bfloat162_rn(__fmul_rn(a.x, sc), __fmul_rn(a.y, sc));
    const __nv_bfloat162 rb = __floats2bfloat162_rn(__fmul_rn(b.x, sc), __fmul_rn(b.y, sc));
    o[2 * i] = *reinterpret_cast<const uint32_t*>(&ra);
    o[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&rb);
  }
  uint4* dst = reinterpret_cast<uint4*>(w) + 2 * c;
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

constexpr int kDqUnroll = 4;

__global__ void __launch_bounds__(256) e4m3_rows_to_bf16_kernel(const uint8_t* __restrict__ q,
                                                                 const float* __restrict__ s,
                                                                 uint16_t* __restrict__ w, int64_t n_chunks,
                                                                 int64_t chunks_per_row) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c0 < n_chunks;
       c0 += kDqUnroll * stride) {
    uint4 v[kDqUnroll];
    float sc[kDqUnroll];
#pragma unroll
    for (int u = 0; u < kDqUnroll; ++u) {
      const int64_t c = c0 + u * stride;
      if (c < n_chunks) {
        v[u] = ldg_stream_v4(reinterpret_cast<const uint4*>(q) + c);
        sc[u] = s[c / chunks_per_row];
      }
    }
#pragma unroll
    for (int u = 0; u < kDqUnroll; ++u) {
      const int64_t c = c0 + u * stride;
      if (c < n_chunks) e4m3x16_rows_to_bf16(v[u], sc[u], w, c);
    }
  }
}

static int launch_e4m3_rows_to_bf16(const uint8_t* q, const float* s, uint16_t* w, int64_t N, int64_t K,
                                    cudaStream_t st) {
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  const int64_t cpr = K / 16, n_chunks = N * cpr;
  int64_t blocks = (n_chunks + 256 * kDqUnroll - 1) / (256 * kDqUnroll);
  const int64_t cap = static_cast<int64_t>(dev->sm_count) * 4;  // one wave (48 registers: <= 5 CTAs per SM)
  if (blocks > cap) blocks = cap;
  e4m3_rows_to_bf16_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(q, s, w, n_chunks, cpr);
  return check_launch("e4m3_rows_to_bf16_kernel");
}

int gemv_status(unsigned int* v, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(v, g_gemv_status, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_gemv_status, &zero, sizeof(unsigned int));
  }
  return e == cudaSuccess ? QFN_OK : set_error(QFN_ERR_CUDA, "gemv status: %s", cudaGetErrorString(e));
}

}  // namespace qfn

using namespace qfn;

extern "C" int qfn_e4m3_rows_to_bf16(const uint8_t* q, const float* s, uint16_t* w, int64_t N, int64_t K,
                                     qfn_stream_t stream) {
  QFN_REQUIRE(q && s && w, QFN_ERR_INVALID_ARG, "qfn_e4m3_rows_to_bf16: null pointer");
  QFN_REQUIRE(N > 0 && K > 0, QFN_ERR_INVALID_ARG, "qfn_e4m3_rows_to_bf16: N=%lld K=%lld must be positive",
              (long long)N, (long long)K);
  QFN_REQUIRE(K % 16 == 0, QFN_ERR_UNSUPPORTED, "qfn_e4m3_rows_to_bf16: K=%lld must be a multiple of 16",
              (long long)K);
  QFN_REQUIRE(aligned(q, 16) && aligned(w, 16), QFN_ERR_ALIGNMENT,
              "qfn_e4m3_rows_to_bf16: q and w must be 16-byte aligned");
  return launch_e4m3_rows_to_bf16(q, s, w, N, K, as_stream(stream));
}

extern "C" int qfn_gemv_e4m3(const uint8_t* q, const float* s, const uint16_t* x, void* y, int y_dtype,
                             int64_t N, int64_t K, qfn_stream_t stream) {
  QFN_REQUIRE(q && s && x && y, QFN_ERR_INVALID_ARG, "qfn_gemv_e4m3: null pointer");
  QFN_REQUIRE(N > 0 && K > 0, QFN_ERR_INVALID_ARG, "qfn_gemv_e4m3: N=%lld K=%lld must be positive",
              (long long)N, (long long)K);
  QFN_REQUIRE(y_dtype == QFN_DTYPE_F32 || y_dtype == QFN_DTYPE_BF16, QFN_ERR_INVALID_ARG,
              "qfn_gemv_e4m3: bad y_dtype %d", y_dtype);
  QFN_REQUIRE(K % 16 == 0 && K <= kGemvMaxK, QFN_ERR_UNSUPPORTED,
              "qfn_gemv_e4m3: K=%lld must be a multiple of 16 and <= %lld", (long long)K, (long long)kGemvMaxK);
  QFN_REQUIRE(aligned(q, 16) && aligned(x, 8), QFN_ERR_ALIGNMENT,
              "qfn_gemv_e4m3: q must be 16-byte and x 8-byte aligned");
  return launch_gemv(q, s, x, y, y_dtype, N, K, as_stream(stream));
}
