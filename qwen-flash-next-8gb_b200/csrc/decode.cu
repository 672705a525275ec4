// bs=1 NVFP4 SwiGLU expert layer over K experts + weighted combine.
//
// Restates qmoe.moe_decode (qmoe.py:77-83) and its two Triton kernels
// _gate_up (qmoe.py:24-51) and _down (qmoe.py:54-74), plus the torch
// reduction out_buf[:K].sum(0) (qmoe.py:83).  Two kernel paths:
//
//  * the slice path (decode_slice.cuh): one cooperative launch per layer for
//    K <= 10 on a 148-SM-class part; the default.
//  * the CUDA-core path below, for any K <= 32 and any part, in two launches:
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
// Helpers of the slice path (decode_slice.cuh).
// ============================================================================


__device__ unsigned int g_decode_status = 0;

__device__ __forceinline__ void note_timeout() { atomicOr(&g_decode_status, kStatusTimeout); }

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

// Exact v * 2^e for |e| <= 252 (two power-of-two factors, each a normal float).
__device__ __forceinline__ float scale_pow2(float v, int e) {
  const int a = e / 2, b = e - a;
  return v * __int_as_float((a + 127) << 23) * __int_as_float((b + 127) << 23);
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

__device__ __forceinline__ float nanmax(float a, float b) { return (isnan(b) || b > a) ? b : a; }

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
  QFN_REQUIRE(variant != 1 && variant != 3, QFN_ERR_UNSUPPORTED,
              "qfn_moe_decode_variant: variants 1 and 3 (the tensor-core and stream paths) were removed");
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
  // the GEMV's and the FP8 linear layer's words (same bit meanings)
  unsigned int g = 0, l = 0;
  int rc = gemv_status(&g, clear != 0);
  if (rc == QFN_OK) rc = linear_status(&l, clear != 0);
  *status |= g | l;
  return rc;
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
// Calls in one stream may share this array because every decode kernel that
// writes h does so only after the previous kernel in the stream has finished:
// the slice kernel and the CUDA-core down kernel (programmatic dependents)
// execute griddepcontrol.wait before their first write of h, and the
// CUDA-core gate/up kernel is launched without programmatic serialisation.
// A kernel that wrote h before its dependency wait would break this.
__device__ __align__(256) float g_noalloc_h[kNoAllocMaxK * qfn::kInter];
struct NoAllocSlot {
  CUcontext ctx;  // the context the address was resolved in
  float* h;
};
NoAllocSlot g_noalloc[64] = {};
std::mutex g_noalloc_mu;
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
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
    // Resolve the device address of the scratch array on the first call in a
    // context (host code must not use the symbol itself: that is a host-side
    // stand-in).  The address is cached per device together with the context
    // it belongs to: after a device reset the module loads again in a new
    // context, and the array may sit at another address.
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_ctx_get_current) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || !fn) return set_error(QFN_ERR_CUDA, "qfn_moe_decode_noalloc: cuCtxGetCurrent unavailable");
      g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    }
    // (before the runtime's first call on this thread no context may be current yet)
    CUcontext ctx = nullptr;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    NoAllocSlot& slot = g_noalloc[dev->device];
    if (!slot.h || !ctx || slot.ctx != ctx) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_h);  // makes the device's primary context current
      if (e != cudaSuccess)
        return set_error(QFN_ERR_CUDA, "qfn_moe_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx)
        return set_error(QFN_ERR_CUDA, "qfn_moe_decode_noalloc: no current CUDA context");
      slot.ctx = ctx;
      slot.h = static_cast<float*>(p);
    }
    h = slot.h;
  }
  rc = check_decode_args(table, n_blocks, sidx, s2, coef, x, x_dtype, h, out, K);
  if (rc) return rc;
  return launch_moe_decode(table, n_blocks, sidx, s2, coef, x, x_dtype, h, out, K, as_stream(stream), 0);
}
