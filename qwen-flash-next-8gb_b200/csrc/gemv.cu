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

static int launch_gemv(const uint8_t* q, const float* s, const uint16_t* x, void* y, int y_dtype, int64_t N,
                       int64_t K, cudaStream_t st) {
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
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

}  // namespace qfn

using namespace qfn;

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
