// NVFP4 -> fp32 dequantization of a weight matrix / an expert block.
//
// Restates qmoe.deq (qmoe.py:93-102) on the GPU: W[n][k] = E2M1[nib] *
// e4m3(s[n][k/16]) * ws2, multiplied in that order in fp32 so the result is
// bit-identical to the reference (the first product is exact: <= 6 bits).
#include "common.cuh"
#include "host.cuh"

namespace qfn {

// One thread per 16 output elements (8 weight bytes = one scale group).
__global__ void __launch_bounds__(256) deq_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ s,
                                                  float ws2, float* __restrict__ out, int64_t n_groups,
                                                  int64_t groups_per_row) {
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < n_groups;
       gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = gi / groups_per_row;
    const int64_t g = gi - row * groups_per_row;
    const uint2 wv = *reinterpret_cast<const uint2*>(w + gi * 8);
    const float sc = e4m3_to_f32(s[row * groups_per_row + g]);
    uint32_t h[8];
    e2m1x8_to_f16x2(wv.x, *reinterpret_cast<uint32_t(*)[4]>(&h[0]));
    e2m1x8_to_f16x2(wv.y, *reinterpret_cast<uint32_t(*)[4]>(&h[4]));
    float4* o = reinterpret_cast<float4*>(out + gi * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 a = f16x2_to_f32x2(h[2 * q]);
      const float2 b = f16x2_to_f32x2(h[2 * q + 1]);
      float4 v;
      v.x = __fmul_rn(__fmul_rn(a.x, sc), ws2);
      v.y = __fmul_rn(__fmul_rn(a.y, sc), ws2);
      v.z = __fmul_rn(__fmul_rn(b.x, sc), ws2);
      v.w = __fmul_rn(__fmul_rn(b.y, sc), ws2);
      o[q] = v;
    }
  }
}

static int launch_deq(const uint8_t* w, const uint8_t* s, float ws2, float* out, int64_t N, int64_t K,
                      cudaStream_t st) {
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  const int64_t gpr = K / 16;
  const int64_t n_groups = N * gpr;
  int64_t blocks = (n_groups + 255) / 256;
  const int64_t cap = static_cast<int64_t>(dev->sm_count) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  deq_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(w, s, ws2, out, n_groups, gpr);
  return check_launch("deq_kernel");
}

}  // namespace qfn

using namespace qfn;

extern "C" int qfn_deq(const uint8_t* w, const uint8_t* s, float ws2, float* out, int64_t N, int64_t K,
                       qfn_stream_t stream) {
  QFN_REQUIRE(w && s && out, QFN_ERR_INVALID_ARG, "qfn_deq: null pointer");
  QFN_REQUIRE(N > 0 && K > 0, QFN_ERR_INVALID_ARG, "qfn_deq: N=%lld K=%lld must be positive", (long long)N,
              (long long)K);
  QFN_REQUIRE(K % 32 == 0, QFN_ERR_UNSUPPORTED, "qfn_deq: K=%lld must be a multiple of 32", (long long)K);
  QFN_REQUIRE(aligned(w, 8) && aligned(out, 16), QFN_ERR_ALIGNMENT,
              "qfn_deq: w must be 8-byte and out 16-byte aligned");
  return launch_deq(w, s, ws2, out, N, K, as_stream(stream));
}

extern "C" int qfn_block_deq(const uint8_t* blk, const float s2[3], float* gate, float* up, float* down,
                             qfn_stream_t stream) {
  QFN_REQUIRE(blk && s2 && gate && up && down, QFN_ERR_INVALID_ARG, "qfn_block_deq: null pointer");
  QFN_REQUIRE(aligned(blk, 16), QFN_ERR_ALIGNMENT, "qfn_block_deq: block must be 16-byte aligned");
  const cudaStream_t st = as_stream(stream);
  int rc = qfn_deq(blk + kOGW, blk + kOGS, s2[0], gate, kInter, kHid, stream);
  if (!rc) rc = qfn_deq(blk + kOUW, blk + kOUS, s2[1], up, kInter, kHid, stream);
  if (!rc) rc = qfn_deq(blk + kODW, blk + kODS, s2[2], down, kHid, kInter, stream);
  (void)st;
  return rc;
}
