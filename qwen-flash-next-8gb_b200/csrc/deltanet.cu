// One-token gated delta rule of the DeltaNet (linear-attention) layers:
// recurrent_gated_delta_rule at T == 1 (qwen_engine.py:158-174), the step the
// engine runs for every linear-attention layer of every decoded token
// (QwenEngine.deltanet, qwen_engine.py:718-719):
//
//   q = l2norm(q) / sqrt(dk), k = l2norm(k)           (l2norm: x * rsqrt(sum x^2 + 1e-6))
//   S = S * exp(g)                                    (per value head)
//   kv_mem = S^T k ;  delta = (v - kv_mem) * beta
//   S = S + k delta^T ;  out = S^T q                  (out rounded to bf16)
//
// with S [heads][dk][dv] fp32 updated in place.  The reference runs this as
// ~15 torch kernels per layer; here it is one launch that reads and writes
// the state once (2 x heads x dk x dv x 4 bytes: the HBM floor of the step).
// Value head h uses key head h / (heads / key heads), the engine's
// repeat_interleave (qwen_engine.py:717).
//
// CTA = (value head, 32 state columns); 256 threads: thread (column c, slice s)
// keeps rows [s dk/8, (s+1) dk/8) of column c in registers.  The dot products
// over dk meet in shared memory, summed in a fixed slice order.  Elementwise
// steps keep the reference's roundings: the decay as one fp32 product, the
// rank-one update as a product then a sum (no fused multiply-add).
#include <cuda_bf16.h>

#include "common.cuh"
#include "host.cuh"

namespace qfn {

constexpr int kDnSlices = 8;      // row slices of dk per CTA (a warp each)
constexpr int kDnCols = 32;       // state columns per CTA (a lane each)

__device__ __forceinline__ uint16_t dn_bf16(float v) {
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<const uint16_t*>(&b);
}

template <int DK>
__global__ void __launch_bounds__(kDnSlices * kDnCols) deltanet_step_kernel(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
    const float* __restrict__ g, const uint16_t* __restrict__ beta, float* __restrict__ S, uint16_t* __restrict__ out,
    int hk_ratio, int dv, float q_scale) {
  constexpr int R = DK / kDnSlices;
  __shared__ float qs[DK], ks_[DK];
  __shared__ float red[kDnSlices][kDnCols];
  __shared__ float nrm[2];
  const int h = blockIdx.x, c = blockIdx.y * kDnCols + (threadIdx.x & 31), sl = threadIdx.x >> 5;
  const int hk = h / hk_ratio;
  float* Sh = S + static_cast<int64_t>(h) * DK * dv;
  float s[R];
#pragma unroll
  for (int j = 0; j < R; ++j) s[j] = Sh[static_cast<int64_t>(sl * R + j) * dv + c];   // issued first
  pdl_wait();   // q, k, v, g, beta come from the previous kernels of the step
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < DK; i += blockDim.x) {
    qs[i] = bf16_bits_to_f32(q[static_cast<int64_t>(hk) * DK + i]);
    ks_[i] = bf16_bits_to_f32(k[static_cast<int64_t>(hk) * DK + i]);
  }
  __syncthreads();
  if (threadIdx.x < 64) {   // warp 0: |q|^2, warp 1: |k|^2
    const float* a = threadIdx.x < 32 ? qs : ks_;
    float acc = 0.f;
    for (int i = threadIdx.x & 31; i < DK; i += 32) acc = fmaf(a[i], a[i], acc);
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) nrm[threadIdx.x >> 5] = acc;
  }
  __syncthreads();
  const float rq = rsqrtf(nrm[0] + 1e-6f), rk = rsqrtf(nrm[1] + 1e-6f);
  const float decay = expf(g[h]);
  float kv = 0.f;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    s[j] = s[j] * decay;
    kv = fmaf(s[j], ks_[sl * R + j] * rk, kv);
  }
  red[sl][threadIdx.x & 31] = kv;
  __syncthreads();
  kv = 0.f;
#pragma unroll
  for (int i = 0; i < kDnSlices; ++i) kv += red[i][threadIdx.x & 31];
  const float delta = (bf16_bits_to_f32(v[static_cast<int64_t>(h) * dv + c]) - kv) * bf16_bits_to_f32(beta[h]);
  float o = 0.f;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const float kn = ks_[sl * R + j] * rk, qn = (qs[sl * R + j] * rq) / q_scale;
    s[j] = __fadd_rn(s[j], __fmul_rn(kn, delta));
    Sh[static_cast<int64_t>(sl * R + j) * dv + c] = s[j];
    o = fmaf(s[j], qn, o);
  }
  __syncthreads();   // every thread has read red[.] for kv
  red[sl][threadIdx.x & 31] = o;
  __syncthreads();
  if (sl == 0) {
    o = 0.f;
#pragma unroll
    for (int i = 0; i < kDnSlices; ++i) o += red[i][threadIdx.x & 31];
    out[static_cast<int64_t>(h) * dv + c] = dn_bf16(o);
  }
}

}  // namespace qfn

using namespace qfn;

extern "C" int qfn_deltanet_step(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                                 const uint16_t* beta, float* S, uint16_t* out, int n_heads, int n_key_heads, int dk,
                                 int dv, qfn_stream_t stream) {
  QFN_REQUIRE(q && k && v && g && beta && S && out, QFN_ERR_INVALID_ARG, "qfn_deltanet_step: null pointer");
  QFN_REQUIRE(n_heads >= 1 && n_key_heads >= 1 && n_heads % n_key_heads == 0, QFN_ERR_INVALID_ARG,
              "qfn_deltanet_step: n_heads=%d must be a multiple of n_key_heads=%d", n_heads, n_key_heads);
  QFN_REQUIRE((dk == 64 || dk == 128 || dk == 256) && dv >= 32 && dv <= 4096 && dv % 32 == 0, QFN_ERR_UNSUPPORTED,
              "qfn_deltanet_step: dk=%d (64, 128 or 256) and dv=%d (a multiple of 32) unsupported", dk, dv);
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_heads, dv / kDnCols);
  cfg.blockDim = dim3(kDnSlices * kDnCols);
  cfg.stream = as_stream(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // the engine divides by dk ** 0.5, a Python float: torch rounds it to the tensor's fp32
  const float q_scale = static_cast<float>(sqrt(static_cast<double>(dk)));
  const int r = n_heads / n_key_heads;
  cudaError_t e;
  if (dk == 64)
    e = cudaLaunchKernelEx(&cfg, deltanet_step_kernel<64>, q, k, v, g, beta, S, out, r, dv, q_scale);
  else if (dk == 128)
    e = cudaLaunchKernelEx(&cfg, deltanet_step_kernel<128>, q, k, v, g, beta, S, out, r, dv, q_scale);
  else
    e = cudaLaunchKernelEx(&cfg, deltanet_step_kernel<256>, q, k, v, g, beta, S, out, r, dv, q_scale);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "deltanet_step_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("deltanet_step_kernel");
}
