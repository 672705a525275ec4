// Fused MoE router of the decode step (QwenEngine.moe, qwen_engine.py:803-806):
//
//   logits = F.linear(x, W_router)                      bf16 [T, E] (fp32 sums, rounded to bf16)
//   probs  = softmax(logits, dtype=float32)
//   tv, ti = topk(probs, k)                             (ties: lower expert id first)
//   tv     = (tv / tv.sum(-1)).to(bf16)
//
// plus the arguments the decode kernel takes for the routed experts
// (qwen_engine.py:821-825): sidx = L * n_experts + ti (the HBM-resident
// table's block rows), coef = tv as fp32, s2 = store.s2[L, ti].  The engine
// computes these with five torch kernels and a host synchronisation
// (ti[0].tolist(), qwen_engine.py:812/815); here one launch produces them on
// the device, so the routed-expert kernel can follow in the same stream (and
// the same CUDA graph) without the host.
//
// Two launches.  Logits: every CTA takes 4 router rows (a warp per row, the
// row's 5,120 bytes held in registers; the router weights are parameters, so
// they are loaded before the programmatic-dependency wait and stream during
// the previous kernel's tail) and multiplies them with the T token rows
// (staged 8 at a time in shared memory): the 2.6 MB of router weights stream
// from HBM once, spread over E / 4 CTAs.  Select (a programmatic dependent of
// the logits kernel): one 256-thread CTA per token: max, exp, sum and
// division as torch's softmax does them in fp32; then each warp takes the
// top k of its experts by k rounds of a 64-bit warp arg-max (probability,
// then lower index: two 32-bit redux.sync reductions a round), and warp 0
// the top k of the warps' candidates the same way; the renormalisation is
// summed in rank order.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host.cuh"

namespace qfn {

constexpr int kRtWarps = 4;                      // router rows per CTA (a warp each)
constexpr int kRtTok = 8;                        // token rows staged in shared memory at a time
constexpr int kRtChunks = kHid / 8 / 32;         // 16-byte chunks of a row per lane: 10
constexpr int kRtMaxExperts = 1024;              // <= 32 logits per lane in phase 2
constexpr int kRtMaxTopk = 32;
constexpr int kSelThreads = 256;                // selection: one CTA per token

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<const uint16_t*>(&b);
}

__device__ __forceinline__ float dot8_bf16(uint4 a, uint4 b) {
  const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    s = fmaf(bf16_bits_to_f32(wa[i] & 0xffffu), bf16_bits_to_f32(wb[i] & 0xffffu), s);
    s = fmaf(bf16_bits_to_f32(wa[i] >> 16), bf16_bits_to_f32(wb[i] >> 16), s);
  }
  return s;
}

__global__ void __launch_bounds__(32 * kRtWarps) moe_route_logits_kernel(const uint16_t* __restrict__ x,
                                                                        const uint16_t* __restrict__ w, int T, int E,
                                                                        uint16_t* __restrict__ logits) {
  __shared__ __align__(16) uint4 xs[kRtTok][kHid / 8];   // 40 KB
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRtWarps + warp;          // E % 4 == 0 (host check): every warp has a row
  uint4 wr[kRtChunks];
  const uint4* wrow = reinterpret_cast<const uint4*>(w + static_cast<int64_t>(row) * kHid);
#pragma unroll
  for (int i = 0; i < kRtChunks; ++i) wr[i] = ldg_stream_v4(wrow + lane + 32 * i);
  pdl_wait();                 // x (and the logits buffer) may belong to the previous kernel in the stream
  pdl_launch_dependents();
  for (int t0 = 0; t0 < T; t0 += kRtTok) {
    const int nt = T - t0 < kRtTok ? T - t0 : kRtTok;
    __syncthreads();
    for (int i = threadIdx.x; i < nt * (kHid / 8); i += blockDim.x)
      xs[i / (kHid / 8)][i % (kHid / 8)] =
          reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0 + i / (kHid / 8)) * kHid)[i % (kHid / 8)];
    __syncthreads();
    for (int t = 0; t < nt; ++t) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < kRtChunks; ++i) s += dot8_bf16(wr[i], xs[t][lane + 32 * i]);
      s = warp_sum(s);
      if (lane == 0) logits[static_cast<int64_t>(t0 + t) * E + row] = f32_to_bf16_bits(s);
    }
  }
}

// Selection keys: probability bits (p >= 0, so the bits order as the values)
// above the complement of the expert id, so that of equal probabilities the
// lower id is the larger key; 0 = no comparable probability (NaN) or taken.
__device__ __forceinline__ uint64_t sel_key(float p, int e) {
  return p == p ? (static_cast<uint64_t>(__float_as_uint(p)) << 32) | (0xffffffffu - static_cast<uint32_t>(e)) : 0ull;
}

// The largest 64-bit key of the warp, from two 32-bit warp reductions.
__device__ __forceinline__ uint64_t warp_max_key(uint64_t k) {
  const uint32_t hi = __reduce_max_sync(0xffffffffu, static_cast<uint32_t>(k >> 32));
  const uint32_t lo = __reduce_max_sync(0xffffffffu, static_cast<uint32_t>(k >> 32) == hi ? static_cast<uint32_t>(k) : 0u);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

// k rounds of a warp arg-max over the keys the lanes hold (kN each); lane r
// returns the r-th largest key (0 once none is left).
template <int kN>
__device__ __forceinline__ uint64_t warp_topk(uint64_t (&key)[kN], int topk, int lane) {
  uint64_t best = 0, mine = 0;
#pragma unroll
  for (int j = 0; j < kN; ++j) best = key[j] > best ? key[j] : best;
  for (int r = 0; r < topk; ++r) {
    const uint64_t w = warp_max_key(best);
    if (lane == r) mine = w;
    if (w != 0 && best == w) {   // the one lane holding the winner takes it out of the race
      best = 0;
#pragma unroll
      for (int j = 0; j < kN; ++j) {
        if (key[j] == w) key[j] = 0;
        best = key[j] > best ? key[j] : best;
      }
    }
  }
  return mine;
}

__global__ void __launch_bounds__(kSelThreads) moe_route_select_kernel(
    const uint16_t* __restrict__ logits, int T, int E, int topk, int64_t sidx_base, const float* __restrict__ s2_layer,
    int32_t* __restrict__ ti, uint16_t* __restrict__ tv, int32_t* __restrict__ sidx, float* __restrict__ coef,
    float* __restrict__ s2_out) {
  constexpr int kW = kSelThreads / 32;
  constexpr int kPer = kRtMaxExperts / kSelThreads;   // experts per thread
  __shared__ float red[kW];
  __shared__ uint64_t cand[kW][kRtMaxTopk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  pdl_wait();                 // the logits kernel has finished
  pdl_launch_dependents();
  const uint16_t* lg = logits + static_cast<int64_t>(t) * E;
  float p[kPer];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = threadIdx.x + kSelThreads * j;
    p[j] = e < E ? bf16_bits_to_f32(__ldcg(lg + e)) : -INFINITY;
    mx = fmaxf(mx, p[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < kW; ++w) mx = fmaxf(mx, red[w]);
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    // exp in double, rounded once to fp32 (correctly rounded in practice): the
    // closest one value per logit that torch's fp32 exp and the host's can land on
    const int e = threadIdx.x + kSelThreads * j;
    p[j] = e < E ? static_cast<float>(exp(static_cast<double>(p[j] - mx))) : 0.f;
    sum += p[j];
  }
  sum = warp_sum(sum);
  __syncthreads();            // every warp has read red[] as maxima
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = red[0];
#pragma unroll
  for (int w = 1; w < kW; ++w) sum += red[w];
  uint64_t key[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = threadIdx.x + kSelThreads * j;
    key[j] = e < E ? sel_key(p[j] / sum, e) : 0ull;
  }
  // top-k of each warp's experts, then of the warps' candidates (in warp 0)
  const uint64_t wk = warp_topk<kPer>(key, topk, lane);
  if (lane < topk) cand[warp][lane] = wk;
  __syncthreads();
  if (warp != 0) return;
  uint64_t ck[kW];
#pragma unroll
  for (int w = 0; w < kW; ++w) ck[w] = lane < topk ? cand[w][lane] : 0ull;
  const uint64_t k = warp_topk<kW>(ck, topk, lane);
  int ek = 0;                  // no comparable probability left (NaN logits): expert 0, weight NaN
  float pk = __int_as_float(0x7fc00000);
  if (k != 0) {
    ek = static_cast<int>(0xffffffffu - static_cast<uint32_t>(k));
    pk = __uint_as_float(static_cast<uint32_t>(k >> 32));
  }
  // renormalise: the k probabilities summed in rank order, as the reference's tv.sum(-1)
  float tsum = 0.f;
  for (int r = 0; r < topk; ++r) tsum += __shfl_sync(0xffffffffu, pk, r);
  if (lane < topk) {
    const int64_t o = static_cast<int64_t>(t) * topk + lane;
    const uint16_t b = f32_to_bf16_bits(pk / tsum);
    ti[o] = ek;
    tv[o] = b;
    if (sidx) sidx[o] = static_cast<int32_t>(sidx_base + ek);
    if (coef) coef[o] = bf16_bits_to_f32(b);
    if (s2_out) {
      s2_out[3 * o] = s2_layer[3 * ek];
      s2_out[3 * o + 1] = s2_layer[3 * ek + 1];
      s2_out[3 * o + 2] = s2_layer[3 * ek + 2];
    }
  }
}

}  // namespace qfn

using namespace qfn;

extern "C" int qfn_moe_route(const uint16_t* x, const uint16_t* w_router, int64_t T, int n_experts, int topk,
                             int64_t sidx_base, const float* s2_layer, int32_t* ti, uint16_t* tv, int32_t* sidx,
                             float* coef, float* s2_out, uint16_t* logits, qfn_stream_t stream) {
  QFN_REQUIRE(x && w_router && ti && tv && logits, QFN_ERR_INVALID_ARG, "qfn_moe_route: null pointer");
  QFN_REQUIRE(T >= 1 && T <= 4096, QFN_ERR_UNSUPPORTED, "qfn_moe_route: T=%lld outside [1, 4096]", (long long)T);
  QFN_REQUIRE(n_experts >= 4 && n_experts <= kRtMaxExperts && n_experts % 4 == 0, QFN_ERR_UNSUPPORTED,
              "qfn_moe_route: n_experts=%d must be a multiple of 4 in [4, %d]", n_experts, kRtMaxExperts);
  QFN_REQUIRE(topk >= 1 && topk <= kRtMaxTopk && topk <= n_experts, QFN_ERR_UNSUPPORTED,
              "qfn_moe_route: topk=%d outside [1, min(%d, n_experts)]", topk, kRtMaxTopk);
  QFN_REQUIRE(!s2_out || s2_layer, QFN_ERR_INVALID_ARG, "qfn_moe_route: s2_out needs s2_layer");
  QFN_REQUIRE(aligned(x, 16) && aligned(w_router, 16), QFN_ERR_ALIGNMENT,
              "qfn_moe_route: x and w_router must be 16-byte aligned");
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(32 * kRtWarps);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(n_experts / kRtWarps);
  const int Ti = static_cast<int>(T);
  cudaError_t e = cudaLaunchKernelEx(&cfg, moe_route_logits_kernel, x, w_router, Ti, n_experts, logits);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "moe_route_logits_kernel launch: %s", cudaGetErrorString(e));
  cfg.gridDim = dim3(static_cast<unsigned>(T));
  cfg.blockDim = dim3(kSelThreads);
  e = cudaLaunchKernelEx(&cfg, moe_route_select_kernel, static_cast<const uint16_t*>(logits), Ti, n_experts, topk,
                         sidx_base, s2_layer, ti, tv, sidx, coef, s2_out);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "moe_route_select_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("moe_route_select_kernel");

}
