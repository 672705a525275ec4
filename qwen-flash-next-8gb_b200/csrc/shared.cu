// Shared expert of the MoE block with bf16 weights (qwen_engine.py:817-818,
// 829-830), and its combine with the routed experts' output:
//
//   sh  = sigmoid(F.linear(x, sh_g)) * sh_down(silu(sh_gate(x)) * sh_up(x))
//   out = y.to(bf16) + sh                         (y: the routed experts, fp32)
//
// Every torch op of the reference rounds its result to bf16, and so do these
// kernels, in the same places:
//   g = bf16(x.Wg), u = bf16(x.Wu), a = bf16(silu(g)), h = bf16(a * u),
//   d = bf16(h.Wd), gt = bf16(sigmoid(bf16(x.wsg))), sh = bf16(gt * d),
//   out = bf16(bf16(y) + sh)
// with fp32 dot products (the reference's GEMMs accumulate in fp32; the
// summation order differs, so a result can differ from the reference by one
// bf16 rounding step when its fp32 sum lies next to a rounding boundary).
//
// Two launches, both HBM streams of the bf16 weights (3 x I x 2560 x 2 bytes)
// that read their weight rows before the programmatic-dependency wait (the
// weights are parameters): gate/up (a warp per feature: its gate and up rows,
// 10 KB, in registers; one more warp for the gate row sh_g) writes h and gt;
// down (a programmatic dependent: a warp per output row) multiplies h into the
// down rows and applies the gate and the combine.  Token rows are staged in
// shared memory 8 at a time.  The two launches are also entry points of their
// own (qfn_shared_expert_gate_up, qfn_shared_expert_down): the gate/up half
// does not depend on the routing and can run on another stream beside the
// router and the routed experts; the down half then follows the routed
// experts in their stream and fuses the combine with their output.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host.cuh"

namespace qfn {

constexpr int kShWarps = 4;
constexpr int kShTok = 8;
constexpr int kShMaxInter = 4096;

__device__ __forceinline__ uint16_t sh_bf16(float v) {
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<const uint16_t*>(&b);
}

__device__ __forceinline__ float sh_dot8(uint4 a, uint4 b) {
  const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    s = fmaf(bf16_bits_to_f32(wa[i] & 0xffffu), bf16_bits_to_f32(wb[i] & 0xffffu), s);
    s = fmaf(bf16_bits_to_f32(wa[i] >> 16), bf16_bits_to_f32(wb[i] >> 16), s);
  }
  return s;
}

// Rows [0, I): gate row n and up row n of feature n; row I: the gate row sh_g.
__global__ void __launch_bounds__(32 * kShWarps) shared_gate_up_kernel(const uint16_t* __restrict__ x, int T,
                                                                      const uint16_t* __restrict__ wg,
                                                                      const uint16_t* __restrict__ wu,
                                                                      const uint16_t* __restrict__ wsg, int I,
                                                                      uint16_t* __restrict__ h,
                                                                      uint16_t* __restrict__ gt) {
  constexpr int kC = kHid / 8 / 32;   // 16-byte chunks of a 2,560-wide row per lane: 10
  __shared__ __align__(16) uint4 xs[kShTok][kHid / 8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kShWarps + warp;
  const bool feat = n < I, gate_row = n == I;
  uint4 rg[kC], ru[kC];
  if (feat || gate_row) {
    const uint4* pg = reinterpret_cast<const uint4*>(feat ? wg + static_cast<int64_t>(n) * kHid : wsg);
    const uint4* pu = reinterpret_cast<const uint4*>(wu + static_cast<int64_t>(feat ? n : 0) * kHid);
#pragma unroll
    for (int i = 0; i < kC; ++i) {
      rg[i] = ldg_stream_v4(pg + lane + 32 * i);
      ru[i] = feat ? ldg_stream_v4(pu + lane + 32 * i) : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  for (int t0 = 0; t0 < T; t0 += kShTok) {
    const int nt = T - t0 < kShTok ? T - t0 : kShTok;
    __syncthreads();
    for (int i = threadIdx.x; i < nt * (kHid / 8); i += blockDim.x)
      xs[i / (kHid / 8)][i % (kHid / 8)] =
          reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0 + i / (kHid / 8)) * kHid)[i % (kHid / 8)];
    __syncthreads();
    if (!feat && !gate_row) continue;
    for (int t = 0; t < nt; ++t) {
      float sg = 0.f, su = 0.f;
#pragma unroll
      for (int i = 0; i < kC; ++i) {
        sg += sh_dot8(rg[i], xs[t][lane + 32 * i]);
        if (feat) su += sh_dot8(ru[i], xs[t][lane + 32 * i]);
      }
      sg = warp_sum(sg);
      su = warp_sum(su);
      if (lane == 0) {
        const float g = bf16_bits_to_f32(sh_bf16(sg));
        if (feat) {
          const float u = bf16_bits_to_f32(sh_bf16(su));
          const float a = bf16_bits_to_f32(sh_bf16(g / (1.0f + expf(-g))));          // F.silu on bf16
          h[static_cast<int64_t>(t0 + t) * I + n] = sh_bf16(a * u);
        } else {
          gt[t0 + t] = sh_bf16(1.0f / (1.0f + expf(-g)));                             // torch.sigmoid on bf16
        }
      }
    }
  }
}

// Output row r of every token: d = bf16(h . Wd[r]), sh = bf16(gt * d), out = bf16(bf16(y) + sh)
// (or sh when y is null).
template <int kCI>
__global__ void __launch_bounds__(32 * kShWarps) shared_down_kernel(const uint16_t* __restrict__ wd, int I, int T,
                                                                   const uint16_t* __restrict__ h,
                                                                   const uint16_t* __restrict__ gt,
                                                                   const float* __restrict__ y,
                                                                   uint16_t* __restrict__ out) {
  extern __shared__ __align__(16) uint4 hs[];   // [kShTok][I / 8]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kShWarps + warp;   // < 2560 (grid = 2560 / 4)
  const int nc = I / 8;                         // 16-byte chunks of a down row
  uint4 rd[kCI];
  const uint4* pd = reinterpret_cast<const uint4*>(wd + static_cast<int64_t>(r) * I);
#pragma unroll
  for (int i = 0; i < kCI; ++i) rd[i] = lane + 32 * i < nc ? ldg_stream_v4(pd + lane + 32 * i) : make_uint4(0, 0, 0, 0);
  pdl_wait();   // h and gt come from the gate/up kernel
  pdl_launch_dependents();
  for (int t0 = 0; t0 < T; t0 += kShTok) {
    const int nt = T - t0 < kShTok ? T - t0 : kShTok;
    __syncthreads();
    for (int i = threadIdx.x; i < nt * nc; i += blockDim.x)
      hs[i] = reinterpret_cast<const uint4*>(h + static_cast<int64_t>(t0) * I)[i];
    __syncthreads();
    for (int t = 0; t < nt; ++t) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < kCI; ++i)
        if (lane + 32 * i < nc) s += sh_dot8(rd[i], hs[t * nc + lane + 32 * i]);
      s = warp_sum(s);
      if (lane == 0) {
        const int64_t o = static_cast<int64_t>(t0 + t) * kHid + r;
        const float d = bf16_bits_to_f32(sh_bf16(s));
        const float sh = bf16_bits_to_f32(sh_bf16(bf16_bits_to_f32(gt[t0 + t]) * d));
        out[o] = y ? sh_bf16(bf16_bits_to_f32(sh_bf16(y[o])) + sh) : sh_bf16(sh);
      }
    }
  }
}

template <int kCI>
static int launch_shared_down(const cudaLaunchConfig_t& cfg0, const uint16_t* wd, int I, int T, const uint16_t* h,
                              const uint16_t* gt, const float* y, uint16_t* out) {
  cudaLaunchConfig_t cfg = cfg0;
  cfg.dynamicSmemBytes = static_cast<size_t>(kShTok) * I * 2;
  auto fn = shared_down_kernel<kCI>;
  if (cfg.dynamicSmemBytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(cfg.dynamicSmemBytes));
    if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "shared down smem attribute: %s", cudaGetErrorString(e));
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, wd, I, T, h, gt, y, out);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "shared_down_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("shared_down_kernel");
}

static cudaLaunchConfig_t shared_cfg(cudaLaunchAttribute* attr, qfn_stream_t stream, unsigned grid) {
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(32 * kShWarps);
  cfg.gridDim = dim3(grid);
  cfg.stream = as_stream(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

static int shared_checks(int64_t T, int inter) {
  QFN_REQUIRE(T >= 1 && T <= 4096, QFN_ERR_UNSUPPORTED, "qfn_shared_expert: T=%lld outside [1, 4096]", (long long)T);
  QFN_REQUIRE(inter >= 8 && inter <= kShMaxInter && inter % 8 == 0, QFN_ERR_UNSUPPORTED,
              "qfn_shared_expert: inter=%d must be a multiple of 8 in [8, %d]", inter, kShMaxInter);
  return QFN_OK;
}

}  // namespace qfn

using namespace qfn;

extern "C" int qfn_shared_expert_gate_up(const uint16_t* x, int64_t T, const uint16_t* w_gate, const uint16_t* w_up,
                                         const uint16_t* w_sg, int inter, uint16_t* h, uint16_t* gt,
                                         qfn_stream_t stream) {
  QFN_REQUIRE(x && w_gate && w_up && w_sg && h && gt, QFN_ERR_INVALID_ARG, "qfn_shared_expert: null pointer");
  int rc = shared_checks(T, inter);
  if (rc) return rc;
  QFN_REQUIRE(aligned(x, 16) && aligned(w_gate, 16) && aligned(w_up, 16) && aligned(w_sg, 16) && aligned(h, 16),
              QFN_ERR_ALIGNMENT, "qfn_shared_expert: x, weights and h must be 16-byte aligned");
  DeviceInfo* dev;
  if ((rc = current_device(&dev))) return rc;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = shared_cfg(attr, stream, (inter + 1 + kShWarps - 1) / kShWarps);   // + the gate row
  cudaError_t e = cudaLaunchKernelEx(&cfg, shared_gate_up_kernel, x, static_cast<int>(T), w_gate, w_up, w_sg, inter,
                                     h, gt);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "shared_gate_up_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("shared_gate_up_kernel");
}

extern "C" int qfn_shared_expert_down(const uint16_t* w_down, int inter, int64_t T, const uint16_t* h,
                                      const uint16_t* gt, const float* y, uint16_t* out, qfn_stream_t stream) {
  QFN_REQUIRE(w_down && h && gt && out, QFN_ERR_INVALID_ARG, "qfn_shared_expert: null pointer");
  int rc = shared_checks(T, inter);
  if (rc) return rc;
  QFN_REQUIRE(aligned(w_down, 16) && aligned(h, 16), QFN_ERR_ALIGNMENT,
              "qfn_shared_expert: weights and h must be 16-byte aligned");
  DeviceInfo* dev;
  if ((rc = current_device(&dev))) return rc;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = shared_cfg(attr, stream, kHid / kShWarps);
  const int Ti = static_cast<int>(T);
  if (inter <= 1024) return launch_shared_down<4>(cfg, w_down, inter, Ti, h, gt, y, out);
  if (inter <= 2048) return launch_shared_down<8>(cfg, w_down, inter, Ti, h, gt, y, out);
  return launch_shared_down<16>(cfg, w_down, inter, Ti, h, gt, y, out);
}

extern "C" int qfn_shared_expert(const uint16_t* x, int64_t T, const uint16_t* w_gate, const uint16_t* w_up,
                                 const uint16_t* w_down, const uint16_t* w_sg, int inter, const float* y,
                                 uint16_t* h, uint16_t* gt, uint16_t* out, qfn_stream_t stream) {
  QFN_REQUIRE(x && w_gate && w_up && w_down && w_sg && h && gt && out, QFN_ERR_INVALID_ARG,
              "qfn_shared_expert: null pointer");
  int rc = shared_checks(T, inter);
  if (rc) return rc;
  QFN_REQUIRE(aligned(x, 16) && aligned(w_gate, 16) && aligned(w_up, 16) && aligned(w_down, 16) && aligned(w_sg, 16) &&
                  aligned(h, 16),
              QFN_ERR_ALIGNMENT, "qfn_shared_expert: x, weights and h must be 16-byte aligned");
  if ((rc = qfn_shared_expert_gate_up(x, T, w_gate, w_up, w_sg, inter, h, gt, stream))) return rc;
  return qfn_shared_expert_down(w_down, inter, T, h, gt, y, out, stream);
}
