// Shared device helpers for the sm_100a kernels of libqfn.
//
// Number formats (the reference's NVFP4 layout, qmoe.py:3,87,95-101):
//  * e2m1: 4-bit code, bit 3 = sign, magnitudes {0,.5,1,1.5,2,3,4,6}; two codes
//    per byte, the LOW nibble is the even k index.
//  * e4m3 ("float8_e4m3fn"): 1-4-3, bias 7, no infinities, 0x7f/0xff = NaN.
// Both convert exactly to f16 with the hardware cvt instructions used below.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace qfn {

constexpr int kHid = 2560;
constexpr int kInter = 640;
constexpr int64_t kBlock = 2764800;
constexpr int64_t kOGW = 0, kOUW = 819200, kODW = 1638400;
constexpr int64_t kOGS = 2457600, kOUS = 2560000, kODS = 2662400;

// Four e2m1 pairs (one 32-bit word = 8 codes) -> four f16x2 words.  Word i
// holds byte i of `w`: low half = low nibble (even k), high half = high nibble.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

// Four e4m3 bytes -> two f16x2 words: lo = bytes (0,1), hi = bytes (2,3); the
// lower byte of each pair lands in the lower half.
__device__ __forceinline__ void e4m3x4_to_f16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\t"
      "mov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

// One e4m3 byte (low 8 bits of b) -> fp32, exact.
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  uint32_t r;
  asm("{\n\t.reg .b16 a;\n\t"
      "cvt.u16.u32 a, %1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\t}"
      : "=r"(r)
      : "r"(b & 0xffu));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(r & 0xffffu)));
}

__device__ __forceinline__ float2 f16x2_to_f32x2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b16) {
  return __uint_as_float(b16 << 16);
}

// Streaming 128/64-bit loads of weights that are read exactly once: bypass L1
// allocation so the x vector / scratch keep the cache.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint2 ldg_stream_v2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ldg_stream_u8(const void* p) {
  uint32_t v;
  asm volatile("{\n\t.reg .u16 t;\n\t"
               "ld.global.nc.L1::no_allocate.u8 t, [%1];\n\t"
               "cvt.u32.u16 %0, t;\n\t}"
               : "=r"(v)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Programmatic dependent launch controls (no-ops when the launch carries no
// programmatic dependency).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 16 e2m1 codes (8 bytes) . 16 fp32 x values held as four float4 -> fp32 sum.
__device__ __forceinline__ float dot16_e2m1(uint2 w, float4 x0, float4 x1, float4 x2, float4 x3) {
  uint32_t h[8];
  e2m1x8_to_f16x2(w.x, *reinterpret_cast<uint32_t(*)[4]>(&h[0]));
  e2m1x8_to_f16x2(w.y, *reinterpret_cast<uint32_t(*)[4]>(&h[4]));
  float2 a;
  float s;
  a = f16x2_to_f32x2(h[0]); s = a.x * x0.x;      s = fmaf(a.y, x0.y, s);
  a = f16x2_to_f32x2(h[1]); s = fmaf(a.x, x0.z, s); s = fmaf(a.y, x0.w, s);
  a = f16x2_to_f32x2(h[2]); s = fmaf(a.x, x1.x, s); s = fmaf(a.y, x1.y, s);
  a = f16x2_to_f32x2(h[3]); s = fmaf(a.x, x1.z, s); s = fmaf(a.y, x1.w, s);
  a = f16x2_to_f32x2(h[4]); s = fmaf(a.x, x2.x, s); s = fmaf(a.y, x2.y, s);
  a = f16x2_to_f32x2(h[5]); s = fmaf(a.x, x2.z, s); s = fmaf(a.y, x2.w, s);
  a = f16x2_to_f32x2(h[6]); s = fmaf(a.x, x3.x, s); s = fmaf(a.y, x3.y, s);
  a = f16x2_to_f32x2(h[7]); s = fmaf(a.x, x3.z, s); s = fmaf(a.y, x3.w, s);
  return s;
}

}  // namespace qfn

// ---------------------------------------------------------------- async copies / barriers
namespace qfn {

// Bound on every spin of a kernel on an mbarrier; a wait that runs out sets
// kStatusTimeout in the device status word of the kernel's translation unit
// and the kernel carries on (its outputs are then garbage; the host reads and
// clears the word with qfn_device_status).
// Every wait of these kernels gives up after kWaitNs of %globaltimer time
// (a working kernel waits microseconds), sets a status bit and lets the
// kernel finish, so that a lost arrival ends in an error status instead of
// holding the GPU.  (A bound on the iteration count alone is no bound in
// time: one mbarrier.try_wait may suspend the thread for a while.)
constexpr unsigned long long kWaitNs = 100ull * 1000 * 1000;   // 100 ms
constexpr uint32_t kStatusTimeout = 1u;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Deadline check for spin loops: true once kWaitNs have passed since t0
// (read every 16th iteration).
__device__ __forceinline__ bool wait_expired(uint32_t i, unsigned long long t0) {
  return (i & 15u) == 0 && global_ns() - t0 > kWaitNs;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// Arrive once and add `bytes` to the transaction count of the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity; false if it timed out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  // a short spin first: most waits end in it without reading the clock
  for (uint32_t i = 0; i < 256; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (wait_expired(i, t0)) return false;
  }
}

// Bulk (non-tensor) TMA copy global -> this CTA's shared memory, completing
// `bytes` of transactions on `bar`.  dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// D += A(16x16, f16, row) * B(16x8, f16, col), fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Two e4m3 scale bytes (low 16 bits of v: byte 0, byte 1) -> two f16x2
// words each holding one scale in both halves.
__device__ __forceinline__ void e4m3x2_to_bcast(uint32_t v, uint32_t& s0, uint32_t& s1) {
  uint32_t r;
  asm("{\n\t.reg .b16 a;\n\t"
      "cvt.u16.u32 a, %1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\t}"
      : "=r"(r)
      : "r"(v & 0xffffu));
  s0 = __byte_perm(r, 0, 0x1010);
  s1 = __byte_perm(r, 0, 0x3232);
}

// Power-of-two scale 2^e that maps max|v| into [2^14, 2^15) so that values
// held as f16 keep 11 significant bits down to max * 2^-28 (e = 0 if max is
// 0 or not finite).
__device__ __forceinline__ int f16_prescale_exp(float maxabs) {
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 0;
  int ex;
  frexpf(maxabs, &ex);  // maxabs in [2^(ex-1), 2^ex)
  return 15 - ex;
}

// v (fp32) -> f16 hi + f16 lo with hi + lo = v to ~22 significant bits.
__device__ __forceinline__ void split_f16(float v, __half& hi, __half& lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

}  // namespace qfn

// ---------------------------------------------------------------- tcgen05 (5th-gen tensor cores)
namespace qfn {

// Shared-memory matrix descriptor (UMMA): K-major, 128-byte swizzle, version 1.
//   addr: start address (advanced by 32 B per K=64 fp4 step inside a 128-B row);
//   sbo: byte distance between consecutive 8-row groups.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor of tcgen05.mma.kind::mxf4nvf4.block_scale.block16:
// A, B e2m1 (K-major), ue4m3 block scales, fp32 accumulate, shape M x N.
__host__ __device__ constexpr uint32_t idesc_mxf4nvf4(int M, int N) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (+)= A(smem desc) x B(smem desc) with block scales read from TMEM.
__device__ __forceinline__ void mma_mxf4nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             bool accumulate, uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate)), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Each thread of a warp writes 4 consecutive 32-bit columns of its TMEM lane.
__device__ __forceinline__ void tmem_st_x4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Each thread of a warp reads 8 consecutive 32-bit columns of its TMEM lane.
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 3-D tiled TMA load (box of the tensor map) into shared memory.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// fp32 -> e4m3 byte, round to nearest even, saturating to +-448.
__device__ __forceinline__ uint32_t f32_to_e4m3_rn(float y) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.f), "f"(y));
  return r & 0xffu;
}
// Two fp32 -> one e2m1 byte (lo -> low nibble), round to nearest even, saturating to +-6.
__device__ __forceinline__ uint32_t f32x2_to_e2m1(float lo, float hi) {
  uint16_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}" : "=h"(r) : "f"(hi), "f"(lo));
  return r & 0xffu;
}

}  // namespace qfn

namespace qfn {
// Each thread of a warp writes 32 / 8 consecutive 32-bit columns of its TMEM lane.
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
}  // namespace qfn

namespace qfn {
// Instruction descriptor of tcgen05.mma.kind::f16: A, B f16 (K-major), fp32
// accumulate (bits 4-5 = 1), shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A(smem desc) x B(smem desc), kind::f16.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}

// Each thread of a warp reads 32 consecutive 32-bit columns of its TMEM lane.
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Each thread of a warp reads 16 consecutive 32-bit columns of its TMEM lane (waits for the load).
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2-D tiled TMA load (box of the tensor map) into shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
}  // namespace qfn

namespace qfn {
// 4-D tiled TMA load (box of the tensor map) into shared memory.
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, int x, int y, int z, int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}
}  // namespace qfn

namespace qfn {
// One lane of a converged warp (the same lane every call): the issuer of
// TMA copies, MMAs and commits in warp-wide producer / MMA loops.  Keeping
// the whole warp in the loop keeps descriptors and addresses in uniform
// registers, which issues tcgen05 instructions about twice as fast as a
// loop run by a single lane.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}
}  // namespace qfn

namespace qfn {
// Prefetch `bytes` (a multiple of 16, 16-byte aligned) of global memory into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
}  // namespace qfn

namespace qfn {
// D[tmem] (+)= A(tmem) x B(smem desc), kind::f16.  A occupies M lanes, K/2
// consecutive 32-bit columns (two f16 per column, lower k in the low half).
__device__ __forceinline__ void mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}
// Each thread of a warp writes 16 consecutive 32-bit columns of its TMEM lane.
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
}  // namespace qfn

