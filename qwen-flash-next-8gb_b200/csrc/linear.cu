// FP8 linear layer for T > 1 tokens (Lin.__call__, qwen_engine.py:79-83):
//
//   y[T][N] = bf16( x[T][K] . W^T ),   W[n][k] = bf16(fp32(q[n][k]) * s[n])
//
// the reference's F.linear(x, (q.to(bf16) * s).to(bf16)) with fp32
// accumulation, as one persistent, warp-specialised tcgen05 GEMM.  The bf16
// weights never reach HBM: every job converts its 128 weight rows K-block by
// K-block from the e4m3 bytes straight into TMEM, where they are the A
// operand of tcgen05.mma kind::f16 (bf16 x bf16 -> fp32).
//
// Job = (128 weight rows, tn tokens: 256, or fewer when that fills the SMs'
// rounds better; 160 for the 2560 x 4096 shape at 2,048 tokens, 54.7 -> 52.4
// us), dealt to the CTAs (one per SM, 480
// threads) in the order row tile fastest, so that the CTAs running at one
// time share the token tiles and walk the whole weight matrix through L2:
//   warp 0       x producer: TMA boxes [tn tokens][64 k] (bf16, 128-byte
//                swizzle) into a ring of kLnStages shared-memory stages;
//   warp 1       MMA issuer: per K-block 4 k-steps of one M = 128, N = tn
//                MMA (A from TMEM, B from shared memory).  The first kLnPre
//                K-blocks of a job go into accumulator half 0 alone (N = tn / 2)
//                and then into half 1, so that the epilogue's reading of the
//                previous job's half 1 overlaps them;
//   warp 2       weight producer: TMA boxes [128 rows][64 B] of the e4m3
//                bytes (64-byte swizzle) into a ring of kLnRawStages stages;
//   warps 3-10   converters, two groups of four warps taking alternate
//                K-blocks: thread = weight row; its 64 bytes of the K-block
//                (four conflict-free 16-byte shared-memory reads) become
//                bf16(fp32(q) * s) with the reference's two roundings and go
//                into one of kLnASlots TMEM A slots; a warp waits for a
//                K-block's TMEM store only after converting its next one;
//   warps 11-14  epilogue: TMEM -> RN bf16 -> y, each accumulator half
//                released as soon as it has been read.
// TMEM: columns [0, tn) the accumulator (the tile's first and second tn / 2
// tokens as halves), [256, 512) eight A slots of 32 columns (one K-block of 64
// bf16 each).
//
// Measured on B200 (T = 2048, the 12288 x 2560 and 2560 x 4096 shapes):
//   - A in TMEM: from shared memory the A tiles would add 32 KB of shared
//     traffic per K-block (written by the converters, read by the MMAs) to
//     the x tile's 64 KB, in the 512 cycles the K-block's MMAs take;
//   - one N = 256 MMA per k-step instead of an N = 128 MMA per half: the A
//     tile is read from TMEM once, 190 -> 168 us for the two shapes;
//   - raw bytes by TMA: loaded by the converter threads (a row per lane)
//     every warp load touched 32 L1 lines and the converters stalled on them
//     (320 -> 199 us);
//   - tiles of 192 tokens with two accumulator buffers (no wait for the
//     epilogue) measured slower for the large shape: 1,056 jobs take 8
//     rounds of the 148 SMs and the conversion per FLOP grows by a third.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <utility>

#include "common.cuh"
#include "host.cuh"

namespace qfn {

constexpr int kLnRows = 128;                          // weight rows per job (MMA M)
constexpr int kLnTok = 256;                           // most tokens per job (two accumulator halves)
constexpr int kLnKB = 64;                             // k per K-block
constexpr int kLnStages = 6;                          // x ring stages
constexpr int kLnRawStages = 4;                       // raw weight ring stages
constexpr int kLnASlots = 8;                          // A slots in TMEM
constexpr int kLnPre = 4;                             // K-blocks of a job issued into half 0 before half 1
constexpr int kLnGroups = 2;                          // converter groups of four warps
constexpr int kLnConv0 = 3;                           // first converter warp
constexpr int kLnEpi0 = kLnConv0 + 4 * kLnGroups;     // first epilogue warp
constexpr int kLnThreads = 32 * (kLnEpi0 + 4);        // 480
constexpr uint32_t kLnXBytes = kLnTok * kLnKB * 2;    // x tile per stage (32 KB)
constexpr uint32_t kLnRawBytes = kLnRows * kLnKB;     // raw rows per stage (8 KB)
constexpr uint32_t kLnTmemA = 256;                    // first A-slot column
constexpr int kLnRaw = kLnStages * static_cast<int>(kLnXBytes);
constexpr int kLnBar = kLnRaw + kLnRawStages * static_cast<int>(kLnRawBytes);
constexpr int kLnSmem = kLnBar + 512 + 1024;          // + barriers + alignment slack

__device__ unsigned int g_linear_status = 0;

// Bounded wait; after the first time-out of a CTA (`abort`) every later wait
// returns at once, so a broken pipeline drains in one time-out.
__device__ __forceinline__ bool ln_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*abort) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort = 1u;
  atomicOr(&g_linear_status, kStatusTimeout);
  return false;
}

__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return idesc_f16(M, N) | (1u << 7) | (1u << 10);   // A and B bf16
}

struct LnArgs {
  const uint8_t* q;   // [N][K] e4m3
  const float* s;     // [N]
  uint16_t* y;        // [T][N] bf16
  int T, N, K;
  int KB;             // K-blocks per job
  int MT;             // row tiles
  int tn, hn;         // tokens per job (a multiple of 32, <= 256) and per accumulator half (tn / 2)
  int n_jobs;
};

// 16 e4m3 weights of one row -> 8 words of bf16 pairs (lower k in the low
// half): fp32(q) exact, one fp32 multiply by the row scale, RN to bf16.
__device__ __forceinline__ void ln_convert16(uint4 v, float sc, uint32_t* o) {
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
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
}

__global__ void __launch_bounds__(kLnThreads, 1)
    ln_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap qmap, const LnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* ld_full = reinterpret_cast<uint64_t*>(smem + kLnBar);  // x tile landed (tx)
  uint64_t* ld_empty = ld_full + kLnStages;                         // MMA commit
  uint64_t* a_full = ld_empty + kLnStages;                          // a converter group
  uint64_t* a_empty = a_full + kLnASlots;                           // MMA commit
  uint64_t* acc_full = a_empty + kLnASlots;                         // [2] MMA commit
  uint64_t* acc_empty = acc_full + 2;                               // [2] 4 epilogue warps
  uint64_t* raw_full = acc_empty + 2;                               // raw rows landed (tx)
  uint64_t* raw_empty = raw_full + kLnRawStages;                    // a converter group
  uint32_t* tslot = reinterpret_cast<uint32_t*>(raw_empty + kLnRawStages);
  volatile uint32_t* abort = tslot + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort = 0u;
    for (int s = 0; s < kLnStages; ++s) {
      mbar_init(&ld_full[s], 1);
      mbar_init(&ld_empty[s], 1);
    }
    for (int j = 0; j < kLnASlots; ++j) {
      mbar_init(&a_full[j], 4);
      mbar_init(&a_empty[j], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&acc_full[h], 1);
      mbar_init(&acc_empty[h], 4);
    }
    for (int s = 0; s < kLnRawStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tslot, 512);
  if (threadIdx.x == 32) {
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&qmap);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_wait();   // x comes from the previous kernel in the stream
  pdl_launch_dependents();

  const int grid = static_cast<int>(gridDim.x);
  // the i-th job of this CTA (-1: none left): row tile fastest
  auto job = [&](int i) -> int {
    const int u = static_cast<int>(blockIdx.x) + i * grid;
    return u < a.n_jobs ? u : -1;
  };
  // a time-out seen by any lane of the warp (warp-uniform, for loop exits)
  auto aborted = [&]() -> bool { return __any_sync(0xffffffffu, *abort != 0u); };
  // accumulator halves a job uses (1 when its token tile holds <= 128 tokens)
  auto halves = [&](int u) -> int { return a.T - (u / a.MT) * a.tn > a.hn ? 2 : 1; };

  if (warp == 0) {
    // ---------------- x producer
    int gkb = 0;
    for (int i = 0;; ++i) {
      const int u = job(i);
      if (u < 0 || aborted()) break;
      const int t0 = (u / a.MT) * a.tn;
      for (int kb = 0; kb < a.KB; ++kb, ++gkb) {
        const int s = gkb % kLnStages;
        ln_wait(&ld_empty[s], ((gkb / kLnStages) & 1) ^ 1, abort);
        if (elect_one()) {
          mbar_arrive_expect_tx(&ld_full[s], static_cast<uint32_t>(a.tn) * kLnKB * 2);
          tma_load_2d(smem + s * kLnXBytes, &xmap, kLnKB * kb, t0, &ld_full[s]);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    const uint32_t idesc = idesc_bf16(kLnRows, a.hn);        // one half
    const uint32_t idesc2 = idesc_bf16(kLnRows, 2 * a.hn);   // both halves (the tile)
    const uint32_t hcol = static_cast<uint32_t>(a.hn);           // half 1's first accumulator column
    const uint32_t hrow = static_cast<uint32_t>(a.hn) * 8u;      // its first x row in the stage, in 16-byte units
    const uint64_t bdesc0 = umma_desc_sw128(smem_u32(smem), 1024);
    uint32_t used[2] = {0u, 0u};
    int gkb = 0;
    for (int i = 0;; ++i) {
      const int u = job(i);
      if (u < 0 || aborted()) break;
      const int nh = halves(u);
      // the first kLnPre K-blocks into half 0 alone (N = 128), then into half 1
      // once the epilogue has read it; then both halves in one N = 256 MMA
      const int pre = nh == 2 ? min(kLnPre, a.KB) : 0;
      ln_wait(&acc_empty[0], (used[0] & 1) ^ 1, abort);
      tc_fence_after();
      for (int kb = 0; kb < pre; ++kb) {
        const int g2 = gkb + kb, s = g2 % kLnStages, j = g2 % kLnASlots;
        ln_wait(&ld_full[s], (g2 / kLnStages) & 1, abort);
        ln_wait(&a_full[j], (g2 / kLnASlots) & 1, abort);
        tc_fence_after();
        if (elect_one()) {
          const uint32_t aslot = tmem + kLnTmemA + 32u * j;
          const uint64_t bd = bdesc0 + ((s * kLnXBytes) >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_f16_ta(tmem, aslot + 8 * k, bd + 2u * k, idesc, (kb | k) != 0);
        }
        __syncwarp();
      }
      if (nh == 2) ln_wait(&acc_empty[1], (used[1] & 1) ^ 1, abort);
      tc_fence_after();
      for (int kb = 0; kb < pre; ++kb, ++gkb) {
        const int s = gkb % kLnStages, j = gkb % kLnASlots;
        if (elect_one()) {
          const uint32_t aslot = tmem + kLnTmemA + 32u * j;
          const uint64_t bd = bdesc0 + ((s * kLnXBytes) >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_f16_ta(tmem + hcol, aslot + 8 * k, bd + (hrow + 2u * k), idesc, (kb | k) != 0);
          mma_commit(&a_empty[j]);
          mma_commit(&ld_empty[s]);
        }
        __syncwarp();
      }
      for (int kb = pre; kb < a.KB; ++kb, ++gkb) {
        const int s = gkb % kLnStages, j = gkb % kLnASlots;
        ln_wait(&ld_full[s], (gkb / kLnStages) & 1, abort);
        ln_wait(&a_full[j], (gkb / kLnASlots) & 1, abort);
        tc_fence_after();
        if (elect_one()) {
          const uint32_t aslot = tmem + kLnTmemA + 32u * j;
          const uint64_t bd = bdesc0 + ((s * kLnXBytes) >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_f16_ta(tmem, aslot + 8 * k, bd + 2u * k, nh == 2 ? idesc2 : idesc, (kb | k) != 0);
          mma_commit(&a_empty[j]);
          mma_commit(&ld_empty[s]);
        }
        __syncwarp();
      }
      if (elect_one()) {
        for (int h = 0; h < nh; ++h) mma_commit(&acc_full[h]);
      }
      __syncwarp();
      for (int h = 0; h < nh; ++h) ++used[h];
    }
  } else if (warp == 2) {
    // ---------------- weight producer: the job's 128 rows of each K-block
    int gkb = 0;
    for (int i = 0;; ++i) {
      const int u = job(i);
      if (u < 0 || aborted()) break;
      const int m0 = (u % a.MT) * kLnRows;
      for (int kb = 0; kb < a.KB; ++kb, ++gkb) {
        const int s = gkb % kLnRawStages;
        ln_wait(&raw_empty[s], ((gkb / kLnRawStages) & 1) ^ 1, abort);
        if (elect_one()) {
          mbar_arrive_expect_tx(&raw_full[s], kLnRawBytes);
          tma_load_2d(smem + kLnRaw + s * kLnRawBytes, &qmap, kLnKB * kb, m0, &raw_full[s]);
        }
        __syncwarp();
      }
    }
  } else if (warp < kLnEpi0) {
    // ---------------- converters: group g takes the CTA's K-blocks g, g + 2, ...
    const int w = warp - kLnConv0;
    const int g = w >> 2;
    const int quarter = warp & 3;                 // TMEM lanes this warp may write
    const int r = 32 * quarter + lane;            // weight row within the job
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    // the CTA's K-blocks in order: job i, K-block kb = gkb - i * KB
    int n_mine = 0;
    while (job(n_mine) >= 0) ++n_mine;
    const int total = n_mine * a.KB;
    // this thread's raw row in a stage: 64-byte rows, 64-byte swizzle
    const int raw_row = r * 64, swz = (r >> 1) & 3;
    int row_job = -1;
    float sc = 0.0f;
    int pend = -1;   // K-block whose TMEM store is in flight
    auto signal = [&](int gk) {   // that store has landed: its A slot is full (one arrival per warp)
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[gk % kLnASlots]);
    };
    for (int gkb = g; gkb < total; gkb += kLnGroups) {
      const int i = gkb / a.KB;
      if (i != row_job) {   // the row scale of this job
        row_job = i;
        const int n = (job(i) % a.MT) * kLnRows + r;
        sc = n < a.N ? a.s[n] : 0.0f;
      }
      const int sr = gkb % kLnRawStages;
      ln_wait(&raw_full[sr], (gkb / kLnRawStages) & 1, abort);
      const uint8_t* raw = smem + kLnRaw + sr * kLnRawBytes + raw_row;
      uint4 rw[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) rw[c] = *reinterpret_cast<const uint4*>(raw + ((c ^ swz) << 4));
      uint32_t v[32];
#pragma unroll
      for (int c = 0; c < 4; ++c) ln_convert16(rw[c], sc, v + 8 * c);
      __syncwarp();
      if (lane == 0) mbar_arrive(&raw_empty[sr]);
      if (pend >= 0) signal(pend);
      const int j = gkb % kLnASlots;
      ln_wait(&a_empty[j], ((gkb / kLnASlots) & 1) ^ 1, abort);
      tc_fence_after();
      tmem_st_x32(tmem + kLnTmemA + 32u * j + lane_base, v);
      pend = gkb;
    }
    if (pend >= 0) signal(pend);
  } else {
    // ---------------- epilogue: warp reads TMEM lanes 32 (warp % 4) ..
    const int quarter = warp & 3;
    uint32_t used[2] = {0u, 0u};
    for (int i = 0;; ++i) {
      const int u = job(i);
      if (u < 0 || aborted()) break;
      const int nh = halves(u);
      const int n = (u % a.MT) * kLnRows + 32 * quarter + lane;
      const int t0 = (u / a.MT) * a.tn;
      for (int h = 0; h < nh; ++h) {
        ln_wait(&acc_full[h], used[h] & 1, abort);
        tc_fence_after();
        const int cols = min(a.hn, a.T - t0 - a.hn * h);
        uint16_t* yc = a.y + static_cast<int64_t>(t0 + a.hn * h) * a.N + n;
        for (int c0 = 0; c0 < cols; c0 += 16) {
          uint32_t v[16];
          tmem_ld_x16(tmem + (static_cast<uint32_t>(32 * quarter) << 16) + a.hn * h + c0, v);
          if (n < a.N) {
            const int lim = cols - c0;
            uint16_t* p = yc + static_cast<int64_t>(c0) * a.N;
#pragma unroll
            for (int c = 0; c < 16; ++c, p += a.N) {
              if (c < lim) *p = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[c])));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[h]);
        ++used[h];
      }
    }
  }
  __syncwarp();   // the role loops end with diverged lanes (elected issuers): reconverge before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// Read (and optionally clear) this file's status word; used by qfn_device_status.
int linear_status(unsigned int* v, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(v, g_linear_status, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_linear_status, &zero, sizeof(unsigned int));
  }
  return e == cudaSuccess ? QFN_OK : set_error(QFN_ERR_CUDA, "linear status: %s", cudaGetErrorString(e));
}

}  // namespace qfn

using namespace qfn;

extern "C" int qfn_linear_e4m3(const uint8_t* q, const float* s, const uint16_t* x, uint16_t* y, int64_t T,
                               int64_t N, int64_t K, qfn_stream_t stream) {
  QFN_REQUIRE(q && s && x && y, QFN_ERR_INVALID_ARG, "qfn_linear_e4m3: null pointer");
  QFN_REQUIRE(T > 0 && N > 0 && K > 0, QFN_ERR_INVALID_ARG, "qfn_linear_e4m3: T=%lld N=%lld K=%lld must be positive",
              (long long)T, (long long)N, (long long)K);
  QFN_REQUIRE(K % 16 == 0, QFN_ERR_UNSUPPORTED, "qfn_linear_e4m3: K=%lld must be a multiple of 16", (long long)K);
  QFN_REQUIRE(T < (int64_t(1) << 30) && N < (int64_t(1) << 30) && K < (int64_t(1) << 30), QFN_ERR_UNSUPPORTED,
              "qfn_linear_e4m3: sizes must be below 2^30");
  QFN_REQUIRE(aligned(q, 16) && aligned(x, 16) && aligned(y, 2), QFN_ERR_ALIGNMENT,
              "qfn_linear_e4m3: q and x must be 16-byte and y 2-byte aligned");
  DeviceInfo* dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  CUtensorMap xmap;
  // tokens per job: the tile (256 down to 128, a multiple of 32) whose jobs fill the
  // SMs' rounds best, each job also paying a fixed cost of about 32 tokens'
  // worth of MMAs (pipeline fill, epilogue)
  const int64_t MT = (N + kLnRows - 1) / kLnRows;
  int tn = kLnTok;
  int64_t best = -1;
  for (int c = kLnTok; c >= 128; c -= 32) {
    const int64_t rounds = (MT * ((T + c - 1) / c) + dev->sm_count - 1) / dev->sm_count;
    if (best < 0 || rounds * (c + 32) < best) {
      best = rounds * (c + 32);
      tn = c;
    }
  }
  if ((rc = tensor_map_2d(x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, T, K * 2, kLnKB, static_cast<uint32_t>(tn),
                          CU_TENSOR_MAP_SWIZZLE_128B, dev->device, &xmap)))
    return rc;
  CUtensorMap qmap;
  if ((rc = tensor_map_2d(q, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, K, kLnKB, kLnRows, CU_TENSOR_MAP_SWIZZLE_64B,
                          dev->device, &qmap)))
    return rc;
  static bool attr_set[64] = {};
  if (!attr_set[dev->device]) {
    cudaError_t e = cudaFuncSetAttribute(ln_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kLnSmem);
    if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "linear smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev->device] = true;
  }
  LnArgs a;
  a.q = q;
  a.s = s;
  a.y = y;
  a.T = static_cast<int>(T);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.KB = static_cast<int>((K + kLnKB - 1) / kLnKB);
  a.MT = static_cast<int>((N + kLnRows - 1) / kLnRows);
  a.tn = tn;
  a.hn = tn / 2;
  const int64_t jobs = MT * ((T + tn - 1) / tn);
  QFN_REQUIRE(jobs < (int64_t(1) << 30), QFN_ERR_UNSUPPORTED, "qfn_linear_e4m3: too many tiles");
  a.n_jobs = static_cast<int>(jobs);
  const unsigned grid = static_cast<unsigned>(jobs < dev->sm_count ? jobs : dev->sm_count);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kLnThreads);
  cfg.dynamicSmemBytes = kLnSmem;
  cfg.stream = as_stream(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, ln_gemm_kernel, xmap, qmap, a);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "ln_gemm launch: %s", cudaGetErrorString(e));
  return check_launch("ln_gemm_kernel");
}
