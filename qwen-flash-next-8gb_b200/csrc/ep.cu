// Expert-parallel MoE layer (batched prefill / batched decode) over an NCCL
// communicator, for callers of the C ABI that run their own NCCL (no torch):
// the all-gather exchange of ep.moe_prefill_ep_ag in one call.
//
//   every rank: its T tokens (x bf16 [T][2560], top-k ids and weights)
//   1. all-gather x and the routing (ids as int32, weights as fp32) over the
//      communicator: every rank sees all W x T tokens;
//   2. map the ids through this rank's `local_of` (expert -> index in this
//      rank's expert table, -1 for experts other ranks own);
//   3. the grouped GEMM of qfn_moe_prefill over all W x T tokens and this
//      rank's experts: fp32 partial sums [W x T][2560] (zero rows for tokens
//      with no expert here);
//   4. reduce-scatter (sum) of the partial sums: rank r keeps rows
//      [r T, (r + 1) T), its own tokens' MoE output.
//
// Every step is queued on the caller's stream (NCCL collectives included);
// nothing synchronises the host.  libnccl is resolved at run time (dlopen of
// libnccl.so.2, reusing the copy the process has already loaded), so the
// library has no link-time dependency on NCCL; the communicator is passed as
// an opaque pointer (ncclComm_t).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "host.cuh"

namespace qfn {

struct NcclApi {
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  const char* (*error_string)(ncclResult_t);
  ncclResult_t (*comm_count)(const ncclComm_t, int*);
  ncclResult_t (*comm_user_rank)(const ncclComm_t, int*);
  ncclResult_t (*comm_cu_device)(const ncclComm_t, int*);
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
};

static NcclApi g_nccl;
static std::mutex g_nccl_mu;
static int g_nccl_state = 0;  // 0: not resolved yet, 1: resolved, -1: unavailable

static int nccl_api(NcclApi** api) {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl_state == 0) {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's own copy, if loaded
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    g_nccl_state = -1;
    if (h) {
      bool ok = true;
      auto sym = [&](const char* name) {
        void* p = dlsym(h, name);
        ok = ok && p != nullptr;
        return p;
      };
      g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(sym("ncclAllGather"));
      g_nccl.reduce_scatter = reinterpret_cast<decltype(g_nccl.reduce_scatter)>(sym("ncclReduceScatter"));
      g_nccl.group_start = reinterpret_cast<decltype(g_nccl.group_start)>(sym("ncclGroupStart"));
      g_nccl.group_end = reinterpret_cast<decltype(g_nccl.group_end)>(sym("ncclGroupEnd"));
      g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(sym("ncclGetErrorString"));
      g_nccl.comm_count = reinterpret_cast<decltype(g_nccl.comm_count)>(sym("ncclCommCount"));
      g_nccl.comm_user_rank = reinterpret_cast<decltype(g_nccl.comm_user_rank)>(sym("ncclCommUserRank"));
      g_nccl.comm_cu_device = reinterpret_cast<decltype(g_nccl.comm_cu_device)>(sym("ncclCommCuDevice"));
      g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(sym("ncclGetUniqueId"));
      g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(sym("ncclCommInitRank"));
      g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(sym("ncclCommDestroy"));
      if (ok) g_nccl_state = 1;
    }
  }
  if (g_nccl_state != 1) return set_error(QFN_ERR_CUDA, "libnccl.so.2 not found or incomplete");
  *api = &g_nccl;
  return QFN_OK;
}

static int nccl_check(NcclApi* api, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return QFN_OK;
  return set_error(QFN_ERR_CUDA, "%s: %s", what, api->error_string(r));
}

// meta[t] = [ids (int32) x K | weights (fp32 bits) x K] of this rank's tokens
template <typename TI>
__global__ void ep_pack_meta_kernel(const TI* __restrict__ ti, const void* __restrict__ tv, bool tv_bf16, int64_t T,
                                    int K, int32_t* __restrict__ meta) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < T * K;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / K, k = i - t * K;
    const float w = tv_bf16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(tv)[i]) : static_cast<const float*>(tv)[i];
    meta[t * 2 * K + k] = static_cast<int32_t>(ti[i]);
    meta[t * 2 * K + K + k] = __float_as_int(w);
  }
}

// all ranks' meta -> this rank's local expert index (-1: another rank's) and the weights
__global__ void ep_local_ids_kernel(const int32_t* __restrict__ meta_all, int64_t rows, int K,
                                    const int32_t* __restrict__ local_of, int n_experts, int32_t* __restrict__ ti_loc,
                                    float* __restrict__ tv_all) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows * K;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / K, k = i - r * K;
    const int32_t e = meta_all[r * 2 * K + k];
    ti_loc[i] = e >= 0 && e < n_experts ? local_of[e] : -1;
    tv_all[i] = __int_as_float(meta_all[r * 2 * K + K + k]);
  }
}

// byte offsets of the call's workspace (each part 256-byte aligned)
struct EpWs {
  size_t meta, x_all, meta_all, ti_loc, tv_all, out_all, pf, total;
};

static size_t ep_up(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static EpWs ep_ws_map(int64_t T, int K, int n_local, int world) {
  EpWs W;
  const size_t rows = static_cast<size_t>(world) * T;
  W.meta = 0;
  W.x_all = ep_up(W.meta + static_cast<size_t>(T) * 2 * K * 4);
  W.meta_all = ep_up(W.x_all + rows * kHid * 2);
  W.ti_loc = ep_up(W.meta_all + rows * 2 * K * 4);
  W.tv_all = ep_up(W.ti_loc + rows * K * 4);
  W.out_all = ep_up(W.tv_all + rows * K * 4);
  W.pf = ep_up(W.out_all + rows * kHid * 4);
  W.total = W.pf + qfn_moe_prefill_workspace(static_cast<int64_t>(rows), K, n_local);
  return W;
}

}  // namespace qfn

using namespace qfn;

extern "C" size_t qfn_moe_prefill_ep_workspace(int64_t T, int topk, int n_local, int world) {
  if (T <= 0 || topk <= 0 || n_local <= 0 || world <= 0) return 0;
  return ep_ws_map(T, topk, n_local, world).total;
}

extern "C" int qfn_moe_prefill_ep(const void* x, int64_t T, const void* ti, int ti_is_int64, const void* tv,
                                  int tv_dtype, int topk, const uint8_t* table, int64_t n_blocks, int64_t base,
                                  const float* s2l, int n_local, const int32_t* local_of, int n_experts, void* comm,
                                  float* out, void* workspace, size_t workspace_bytes, qfn_stream_t stream) {
  QFN_REQUIRE(x && ti && tv && table && s2l && local_of && comm && out && workspace, QFN_ERR_INVALID_ARG,
              "qfn_moe_prefill_ep: null pointer");
  QFN_REQUIRE(T >= 1 && topk >= 1 && topk <= QFN_MAX_TOPK, QFN_ERR_INVALID_ARG, "qfn_moe_prefill_ep: T=%lld topk=%d",
              (long long)T, topk);
  QFN_REQUIRE(n_local >= 1 && n_experts >= 1, QFN_ERR_INVALID_ARG, "qfn_moe_prefill_ep: n_local=%d n_experts=%d",
              n_local, n_experts);
  QFN_REQUIRE(tv_dtype == QFN_DTYPE_F32 || tv_dtype == QFN_DTYPE_BF16, QFN_ERR_INVALID_ARG,
              "qfn_moe_prefill_ep: bad tv dtype %d", tv_dtype);
  QFN_REQUIRE(aligned(x, 16) && aligned(out, 16) && aligned(workspace, 256), QFN_ERR_ALIGNMENT,
              "qfn_moe_prefill_ep: x, out must be 16-byte and workspace 256-byte aligned");
  NcclApi* api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  int world = 0, rank = 0;
  if ((rc = nccl_check(api, api->comm_count(c, &world), "ncclCommCount"))) return rc;
  if ((rc = nccl_check(api, api->comm_user_rank(c, &rank), "ncclCommUserRank"))) return rc;
  const EpWs W = ep_ws_map(T, topk, n_local, world);
  QFN_REQUIRE(workspace_bytes >= W.total, QFN_ERR_WORKSPACE, "qfn_moe_prefill_ep: workspace %zu < %zu bytes",
              workspace_bytes, W.total);
  cudaStream_t st = as_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* meta = reinterpret_cast<int32_t*>(ws + W.meta);
  uint16_t* x_all = reinterpret_cast<uint16_t*>(ws + W.x_all);
  int32_t* meta_all = reinterpret_cast<int32_t*>(ws + W.meta_all);
  int32_t* ti_loc = reinterpret_cast<int32_t*>(ws + W.ti_loc);
  float* tv_all = reinterpret_cast<float*>(ws + W.tv_all);
  float* out_all = reinterpret_cast<float*>(ws + W.out_all);
  const int64_t rows = static_cast<int64_t>(world) * T;
  const unsigned grid = static_cast<unsigned>((T * topk + 255) / 256 < 1184 ? (T * topk + 255) / 256 : 1184);
  const bool bf = tv_dtype == QFN_DTYPE_BF16;
  if (ti_is_int64)
    ep_pack_meta_kernel<int64_t><<<grid, 256, 0, st>>>(static_cast<const int64_t*>(ti), tv, bf, T, topk, meta);
  else
    ep_pack_meta_kernel<int32_t><<<grid, 256, 0, st>>>(static_cast<const int32_t*>(ti), tv, bf, T, topk, meta);
  if ((rc = check_launch("ep_pack_meta"))) return rc;
  // 1. all-gather x and the routing
  if ((rc = nccl_check(api, api->group_start(), "ncclGroupStart"))) return rc;
  ncclResult_t r1 = api->all_gather(x, x_all, static_cast<size_t>(T) * kHid, ncclBfloat16, c, st);
  ncclResult_t r2 = api->all_gather(meta, meta_all, static_cast<size_t>(T) * 2 * topk, ncclInt32, c, st);
  ncclResult_t r3 = api->group_end();
  if ((rc = nccl_check(api, r1, "ncclAllGather (x)")) || (rc = nccl_check(api, r2, "ncclAllGather (routing)")) ||
      (rc = nccl_check(api, r3, "ncclGroupEnd")))
    return rc;
  // 2. this rank's expert indices
  const unsigned grid2 = static_cast<unsigned>((rows * topk + 255) / 256 < 1184 ? (rows * topk + 255) / 256 : 1184);
  ep_local_ids_kernel<<<grid2, 256, 0, st>>>(meta_all, rows, topk, local_of, n_experts, ti_loc, tv_all);
  if ((rc = check_launch("ep_local_ids"))) return rc;
  // 3. the grouped GEMM over all ranks' tokens and this rank's experts
  if ((rc = qfn_moe_prefill(x_all, rows, ti_loc, 0, tv_all, QFN_DTYPE_F32, topk, table, n_blocks, base, s2l, n_local,
                            out_all, ws + W.pf, W.total - W.pf, stream)))
    return rc;
  // 4. reduce-scatter: this rank's tokens' sums
  return nccl_check(api, api->reduce_scatter(out_all, out, static_cast<size_t>(T) * kHid, ncclFloat32, ncclSum, c, st),
                    "ncclReduceScatter");
}

// NCCL bootstrap for callers without one of their own (and the tests): the
// 128-byte unique id (rank 0 creates it, every rank receives it by its own
// means), a communicator per rank on the current device, and its release.
extern "C" int qfn_nccl_unique_id(void* id_out) {
  QFN_REQUIRE(id_out, QFN_ERR_INVALID_ARG, "qfn_nccl_unique_id: null pointer");
  NcclApi* api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  ncclUniqueId id;
  if ((rc = nccl_check(api, api->get_unique_id(&id), "ncclGetUniqueId"))) return rc;
  memcpy(id_out, &id, sizeof(id));
  return QFN_OK;
}

extern "C" int qfn_nccl_comm_init(void** comm_out, int world, int rank, const void* id) {
  QFN_REQUIRE(comm_out && id, QFN_ERR_INVALID_ARG, "qfn_nccl_comm_init: null pointer");
  QFN_REQUIRE(world >= 1 && rank >= 0 && rank < world, QFN_ERR_INVALID_ARG, "qfn_nccl_comm_init: rank %d of %d",
              rank, world);
  NcclApi* api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  if ((rc = nccl_check(api, api->comm_init_rank(&c, world, uid, rank), "ncclCommInitRank"))) return rc;
  *comm_out = c;
  return QFN_OK;
}

extern "C" int qfn_nccl_comm_destroy(void* comm) {
  QFN_REQUIRE(comm, QFN_ERR_INVALID_ARG, "qfn_nccl_comm_destroy: null pointer");
  NcclApi* api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  return nccl_check(api, api->comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}
