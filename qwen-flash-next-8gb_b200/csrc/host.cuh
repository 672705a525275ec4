// Host-side helpers shared by the C-ABI entry points: status/message
// handling, per-device properties, launch checking.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/qfn.h"

namespace qfn {

// Record a message for qfn_last_error() on this host thread; returns status.
int set_error(int status, const char* fmt, ...);

struct DeviceInfo {
  int device;
  int sm_count;
  int cc_major, cc_minor;
  size_t smem_optin;
  int pf_ctas;   // CTAs of the persistent prefill GEMMs (qfn_set_prefill_sm_budget; 0 = one per SM)
};

// Properties of the current device (cached per device).  Returns QFN_OK,
// QFN_ERR_CUDA or QFN_ERR_DEVICE (not compute capability 10.x).
int current_device(DeviceInfo** out);

inline cudaStream_t as_stream(qfn_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Check the launch that was just queued.
int check_launch(const char* what);

// Read (clear != false: and reset) the status words of the GEMV and of the
// FP8 linear layer on the current device (bit 0: a bounded wait ran out).
int gemv_status(unsigned int* v, bool clear);
int linear_status(unsigned int* v, bool clear);

}  // namespace qfn

#define QFN_REQUIRE(cond, status, ...)                 \
  do {                                                 \
    if (!(cond)) return ::qfn::set_error((status), __VA_ARGS__); \
  } while (0)

#include <cuda.h>

namespace qfn {

// 2-D TMA tensor map over `rows` rows of `inner` elements (row stride in
// bytes), box [box_rows][box_inner], cached per (device, all arguments).
int tensor_map_2d(const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle,
                  int device, CUtensorMap* out);

// N-D (rank <= 5) TMA tensor map, cached per (device, arguments).
// dims[0] is the contiguous dimension; strides[i] is the byte stride of
// dimension i + 1.
int tensor_map_nd(const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, int device, CUtensorMap* out,
                  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE,
                  CUtensorMapL2promotion promotion = CU_TENSOR_MAP_L2_PROMOTION_L2_128B);

}  // namespace qfn
