// The thin torch extension over libqfn's C ABI: the parts of the hot path
// as torch operators (torch.ops.qfn.*), so that PyTorch callers reach the
// kernels through one dispatcher call instead of ctypes.  Each operator
// checks its tensors (type errors raise TypeError, shape / device errors
// ValueError, as the Python wrappers did), makes the tensors' device current,
// and calls the C entry point on torch's current stream; a non-zero status
// raises RuntimeError with the library's message.  No computation happens
// here: a missing libqfn.so fails at load time.
//
//   qfn::moe_decode  -> qfn_moe_decode_variant  (qmoe.moe_decode, qmoe.py:77-83)
//   qfn::moe_prefill -> qfn_moe_prefill         (the expert loop of QwenEngine.moe, qwen_engine.py:835-852)
//   qfn::gemv        -> qfn_gemv_e4m3           (fp8gemv.gemv, fp8gemv.py:5-26)
//   qfn::linear      -> qfn_linear_e4m3         (Lin.__call__ for T > 1, qwen_engine.py:79-83)
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "qfn.h"

namespace {

void req_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.is_cuda(), name, " must be a CUDA tensor (libqfn has no CPU path)");
  TORCH_CHECK_VALUE(t.is_contiguous(), name, " must be contiguous");
}

void req_type(const at::Tensor& t, const char* name, at::ScalarType dt) {
  TORCH_CHECK_TYPE(t.scalar_type() == dt, name, " must be ", dt, ", got ", t.scalar_type());
}

void same_device(const at::Tensor& t, const char* name, const at::Tensor& ref, const char* ref_name) {
  TORCH_CHECK_VALUE(t.device() == ref.device(), name, " is on ", t.device(), ", ", ref_name, " on ", ref.device());
}

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == QFN_OK, what, ": ", qfn_strerror(rc), " (", qfn_last_error(), ")");
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

at::Tensor moe_decode(const at::Tensor& slots, const at::Tensor& sidx, const at::Tensor& s2, const at::Tensor& coef,
                      const at::Tensor& x, at::Tensor h_buf, int64_t variant) {
  const std::pair<const at::Tensor*, const char*> all[] = {
      {&slots, "slots_u8"}, {&sidx, "sidx"}, {&s2, "s2"}, {&coef, "coef"}, {&x, "x"}, {&h_buf, "h_buf"}};
  for (const auto& a : all) req_cuda(*a.first, a.second);
  req_type(slots, "slots_u8", at::kByte);
  req_type(sidx, "sidx", at::kInt);
  req_type(s2, "s2", at::kFloat);
  req_type(coef, "coef", at::kFloat);
  req_type(h_buf, "h_buf", at::kFloat);
  const int64_t K = sidx.numel();
  TORCH_CHECK_VALUE(slots.dim() == 2 && slots.size(1) == QFN_BLOCK_BYTES, "slots_u8 must be [S, ", QFN_BLOCK_BYTES,
                    "], got ", slots.sizes());
  TORCH_CHECK_VALUE(sidx.dim() == 1 && K >= 1 && K <= QFN_MAX_TOPK, "sidx must be int32[K] with 1 <= K <= ",
                    QFN_MAX_TOPK);
  TORCH_CHECK_VALUE(s2.dim() == 2 && s2.size(0) == K && s2.size(1) == 3 && coef.dim() == 1 && coef.size(0) == K,
                    "s2 must be [K,3] and coef [K]; got ", s2.sizes(), ", ", coef.sizes());
  TORCH_CHECK_VALUE(x.numel() == QFN_HID && (x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat),
                    "x must be bf16/fp32 with ", QFN_HID, " elements");
  TORCH_CHECK_VALUE(h_buf.dim() == 2 && h_buf.size(0) >= K && h_buf.size(1) == QFN_INTER, "h_buf must be f32[>=K, ",
                    QFN_INTER, "]");
  for (const auto& a : all) same_device(*a.first, a.second, slots, "slots_u8");
  c10::cuda::CUDAGuard guard(slots.device());
  at::Tensor out = at::empty({QFN_HID}, slots.options().dtype(at::kFloat));
  check_rc(qfn_moe_decode_variant(slots.data_ptr<uint8_t>(), slots.size(0), sidx.data_ptr<int32_t>(),
                                  s2.data_ptr<float>(), coef.data_ptr<float>(), x.data_ptr(),
                                  x.scalar_type() == at::kFloat ? QFN_DTYPE_F32 : QFN_DTYPE_BF16,
                                  h_buf.data_ptr<float>(), out.data_ptr<float>(), static_cast<int>(K),
                                  static_cast<int>(variant), stream_of(out)),
           "qfn_moe_decode");
  return out;
}

at::Tensor moe_prefill(const at::Tensor& x, const at::Tensor& ti, const at::Tensor& tv, const at::Tensor& table,
                       const at::Tensor& s2, int64_t L) {
  const std::pair<const at::Tensor*, const char*> all[] = {
      {&x, "x"}, {&ti, "ti"}, {&tv, "tv"}, {&table, "table"}, {&s2, "s2"}};
  for (const auto& a : all) req_cuda(*a.first, a.second);
  req_type(x, "x", at::kBFloat16);
  req_type(table, "table", at::kByte);
  req_type(s2, "s2", at::kFloat);
  TORCH_CHECK_VALUE(x.dim() == 2 && x.size(1) == QFN_HID, "x must be bf16[T, ", QFN_HID, "], got ", x.sizes());
  const int64_t T = x.size(0);
  TORCH_CHECK_VALUE(ti.dim() == 2 && ti.size(0) == T && tv.sizes() == ti.sizes(),
                    "ti and tv must be [T, topk] with T=", T, "; got ", ti.sizes(), ", ", tv.sizes());
  TORCH_CHECK_TYPE(ti.scalar_type() == at::kLong || ti.scalar_type() == at::kInt, "ti must be int64 or int32");
  TORCH_CHECK_TYPE(tv.scalar_type() == at::kBFloat16 || tv.scalar_type() == at::kFloat, "tv must be bf16 or fp32");
  TORCH_CHECK_VALUE(s2.dim() == 2 && s2.size(1) == 3, "s2 must be f32[n_experts, 3], got ", s2.sizes());
  TORCH_CHECK_VALUE(table.dim() == 2 && table.size(1) == QFN_BLOCK_BYTES, "table must be [NB, ", QFN_BLOCK_BYTES,
                    "]");
  for (const auto& a : all) same_device(*a.first, a.second, x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  const int topk = static_cast<int>(ti.size(1));
  const int E = static_cast<int>(s2.size(0));
  at::Tensor out = at::empty({T, QFN_HID}, x.options().dtype(at::kFloat));
  if (T == 0) return out;
  const size_t nbytes = qfn_moe_prefill_workspace(T, topk, E);
  at::Tensor ws = at::empty({static_cast<int64_t>(nbytes)}, x.options().dtype(at::kByte));
  check_rc(qfn_moe_prefill(x.data_ptr(), T, ti.data_ptr(), ti.scalar_type() == at::kLong ? 1 : 0, tv.data_ptr(),
                           tv.scalar_type() == at::kBFloat16 ? QFN_DTYPE_BF16 : QFN_DTYPE_F32, topk,
                           table.data_ptr<uint8_t>(), table.size(0), L * E, s2.data_ptr<float>(), E,
                           out.data_ptr<float>(), ws.data_ptr(), nbytes, stream_of(out)),
           "qfn_moe_prefill");
  return out;
}

at::Tensor gemv(const at::Tensor& q, const at::Tensor& s, const at::Tensor& x, bool out_f32) {
  req_cuda(q, "q");
  TORCH_CHECK_TYPE(q.scalar_type() == at::kFloat8_e4m3fn || q.scalar_type() == at::kByte,
                   "q must be float8_e4m3fn (or its raw uint8 bytes), got ", q.scalar_type());
  req_cuda(s, "s");
  req_type(s, "s", at::kFloat);
  req_cuda(x, "x");
  req_type(x, "x", at::kBFloat16);
  TORCH_CHECK_VALUE(q.dim() == 2, "q must be [N, K]");
  const int64_t N = q.size(0), K = q.size(1);
  TORCH_CHECK_VALUE(s.numel() == N && x.numel() == K, "s must have ", N, " and x ", K, " elements; got ", s.numel(),
                    ", ", x.numel());
  same_device(s, "s", q, "q");
  same_device(x, "x", q, "q");
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor y = at::empty({N}, q.options().dtype(out_f32 ? at::kFloat : at::kBFloat16));
  check_rc(qfn_gemv_e4m3(static_cast<const uint8_t*>(q.data_ptr()), s.data_ptr<float>(),
                         static_cast<const uint16_t*>(x.data_ptr()), y.data_ptr(),
                         out_f32 ? QFN_DTYPE_F32 : QFN_DTYPE_BF16, N, K, stream_of(y)),
           "qfn_gemv_e4m3");
  return y;
}

// Lin.__call__ for T > 1 (qwen_engine.py:79-83): x [T, K] bf16 -> [T, N] bf16.
at::Tensor linear(const at::Tensor& x, const at::Tensor& q, const at::Tensor& s) {
  req_cuda(q, "q");
  TORCH_CHECK_TYPE(q.scalar_type() == at::kFloat8_e4m3fn || q.scalar_type() == at::kByte,
                   "q must be float8_e4m3fn (or its raw uint8 bytes), got ", q.scalar_type());
  req_cuda(s, "s");
  req_type(s, "s", at::kFloat);
  req_cuda(x, "x");
  req_type(x, "x", at::kBFloat16);
  TORCH_CHECK_VALUE(q.dim() == 2 && x.dim() == 2, "q must be [N, K] and x [T, K]");
  const int64_t N = q.size(0), K = q.size(1), T = x.size(0);
  TORCH_CHECK_VALUE(x.size(1) == K && s.numel() == N, "x must be [T, ", K, "] and s have ", N, " elements; got ",
                    x.sizes(), ", ", s.numel());
  same_device(s, "s", q, "q");
  same_device(x, "x", q, "q");
  c10::cuda::CUDAGuard guard(q.device());
  // the kernel's TMA reads x from a 16-byte aligned base (a view may start anywhere)
  const at::Tensor xa = reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 ? x.clone() : x;
  at::Tensor y = at::empty({T, N}, x.options());
  if (T == 0 || N == 0) return y;
  check_rc(qfn_linear_e4m3(static_cast<const uint8_t*>(q.data_ptr()), s.data_ptr<float>(),
                           static_cast<const uint16_t*>(xa.data_ptr()), static_cast<uint16_t*>(y.data_ptr()), T, N, K,
                           stream_of(y)),
           "qfn_linear_e4m3");
  return y;
}

}  // namespace

// Catch-all kernels (not per dispatch key): a CPU tensor reaches the checks
// above and raises ValueError rather than a missing-kernel error.
TORCH_LIBRARY(qfn, m) {
  m.def("moe_decode(Tensor slots, Tensor sidx, Tensor s2, Tensor coef, Tensor x, Tensor(a!) h_buf, int variant) -> Tensor",
        &moe_decode);
  m.def("moe_prefill(Tensor x, Tensor ti, Tensor tv, Tensor table, Tensor s2, int L) -> Tensor", &moe_prefill);
  m.def("gemv(Tensor q, Tensor s, Tensor x, bool out_f32) -> Tensor", &gemv);
  m.def("linear(Tensor x, Tensor q, Tensor s) -> Tensor", &linear);
}
