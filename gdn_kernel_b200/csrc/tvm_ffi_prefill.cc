// TVM-FFI export `kernel` for GDN chunked prefill: the drop-in for the
// reference's prefill entry point (ref solution/cuda/kernel_prefill.cu:300-339,
// exported there with TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel, GDNPrefillKernel)).
// Same argument order; cu_seqlens may be int32 or int64 (the reference reads
// int64 only, kernel_prefill.cu:323).
#include "tvm_ffi_common.h"

namespace gdn_tvm {

void GdnPrefill(TensorView q, TensorView k, TensorView v, TensorView state, TensorView A_log,
                TensorView a, TensorView dt_bias, TensorView b, TensorView cu_seqlens,
                double scale, TensorView output, TensorView new_state) {
  require(q.ndim() == 3 && v.ndim() == 3, "q and v must be packed [T, H, D]");
  const DLDevice dev = q.device();
  require(dev.device_type == kDLCUDA, "q must be a CUDA tensor");
  const int64_t T = q.size(0), H_qk = q.size(1), D = q.size(2), H_v = v.size(1);
  require(cu_seqlens.ndim() == 1 && cu_seqlens.size(0) >= 1, "cu_seqlens must be [N + 1]");
  const int64_t N = cu_seqlens.size(0) - 1;
  const bool cu64 = is_dtype(cu_seqlens, kDLInt, 64);
  require(cu64 || is_dtype(cu_seqlens, kDLInt, 32), "cu_seqlens must be int32 or int64");
  check_tensor(cu_seqlens, "cu_seqlens", kDLInt, cu64 ? 64 : 32, {N + 1}, dev);
  check_tensor(q, "q", kDLBfloat, 16, {T, H_qk, D}, dev);
  check_tensor(k, "k", kDLBfloat, 16, {T, H_qk, D}, dev);
  check_tensor(v, "v", kDLBfloat, 16, {T, H_v, D}, dev);
  check_tensor(A_log, "A_log", kDLFloat, 32, {H_v}, dev);
  check_tensor(a, "a", kDLBfloat, 16, {T, H_v}, dev);
  check_tensor(dt_bias, "dt_bias", kDLFloat, 32, {H_v}, dev);
  check_tensor(b, "b", kDLBfloat, 16, {T, H_v}, dev);
  check_tensor(output, "output", kDLBfloat, 16, {T, H_v, D}, dev);
  check_tensor(new_state, "new_state", kDLFloat, 32, {N, H_v, D, D}, dev);
  const float* st = optional_state(state, "state", {N, H_v, D, D}, dev);
  // The reference signature carries no workspace, and gdn_b200_prefill needs
  // none: it works in the library's static record ring (no allocation).
  DeviceGuard guard(dev);
  const int rc = gdn_b200_prefill(ptr(q), ptr(k), ptr(v), st,
                                  static_cast<const float*>(ptr(A_log)), ptr(a),
                                  static_cast<const float*>(ptr(dt_bias)), ptr(b),
                                  ptr(cu_seqlens), cu64 ? 1 : 0, scale, ptr(output),
                                  static_cast<float*>(ptr(new_state)), N, T,
                                  static_cast<int32_t>(H_qk), static_cast<int32_t>(H_v),
                                  static_cast<int32_t>(D), env_stream(dev));
  check_rc(rc);
}

}  // namespace gdn_tvm

TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel, gdn_tvm::GdnPrefill);
