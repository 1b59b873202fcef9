// TVM-FFI export `kernel` for GDN decode: the drop-in for the reference's
// decode entry point (ref solution/cuda/kernel.cu:101-150, exported there with
// TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel, GDNDecodeKernel)).  Same argument order,
// destination-passing style, stream taken from TVMFFIEnvGetStream.
#include "tvm_ffi_common.h"

namespace gdn_tvm {

void GdnDecode(TensorView q, TensorView k, TensorView v, TensorView state, TensorView A_log,
               TensorView a, TensorView dt_bias, TensorView b, double scale, TensorView output,
               TensorView new_state) {
  require(q.ndim() == 4 && v.ndim() == 4, "q and v must be [B, 1, H, D]");
  const DLDevice dev = q.device();
  require(dev.device_type == kDLCUDA, "q must be a CUDA tensor");
  const int64_t B = q.size(0), H_qk = q.size(2), D = q.size(3), H_v = v.size(2);
  require(q.size(1) == 1, "decode takes T == 1");
  check_tensor(q, "q", kDLBfloat, 16, {B, 1, H_qk, D}, dev);
  check_tensor(k, "k", kDLBfloat, 16, {B, 1, H_qk, D}, dev);
  check_tensor(v, "v", kDLBfloat, 16, {B, 1, H_v, D}, dev);
  check_tensor(A_log, "A_log", kDLFloat, 32, {H_v}, dev);
  check_tensor(a, "a", kDLBfloat, 16, {B, 1, H_v}, dev);
  check_tensor(dt_bias, "dt_bias", kDLFloat, 32, {H_v}, dev);
  check_tensor(b, "b", kDLBfloat, 16, {B, 1, H_v}, dev);
  check_tensor(output, "output", kDLBfloat, 16, {B, 1, H_v, D}, dev);
  check_tensor(new_state, "new_state", kDLFloat, 32, {B, H_v, D, D}, dev);
  const float* st = optional_state(state, "state", {B, H_v, D, D}, dev);
  DeviceGuard guard(dev);
  check_rc(gdn_b200_decode(ptr(q), ptr(k), ptr(v), st, static_cast<const float*>(ptr(A_log)),
                           ptr(a), static_cast<const float*>(ptr(dt_bias)), ptr(b), scale,
                           ptr(output), static_cast<float*>(ptr(new_state)), B,
                           static_cast<int32_t>(H_qk), static_cast<int32_t>(H_v),
                           static_cast<int32_t>(D), env_stream(dev)));
}

}  // namespace gdn_tvm

TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel, gdn_tvm::GdnDecode);
