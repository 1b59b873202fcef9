// Shared DLPack validation for the TVM-FFI `kernel` exports.  The reference's
// exports (ref solution/cuda/kernel.cu:101-150, kernel_prefill.cu:300-339)
// check nothing; these raise tvm-ffi ValueError on a dtype, device, shape or
// layout mismatch instead of launching on bad memory.
#pragma once

#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "gdn_b200.h"

namespace gdn_tvm {

using tvm::ffi::TensorView;

inline bool is_dtype(const TensorView& t, uint8_t code, uint8_t bits) {
  DLDataType d = t.dtype();
  return d.code == code && d.bits == bits && d.lanes == 1;
}

inline void require(bool cond, const std::string& msg) {
  if (!cond) TVM_FFI_THROW(ValueError) << msg;
}

inline void* ptr(const TensorView& t) {
  return static_cast<char*>(t.data_ptr()) + t.byte_offset();
}

inline void check_tensor(const TensorView& t, const char* name, uint8_t code, uint8_t bits,
                         const std::vector<int64_t>& shape, const DLDevice& dev) {
  require(is_dtype(t, code, bits), std::string(name) + ": wrong dtype");
  require(t.device().device_type == kDLCUDA && t.device().device_id == dev.device_id,
          std::string(name) + ": must live on the same CUDA device as q");
  require(t.ndim() == static_cast<int32_t>(shape.size()), std::string(name) + ": wrong rank");
  for (size_t i = 0; i < shape.size(); ++i)
    require(t.size(static_cast<int64_t>(i)) == shape[i],
            std::string(name) + ": wrong extent in dim " + std::to_string(i));
  require(t.numel() == 0 || t.IsContiguous(), std::string(name) + ": must be contiguous");
}

inline void check_rc(int rc) {
  if (rc == GDN_B200_ERR_INVALID_ARGUMENT) TVM_FFI_THROW(ValueError) << gdn_b200_last_error();
  if (rc != GDN_B200_OK) TVM_FFI_THROW(RuntimeError) << gdn_b200_last_error();
}

// Makes the tensors' device current for the whole call (the C ABI launches on,
// and looks up per-device state for, the current device) and restores the
// caller's device on exit.
class DeviceGuard {
 public:
  explicit DeviceGuard(const DLDevice& dev) {
    if (cudaGetDevice(&prev_) != cudaSuccess)
      TVM_FFI_THROW(RuntimeError) << "cudaGetDevice failed";
    if (prev_ != dev.device_id) {
      cudaError_t e = cudaSetDevice(dev.device_id);
      if (e != cudaSuccess) TVM_FFI_THROW(RuntimeError) << "cudaSetDevice: " << cudaGetErrorString(e);
      switched_ = true;
    }
  }
  ~DeviceGuard() {
    if (switched_) cudaSetDevice(prev_);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;

 private:
  int prev_ = 0;
  bool switched_ = false;
};

inline void* env_stream(const DLDevice& dev) {
  return TVMFFIEnvGetStream(dev.device_type, dev.device_id);
}

// A state argument whose data pointer is null (or that has no elements) means
// "zero initial state", as in the reference (kernel.cu:135-139).
inline const float* optional_state(const TensorView& state, const char* name,
                                   const std::vector<int64_t>& shape, const DLDevice& dev) {
  if (state.data_ptr() == nullptr) return nullptr;
  check_tensor(state, name, kDLFloat, 32, shape, dev);
  return static_cast<const float*>(ptr(state));
}

}  // namespace gdn_tvm
