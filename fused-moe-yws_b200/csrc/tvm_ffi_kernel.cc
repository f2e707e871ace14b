// tvm_ffi_kernel.cc -- TVM-FFI export `kernel` with the reference operator's signature.
//
// Drop-in for solution/cuda/kernel.cu:1727-1839 (TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel,
// kernel), solution spec entry_point "kernel.cu::kernel", binding "tvm-ffi",
// destination_passing_style = false). It keeps the reference's tensor contract checks
// (CheckTensor / CheckScalarVector / CheckSameDevice, kernel.cu:121-168 and :1746-1769)
// and exception types, allocates the bf16 output and a scratch workspace through the TVM-FFI
// environment allocator, and runs the whole operator through the C ABI (include/fmoe.h)
// on the environment stream. Unlike the reference (kernel.cu:1834) it does not
// synchronise the stream before returning.
//
// Device-side failures (a bounded wait inside a GEMM that ran out) cannot be seen when an
// asynchronous call returns. Each call's last kernel reports its device error word to a
// host-mapped word of the library, and every call starts by polling it
// (fmoe_poll_device_error): a failure of an earlier call on the device raises RuntimeError
// at the next call, as the reference's CHECK_CUDA (kernel.cu:53-62) raises on CUDA errors.
// With FMOE_SYNC_CHECK=1 in the environment the call also synchronises the stream before
// returning, like the reference, and raises for its own failure.
//
// Geometry is derived from the tensor shapes rather than hard-coded (kernel.cu:32-40):
// E_global from routing_logits, E_local / 2I / H from gemm1_weights. n_group, topk_group
// and top_k come from the definition table keyed by E_global (256 -> 8/4/8 for
// DeepSeek-V3, 16 -> 4/2/4 for the tiny contest geometry).
#include <tvm/ffi/container/shape.h>
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include <cuda_runtime.h>

#include <cstdlib>
#include <string>

#include "fmoe.h"

namespace ffi = tvm::ffi;

namespace {

void CheckTensor(const ffi::TensorView& t, const char* name, int32_t ndim,
                 std::initializer_list<int64_t> shape, DLDataType dtype) {
  if (t.device().device_type != kDLCUDA) TVM_FFI_THROW(ValueError) << name << " must be a CUDA tensor";
  if (!t.IsContiguous()) TVM_FFI_THROW(ValueError) << name << " must be contiguous";
  if (t.ndim() != ndim)
    TVM_FFI_THROW(ValueError) << name << " must be " << ndim << "D, got " << t.ndim();
  int i = 0;
  for (int64_t s : shape) {
    if (t.size(i) != s)
      TVM_FFI_THROW(ValueError) << name << " shape mismatch at dim " << i << ": expected " << s
                                << ", got " << t.size(i);
    ++i;
  }
  const DLDataType d = t.dtype();
  if (d.code != dtype.code || d.bits != dtype.bits || d.lanes != dtype.lanes)
    TVM_FFI_THROW(TypeError) << name << " dtype mismatch: expected "
                             << ffi::DLDataTypeToString(dtype) << ", got "
                             << ffi::DLDataTypeToString(d);
}

void CheckSameDevice(const ffi::TensorView& a, const ffi::TensorView& b, const char* an,
                     const char* bn) {
  if (a.device().device_type != b.device().device_type ||
      a.device().device_id != b.device().device_id)
    TVM_FFI_THROW(ValueError) << an << " and " << bn << " must be on the same device";
}

// Makes the tensors' device current for the call and restores the caller's device after.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess)
      TVM_FFI_THROW(RuntimeError) << "cudaSetDevice(" << dev << ") failed";
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

bool SyncCheckEnabled() {
  static const bool on = [] {
    const char* e = std::getenv("FMOE_SYNC_CHECK");
    return e && e[0] == '1';
  }();
  return on;
}

// Raise RuntimeError if a call on the current device has reported a device error word.
void ThrowIfDeviceError(const char* when) {
  int32_t bits = 0;
  if (fmoe_poll_device_error(&bits) != FMOE_OK)
    TVM_FFI_THROW(RuntimeError) << fmoe_last_error();
  if (bits != 0)
    TVM_FFI_THROW(RuntimeError) << when << ": the fused MoE kernels reported device error 0x"
                                << std::hex << bits
                                << " (a bounded wait expired); that call's output is invalid";
}

void ThrowStatus(int rc) {
  const std::string msg = fmoe_last_error();
  if (rc == FMOE_ERR_VALUE || rc == FMOE_ERR_WORKSPACE) TVM_FFI_THROW(ValueError) << msg;
  if (rc == FMOE_ERR_TYPE) TVM_FFI_THROW(TypeError) << msg;
  TVM_FFI_THROW(RuntimeError) << msg;
}

}  // namespace

ffi::Tensor kernel(const ffi::TensorView& routing_logits, const ffi::TensorView& routing_bias,
                   const ffi::TensorView& hidden_states,
                   const ffi::TensorView& hidden_states_scale,
                   const ffi::TensorView& gemm1_weights,
                   const ffi::TensorView& gemm1_weights_scale,
                   const ffi::TensorView& gemm2_weights,
                   const ffi::TensorView& gemm2_weights_scale, int32_t local_expert_offset,
                   float routed_scaling_factor) {
  const DLDataType f32{kDLFloat, 32, 1}, bf16{kDLBfloat, 16, 1}, f8{kDLFloat8_e4m3fn, 8, 1};
  if (routing_logits.ndim() != 2) TVM_FFI_THROW(ValueError) << "routing_logits must be 2D";
  if (gemm1_weights.ndim() != 3) TVM_FFI_THROW(ValueError) << "gemm1_weights must be 3D";
  const int64_t T = routing_logits.size(0), E = routing_logits.size(1);
  const int64_t EL = gemm1_weights.size(0), I = gemm1_weights.size(1) / 2,
                H = gemm1_weights.size(2);
  int n_group = 0, topk_group = 0, top_k = 0;
  if (E == 256) {
    n_group = 8, topk_group = 4, top_k = 8;
  } else if (E == 16) {
    n_group = 4, topk_group = 2, top_k = 4;
  } else {
    TVM_FFI_THROW(ValueError) << "routing_logits: unsupported number of experts " << E;
  }
  if (H % 128 != 0 || I % 128 != 0 || H <= 0 || I <= 0)
    TVM_FFI_THROW(ValueError) << "gemm1_weights: hidden and intermediate sizes must be multiples of 128";
  CheckTensor(routing_logits, "routing_logits", 2, {T, E}, f32);
  CheckTensor(routing_bias, "routing_bias", 1, {E}, bf16);
  CheckTensor(hidden_states, "hidden_states", 2, {T, H}, f8);
  CheckTensor(hidden_states_scale, "hidden_states_scale", 2, {H / 128, T}, f32);
  CheckTensor(gemm1_weights, "gemm1_weights", 3, {EL, 2 * I, H}, f8);
  CheckTensor(gemm1_weights_scale, "gemm1_weights_scale", 3, {EL, 2 * I / 128, H / 128}, f32);
  CheckTensor(gemm2_weights, "gemm2_weights", 3, {EL, H, I}, f8);
  CheckTensor(gemm2_weights_scale, "gemm2_weights_scale", 3, {EL, H / 128, I / 128}, f32);
  CheckSameDevice(routing_logits, routing_bias, "routing_logits", "routing_bias");
  CheckSameDevice(routing_logits, hidden_states, "routing_logits", "hidden_states");
  CheckSameDevice(routing_logits, hidden_states_scale, "routing_logits", "hidden_states_scale");
  CheckSameDevice(routing_logits, gemm1_weights, "routing_logits", "gemm1_weights");
  CheckSameDevice(routing_logits, gemm1_weights_scale, "routing_logits", "gemm1_weights_scale");
  CheckSameDevice(routing_logits, gemm2_weights, "routing_logits", "gemm2_weights");
  CheckSameDevice(routing_logits, gemm2_weights_scale, "routing_logits", "gemm2_weights_scale");

  fmoe_problem p{};
  p.num_tokens = T;
  p.num_experts = (int32_t)E;
  p.num_local_experts = (int32_t)EL;
  p.hidden_size = (int32_t)H;
  p.intermediate_size = (int32_t)I;
  p.top_k = top_k;
  p.n_group = n_group;
  p.topk_group = topk_group;
  p.local_expert_offset = local_expert_offset;
  p.routed_scaling_factor = routed_scaling_factor;
  p.tile_n = 0;
  if (fmoe_validate(&p) != FMOE_OK) ThrowStatus(FMOE_ERR_VALUE);

  const DLDevice device = routing_logits.device();
  DeviceGuard guard(device.device_id);
  ThrowIfDeviceError("an earlier call on this device");
  void* stream = TVMFFIEnvGetStream(device.device_type, device.device_id);
  ffi::Tensor out = ffi::Tensor::FromEnvAlloc(TVMFFIEnvTensorAlloc, ffi::Shape({T, H}), bf16, device);
  if (T == 0) return out;
  size_t ws_bytes = 0;
  if (fmoe_workspace_size(&p, &ws_bytes) != FMOE_OK) ThrowStatus(FMOE_ERR_VALUE);
  ffi::Tensor ws = ffi::Tensor::FromEnvAlloc(TVMFFIEnvTensorAlloc,
                                             ffi::Shape({(int64_t)ws_bytes}),
                                             DLDataType{kDLUInt, 8, 1}, device);
  fmoe_tensors t{};
  t.routing_logits = static_cast<const float*>(routing_logits.data_ptr());
  t.routing_bias = routing_bias.data_ptr();
  t.hidden_states = hidden_states.data_ptr();
  t.hidden_states_scale = static_cast<const float*>(hidden_states_scale.data_ptr());
  t.gemm1_weights = gemm1_weights.data_ptr();
  t.gemm1_weights_scale = static_cast<const float*>(gemm1_weights_scale.data_ptr());
  t.gemm2_weights = gemm2_weights.data_ptr();
  t.gemm2_weights_scale = static_cast<const float*>(gemm2_weights_scale.data_ptr());
  t.output = out.data_ptr();
  const int rc = fmoe_forward(&p, &t, ws.data_ptr(), ws_bytes, stream);
  if (rc != FMOE_OK) ThrowStatus(rc);
  if (SyncCheckEnabled()) {
    const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) TVM_FFI_THROW(RuntimeError) << "CUDA error: " << cudaGetErrorString(e);
    ThrowIfDeviceError("this call");
  }
  return out;
}

TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel, kernel);
