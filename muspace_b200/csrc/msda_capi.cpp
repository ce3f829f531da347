// extern "C" boundary of libmuspace_ops.so (declared in include/muspace_msda.h).
//
// Takes the place of the TVM-FFI binding of muSPACE's MSDA
// (csrc/ms_deformable_attn/ms_deform_attn_musa.mu:507-628 and the checks of
// csrc/ffi/tensor_utils.hpp:13-34): it validates DLPack views with the same
// dtype / contiguity / im2col_step rules, adds the cross-tensor device check
// the reference left out, and turns every failure into a status code plus a
// per-thread message instead of an exception.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <limits>
#include <string>

#include "../../include/muspace_msda.h"
#include "deform_agg.h"
#include "flash_sca.h"
#include "msda_kernels.h"

namespace {

thread_local std::string g_last_error;

struct Failure {
  int status;
};

[[noreturn]] void fail(int status, const std::string& msg) {
  g_last_error = msg;
  throw Failure{status};
}

void require(bool ok, const std::string& msg) {
  if (!ok) fail(MSDA_STATUS_INVALID_ARGUMENT, msg);
}

std::string dtype_name(DLDataType t) {
  if (t.code == kDLFloat && t.bits == 32) return "float32";
  if (t.code == kDLBfloat && t.bits == 16) return "bfloat16";
  if (t.code == kDLFloat && t.bits == 16) return "float16";
  if (t.code == kDLFloat && t.bits == 64) return "float64";
  if (t.code == kDLInt && t.bits == 64) return "int64";
  if (t.code == kDLInt && t.bits == 32) return "int32";
  char buf[48];
  std::snprintf(buf, sizeof(buf), "dtype(code=%u,bits=%u)", t.code, t.bits);
  return buf;
}

bool same_dtype(DLDataType t, uint8_t code, uint8_t bits) { return t.code == code && t.bits == bits && t.lanes == 1; }

// Device, dtype, rank and row-major contiguity of one view (size-1 dims may
// carry any stride, as in DLPack's compactness rule).
void check_tensor(const DLTensor* t, const char* name, uint8_t code, uint8_t bits, int ndim, int device_id) {
  require(t != nullptr, std::string(name) + " is null");
  require(t->device.device_type == kDLCUDA,
          std::string(name) + " must be a CUDA tensor (DLPack device type kDLCUDA)");
  require(t->device.device_id == device_id, std::string(name) + " is on CUDA device " +
                                                std::to_string(t->device.device_id) + ", value is on device " +
                                                std::to_string(device_id));
  require(same_dtype(t->dtype, code, bits), std::string(name) + " must be " +
                                                dtype_name(DLDataType{code, bits, 1}) + ", got " +
                                                dtype_name(t->dtype));
  require(t->ndim == ndim, std::string(name) + " must have " + std::to_string(ndim) + " dims, got " +
                               std::to_string(t->ndim));
  bool empty = false;
  for (int i = 0; i < ndim; ++i) {
    require(t->shape[i] >= 0, std::string(name) + " has a negative extent");
    empty = empty || t->shape[i] == 0;
  }
  if (t->strides != nullptr && !empty) {  // a view without elements has no layout to check
    int64_t expect = 1;
    for (int i = ndim - 1; i >= 0; --i) {
      if (t->shape[i] != 1)
        require(t->strides[i] == expect, std::string(name) + " must be contiguous");
      expect *= t->shape[i];
    }
  }
}

void* data_of(const DLTensor* t) { return static_cast<char*>(t->data) + t->byte_offset; }

void check_dims(const msda_dims_t& d) {
  const int64_t kMax = std::numeric_limits<int32_t>::max();
  require(d.batch >= 0 && d.spatial_size >= 0 && d.heads >= 0 && d.channels >= 0 && d.levels >= 0 &&
              d.queries >= 0 && d.points >= 0,
          "sizes must be non-negative");
  require(d.batch <= kMax && d.spatial_size <= kMax && d.queries <= kMax && d.levels <= 4096 && d.points <= 4096,
          "a size exceeds the supported range (B, Lin, Lq < 2^31; L, P <= 4096)");
  require(d.heads * d.channels <= kMax && d.levels * d.points <= kMax, "Hh * D or L * P exceeds 2^31");
}

msda::Dims to_kernel_dims(const msda_dims_t& d) {
  return msda::Dims{static_cast<int>(d.batch),   static_cast<int>(d.spatial_size), static_cast<int>(d.heads),
                    static_cast<int>(d.channels), static_cast<int>(d.levels),       static_cast<int>(d.queries),
                    static_cast<int>(d.points),
                    msda::points_magic(static_cast<int>(d.levels), static_cast<int>(d.points))};
}

void check_launch(cudaError_t err, const char* what) {
  if (err != cudaSuccess)
    fail(MSDA_STATUS_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorName(err) + ": " + cudaGetErrorString(err));
}

// Makes `device` current for the launch and restores the caller's device.
struct DeviceGuard {
  int previous = -1;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
    if (previous != device) check_launch(cudaSetDevice(device), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int now = -1;
    if (previous >= 0 && cudaGetDevice(&now) == cudaSuccess && now != previous) cudaSetDevice(previous);
  }
};

// Shape checks shared by both directions; fills dims from the views the way
// the reference does (ms_deform_attn_musa.mu:521-522).
msda_dims_t dims_from_views(const DLTensor* value, const DLTensor* spatial, const DLTensor* start,
                            const DLTensor* loc, const DLTensor* weight, int im2col_step) {
  msda_dims_t d{};
  d.batch = value->shape[0];
  d.spatial_size = value->shape[1];
  d.heads = value->shape[2];
  d.channels = value->shape[3];
  d.levels = spatial->shape[0];
  d.queries = loc->shape[1];
  d.points = loc->shape[4];
  require(spatial->shape[1] == 2, "spatial_shapes must have shape (L, 2)");
  require(start->shape[0] == d.levels, "level_start_index must have shape (L,)");
  require(loc->shape[0] == d.batch && loc->shape[2] == d.heads && loc->shape[3] == d.levels && loc->shape[5] == 2,
          "sampling_locations must have shape (B, Lq, Hh, L, P, 2)");
  require(weight->shape[0] == d.batch && weight->shape[1] == d.queries && weight->shape[2] == d.heads &&
              weight->shape[3] == d.levels && weight->shape[4] == d.points,
          "attention_weights must have shape (B, Lq, Hh, L, P)");
  const int64_t step = d.batch < im2col_step ? d.batch : im2col_step;
  require(step > 0, "im2col_step chunk must be positive (min(batch, im2col_step) = " + std::to_string(step) + ")");
  require(d.batch % step == 0, "batch (" + std::to_string(d.batch) + ") must be divisible by im2col_step chunk (" +
                                   std::to_string(step) + ")");
  check_dims(d);
  return d;
}

msda::DType storage_dtype(const DLTensor* value) {
  require(value != nullptr, "value is null");
  if (same_dtype(value->dtype, kDLFloat, 32)) return msda::DType::kF32;
  if (same_dtype(value->dtype, kDLBfloat, 16)) return msda::DType::kBF16;
  fail(MSDA_STATUS_INVALID_ARGUMENT, "value must be float32 or bfloat16, got " + dtype_name(value->dtype));
}

template <typename F>
int guarded(F&& body) {
  try {
    body();
    g_last_error.clear();
    return MSDA_STATUS_OK;
  } catch (const Failure& f) {
    return f.status;
  } catch (...) {
    g_last_error = "internal error";
    return MSDA_STATUS_CUDA_ERROR;
  }
}

}  // namespace

extern "C" {

int ms_deform_attn_forward(const DLTensor* value, const DLTensor* spatial_shapes, const DLTensor* level_start_index,
                           const DLTensor* sampling_locations, const DLTensor* attention_weights, DLTensor* output,
                           int im2col_step, void* stream) {
  return guarded([&] {
    const msda::DType dt = storage_dtype(value);
    const uint8_t code = dt == msda::DType::kBF16 ? kDLBfloat : kDLFloat;
    const uint8_t bits = dt == msda::DType::kBF16 ? 16 : 32;
    const int dev = value->device.device_id;
    check_tensor(value, "value", code, bits, 4, dev);
    check_tensor(spatial_shapes, "spatial_shapes", kDLInt, 64, 2, dev);
    check_tensor(level_start_index, "level_start_index", kDLInt, 64, 1, dev);
    check_tensor(sampling_locations, "sampling_locations", code, bits, 6, dev);
    check_tensor(attention_weights, "attention_weights", code, bits, 5, dev);
    check_tensor(output, "out", code, bits, 3, dev);
    const msda_dims_t d =
        dims_from_views(value, spatial_shapes, level_start_index, sampling_locations, attention_weights, im2col_step);
    require(output->shape[0] == d.batch && output->shape[1] == d.queries &&
                output->shape[2] == d.heads * d.channels,
            "out must have shape (B, Lq, Hh * D)");
    DeviceGuard guard(dev);
    msda::Args a{};
    a.value = data_of(value);
    a.shapes = static_cast<const int64_t*>(data_of(spatial_shapes));
    a.starts = static_cast<const int64_t*>(data_of(level_start_index));
    a.loc = data_of(sampling_locations);
    a.weight = data_of(attention_weights);
    a.out = data_of(output);
    check_launch(msda::launch_forward(dt, to_kernel_dims(d), a, static_cast<cudaStream_t>(stream)),
                 "ms_deform_attn_forward");
  });
}

int ms_deform_attn_backward(const DLTensor* value, const DLTensor* spatial_shapes, const DLTensor* level_start_index,
                            const DLTensor* sampling_locations, const DLTensor* attention_weights,
                            const DLTensor* grad_output, DLTensor* grad_value, DLTensor* grad_sampling_loc,
                            DLTensor* grad_attn_weight, int im2col_step, void* stream) {
  return guarded([&] {
    const msda::DType dt = storage_dtype(value);
    const uint8_t code = dt == msda::DType::kBF16 ? kDLBfloat : kDLFloat;
    const uint8_t bits = dt == msda::DType::kBF16 ? 16 : 32;
    const int dev = value->device.device_id;
    check_tensor(value, "value", code, bits, 4, dev);
    check_tensor(spatial_shapes, "spatial_shapes", kDLInt, 64, 2, dev);
    check_tensor(level_start_index, "level_start_index", kDLInt, 64, 1, dev);
    check_tensor(sampling_locations, "sampling_locations", code, bits, 6, dev);
    check_tensor(attention_weights, "attention_weights", code, bits, 5, dev);
    check_tensor(grad_output, "grad", code, bits, 3, dev);
    check_tensor(grad_value, "grad_value", kDLFloat, 32, 4, dev);
    check_tensor(grad_sampling_loc, "grad_sampling_locations", kDLFloat, 32, 6, dev);
    check_tensor(grad_attn_weight, "grad_attention_weights", kDLFloat, 32, 5, dev);
    const msda_dims_t d =
        dims_from_views(value, spatial_shapes, level_start_index, sampling_locations, attention_weights, im2col_step);
    require(grad_output->shape[0] == d.batch && grad_output->shape[1] == d.queries &&
                grad_output->shape[2] == d.heads * d.channels,
            "grad must have shape (B, Lq, Hh * D)");
    for (int i = 0; i < 4; ++i)
      require(grad_value->shape[i] == value->shape[i], "grad_value must have the shape of value");
    for (int i = 0; i < 6; ++i)
      require(grad_sampling_loc->shape[i] == sampling_locations->shape[i],
              "grad_sampling_locations must have the shape of sampling_locations");
    for (int i = 0; i < 5; ++i)
      require(grad_attn_weight->shape[i] == attention_weights->shape[i],
              "grad_attention_weights must have the shape of attention_weights");
    DeviceGuard guard(dev);
    msda::Args a{};
    a.value = data_of(value);
    a.shapes = static_cast<const int64_t*>(data_of(spatial_shapes));
    a.starts = static_cast<const int64_t*>(data_of(level_start_index));
    a.loc = data_of(sampling_locations);
    a.weight = data_of(attention_weights);
    a.grad_out = data_of(grad_output);
    a.grad_value = static_cast<float*>(data_of(grad_value));
    a.grad_loc = static_cast<float*>(data_of(grad_sampling_loc));
    a.grad_weight = static_cast<float*>(data_of(grad_attn_weight));
    check_launch(msda::launch_backward(dt, to_kernel_dims(d), a, static_cast<cudaStream_t>(stream)),
                 "ms_deform_attn_backward");
  });
}

int msda_forward(msda_dtype_t dtype, const msda_dims_t* dims, const void* value, const int64_t* spatial_shapes,
                 const int64_t* level_start_index, const void* sampling_locations, const void* attention_weights,
                 void* output, void* stream) {
  return guarded([&] {
    require(dtype == MSDA_DTYPE_FLOAT32 || dtype == MSDA_DTYPE_BFLOAT16, "dtype must be float32 or bfloat16");
    require(dims != nullptr, "dims is null");
    check_dims(*dims);
    const bool empty = dims->batch * dims->queries * dims->heads * dims->channels == 0;
    require(empty || (value && spatial_shapes && level_start_index && sampling_locations && attention_weights && output),
            "a required pointer is null");
    msda::Args a{};
    a.value = value;
    a.shapes = spatial_shapes;
    a.starts = level_start_index;
    a.loc = sampling_locations;
    a.weight = attention_weights;
    a.out = output;
    const msda::DType dt = dtype == MSDA_DTYPE_BFLOAT16 ? msda::DType::kBF16 : msda::DType::kF32;
    check_launch(msda::launch_forward(dt, to_kernel_dims(*dims), a, static_cast<cudaStream_t>(stream)),
                 "msda_forward");
  });
}

int msda_backward(msda_dtype_t dtype, const msda_dims_t* dims, const void* value, const int64_t* spatial_shapes,
                  const int64_t* level_start_index, const void* sampling_locations, const void* attention_weights,
                  const void* grad_output, float* grad_value, float* grad_sampling_loc, float* grad_attn_weight,
                  void* stream) {
  return guarded([&] {
    require(dtype == MSDA_DTYPE_FLOAT32 || dtype == MSDA_DTYPE_BFLOAT16, "dtype must be float32 or bfloat16");
    require(dims != nullptr, "dims is null");
    check_dims(*dims);
    const bool empty = dims->batch * dims->queries * dims->heads == 0;
    require(empty || (value && spatial_shapes && level_start_index && sampling_locations && attention_weights &&
                      grad_output && grad_value && grad_sampling_loc && grad_attn_weight),
            "a required pointer is null");
    msda::Args a{};
    a.value = value;
    a.shapes = spatial_shapes;
    a.starts = level_start_index;
    a.loc = sampling_locations;
    a.weight = attention_weights;
    a.grad_out = grad_output;
    a.grad_value = grad_value;
    a.grad_loc = grad_sampling_loc;
    a.grad_weight = grad_attn_weight;
    const msda::DType dt = dtype == MSDA_DTYPE_BFLOAT16 ? msda::DType::kBF16 : msda::DType::kF32;
    check_launch(msda::launch_backward(dt, to_kernel_dims(*dims), a, static_cast<cudaStream_t>(stream)),
                 "msda_backward");
  });
}

int msda_deterministic_workspace_bytes(const msda_dims_t* dims, size_t* bytes) {
  return guarded([&] {
    require(dims != nullptr && bytes != nullptr, "dims or bytes is null");
    check_dims(*dims);
    *bytes = msda::deterministic_workspace_bytes(to_kernel_dims(*dims));
  });
}

int ms_deform_attn_backward_deterministic(const DLTensor* value, const DLTensor* spatial_shapes,
                                          const DLTensor* level_start_index, const DLTensor* sampling_locations,
                                          const DLTensor* attention_weights, const DLTensor* grad_output,
                                          DLTensor* grad_value, DLTensor* grad_sampling_loc,
                                          DLTensor* grad_attn_weight, DLTensor* workspace, int im2col_step,
                                          void* stream) {
  return guarded([&] {
    const msda::DType dt = storage_dtype(value);
    const uint8_t code = dt == msda::DType::kBF16 ? kDLBfloat : kDLFloat;
    const uint8_t bits = dt == msda::DType::kBF16 ? 16 : 32;
    const int dev = value->device.device_id;
    check_tensor(value, "value", code, bits, 4, dev);
    check_tensor(spatial_shapes, "spatial_shapes", kDLInt, 64, 2, dev);
    check_tensor(level_start_index, "level_start_index", kDLInt, 64, 1, dev);
    check_tensor(sampling_locations, "sampling_locations", code, bits, 6, dev);
    check_tensor(attention_weights, "attention_weights", code, bits, 5, dev);
    check_tensor(grad_output, "grad", code, bits, 3, dev);
    check_tensor(grad_value, "grad_value", kDLFloat, 32, 4, dev);
    check_tensor(grad_sampling_loc, "grad_sampling_locations", kDLFloat, 32, 6, dev);
    check_tensor(grad_attn_weight, "grad_attention_weights", kDLFloat, 32, 5, dev);
    check_tensor(workspace, "workspace", kDLUInt, 8, 1, dev);
    const msda_dims_t d =
        dims_from_views(value, spatial_shapes, level_start_index, sampling_locations, attention_weights, im2col_step);
    require(grad_output->shape[0] == d.batch && grad_output->shape[1] == d.queries &&
                grad_output->shape[2] == d.heads * d.channels,
            "grad must have shape (B, Lq, Hh * D)");
    for (int i = 0; i < 4; ++i)
      require(grad_value->shape[i] == value->shape[i], "grad_value must have the shape of value");
    for (int i = 0; i < 6; ++i)
      require(grad_sampling_loc->shape[i] == sampling_locations->shape[i],
              "grad_sampling_locations must have the shape of sampling_locations");
    for (int i = 0; i < 5; ++i)
      require(grad_attn_weight->shape[i] == attention_weights->shape[i],
              "grad_attention_weights must have the shape of attention_weights");
    const msda::Dims kd = to_kernel_dims(d);
    const size_t need = msda::deterministic_workspace_bytes(kd);
    require(static_cast<size_t>(workspace->shape[0]) >= need,
            "workspace holds " + std::to_string(workspace->shape[0]) + " bytes, the call needs " +
                std::to_string(need) + " (msda_deterministic_workspace_bytes)");
    require((reinterpret_cast<uintptr_t>(data_of(workspace)) & 255u) == 0, "workspace must be 256-byte aligned");
    DeviceGuard guard(dev);
    msda::Args a{};
    a.value = data_of(value);
    a.shapes = static_cast<const int64_t*>(data_of(spatial_shapes));
    a.starts = static_cast<const int64_t*>(data_of(level_start_index));
    a.loc = data_of(sampling_locations);
    a.weight = data_of(attention_weights);
    a.grad_out = data_of(grad_output);
    a.grad_value = static_cast<float*>(data_of(grad_value));
    a.grad_loc = static_cast<float*>(data_of(grad_sampling_loc));
    a.grad_weight = static_cast<float*>(data_of(grad_attn_weight));
    check_launch(msda::launch_backward_deterministic(dt, kd, a, data_of(workspace), static_cast<cudaStream_t>(stream)),
                 "ms_deform_attn_backward_deterministic");
  });
}

int msda_backward_deterministic(msda_dtype_t dtype, const msda_dims_t* dims, const void* value,
                                const int64_t* spatial_shapes, const int64_t* level_start_index,
                                const void* sampling_locations, const void* attention_weights,
                                const void* grad_output, float* grad_value, float* grad_sampling_loc,
                                float* grad_attn_weight, void* workspace, size_t workspace_bytes, void* stream) {
  return guarded([&] {
    require(dtype == MSDA_DTYPE_FLOAT32 || dtype == MSDA_DTYPE_BFLOAT16, "dtype must be float32 or bfloat16");
    require(dims != nullptr, "dims is null");
    check_dims(*dims);
    const bool empty = dims->batch * dims->queries * dims->heads == 0;
    require(empty || (value && spatial_shapes && level_start_index && sampling_locations && attention_weights &&
                      grad_output && grad_value && grad_sampling_loc && grad_attn_weight && workspace),
            "a required pointer is null");
    const msda::Dims kd = to_kernel_dims(*dims);
    const size_t need = msda::deterministic_workspace_bytes(kd);
    require(empty || workspace_bytes >= need,
            "workspace holds " + std::to_string(workspace_bytes) + " bytes, the call needs " + std::to_string(need));
    require(empty || (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, "workspace must be 256-byte aligned");
    msda::Args a{};
    a.value = value;
    a.shapes = spatial_shapes;
    a.starts = level_start_index;
    a.loc = sampling_locations;
    a.weight = attention_weights;
    a.grad_out = grad_output;
    a.grad_value = grad_value;
    a.grad_loc = grad_sampling_loc;
    a.grad_weight = grad_attn_weight;
    const msda::DType dt = dtype == MSDA_DTYPE_BFLOAT16 ? msda::DType::kBF16 : msda::DType::kF32;
    check_launch(msda::launch_backward_deterministic(dt, kd, a, workspace, static_cast<cudaStream_t>(stream)),
                 "msda_backward_deterministic");
  });
}

int msda_backward_static_scratch(msda_dtype_t dtype, const msda_dims_t* dims, const void* value,
                                 const int64_t* spatial_shapes, const int64_t* level_start_index,
                                 const void* sampling_locations, const void* attention_weights,
                                 const void* grad_output, float* grad_value, float* grad_sampling_loc,
                                 float* grad_attn_weight, void* stream) {
  return guarded([&] {
    require(dtype == MSDA_DTYPE_FLOAT32 || dtype == MSDA_DTYPE_BFLOAT16, "dtype must be float32 or bfloat16");
    require(dims != nullptr, "dims is null");
    check_dims(*dims);
    const bool empty = dims->batch * dims->queries * dims->heads == 0;
    require(empty || (value && spatial_shapes && level_start_index && sampling_locations && attention_weights &&
                      grad_output && grad_value && grad_sampling_loc && grad_attn_weight),
            "a required pointer is null");
    msda::Args a{};
    a.value = value;
    a.shapes = spatial_shapes;
    a.starts = level_start_index;
    a.loc = sampling_locations;
    a.weight = attention_weights;
    a.grad_out = grad_output;
    a.grad_value = grad_value;
    a.grad_loc = grad_sampling_loc;
    a.grad_weight = grad_attn_weight;
    const msda::DType dt = dtype == MSDA_DTYPE_BFLOAT16 ? msda::DType::kBF16 : msda::DType::kF32;
    const msda::Dims kd = to_kernel_dims(*dims);
    const size_t need = msda::backward_scratch_bytes(dt, kd, a);
    require(need <= msda::static_scratch_capacity(),
            "problem needs " + std::to_string(need) + " bytes of scratch, the static scratch holds " +
                std::to_string(msda::static_scratch_capacity()) +
                " (about 1M head-rows B * Lq * Hh); use msda_backward for larger calls");
    if (!empty) {
      // The scratch address is the current device's; the stream and the data
      // must belong to that device, or the kernels would get another GPU's
      // array.
      int current = -1, stream_device = -1;
      check_launch(cudaGetDevice(&current), "cudaGetDevice");
      check_launch(cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &stream_device), "cudaStreamGetDevice");
      require(stream_device == current, "stream is on CUDA device " + std::to_string(stream_device) +
                                            ", the current device is " + std::to_string(current));
      cudaPointerAttributes attr{};
      check_launch(cudaPointerGetAttributes(&attr, value), "cudaPointerGetAttributes");
      require(attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged,
              "value is not device memory");
      require(attr.device == current, "value is on CUDA device " + std::to_string(attr.device) +
                                          ", the current device is " + std::to_string(current));
    }
    void* scratch = nullptr;
    if (need > 0) check_launch(msda::static_scratch_address(&scratch), "static scratch set-up");
    check_launch(msda::launch_backward_on_scratch(dt, kd, a, scratch, static_cast<cudaStream_t>(stream)),
                 "msda_backward_static_scratch");
  });
}

int ms_deform_attn_scatter_div_forward(const DLTensor* value, const DLTensor* spatial_shapes,
                                      const DLTensor* level_start_index, const DLTensor* sampling_locations,
                                      const DLTensor* attention_weights, const DLTensor* index, const DLTensor* count,
                                      DLTensor* slots, int cam_id, void* stream) {
  return guarded([&] {
    const msda::DType dt = storage_dtype(value);
    const uint8_t code = dt == msda::DType::kBF16 ? kDLBfloat : kDLFloat;
    const uint8_t bits = dt == msda::DType::kBF16 ? 16 : 32;
    const int dev = value->device.device_id;
    check_tensor(value, "value", code, bits, 4, dev);
    check_tensor(spatial_shapes, "spatial_shapes", kDLInt, 64, 2, dev);
    check_tensor(level_start_index, "level_start_index", kDLInt, 64, 1, dev);
    check_tensor(sampling_locations, "sampling_locations", code, bits, 6, dev);
    check_tensor(attention_weights, "attention_weights", code, bits, 5, dev);
    check_tensor(index, "index", kDLInt, 64, 1, dev);
    check_tensor(count, "count", code, bits, 2, dev);
    check_tensor(slots, "slots", code, bits, 3, dev);
    // the rebatched call: B * cams images, max_len query slots per image
    const msda_dims_t d =
        dims_from_views(value, spatial_shapes, level_start_index, sampling_locations, attention_weights, 1 << 30);
    msda_slot_dims_t sd{};
    sd.batch = count->shape[0];
    sd.num_query = count->shape[1];
    sd.valid_len = index->shape[0];
    sd.cam = cam_id;
    require(sd.batch > 0 && d.batch % sd.batch == 0,
            "value batch (" + std::to_string(d.batch) + ") must be count batch (" + std::to_string(sd.batch) +
                ") times the number of cameras");
    sd.cams = d.batch / sd.batch;
    require(cam_id >= 0 && cam_id < sd.cams,
            "cam_id " + std::to_string(cam_id) + " outside [0, " + std::to_string(sd.cams) + ")");
    require(sd.valid_len <= d.queries, "index is longer than the rebatched query dimension (max_len)");
    require(slots->shape[0] == sd.batch && slots->shape[1] == sd.num_query && slots->shape[2] == d.heads * d.channels,
            "slots must have shape (B, num_query, Hh * D)");
    require(sd.num_query <= std::numeric_limits<int32_t>::max(), "num_query exceeds 2^31");
    DeviceGuard guard(dev);
    msda::Args a{};
    a.value = data_of(value);
    a.shapes = static_cast<const int64_t*>(data_of(spatial_shapes));
    a.starts = static_cast<const int64_t*>(data_of(level_start_index));
    a.loc = data_of(sampling_locations);
    a.weight = data_of(attention_weights);
    const msda::SlotDims ks{static_cast<int>(sd.batch), static_cast<int>(sd.cams), static_cast<int>(sd.cam),
                            static_cast<int>(sd.valid_len), static_cast<int>(sd.num_query)};
    const cudaError_t err = msda::launch_scatter_div(dt, to_kernel_dims(d), ks, a,
                                                     static_cast<const int64_t*>(data_of(index)), data_of(count),
                                                     data_of(slots), static_cast<cudaStream_t>(stream));
    require(err != cudaErrorInvalidValue,
            "ms_deform_attn_scatter_div_forward needs Hh * D rows in 16-byte lane slices (D * element size a "
            "multiple of 16 up to 512 bytes) and 16-byte aligned tensors");
    check_launch(err, "ms_deform_attn_scatter_div_forward");
  });
}

int msda_scatter_div_forward(msda_dtype_t dtype, const msda_dims_t* dims, const msda_slot_dims_t* slot_dims,
                             const void* value, const int64_t* spatial_shapes, const int64_t* level_start_index,
                             const void* sampling_locations, const void* attention_weights, const int64_t* index,
                             const void* count, void* slots, void* stream) {
  return guarded([&] {
    require(dtype == MSDA_DTYPE_FLOAT32 || dtype == MSDA_DTYPE_BFLOAT16, "dtype must be float32 or bfloat16");
    require(dims != nullptr && slot_dims != nullptr, "dims is null");
    check_dims(*dims);
    const msda_slot_dims_t& sd = *slot_dims;
    const int64_t kMax = std::numeric_limits<int32_t>::max();
    require(sd.batch >= 0 && sd.cams > 0 && sd.valid_len >= 0 && sd.num_query >= 0 && sd.num_query <= kMax,
            "slot sizes must be non-negative (cams positive, num_query < 2^31)");
    require(dims->batch == sd.batch * sd.cams, "dims->batch must be slot_dims->batch * slot_dims->cams");
    require(sd.cam >= 0 && sd.cam < sd.cams, "cam outside [0, cams)");
    require(sd.valid_len <= dims->queries, "valid_len exceeds the rebatched query dimension (dims->queries)");
    const bool empty = sd.batch * sd.valid_len * dims->heads * dims->channels == 0;
    require(empty || (value && spatial_shapes && level_start_index && sampling_locations && attention_weights &&
                      index && count && slots),
            "a required pointer is null");
    msda::Args a{};
    a.value = value;
    a.shapes = spatial_shapes;
    a.starts = level_start_index;
    a.loc = sampling_locations;
    a.weight = attention_weights;
    const msda::DType dt = dtype == MSDA_DTYPE_BFLOAT16 ? msda::DType::kBF16 : msda::DType::kF32;
    const msda::SlotDims ks{static_cast<int>(sd.batch), static_cast<int>(sd.cams), static_cast<int>(sd.cam),
                            static_cast<int>(sd.valid_len), static_cast<int>(sd.num_query)};
    const cudaError_t err =
        msda::launch_scatter_div(dt, to_kernel_dims(*dims), ks, a, index, count, slots, static_cast<cudaStream_t>(stream));
    require(err != cudaErrorInvalidValue,
            "msda_scatter_div_forward needs Hh * D rows in 16-byte lane slices and 16-byte aligned pointers");
    check_launch(err, "msda_scatter_div_forward");
  });
}

// ---------------------------------------------------------------------------
// deformable aggregation (csrc/deformable_aggregation/deformable_aggregation_musa.mu:643-751)
// ---------------------------------------------------------------------------
namespace {

struct DaViews {
  da::Dims dims;
  da::Args args;
  int device;
};

// The reference's validate() (fp32 / int32, contiguous, ranks) plus the shape
// agreements it left to the Python layer (mu_space/ops/deformable_aggregation.py:35-79).
DaViews da_views(const DLTensor* mc, const DLTensor* sp, const DLTensor* st, const DLTensor* loc, const DLTensor* w) {
  require(mc != nullptr, "mc_ms_feat is null");
  const int dev = mc->device.device_id;
  check_tensor(mc, "mc_ms_feat", kDLFloat, 32, 3, dev);
  check_tensor(sp, "spatial_shape", kDLInt, 32, 3, dev);
  check_tensor(st, "scale_start_index", kDLInt, 32, 2, dev);
  check_tensor(loc, "sampling_location", kDLFloat, 32, 5, dev);
  check_tensor(w, "weights", kDLFloat, 32, 6, dev);
  const int64_t batch = mc->shape[0], num_feat = mc->shape[1], channels = mc->shape[2];
  const int64_t cams = sp->shape[0], scales = sp->shape[1];
  const int64_t anchors = loc->shape[1], pts = loc->shape[2], groups = w->shape[5];
  require(sp->shape[2] == 2, "spatial_shape must have shape [num_cams, num_scale, 2]");
  require(st->shape[0] == cams && st->shape[1] == scales, "scale_start_index must have shape [num_cams, num_scale]");
  require(loc->shape[0] == batch && loc->shape[3] == cams && loc->shape[4] == 2,
          "sampling_location must have shape [B, anchors, pts, cams, 2]");
  require(w->shape[0] == batch && w->shape[1] == anchors && w->shape[2] == pts && w->shape[3] == cams &&
              w->shape[4] == scales,
          "weights must have shape [B, anchors, pts, cams, scale, groups]");
  require(groups >= 1 && groups <= 8, "num_groups must be in [1, 8]");
  require(channels % groups == 0, "num_embeds must be divisible by num_groups");
  const int64_t kMax = std::numeric_limits<int32_t>::max();
  require(batch <= kMax && num_feat <= kMax && channels <= kMax && anchors <= kMax && pts <= 65536,
          "a size exceeds the supported range");
  require(cams * scales <= 1024 && pts * cams <= kMax, "num_cams * num_scale exceeds 1024");
  DaViews v{};
  v.dims = da::Dims{static_cast<int>(batch), static_cast<int>(num_feat), static_cast<int>(channels),
                    static_cast<int>(cams), static_cast<int>(scales), static_cast<int>(anchors),
                    static_cast<int>(pts), static_cast<int>(groups)};
  v.args.feat = static_cast<const float*>(data_of(mc));
  v.args.shape = static_cast<const int*>(data_of(sp));
  v.args.start = static_cast<const int*>(data_of(st));
  v.args.loc = static_cast<const float*>(data_of(loc));
  v.args.weights = static_cast<const float*>(data_of(w));
  v.device = dev;
  return v;
}

int da_forward_entry(const DLTensor* mc, const DLTensor* sp, const DLTensor* st, const DLTensor* loc,
                     const DLTensor* w, DLTensor* out, void* stream, bool optimized, const char* name) {
  return guarded([&] {
    DaViews v = da_views(mc, sp, st, loc, w);
    check_tensor(out, "out", kDLFloat, 32, 3, v.device);
    require(out->shape[0] == mc->shape[0] && out->shape[1] == loc->shape[1] && out->shape[2] == mc->shape[2],
            "out must have shape [B, anchors, C]");
    v.args.out = static_cast<float*>(data_of(out));
    DeviceGuard guard(v.device);
    check_launch(da::forward(v.dims, v.args, optimized, static_cast<cudaStream_t>(stream)), name);
  });
}

int da_backward_entry(const DLTensor* mc, const DLTensor* sp, const DLTensor* st, const DLTensor* loc,
                      const DLTensor* w, const DLTensor* grad, DLTensor* grad_mc, DLTensor* grad_loc,
                      DLTensor* grad_w, void* stream, bool optimized, const char* name) {
  return guarded([&] {
    DaViews v = da_views(mc, sp, st, loc, w);
    check_tensor(grad, "grad_output", kDLFloat, 32, 3, v.device);
    check_tensor(grad_mc, "grad_mc_ms_feat", kDLFloat, 32, 3, v.device);
    check_tensor(grad_loc, "grad_sampling_location", kDLFloat, 32, 5, v.device);
    check_tensor(grad_w, "grad_weights", kDLFloat, 32, 6, v.device);
    require(grad->shape[0] == mc->shape[0] && grad->shape[1] == loc->shape[1] && grad->shape[2] == mc->shape[2],
            "grad_output must have shape [B, anchors, C]");
    for (int i = 0; i < 3; ++i) require(grad_mc->shape[i] == mc->shape[i], "grad_mc_ms_feat must have the shape of mc_ms_feat");
    for (int i = 0; i < 5; ++i)
      require(grad_loc->shape[i] == loc->shape[i], "grad_sampling_location must have the shape of sampling_location");
    for (int i = 0; i < 6; ++i) require(grad_w->shape[i] == w->shape[i], "grad_weights must have the shape of weights");
    v.args.grad_out = static_cast<const float*>(data_of(grad));
    v.args.grad_feat = static_cast<float*>(data_of(grad_mc));
    v.args.grad_loc = static_cast<float*>(data_of(grad_loc));
    v.args.grad_weights = static_cast<float*>(data_of(grad_w));
    DeviceGuard guard(v.device);
    check_launch(da::backward(v.dims, v.args, optimized, static_cast<cudaStream_t>(stream)), name);
  });
}

}  // namespace

int deformable_aggregation_forward_opt(const DLTensor* mc_ms_feat, const DLTensor* spatial_shape,
                                       const DLTensor* scale_start_index, const DLTensor* sampling_location,
                                       const DLTensor* weights, DLTensor* output, void* stream) {
  return da_forward_entry(mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights, output, stream,
                          true, "deformable_aggregation_forward_opt");
}

int deformable_aggregation_forward_base(const DLTensor* mc_ms_feat, const DLTensor* spatial_shape,
                                        const DLTensor* scale_start_index, const DLTensor* sampling_location,
                                        const DLTensor* weights, DLTensor* output, void* stream) {
  return da_forward_entry(mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights, output, stream,
                          false, "deformable_aggregation_forward_base");
}

int deformable_aggregation_backward_opt(const DLTensor* mc_ms_feat, const DLTensor* spatial_shape,
                                        const DLTensor* scale_start_index, const DLTensor* sampling_location,
                                        const DLTensor* weights, const DLTensor* grad_output,
                                        DLTensor* grad_mc_ms_feat, DLTensor* grad_sampling_location,
                                        DLTensor* grad_weights, void* stream) {
  return da_backward_entry(mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights, grad_output,
                           grad_mc_ms_feat, grad_sampling_location, grad_weights, stream, true,
                           "deformable_aggregation_backward_opt");
}

int deformable_aggregation_backward_base(const DLTensor* mc_ms_feat, const DLTensor* spatial_shape,
                                         const DLTensor* scale_start_index, const DLTensor* sampling_location,
                                         const DLTensor* weights, const DLTensor* grad_output,
                                         DLTensor* grad_mc_ms_feat, DLTensor* grad_sampling_location,
                                         DLTensor* grad_weights, void* stream) {
  return da_backward_entry(mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights, grad_output,
                           grad_mc_ms_feat, grad_sampling_location, grad_weights, stream, false,
                           "deformable_aggregation_backward_base");
}

// ---------------------------------------------------------------------------
// FlashSCA (csrc/flashbev/flash_bevpool_sca_musa.mu:262-399)
// ---------------------------------------------------------------------------
namespace {

struct FscaViews {
  fsca::Dims dims;
  fsca::Args args;
  int device;
};

// The reference's checks (fp32 / int32, contiguous, value rank 4, heads and
// grid positive, C % heads == 0) plus the shape agreements its Python layer
// made (mu_space/ops/flashbev.py:560-640).
FscaViews fsca_views(const DLTensor* value, const DLTensor* proj, const DLTensor* spatial, const DLTensor* start,
                     const DLTensor* image_size, const DLTensor* offsets, const DLTensor* weights, int heads,
                     int points, int gx, int gy, int gz, int value_stride_n) {
  require(value != nullptr, "value is null");
  const int dev = value->device.device_id;
  check_tensor(value, "value", kDLFloat, 32, 4, dev);
  check_tensor(proj, "projection_matrices", kDLFloat, 32, 4, dev);
  check_tensor(spatial, "spatial_shapes", kDLInt, 32, 2, dev);
  check_tensor(start, "level_start_index", kDLInt, 32, 1, dev);
  check_tensor(image_size, "image_size", kDLInt, 32, 1, dev);
  check_tensor(offsets, "sampling_offsets", kDLFloat, 32, 8, dev);
  check_tensor(weights, "attention_weights", kDLFloat, 32, 7, dev);
  require(heads > 0 && points > 0, "num_heads and num_points must be positive");
  require(gx > 0 && gy > 0 && gz > 0, "grid sizes must be positive");
  const int64_t batch = value->shape[0], cams = value->shape[1], stride = value->shape[2], channels = value->shape[3];
  const int64_t levels = spatial->shape[0];
  require(channels % heads == 0, "channels must be divisible by num_heads");
  require(proj->shape[0] == batch && proj->shape[1] == cams && proj->shape[2] == 3 && proj->shape[3] == 4,
          "projection_matrices must have shape [B,N,3,4]");
  require(spatial->shape[1] == 2 && start->shape[0] == levels && image_size->shape[0] == 2,
          "level_start_index/image_size shapes must be [levels]/[2]");
  const int64_t want[8] = {batch, gy, gx, heads, levels, points, gz, 2};
  for (int i = 0; i < 8; ++i) require(offsets->shape[i] == want[i], "sampling_offsets must have shape [B,gy,gx,heads,L,P,gz,2]");
  for (int i = 0; i < 7; ++i) require(weights->shape[i] == want[i], "attention_weights must have shape [B,gy,gx,heads,L,P,gz]");
  require(value_stride_n >= 1 && value_stride_n <= stride, "value_stride_n must be in [1, value.size(2)]");
  require(levels <= fsca::kMaxLevels, "at most 16 levels");
  require(cams * gz <= fsca::kMaxPairs, "num_cams * grid_z must be at most 64");
  const int64_t kMax = std::numeric_limits<int32_t>::max();
  require(cams * stride <= kMax && batch * gx * gy <= kMax && channels <= kMax, "a size exceeds the supported range");
  FscaViews v{};
  // floor(x / d) == umulhi(x, ceil(2^32 / d)) whenever x * d < 2^32; the kernels divide sample
  // indices below kMaxPairs * L * P by P and by L * P, and within one (cell, head) indices below
  // that many by P
  const auto magic = [](uint64_t d, uint64_t x_max) -> uint32_t {
    if (d <= 1 || x_max * d >= (uint64_t{1} << 32)) return 0;
    return static_cast<uint32_t>(((uint64_t{1} << 32) + d - 1) / d);
  };
  const uint64_t lp = static_cast<uint64_t>(levels) * static_cast<uint64_t>(points);
  v.dims = fsca::Dims{static_cast<int>(batch), static_cast<int>(cams), static_cast<int>(stride),
                      static_cast<int>(channels), static_cast<int>(levels), heads, points, gx, gy, gz,
                      magic(static_cast<uint64_t>(points), fsca::kMaxPairs * lp),
                      magic(lp, fsca::kMaxPairs * lp)};
  v.args.value = static_cast<const float*>(data_of(value));
  v.args.projection = static_cast<const float*>(data_of(proj));
  v.args.shapes = static_cast<const int*>(data_of(spatial));
  v.args.starts = static_cast<const int*>(data_of(start));
  v.args.image_size = static_cast<const int*>(data_of(image_size));
  v.args.offsets = static_cast<const float*>(data_of(offsets));
  v.args.weights = static_cast<const float*>(data_of(weights));
  v.device = dev;
  return v;
}

void fsca_require_lanes(const FscaViews& v, bool backward) {
  require(fsca::lanes_per_head(v.dims, v.args, backward) != 0,
          "flash_bevpool_sca needs channels / num_heads = 4 * {1, 2, 4, 8, 16, 32} and 16-byte aligned tensors");
}

}  // namespace

int flash_bevpool_sca_forward(const DLTensor* value, const DLTensor* projection_matrices, const DLTensor* spatial_shapes,
                              const DLTensor* level_start_index, const DLTensor* image_size,
                              const DLTensor* sampling_offsets, const DLTensor* attention_weights, DLTensor* out,
                              int num_heads, int num_points, int grid_x, int grid_y, int grid_z, float voxel_size_x,
                              float voxel_size_y, float voxel_size_z, float voxel_x_min, float voxel_y_min,
                              float voxel_z_min, int value_stride_n, float epsilon, void* stream) {
  return guarded([&] {
    FscaViews v = fsca_views(value, projection_matrices, spatial_shapes, level_start_index, image_size,
                             sampling_offsets, attention_weights, num_heads, num_points, grid_x, grid_y, grid_z,
                             value_stride_n);
    check_tensor(out, "out", kDLFloat, 32, 4, v.device);
    require(out->shape[0] == value->shape[0] && out->shape[1] == grid_y && out->shape[2] == grid_x &&
                out->shape[3] == value->shape[3],
            "out must have shape [B, gy, gx, C]");
    v.args.out = static_cast<float*>(data_of(out));
    fsca_require_lanes(v, false);
    DeviceGuard guard(v.device);
    const fsca::Grid grid{voxel_size_x, voxel_size_y, voxel_size_z, voxel_x_min, voxel_y_min, voxel_z_min};
    check_launch(fsca::forward(v.dims, grid, epsilon, v.args, static_cast<cudaStream_t>(stream)),
                 "flash_bevpool_sca_forward");
  });
}

int flash_bevpool_sca_backward(const DLTensor* out_grad, const DLTensor* value, const DLTensor* projection_matrices,
                               const DLTensor* spatial_shapes, const DLTensor* level_start_index,
                               const DLTensor* image_size, const DLTensor* roi_range,
                               const DLTensor* sampling_offsets, const DLTensor* attention_weights,
                               DLTensor* value_grad, DLTensor* sampling_offsets_grad,
                               DLTensor* attention_weights_grad, int num_heads, int num_points, int grid_x,
                               int grid_y, int grid_z, int value_stride_n, float epsilon, void* stream) {
  return guarded([&] {
    FscaViews v = fsca_views(value, projection_matrices, spatial_shapes, level_start_index, image_size,
                             sampling_offsets, attention_weights, num_heads, num_points, grid_x, grid_y, grid_z,
                             value_stride_n);
    check_tensor(out_grad, "out_grad", kDLFloat, 32, 4, v.device);
    check_tensor(roi_range, "roi_range", kDLFloat, 32, 1, v.device);
    check_tensor(value_grad, "value_grad", kDLFloat, 32, 4, v.device);
    check_tensor(sampling_offsets_grad, "sampling_offsets_grad", kDLFloat, 32, 8, v.device);
    check_tensor(attention_weights_grad, "attention_weights_grad", kDLFloat, 32, 7, v.device);
    require(roi_range->shape[0] == 6, "roi_range must have shape [6]");
    require(out_grad->shape[0] == value->shape[0] && out_grad->shape[1] == grid_y && out_grad->shape[2] == grid_x &&
                out_grad->shape[3] == value->shape[3],
            "out_grad must have shape [B, gy, gx, C]");
    for (int i = 0; i < 4; ++i) require(value_grad->shape[i] == value->shape[i], "value_grad must have the shape of value");
    for (int i = 0; i < 8; ++i)
      require(sampling_offsets_grad->shape[i] == sampling_offsets->shape[i],
              "sampling_offsets_grad must have the shape of sampling_offsets");
    for (int i = 0; i < 7; ++i)
      require(attention_weights_grad->shape[i] == attention_weights->shape[i],
              "attention_weights_grad must have the shape of attention_weights");
    v.args.roi = static_cast<const float*>(data_of(roi_range));
    v.args.grad_out = static_cast<const float*>(data_of(out_grad));
    v.args.grad_value = static_cast<float*>(data_of(value_grad));
    v.args.grad_offsets = static_cast<float*>(data_of(sampling_offsets_grad));
    v.args.grad_weights = static_cast<float*>(data_of(attention_weights_grad));
    fsca_require_lanes(v, true);
    DeviceGuard guard(v.device);
    check_launch(fsca::backward(v.dims, epsilon, v.args, static_cast<cudaStream_t>(stream)),
                 "flash_bevpool_sca_backward");
  });
}

const char* msda_last_error(void) { return g_last_error.c_str(); }

int msda_stage_wait_timeouts(unsigned int* count) {
  return guarded([&] {
    require(count != nullptr, "count is null");
    const unsigned int v = msda::staged_wait_timeouts();
    if (v == ~0u) fail(MSDA_STATUS_CUDA_ERROR, "the staged forward's wait counter could not be read");
    *count = v;
  });
}

const char* msda_version(void) { return "0.1.0"; }

}  // extern "C"
