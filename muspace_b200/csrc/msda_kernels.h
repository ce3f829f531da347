// Host-side interface between the C-ABI shim (msda_capi.cpp) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace msda {

struct Dims {
  int batch, spatial_size, heads, channels, levels, queries, points;
};

// One level of the level table, staged in shared memory by every CTA.
struct Level {
  int height, width, start;
};

enum class DType { kF32 = 0, kBF16 = 1 };

// Raw device pointers of one call. Forward uses value..out; backward uses
// value..weight, grad_out and the three gradient buffers.
struct Args {
  const void* value;
  const int64_t* shapes;
  const int64_t* starts;
  const void* loc;
  const void* weight;
  void* out;
  const void* grad_out;
  float* grad_value;
  float* grad_loc;
  float* grad_weight;
  const int* order;  // optional head-row visiting order (row-wise kernels); null = natural
  bool skip_grad_value;  // row-wise backward: grad_loc / grad_w only (grad_value comes from elsewhere)
};

// Grid-stride kernels never need more CTAs than this; 148 SMs x 8 resident
// 256-thread CTAs x 16 waves keeps every SM busy without a tail of idle CTAs.
inline int64_t grid_cap() { return 148LL * 8 * 16; }

inline size_t level_smem(const Dims& d) { return sizeof(Level) * static_cast<size_t>(d.levels > 0 ? d.levels : 1); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Lanes per head-row for the 16-byte vector kernels, or 0 when the channel
// count / alignment needs the scalar kernels.
inline int vec_group(int channels, size_t elem, const Args& a) {
  const size_t row_bytes = static_cast<size_t>(channels) * elem;
  if (row_bytes == 0 || row_bytes % 16 != 0) return 0;
  const size_t g = row_bytes / 16;
  if (g != 1 && g != 2 && g != 4 && g != 8 && g != 16 && g != 32) return 0;
  if (!aligned16(a.value)) return 0;
  if ((reinterpret_cast<uintptr_t>(a.loc) % (2 * elem)) != 0) return 0;  // (x, y) pairs load as one word
  if (a.out && !aligned16(a.out)) return 0;
  if (a.grad_out && !aligned16(a.grad_out)) return 0;
  if (a.grad_value && !aligned16(a.grad_value)) return 0;
  if ((reinterpret_cast<uintptr_t>(a.grad_loc) & 7u) != 0) return 0;  // (x, y) gradients store as one float2
  return static_cast<int>(g);
}

// Entry points used by the C-ABI: pick the tiled path when it applies and
// fall back to the row-wise kernels otherwise (msda_tiled.cu).
cudaError_t launch_forward(DType dtype, const Dims& d, const Args& a, cudaStream_t stream);
cudaError_t launch_backward(DType dtype, const Dims& d, const Args& a, cudaStream_t stream);

// Backward on caller-provided scratch (used by the static-scratch entry point):
// the scratch bytes the call needs (0 when the bucketed kernels do not apply
// and the scratch-free row-wise kernels run instead), and the launch itself.
size_t backward_scratch_bytes(DType dtype, const Dims& d, const Args& a);
cudaError_t launch_backward_on_scratch(DType dtype, const Dims& d, const Args& a, void* scratch, cudaStream_t stream);

// The fixed per-device scratch array (msda_noalloc.cu).
size_t static_scratch_capacity();
cudaError_t static_scratch_address(void** out);

// Row-wise kernels: one item per lane group in natural (b, q, h) order; any
// channel count (msda_forward.cu, msda_backward.cu).
cudaError_t launch_forward_rowwise(DType dtype, const Dims& d, const Args& a, cudaStream_t stream);
cudaError_t launch_backward_rowwise(DType dtype, const Dims& d, const Args& a, cudaStream_t stream);

}  // namespace msda
