// Host-side interface between the C-ABI shim (msda_capi.cpp) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace msda {

struct Dims {
  int batch, spatial_size, heads, channels, levels, queries, points;
  // ceil(2^32 / points) when levels * points^2 < 2^32 and points > 1: then the
  // level of sample s (0 <= s < levels * points) is __umulhi(s, points_magic)
  // exactly; 0 means divide (LevelOf in msda_device.cuh)
  uint32_t points_magic;
};
// The multiply-high constant of Dims::points_magic (0 when it would not be exact).
inline uint32_t points_magic(int levels, int points) {
  if (points <= 1 || levels <= 0) return 0;
  const uint64_t p = static_cast<uint64_t>(points);
  if (static_cast<uint64_t>(levels) * p * p >= (uint64_t{1} << 32)) return 0;
  return static_cast<uint32_t>(((uint64_t{1} << 32) + p - 1) / p);
}

// One level of the level table, staged in shared memory by every CTA.
struct Level {
  int height, width, start;
};

enum class DType { kF32 = 0, kBF16 = 1 };

// The rebatch side of the fused spatial-cross-attention scatter (one camera):
// batch entries, cameras per batch entry, the camera, its valid rebatched
// queries and the BEV queries of the slots tensor.
struct SlotDims {
  int batch, cams, cam, valid_len, num_query;
};

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

// Most CTAs a launch asks for; beyond it the kernels' grid-stride loops take
// over. Items are meant to be visited roughly in order (batch-major) so the
// CTAs in flight share one camera's value map and grad_value lines in L2; a
// small cap makes each CTA stride across many cameras and spreads the working
// set beyond L2, so the cap only guards gridDim.x.
#ifndef MSDA_GRID_CAP
#define MSDA_GRID_CAP (1LL << 30)
#endif
inline int64_t grid_cap() { return MSDA_GRID_CAP; }

inline size_t level_smem(const Dims& d) { return sizeof(Level) * static_cast<size_t>(d.levels > 0 ? d.levels : 1); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Lanes per head-row when each lane holds lane_bytes (8 or 16) of channels,
// or 0 when the channel count / alignment rules that layout out: G must be a
// power of two up to a warp, the channel slices must be aligned to lane_bytes
// and the fp32 gradient slices to 16 bytes.
inline int vec_lanes(int channels, size_t elem, size_t lane_bytes, const Args& a) {
  const size_t row_bytes = static_cast<size_t>(channels) * elem;
  if (row_bytes == 0 || row_bytes % lane_bytes != 0) return 0;
  const size_t g = row_bytes / lane_bytes;
  if (g != 1 && g != 2 && g != 4 && g != 8 && g != 16 && g != 32) return 0;
  if (lane_bytes / elem < 4) return 0;  // a lane's fp32 gradient slice must fill whole 16-byte REDs
  const auto aligned = [lane_bytes](const void* p) { return (reinterpret_cast<uintptr_t>(p) % lane_bytes) == 0; };
  if (!aligned(a.value)) return 0;
  if ((reinterpret_cast<uintptr_t>(a.loc) % (2 * elem)) != 0) return 0;  // (x, y) pairs load as one word
  if (a.out && !aligned(a.out)) return 0;
  if (a.grad_out && !aligned(a.grad_out)) return 0;
  if (a.grad_value && !aligned16(a.grad_value)) return 0;
  if ((reinterpret_cast<uintptr_t>(a.grad_loc) & 7u) != 0) return 0;  // (x, y) gradients store as one float2
  return static_cast<int>(g);
}

// Lanes per head-row for the 16-byte vector kernels (forward, bucketed scatter).
inline int vec_group(int channels, size_t elem, const Args& a) { return vec_lanes(channels, elem, 16, a); }

// Entry points used by the C-ABI (msda_bucketed.cu): the row-wise kernels, or
// the bucketed backward in builds with MSDA_BUCKETED_BACKWARD=1.
cudaError_t launch_forward(DType dtype, const Dims& d, const Args& a, cudaStream_t stream);
cudaError_t launch_backward(DType dtype, const Dims& d, const Args& a, cudaStream_t stream);

// Backward on caller-provided scratch (used by the static-scratch entry point):
// the scratch bytes the call needs (0 when the bucketed kernels do not apply
// and the scratch-free row-wise kernels run instead), and the launch itself.
size_t backward_scratch_bytes(DType dtype, const Dims& d, const Args& a);
cudaError_t launch_backward_on_scratch(DType dtype, const Dims& d, const Args& a, void* scratch, cudaStream_t stream);

// Deterministic backward (msda_deterministic.cu): grad_value summed in 64-bit
// fixed point on a caller-provided workspace of deterministic_workspace_bytes
// (256-byte aligned), grad_loc / grad_w from the row-wise kernels.
size_t deterministic_workspace_bytes(const Dims& d);
cudaError_t launch_backward_deterministic(DType dtype, const Dims& d, const Args& a, void* workspace,
                                          cudaStream_t stream);

// The fixed per-device scratch array (msda_noalloc.cu).
size_t static_scratch_capacity();
cudaError_t static_scratch_address(void** out);

// Row-wise kernels: one item per lane group in natural (b, q, h) order; any
// channel count (msda_forward.cu, msda_backward.cu).
cudaError_t launch_forward_rowwise(DType dtype, const Dims& d, const Args& a, cudaStream_t stream);
cudaError_t launch_backward_rowwise(DType dtype, const Dims& d, const Args& a, cudaStream_t stream);

// bf16 D = 32 forward with the smallest levels staged in shared memory by TMA
// (msda_staged.cu; opt-in, MUSPACE_FWD_STAGED=1); *used = false when it is off
// or the call does not suit it, and the row-wise kernels take the call.
cudaError_t launch_forward_staged(const Dims& d, const Args& a, cudaStream_t stream, bool* used);
// Copy waits of the staged forward that gave up so far (this device; ~0u when
// it cannot be read).
unsigned int staged_wait_timeouts();
// Fused MSDA forward + rebatch scatter + count normalisation for one camera
// (msda_forward.cu); d describes the rebatched call (batch = B * cams,
// queries = max_len). cudaErrorInvalidValue when the channel count has no
// 16-byte lane layout.
cudaError_t launch_scatter_div(DType dtype, const Dims& d, const SlotDims& sd, const Args& a, const int64_t* index,
                               const void* count, void* slots, cudaStream_t stream);

}  // namespace msda
