// Host-side interface of the FlashSCA kernels (flash_sca.cu).
//
// FlashSCA is BEVFormer's spatial cross-attention without the rebatching: for
// every BEV cell the voxel centre at each height is projected into every
// camera, and the cell's queries sample the cameras' multi-level feature maps
// around the projections (mu_space/ops/flashbev.py:368-454,
// csrc/flashbev/flash_bevpool_sca_musa.mu). Layouts (contiguous):
//   value               [B, cams, S, C]         float32 (S >= every level's end)
//   projection          [B, cams, 3, 4]         float32 (image = P [x y z 1])
//   spatial_shapes      [L, 2] int32 (h, w);  level_start [L] int32;  image_size [2] int32 (H, W)
//   sampling_offsets    [B, gy, gx, heads, L, P, gz, 2]   float32 (pixels of the level)
//   attention_weights   [B, gy, gx, heads, L, P, gz]      float32
//   output              [B, gy, gx, C]          float32
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fsca {

struct Dims {
  int batch, cams, stride_n, channels, levels, heads, points;
  int gx, gy, gz;
  // ceil(2^32 / d) for d = points and d = levels * points, set by the host
  // where a multiply-high by it equals the division for every sample index the
  // kernels divide (kMaxPairs pairs of levels * points samples); 0: divide
  uint32_t points_magic, lp_magic;
};

// Voxel grid: centre of cell (ix, iy, iz) = min + (i + 0.5) * size. The
// forward takes it as numbers; the backward, like the reference, reads the
// 6-float roi [xmin, xmax, ymin, ymax, zmin, zmax] from device memory and
// derives size = (max - min) / g.
struct Grid {
  float sx, sy, sz, xmin, ymin, zmin;
};

struct Args {
  const float* value;
  const float* projection;
  const int* shapes;
  const int* starts;
  const int* image_size;
  const float* offsets;
  const float* weights;
  const float* roi;          // backward only
  float* out;                // forward
  const float* grad_out;     // backward
  float* grad_value;         // accumulated into
  float* grad_offsets;       // accumulated into
  float* grad_weights;       // accumulated into
};

// Lanes per head for the channel count, or 0 when it is unsupported (C / heads
// must be 4 * {1, 2, 4, 8, 16, 32} with 16-byte aligned float tensors).
int lanes_per_head(const Dims& d, const Args& a, bool backward);

cudaError_t forward(const Dims& d, const Grid& g, float epsilon, const Args& a, cudaStream_t stream);
cudaError_t backward(const Dims& d, float epsilon, const Args& a, cudaStream_t stream);

// Limits of the kernels' per-cell tables.
constexpr int kMaxPairs = 64;   // cams * gz
constexpr int kMaxLevels = 16;

}  // namespace fsca
