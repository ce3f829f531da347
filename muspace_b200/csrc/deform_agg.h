// Host-side interface of the deformable-aggregation kernels (deform_agg.cu).
//
// SparseDrive's multi-camera, multi-scale deformable feature aggregation, as
// muSPACE defines it (mu_space/ops/deformable_aggregation.py:113-156 for the
// semantics, csrc/deformable_aggregation/deformable_aggregation_musa.mu for
// the kernels). Layouts (row-major, contiguous, fp32 / int32):
//   mc_ms_feat         (B, num_feat, C)                    features of every camera and scale
//   spatial_shape      (cams, scales, 2)  int32            (H, W) per camera and scale
//   scale_start_index  (cams, scales)     int32            first row of each map in mc_ms_feat
//   sampling_location  (B, anchors, pts, cams, 2)          (x, y) normalised to the image
//   weights            (B, anchors, pts, cams, scales, groups)
//   output             (B, anchors, C)
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace da {

struct Dims {
  int batch, num_feat, channels, cams, scales, anchors, pts, groups;
};

struct Args {
  const float* feat;
  const int* shape;
  const int* start;
  const float* loc;
  const float* weights;
  float* out;              // forward: written
  const float* grad_out;   // backward
  float* grad_feat;        // accumulated into (the caller zeroes it)
  float* grad_loc;         // written for every (anchor, pt, cam)
  float* grad_weights;     // written for every (anchor, pt, cam, scale, group)
};

// optimized = the warp-per-anchor vector kernels when the shape allows
// (C a multiple of 4 up to 512, C / groups a multiple of 4 whose quarter is a
// power of two, 16-byte aligned tensors), else the scalar kernels;
// optimized = false always takes the scalar kernels.
cudaError_t forward(const Dims& d, const Args& a, bool optimized, cudaStream_t stream);
cudaError_t backward(const Dims& d, const Args& a, bool optimized, cudaStream_t stream);

}  // namespace da
