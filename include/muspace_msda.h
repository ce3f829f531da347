/*
 * muspace_msda.h -- C ABI of the B200 multi-scale deformable attention (MSDA)
 * library, libmuspace_ops.so.
 *
 * The library replaces the MSDA exports of muSPACE's TVM-FFI module
 * (csrc/ms_deformable_attn/ms_deform_attn_musa.mu:627-628): the same two entry
 * points, the same argument order, dtype rules and validation, but bound as
 * plain C over DLPack DLTensor views instead of tvm::ffi::TensorView, plus an
 * explicit CUDA stream and an int status instead of a thrown ICHECK.
 *
 * Conventions shared by every entry point:
 *   - All tensors live on the same CUDA device and are row-major contiguous.
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *     stream) and returns without synchronising. Calls on different streams
 *     are independent; the library keeps no global state besides the
 *     per-thread error message.
 *   - Return 0 on success. On failure nothing is launched, a non-zero
 *     msda_status_t is returned and msda_last_error() describes it.
 *   - value, sampling_locations, attention_weights, output and grad_output
 *     share one storage dtype, float32 or bfloat16; geometry, interpolation
 *     and every sum are evaluated in fp32 whatever the storage dtype.
 *     spatial_shapes and level_start_index are int64; the three gradient
 *     buffers are always float32.
 *   - Layouts: value (B, Lin, Hh, D); spatial_shapes (L, 2) as (H, W);
 *     level_start_index (L); sampling_locations (B, Lq, Hh, L, P, 2) with the
 *     last dim (x, y) in [0, 1]; attention_weights (B, Lq, Hh, L, P);
 *     output / grad_output (B, Lq, Hh * D).
 *   - Sampling follows torch.nn.functional.grid_sample(mode="bilinear",
 *     padding_mode="zeros", align_corners=False): corners outside a level
 *     read as zero and receive no gradient.
 */
#ifndef MUSPACE_MSDA_H_
#define MUSPACE_MSDA_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MSDA_API __attribute__((visibility("default")))
#else
#define MSDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#ifndef DLPACK_DLPACK_H_
/* ABI-compatible subset of DLPack (v0.6 .. v1.x). Include <dlpack/dlpack.h>
 * before this header to use the full definitions instead. */
typedef enum {
  kDLCPU = 1,
  kDLCUDA = 2,
  kDLCUDAHost = 3,
  kDLCUDAManaged = 13,
} DLDeviceType;

typedef struct {
  DLDeviceType device_type;
  int32_t device_id;
} DLDevice;

typedef enum {
  kDLInt = 0U,
  kDLUInt = 1U,
  kDLFloat = 2U,
  kDLBfloat = 4U,
} DLDataTypeCode;

typedef struct {
  uint8_t code;
  uint8_t bits;
  uint16_t lanes;
} DLDataType;

typedef struct {
  void *data;
  DLDevice device;
  int32_t ndim;
  DLDataType dtype;
  int64_t *shape;
  int64_t *strides; /* NULL = compact row-major */
  uint64_t byte_offset;
} DLTensor;
#endif /* DLPACK_DLPACK_H_ */

typedef enum {
  MSDA_STATUS_OK = 0,
  MSDA_STATUS_INVALID_ARGUMENT = 1, /* dtype, device, layout or shape rejected */
  MSDA_STATUS_CUDA_ERROR = 2,       /* the CUDA runtime refused a launch */
} msda_status_t;

typedef enum {
  MSDA_DTYPE_FLOAT32 = 0,
  MSDA_DTYPE_BFLOAT16 = 1,
} msda_dtype_t;

/* Problem sizes for the plain-pointer entry points. */
typedef struct {
  int64_t batch;        /* B   */
  int64_t spatial_size; /* Lin = sum over levels of H * W */
  int64_t heads;        /* Hh  */
  int64_t channels;     /* D   */
  int64_t levels;       /* L   */
  int64_t queries;      /* Lq  */
  int64_t points;       /* P   */
} msda_dims_t;

/*
 * Forward: output = MSDA(value, spatial_shapes, level_start_index,
 * sampling_locations, attention_weights).
 *
 * Replaces ms_deform_attn_forward, csrc/ms_deformable_attn/ms_deform_attn_musa.mu:507-560
 * (same argument order; `stream` is new). As there, B is read from value,
 * L from spatial_shapes, Lq from sampling_locations dim 1 and P from its dim
 * 4, and im2col_step must satisfy step = min(B, im2col_step) > 0 with
 * B % step == 0. The reference launched once per chunk of `step` batch
 * entries; here the whole batch is one launch, which gives the same result.
 */
MSDA_API int ms_deform_attn_forward(const DLTensor *value, const DLTensor *spatial_shapes,
                           const DLTensor *level_start_index, const DLTensor *sampling_locations,
                           const DLTensor *attention_weights, DLTensor *output, int im2col_step,
                           void *stream);

/*
 * Backward.
 *
 * Replaces ms_deform_attn_backward, csrc/ms_deformable_attn/ms_deform_attn_musa.mu:561-626
 * (same argument order; `stream` is new). grad_value, grad_sampling_loc and
 * grad_attn_weight must be float32. As in the reference, grad_value is
 * ACCUMULATED into, so the caller zeroes it first; grad_sampling_loc and
 * grad_attn_weight are overwritten for every sample.
 */
MSDA_API int ms_deform_attn_backward(const DLTensor *value, const DLTensor *spatial_shapes,
                            const DLTensor *level_start_index, const DLTensor *sampling_locations,
                            const DLTensor *attention_weights, const DLTensor *grad_output,
                            DLTensor *grad_value, DLTensor *grad_sampling_loc, DLTensor *grad_attn_weight,
                            int im2col_step, void *stream);

/*
 * Plain-pointer forms of the two calls above for callers without DLPack: raw
 * device pointers plus the sizes in `dims`. They perform the size checks but
 * cannot see devices or strides, so the pointers must be contiguous device
 * memory of the documented shapes on the current device. Same semantics as
 * ms_deform_attn_forward / ms_deform_attn_backward (the reference has no
 * plain-pointer export; these are the pointer-level core both wrap).
 */
MSDA_API int msda_forward(msda_dtype_t dtype, const msda_dims_t *dims, const void *value, const int64_t *spatial_shapes,
                 const int64_t *level_start_index, const void *sampling_locations,
                 const void *attention_weights, void *output, void *stream);

MSDA_API int msda_backward(msda_dtype_t dtype, const msda_dims_t *dims, const void *value, const int64_t *spatial_shapes,
                  const int64_t *level_start_index, const void *sampling_locations,
                  const void *attention_weights, const void *grad_output, float *grad_value,
                  float *grad_sampling_loc, float *grad_attn_weight, void *stream);

/*
 * msda_backward without any device allocation. No counterpart in the
 * reference: this entry point exists for callers that may not allocate GPU
 * memory once they run, such as deployments that plan all device memory
 * before start-up and forbid allocation afterwards (automotive and other
 * real-time inference runtimes), and plugin hosts that own the device memory
 * and do not let a plugin call the CUDA allocator.
 *
 * Same arguments, layouts and results as msda_backward (grad_value is
 * accumulated into, so the caller zeroes it). It runs the bucketed backward
 * (head-rows sorted into spatial buckets, grad_value updates merged per pixel
 * before they are sent), whose bucket plan lives in one fixed 8 MiB array in
 * device memory that this library declares; every GPU that loads the library
 * keeps it until the process exits. It is enough for about one million
 * head-rows (B * Lq * Hh); larger calls are rejected with
 * MSDA_STATUS_INVALID_ARGUMENT and nothing runs. The function allocates
 * nothing: no cudaMalloc, cudaMallocAsync, cudaFree, no allocating library.
 *
 * Cost: the bucketed backward is slower than the fused backward that
 * msda_backward runs by default (measured on B200, bf16, BEVFormer SCA shapes:
 * 2.41 ms against 0.94 ms for 6 camera images, 0.87 against 0.34 ms for 2).
 * msda_backward itself allocates nothing either in a default build (its fused
 * kernels need no work space); only builds with -DMSDA_BUCKETED_BACKWARD=1
 * make it take the bucket plan from the stream-ordered allocator. Callers that
 * merely must not allocate can therefore call msda_backward.
 *
 * The current device must be the device of every pointer and of `stream`:
 * the array's address is the current device's. The call checks the stream's
 * device and value's device against it and returns
 * MSDA_STATUS_INVALID_ARGUMENT (nothing runs) when they differ.
 *
 * The array is shared by every call on a device and keeps the last call's
 * contents; each call clears what must start at zero. Calls whose work
 * overlaps on the GPU (different streams, or different host threads on one
 * device without ordering between them) race on the array: order them on one
 * stream, or synchronise between them.
 *
 * The first call on a device looks up the array's device address (with that
 * device current) and caches it; make that first call before capturing any
 * stream on that device.
 */
MSDA_API int msda_backward_static_scratch(msda_dtype_t dtype, const msda_dims_t *dims, const void *value,
                                          const int64_t *spatial_shapes, const int64_t *level_start_index,
                                          const void *sampling_locations, const void *attention_weights,
                                          const void *grad_output, float *grad_value, float *grad_sampling_loc,
                                          float *grad_attn_weight, void *stream);

/*
 * Deterministic backward (no counterpart in the reference, whose atomicAdd
 * backward is not reproducible either): the same arguments and results as
 * ms_deform_attn_backward / msda_backward, but grad_value is bit-identical
 * from run to run. Contributions to grad_value are summed as 64-bit fixed-point
 * integers (associative, so the order of the additions no longer matters) at a
 * power-of-two scale taken on the device from max |grad_output| and
 * max |attention_weights|, converted back once and added into grad_value;
 * grad_sampling_loc / grad_attn_weight come from the same kernels as the
 * default path, which are already reproducible. The result equals the exactly
 * rounded sum of the fp32 contributions, each kept to 2^-(61 - k) of the
 * largest possible one, k = ceil(log2(Lq * L * P)) + 1. With a non-finite value
 * in grad_output or attention_weights, grad_value receives fp32 atomic
 * additions instead (not reproducible in its finite elements).
 *
 * The caller provides the work space: `workspace` of at least
 * msda_deterministic_workspace_bytes bytes (256 + 8 * B * Lin * Hh * D),
 * 256-byte aligned, uint8 for the DLPack form. The call clears it itself. Calls
 * that share a work space must be ordered on the GPU.
 */
MSDA_API int msda_deterministic_workspace_bytes(const msda_dims_t *dims, size_t *bytes);

MSDA_API int ms_deform_attn_backward_deterministic(const DLTensor *value, const DLTensor *spatial_shapes,
                                                   const DLTensor *level_start_index,
                                                   const DLTensor *sampling_locations,
                                                   const DLTensor *attention_weights, const DLTensor *grad_output,
                                                   DLTensor *grad_value, DLTensor *grad_sampling_loc,
                                                   DLTensor *grad_attn_weight, DLTensor *workspace, int im2col_step,
                                                   void *stream);

MSDA_API int msda_backward_deterministic(msda_dtype_t dtype, const msda_dims_t *dims, const void *value,
                                         const int64_t *spatial_shapes, const int64_t *level_start_index,
                                         const void *sampling_locations, const void *attention_weights,
                                         const void *grad_output, float *grad_value, float *grad_sampling_loc,
                                         float *grad_attn_weight, void *workspace, size_t workspace_bytes,
                                         void *stream);

/*
 * BEVFormer spatial cross-attention, forward fused with the rebatch scatter
 * and the camera-count normalisation, for ONE camera:
 *
 *   for b < B, q < valid_len, h < Hh:
 *     slots[b, index[q], h, :] += MSDA(b * cams + cam_id, q, h) / count[b, index[q]]
 *
 * Replaces ms_deformable_im2col_scatter_div_musa,
 * csrc/ms_deformable_attn/ms_deform_attn_musa.mu:455-505 (kernel
 * ms_deform_attn_musa_kernel.muh:419-486), which the reference compiled but
 * never exported; its argument list (batch_size, num_cams, cam_id,
 * valid_len, max_len, num_query, ...) is read here from the views:
 *   value               (B * cams, Lin, Hh, D)       storage dtype
 *   sampling_locations  (B * cams, max_len, Hh, L, P, 2), attention_weights
 *                       (B * cams, max_len, Hh, L, P): the rebatched queries
 *   index               (valid_len,) int64, valid_len <= max_len: the BEV
 *                       query of each of this camera's first valid_len rows;
 *                       distinct entries (a BEV query appears once per camera)
 *   count               (B, num_query) storage dtype: cameras per BEV query
 *   slots               (B, num_query, Hh * D) storage dtype, updated in place
 * The update is a read-modify-write in the storage dtype (as in the
 * reference), race-free because index holds distinct queries; call the
 * cameras one after another (one stream) to accumulate all of them. An index
 * entry outside [0, num_query) updates nothing. The MSDA term is the same
 * sampling as ms_deform_attn_forward (grid_sample convention). Needs D *
 * element size a multiple of 16 bytes up to 512 (D = 32 in BEVFormer).
 */
MSDA_API int ms_deform_attn_scatter_div_forward(const DLTensor *value, const DLTensor *spatial_shapes,
                                               const DLTensor *level_start_index, const DLTensor *sampling_locations,
                                               const DLTensor *attention_weights, const DLTensor *index,
                                               const DLTensor *count, DLTensor *slots, int cam_id, void *stream);

/* Sizes of the rebatch side of the fused scatter (plain-pointer form). */
typedef struct {
  int64_t batch;     /* B: batch entries (count / slots dim 0) */
  int64_t cams;      /* cameras per batch entry; dims->batch = batch * cams */
  int64_t cam;       /* the camera of this call */
  int64_t valid_len; /* rows of this camera that carry a BEV query (index length) */
  int64_t num_query; /* BEV queries (count / slots dim 1) */
} msda_slot_dims_t;

/* Plain-pointer form of ms_deform_attn_scatter_div_forward; dims describes the
 * rebatched MSDA call (batch = B * cams, queries = max_len). */
MSDA_API int msda_scatter_div_forward(msda_dtype_t dtype, const msda_dims_t *dims, const msda_slot_dims_t *slot_dims,
                                      const void *value, const int64_t *spatial_shapes,
                                      const int64_t *level_start_index, const void *sampling_locations,
                                      const void *attention_weights, const int64_t *index, const void *count,
                                      void *slots, void *stream);

/*
 * SparseDrive deformable aggregation (multi-camera, multi-scale feature
 * gather with per-group weights), float32:
 *
 *   output[b, a, :] = sum over (pt, cam) whose sampling_location lies in the
 *                     open square (0, 1)^2, and over scales s, of
 *                     weights[b, a, pt, cam, s, group] * bilinear(map(cam, s), location)
 *
 * with the bilinear sample at h = y * H - 0.5, w = x * W - 0.5 and corners
 * outside the map read as zero. Layouts (contiguous):
 *   mc_ms_feat          [B, num_feat, C]                  float32
 *   spatial_shape       [num_cams, num_scale, 2]          int32 (H, W)
 *   scale_start_index   [num_cams, num_scale]             int32 (first row of each map)
 *   sampling_location   [B, anchors, pts, num_cams, 2]    float32 (x, y)
 *   weights             [B, anchors, pts, num_cams, num_scale, groups], 1 <= groups <= 8, C % groups == 0
 *   output              [B, anchors, C]                   float32, overwritten
 *
 * Replace the reference exports of the same names and argument order
 * (csrc/deformable_aggregation/deformable_aggregation_musa.mu:718-751;
 * `stream` is new). *_opt run the warp-per-anchor kernels when
 * C % 4 == 0, C <= 512, C / groups is 4 times a power of two and the float
 * tensors are 16-byte aligned, the scalar kernels otherwise; *_base always run
 * the scalar kernels (the reference's baseline pair, kept for comparison).
 *
 * Backward: grad_mc_ms_feat is ACCUMULATED into (the caller zeroes it, as the
 * reference's Python layer does); grad_sampling_location and grad_weights are
 * written for every entry (zero where the location is outside the image).
 */
MSDA_API int deformable_aggregation_forward_opt(const DLTensor *mc_ms_feat, const DLTensor *spatial_shape,
                                                const DLTensor *scale_start_index, const DLTensor *sampling_location,
                                                const DLTensor *weights, DLTensor *output, void *stream);
MSDA_API int deformable_aggregation_forward_base(const DLTensor *mc_ms_feat, const DLTensor *spatial_shape,
                                                 const DLTensor *scale_start_index, const DLTensor *sampling_location,
                                                 const DLTensor *weights, DLTensor *output, void *stream);
MSDA_API int deformable_aggregation_backward_opt(const DLTensor *mc_ms_feat, const DLTensor *spatial_shape,
                                                 const DLTensor *scale_start_index, const DLTensor *sampling_location,
                                                 const DLTensor *weights, const DLTensor *grad_output,
                                                 DLTensor *grad_mc_ms_feat, DLTensor *grad_sampling_location,
                                                 DLTensor *grad_weights, void *stream);
MSDA_API int deformable_aggregation_backward_base(const DLTensor *mc_ms_feat, const DLTensor *spatial_shape,
                                                  const DLTensor *scale_start_index, const DLTensor *sampling_location,
                                                  const DLTensor *weights, const DLTensor *grad_output,
                                                  DLTensor *grad_mc_ms_feat, DLTensor *grad_sampling_location,
                                                  DLTensor *grad_weights, void *stream);

/*
 * FlashSCA (flash_bevpool_sca): BEVFormer spatial cross-attention without the
 * rebatching, float32. For every BEV cell (gy x gx) the voxel centre at each of
 * gz heights is projected into every camera (image = P [x y z 1], depth > 0,
 * u = row0 / max(depth, eps), landing in [0, W) x [0, H)); the cell's output
 * channel c sums, over the landing (camera, height) pairs, the levels and the
 * points of head(c), weight * bilinear(level map, base + offset) with
 * base = (u / W * w - 0.5, v / H * h - 0.5), zero padding and non-finite
 * feature values read as 0, divided by the number of cameras in which any
 * height lands.
 *   value               [B, N, S, C]                         float32
 *   projection_matrices [B, N, 3, 4]                         float32
 *   spatial_shapes      [L, 2] int32 (h, w); level_start_index [L] int32; image_size [2] int32 (H, W)
 *   sampling_offsets    [B, gy, gx, heads, L, P, gz, 2]      float32 (level pixels)
 *   attention_weights   [B, gy, gx, heads, L, P, gz]         float32
 *   out                 [B, gy, gx, C]                       float32, overwritten
 * Replace the reference exports of the same names and argument order
 * (csrc/flashbev/flash_bevpool_sca_musa.mu:262-399; `stream` is new). The
 * backward reads the voxel grid from roi_range [xmin, xmax, ymin, ymax, zmin,
 * zmax] as the reference does and ACCUMULATES into value_grad,
 * sampling_offsets_grad and attention_weights_grad (the caller zeroes them).
 * value_stride_n is validated (1 <= it <= S) but rows are addressed with the
 * tensor's own S, as the reference's PyTorch path does. Limits: C / heads =
 * 4 * {1, 2, 4, 8, 16, 32}, N * gz <= 64, L <= 16.
 */
MSDA_API int flash_bevpool_sca_forward(const DLTensor *value, const DLTensor *projection_matrices,
                                       const DLTensor *spatial_shapes, const DLTensor *level_start_index,
                                       const DLTensor *image_size, const DLTensor *sampling_offsets,
                                       const DLTensor *attention_weights, DLTensor *out, int num_heads,
                                       int num_points, int grid_x, int grid_y, int grid_z, float voxel_size_x,
                                       float voxel_size_y, float voxel_size_z, float voxel_x_min, float voxel_y_min,
                                       float voxel_z_min, int value_stride_n, float epsilon, void *stream);
MSDA_API int flash_bevpool_sca_backward(const DLTensor *out_grad, const DLTensor *value,
                                        const DLTensor *projection_matrices, const DLTensor *spatial_shapes,
                                        const DLTensor *level_start_index, const DLTensor *image_size,
                                        const DLTensor *roi_range, const DLTensor *sampling_offsets,
                                        const DLTensor *attention_weights, DLTensor *value_grad,
                                        DLTensor *sampling_offsets_grad, DLTensor *attention_weights_grad,
                                        int num_heads, int num_points, int grid_x, int grid_y, int grid_z,
                                        int value_stride_n, float epsilon, void *stream);

/* Message of the last failed call on this thread ("" after a success). The
 * reference raised it as a TVM-FFI exception (csrc/ffi/tensor_utils.hpp:13-34). */
MSDA_API const char *msda_last_error(void);

/* Waits of the staged bf16 forward (opt-in through MUSPACE_FWD_STAGED=1: the
 * kernel that copies each head's smallest levels into shared memory with TMA;
 * measured slower than the default forward) that gave up on the copies on the current
 * device since the library loaded; such a thread reads the rows from global
 * memory instead, so results are unchanged. A diagnostic: 0 is expected.
 * Returns MSDA_STATUS_CUDA_ERROR when the counter cannot be read. */
MSDA_API int msda_stage_wait_timeouts(unsigned int *count);

/* Library version string, "<major>.<minor>.<patch>". */
MSDA_API const char *msda_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MUSPACE_MSDA_H_ */
