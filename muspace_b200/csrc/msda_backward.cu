// MSDA backward on sm_100a.
//
// For every sample (b, q, h, l, p) with attention weight a and incoming
// gradient g[c] = grad_out[b, q, h, c]:
//   grad_value[corner k, c] += w_k * a * g[c]                    (scatter)
//   grad_w[s]               = sum_c g[c] * bilinear_c
//   grad_loc[s]             = (W * a * sum_c g[c] * d bilinear_c / dx,
//                              H * a * sum_c g[c] * d bilinear_c / dy)
// grad_value is accumulated into a caller-zeroed fp32 buffer; grad_loc and
// grad_w are written (every sample, zero when it has no in-bounds corner).
//
// Replaces muSPACE's MUSA backward kernels
// (csrc/ms_deformable_attn/ms_deform_attn_musa_kernel.muh:93-166 and 625-733,
// launched by ms_deform_attn_musa.mu:114-453), which issue 4 x 32 scalar fp32
// atomics per sample from one warp per head-row and serialise location /
// weight loads through lane 0.
//
// B200 design: the same G-lane group per head-row as the forward. Each lane
// scatters its 16-byte channel slice of every in-bounds corner with
// red.global.add.v4.f32 (one vector reduction per 4 channels, no return
// value), so a bf16 D=32 corner costs 8 vector REDs instead of 32 scalar
// atomics. Per sample and corner k each lane forms T_k = sum_c g_c v_k,c over
// its channels (packed fp32x2 FMAs); xor shuffles sum the four T_k over the
// group and one lane derives grad_w and grad_loc from them.
#include "msda_device.cuh"

namespace msda {


// kScatter = false computes grad_loc / grad_w only; grad_value then comes from
// the bucketed scatter kernel (msda_bucketed.cu).
template <typename T, int G, bool kScatter>
__global__ void __launch_bounds__(256, 3) backward_vec_kernel(Dims d, const T* __restrict__ value,
                                                           const int64_t* __restrict__ shapes,
                                                           const int64_t* __restrict__ starts,
                                                           const T* __restrict__ loc, const T* __restrict__ weight,
                                                           const T* __restrict__ grad_out,
                                                           float* __restrict__ grad_value,
                                                           float* __restrict__ grad_loc,
                                                           float* __restrict__ grad_weight,
                                                           const int* __restrict__ order) {
  using V = Vec16<T>;
  constexpr int kVec = V::kLanes;
  extern __shared__ Level levels[];
  stage_levels(levels, shapes, starts, d);

  const int sub = threadIdx.x % G;
  const int groups_per_cta = blockDim.x / G;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int row_stride = d.heads * d.channels;
  const int samples = d.levels * d.points;

  // Every lane of a warp runs the same number of loop trips (whole warps map
  // to whole groups and the trip count only depends on the warp's first
  // item), so the full-mask shuffles below are always convergent.
  const int64_t stride = static_cast<int64_t>(gridDim.x) * groups_per_cta;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * groups_per_cta + threadIdx.x / G;
       item - (threadIdx.x % 32) / G < items; item += stride) {
    const bool live = item < items;
    const int64_t slot = live ? item : items - 1;
    const int64_t it = order ? order[slot] : slot;
    const int h = static_cast<int>(it % d.heads);
    const int64_t b = it / (static_cast<int64_t>(d.queries) * d.heads);
    const int64_t head0 = (b * d.spatial_size) * row_stride + h * d.channels;
    const T* vbase = value + head0 + sub * kVec;
    float* gbase = grad_value + head0;
    const T* lp = loc + it * samples * 2;
    const T* wp = weight + it * samples;

    // g in the lane's 16-byte load slice (for the dot products, as channel
    // pairs) and in the slice it scatters (for grad_value); see RedSlice.
    float g[kVec], gr[kVec];
    const T* grow = grad_out + it * d.channels;
    V::unpack(ld_stream16(grow + sub * kVec, evict_first_policy()), g);
    RedSlice<T, G>::load(grow, sub, g, gr);
    float2 g2[kVec / 2];
#pragma unroll
    for (int i = 0; i < kVec / 2; ++i) g2[i] = make_float2(g[2 * i], g[2 * i + 1]);

    for (int l = 0; l < d.levels; ++l) {
      const Level lv = levels[l];
#pragma unroll 2
      for (int p = 0; p < d.points; ++p) {
        const int s = l * d.points + p;
        const float2 xy = load_loc(lp + 2 * s);
        const float a = to_f32(wp[s]);
        Corners c;
        // T_k = sum_c g_c v_k,c over this lane's channels, one per corner k
        float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const bool valid = live && corners(lv, xy.x, xy.y, c);
        if (valid) {
          uint4 raw[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            raw[k] = c.row[k] >= 0 ? ldg16(vbase + static_cast<int64_t>(c.row[k]) * row_stride)
                                   : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
            float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < kVec / 2; ++i) {
              const float2 v2 = sizeof(T) == 2 ? bf16x2_to_float2(w[i])
                                               : make_float2(__uint_as_float(w[2 * i]), __uint_as_float(w[2 * i + 1]));
              acc = ffma2(g2[i], v2, acc);
            }
            t[k] = acc.x + acc.y;
          }
          if (kScatter) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (c.row[k] < 0) continue;
              RedSlice<T, G>::scatter(gbase + static_cast<int64_t>(c.row[k]) * row_stride, sub, c.w[k] * a, gr);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) t[k] = group_sum<G>(t[k]);
        if (live && sub == 0) {
          // grad_w = sum_k w_k T_k; grad_x = W a (hh (T_01 - T_00) + lh (T_11 - T_10));
          // grad_y = H a (hw (T_10 - T_00) + lw (T_11 - T_01)); zero for a skipped sample
          float gw = 0.0f, gx = 0.0f, gy = 0.0f;
          if (valid) {
            gw = c.w[0] * t[0] + c.w[1] * t[1] + c.w[2] * t[2] + c.w[3] * t[3];
            gx = static_cast<float>(lv.width) * a * (c.hh * (t[1] - t[0]) + c.lh * (t[3] - t[2]));
            gy = static_cast<float>(lv.height) * a * (c.hw * (t[2] - t[0]) + c.lw * (t[3] - t[1]));
          }
          const int64_t so = it * samples + s;
          grad_weight[so] = gw;
          *reinterpret_cast<float2*>(grad_loc + 2 * so) = make_float2(gx, gy);
        }
      }
    }
  }
}

// Any D: one thread per head-row, channels in a loop (no cross-thread
// reduction needed); grad_value through scalar fp32 atomics.
template <typename T>
__global__ void __launch_bounds__(256) backward_scalar_kernel(Dims d, const T* __restrict__ value,
                                                              const int64_t* __restrict__ shapes,
                                                              const int64_t* __restrict__ starts,
                                                              const T* __restrict__ loc,
                                                              const T* __restrict__ weight,
                                                              const T* __restrict__ grad_out,
                                                              float* __restrict__ grad_value,
                                                              float* __restrict__ grad_loc,
                                                              float* __restrict__ grad_weight) {
  extern __shared__ Level levels[];
  stage_levels(levels, shapes, starts, d);
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int row_stride = d.heads * d.channels;
  const int samples = d.levels * d.points;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < items;
       item += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int h = static_cast<int>(item % d.heads);
    const int64_t b = item / (static_cast<int64_t>(d.queries) * d.heads);
    const int64_t vrow0 = (b * d.spatial_size) * row_stride + h * d.channels;
    const T* g = grad_out + item * d.channels;
    for (int l = 0; l < d.levels; ++l) {
      const Level lv = levels[l];
      for (int p = 0; p < d.points; ++p) {
        const int64_t so = item * samples + l * d.points + p;
        const float x = to_f32(loc[2 * so]), y = to_f32(loc[2 * so + 1]);
        const float a = to_f32(weight[so]);
        Corners c;
        float part_w = 0.0f, part_x = 0.0f, part_y = 0.0f;
        if (corners(lv, x, y, c)) {
          for (int ch = 0; ch < d.channels; ++ch) {
            const float gc = to_f32(g[ch]);
            float v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
              v[k] = c.row[k] >= 0 ? to_f32(value[vrow0 + static_cast<int64_t>(c.row[k]) * row_stride + ch]) : 0.0f;
            const float bil = c.w[0] * v[0] + c.w[1] * v[1] + c.w[2] * v[2] + c.w[3] * v[3];
            part_w = fmaf(gc, bil, part_w);
            part_x = fmaf(gc, c.hh * (v[1] - v[0]) + c.lh * (v[3] - v[2]), part_x);
            part_y = fmaf(gc, c.hw * (v[2] - v[0]) + c.lw * (v[3] - v[1]), part_y);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (c.row[k] >= 0)
                atomicAdd(grad_value + vrow0 + static_cast<int64_t>(c.row[k]) * row_stride + ch, c.w[k] * a * gc);
          }
        }
        grad_weight[so] = part_w;
        grad_loc[2 * so] = static_cast<float>(lv.width) * part_x * a;
        grad_loc[2 * so + 1] = static_cast<float>(lv.height) * part_y * a;
      }
    }
  }
}

template <typename T, int G>
static cudaError_t launch_backward_vec(const Dims& d, const Args& a, cudaStream_t stream) {
  constexpr int kThreads = 256;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t groups_per_cta = kThreads / G;
  const int64_t blocks = (items + groups_per_cta - 1) / groups_per_cta;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  auto kernel = a.skip_grad_value ? backward_vec_kernel<T, G, false> : backward_vec_kernel<T, G, true>;
  kernel<<<grid, kThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<const T*>(a.grad_out), a.grad_value, a.grad_loc, a.grad_weight,
      a.order);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_backward_t(const Dims& d, const Args& a, cudaStream_t stream) {
  switch (vec_group(d.channels, sizeof(T), a)) {
    case 1: return launch_backward_vec<T, 1>(d, a, stream);
    case 2: return launch_backward_vec<T, 2>(d, a, stream);
    case 4: return launch_backward_vec<T, 4>(d, a, stream);
    case 8: return launch_backward_vec<T, 8>(d, a, stream);
    case 16: return launch_backward_vec<T, 16>(d, a, stream);
    case 32: return launch_backward_vec<T, 32>(d, a, stream);
    default: break;
  }
  if (a.skip_grad_value) return cudaErrorInvalidValue;  // the scalar kernel always scatters
  constexpr int kThreads = 256;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t blocks = (items + kThreads - 1) / kThreads;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  backward_scalar_kernel<T><<<grid, kThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<const T*>(a.grad_out), a.grad_value, a.grad_loc, a.grad_weight);
  return cudaGetLastError();
}

cudaError_t launch_backward_rowwise(DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0) return cudaSuccess;
  return dtype == DType::kBF16 ? launch_backward_t<__nv_bfloat16>(d, a, stream)
                               : launch_backward_t<float>(d, a, stream);
}

}  // namespace msda
