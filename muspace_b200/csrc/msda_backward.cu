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
// B200 design. A group of G lanes owns a head-row; each lane holds kBytes of
// its channels (bf16: 8 bytes = 4 channels, fp32: 16 bytes = 4 channels, so
// bf16 D = 32 runs 8 lanes and one RED instruction of the group covers the
// corner's whole 128-byte fp32 grad_value line). Samples are taken in chunks
// of C = min(G, 4) (2 for fp32): the lane at sub = i * G / C computes the geometry of
// chunk sample i once and stages its corner rows and w_k * a in shared
// memory. Every lane then, per sample, gathers its slice of the four corners,
// forms the corner dots T_k = sum_c g_c v_k,c over its channels (packed fp32x2
// FMAs) and scatters w_k * a * g with red.global.add.v4.f32 (no return value).
// A transpose reduction hands each staging lane the four T_k of its own sample,
// from which it writes
//   grad_w = sum_k w_k T_k,
//   grad_x = W a (hh (T_1 - T_0) + lh (T_3 - T_2)),
//   grad_y = H a (hw (T_2 - T_0) + lw (T_3 - T_1)),
// so the C staging lanes of a group store C consecutive samples' gradients.
#include "msda_device.cuh"

namespace msda {

#ifndef MSDA_BWD_CHUNK_F32
#define MSDA_BWD_CHUNK_F32 2
#endif
#ifndef MSDA_BWD_MINBLOCKS_F32
#define MSDA_BWD_MINBLOCKS_F32 3
#endif
// Samples staged per chunk (the partial dots of a chunk live in registers:
// 4 per sample) and CTAs per SM the register budget is sized for; measured
// on B200 (fp32 D = 32: chunk 2 at 3 CTAs/SM beats chunk 4 at 2 or 3).
template <typename T>
constexpr int kChunk = sizeof(T) == 2 ? 4 : MSDA_BWD_CHUNK_F32;
template <typename T, int kBytes>
constexpr int kMinBlocks = sizeof(T) == 2 ? (kBytes == 8 ? 3 : 2) : MSDA_BWD_MINBLOCKS_F32;

// kScatter = false computes grad_loc / grad_w only; grad_value then comes from
// the bucketed scatter kernel (msda_bucketed.cu).
template <typename T, int G, int kBytes, bool kScatter>
__global__ void __launch_bounds__(kCtaThreads, kMinBlocks<T, kBytes>) backward_vec_kernel(Dims d, const T* __restrict__ value,
                                                                      const int64_t* __restrict__ shapes,
                                                                      const int64_t* __restrict__ starts,
                                                                      const T* __restrict__ loc,
                                                                      const T* __restrict__ weight,
                                                                      const T* __restrict__ grad_out,
                                                                      float* __restrict__ grad_value,
                                                                      float* __restrict__ grad_loc,
                                                                      float* __restrict__ grad_weight,
                                                                      const int* __restrict__ order) {
  using S = Slice<T, kBytes>;
  constexpr int kCh = S::kChannels, kPairs = S::kPairs, kWords = kBytes / 4;
  constexpr int C = Chunk<G, kChunk<T>>::kSamples, kOwn = Chunk<G, kChunk<T>>::kStagerStride;
  constexpr int kGroups = kCtaThreads / G;
  extern __shared__ Level levels[];
  __shared__ int4 s_row[kCtaThreads];
  __shared__ float4 s_wa[kCtaThreads];
  stage_levels(levels, shapes, starts, d);

  const int sub = threadIdx.x % G;
  const int base = threadIdx.x - sub;
  const bool stager = sub % kOwn == 0;
  const int mine = sub / kOwn;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int row_stride = d.heads * d.channels;
  const int samples = d.levels * d.points;

  // Whole warps take the same number of trips (the trip count depends only on
  // the warp's first item), so the full-mask shuffles and warp syncs below
  // are always convergent.
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kGroups;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * kGroups + threadIdx.x / G;
       item - (threadIdx.x % 32) / G < items; item += stride) {
    const bool live = item < items;
    const int64_t slot = live ? item : items - 1;
    const int64_t it = order ? order[slot] : slot;
    const int h = static_cast<int>(it % d.heads);
    const int64_t b = it / (static_cast<int64_t>(d.queries) * d.heads);
    const int64_t head0 = (b * d.spatial_size) * row_stride + h * d.channels + sub * kCh;
    const T* vbase = value + head0;
    float* gbase = grad_value + head0;
    const T* lp = loc + it * samples * 2;
    const T* wp = weight + it * samples;

    float2 g2[kPairs];
    {
      const Words<kWords> graw = ld_stream_words<kBytes>(grad_out + it * d.channels + sub * kCh, evict_first_policy());
#pragma unroll
      for (int q = 0; q < kPairs; ++q) g2[q] = S::pair(graw, q);
    }

    for (int s0 = 0; s0 < samples; s0 += C) {
      float4 geo = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      bool valid = false;
      if (stager) valid = stage_sample(levels, d.points, samples, live, s0 + mine, lp, wp, s_row + threadIdx.x,
                                       s_wa + threadIdx.x, &geo);
      __syncwarp();
      float t[C][4];
#pragma unroll
      for (int i = 0; i < C; ++i) {
        const int4 r4 = s_row[base + i * kOwn];
        const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
        Words<kWords> raw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          raw[k] = rows[k] >= 0 ? ldg_words<kBytes>(vbase + static_cast<int64_t>(rows[k]) * row_stride)
                                : zero_words<kWords>();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int q = 0; q < kPairs; ++q) acc = ffma2(g2[q], S::pair(raw[k], q), acc);
          t[i][k] = acc.x + acc.y;
        }
        if constexpr (kScatter) {
          const float4 w4 = s_wa[base + i * kOwn];
          const float wa[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (rows[k] >= 0) scatter_slice<kPairs>(gbase + static_cast<int64_t>(rows[k]) * row_stride, wa[k], g2);
        }
      }
      __syncwarp();  // the next chunk's staging overwrites the slots read above
      reduce_to_stagers<G, C>(t, sub);
      const int s = s0 + mine;
      if (stager && live && s < samples) {
        float gw = 0.0f, gx = 0.0f, gy = 0.0f;
        if (valid) {
          const Level lv = levels[s / d.points];
          const float lh = geo.x, lw = geo.y, a = geo.z;
          const float hh = __fsub_rn(1.0f, lh), hw = __fsub_rn(1.0f, lw);
          const float* tt = t[0];
          gw = __fmul_rn(hh, hw) * tt[0] + __fmul_rn(hh, lw) * tt[1] + __fmul_rn(lh, hw) * tt[2] +
               __fmul_rn(lh, lw) * tt[3];
          gx = static_cast<float>(lv.width) * a * (hh * (tt[1] - tt[0]) + lh * (tt[3] - tt[2]));
          gy = static_cast<float>(lv.height) * a * (hw * (tt[2] - tt[0]) + lw * (tt[3] - tt[1]));
        }
        const int64_t so = it * samples + s;
        grad_weight[so] = gw;
        *reinterpret_cast<float2*>(grad_loc + 2 * so) = make_float2(gx, gy);
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

template <typename T, int G, int kBytes>
static cudaError_t launch_backward_vec(const Dims& d, const Args& a, cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t groups_per_cta = kCtaThreads / G;
  const int64_t blocks = (items + groups_per_cta - 1) / groups_per_cta;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  auto kernel = a.skip_grad_value ? backward_vec_kernel<T, G, kBytes, false> : backward_vec_kernel<T, G, kBytes, true>;
  kernel<<<grid, kCtaThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<const T*>(a.grad_out), a.grad_value, a.grad_loc, a.grad_weight,
      a.order);
  return cudaGetLastError();
}

template <typename T, int kBytes>
static cudaError_t launch_backward_lanes(int g, const Dims& d, const Args& a, cudaStream_t stream) {
  switch (g) {
    case 1: return launch_backward_vec<T, 1, kBytes>(d, a, stream);
    case 2: return launch_backward_vec<T, 2, kBytes>(d, a, stream);
    case 4: return launch_backward_vec<T, 4, kBytes>(d, a, stream);
    case 8: return launch_backward_vec<T, 8, kBytes>(d, a, stream);
    case 16: return launch_backward_vec<T, 16, kBytes>(d, a, stream);
    case 32: return launch_backward_vec<T, 32, kBytes>(d, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_backward_t(const Dims& d, const Args& a, cudaStream_t stream) {
  // bf16: 8-byte lanes (4 channels, whole-line REDs) up to D = 128, 16-byte
  // lanes for D = 256; fp32: 16-byte lanes (4 channels).
  if constexpr (sizeof(T) == 2) {
    if (const int g = vec_lanes(d.channels, sizeof(T), 8, a)) return launch_backward_lanes<T, 8>(g, d, a, stream);
    if (vec_lanes(d.channels, sizeof(T), 16, a) == 32) return launch_backward_vec<T, 32, 16>(d, a, stream);
  } else {
    if (const int g = vec_lanes(d.channels, sizeof(T), 16, a)) return launch_backward_lanes<T, 16>(g, d, a, stream);
  }
  if (a.skip_grad_value) return cudaErrorInvalidValue;  // the scalar kernel always scatters
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t blocks = (items + kCtaThreads - 1) / kCtaThreads;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  backward_scalar_kernel<T><<<grid, kCtaThreads, level_smem(d), stream>>>(
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
