// MSDA forward on sm_100a.
//
// out[b, q, h, c] = sum_l sum_p  a[b,q,h,l,p] * bilinear(value_l[b, :, :, h, c], x, y)
//
// Replaces the MUSA forward kernels of muSPACE
// (csrc/ms_deformable_attn/ms_deform_attn_musa_kernel.muh:243-417, launched by
// ms_deform_attn_musa.mu:47-112), which run one thread per output channel and
// make every lane re-read the sample's location and weight.
//
// B200 design. One work item is one (b, q, h) head-row of D channels; a group
// of G = D * sizeof(T) / 16 lanes owns it and each lane holds 16 bytes of
// channels (8 bf16 or 4 fp32). For D = 32 that is 4 lanes (bf16) or 8 lanes
// (fp32), so a warp runs 8 or 4 head-rows at once and every corner gather is
// one 16-byte load per lane, 64 / 128 contiguous bytes per group.
//
// The sample geometry (level, unnormalised coordinate, the four corner rows
// and bilinear weights) is the same for every lane of a group, so it is not
// computed G times: the samples are taken in chunks of 8 (4 for head-rows of
// at most 4 samples; at most 4 G), lane sub computes samples sub, sub + G, ...
// of the chunk and stages their four corner rows and w_k * a in shared
// memory, and the whole group then reads them back (one broadcast load each)
// while it gathers. Items are ordered
// batch-major, so at any moment the CTAs in flight gather from one or two
// cameras' value maps, which stay resident in L2. Any other D takes the
// scalar kernel below.
#include "msda_device.cuh"

namespace msda {

#ifndef MSDA_FWD_PACKED
#define MSDA_FWD_PACKED 1
#endif
// CTAs per SM the forward's register budget is sized for: occupancy pays
// (5 x 256 threads at <= 48 registers, bf16 D = 32 without spills; c4 forward
// 2.40 -> 2.36 ms against 4 x 256 at 64, bevformer-1l fp32 unchanged).
#ifndef MSDA_FWD_MINBLOCKS
#define MSDA_FWD_MINBLOCKS 5
#endif
// Samples of a chunk whose corner gathers are issued together (the loads of
// the unrolled samples are in flight at once).
#ifndef MSDA_FWD_UNROLL
#define MSDA_FWD_UNROLL 1
#endif
constexpr int kFwdUnroll = MSDA_FWD_UNROLL;

// Samples staged per chunk by the forward kernels (lane sub stages samples
// sub, sub + G, ... of the chunk), and their shared slots: one per sample plus
// one of padding per group, so the groups of a warp reading slot i at once hit
// different shared-memory banks.
#ifndef MSDA_FWD_CHUNK
#define MSDA_FWD_CHUNK 8
#endif
template <int G, int kChunk = MSDA_FWD_CHUNK>
struct FwdSlots {  // 1-lane groups (256 per CTA) stage 4 samples so the slots fit 48 KB
  static constexpr int kSamples = kChunk < 4 * G ? kChunk : 4 * G;
  static constexpr int kPerGroup = kSamples + 1;
};

// Lane bytes of the forward for bf16 / fp32 storage (16: one 16-byte load per
// corner; 32: two, half the lanes per head-row).
// 1: corners outside their level are gathered from an in-level row of the same
// sample with weight 0 instead of being skipped (no compare and zero-fill per
// corner); a head-row whose sum comes out non-finite (which a non-finite
// value read that way could cause) is summed again the exact way.
#ifndef MSDA_FWD_SUBST
#define MSDA_FWD_SUBST 1
#endif
// Bytes of channels per lane (16 or 32; 32 falls back to 16 where D or the
// alignment does not allow it). Measured on B200: bf16 16 (32 was slower at
// c4); fp32 32 (bevformer-1l forward 0.153 -> 0.119 ms, c1 0.191 -> 0.188 ms).
#ifndef MSDA_FWD_LANE_BYTES_BF16
#define MSDA_FWD_LANE_BYTES_BF16 16
#endif
#ifndef MSDA_FWD_LANE_BYTES_F32
#define MSDA_FWD_LANE_BYTES_F32 32
#endif

// The staged corners of a sample for the substituting gather: every corner
// outside its level takes the row of an in-level corner of the same sample
// (row 0 of the map when it has none, which the caller guarantees exists) and
// weight 0, so every corner can be loaded unconditionally.
__device__ __forceinline__ void substitute_outside_corners(int4* row, float4* wa) {
  int4 r = *row;
  float4 w = *wa;
  const int any = r.x >= 0 ? r.x : r.y >= 0 ? r.y : r.z >= 0 ? r.z : r.w >= 0 ? r.w : 0;
  if (r.x < 0) r.x = any, w.x = 0.0f;
  if (r.y < 0) r.y = any, w.y = 0.0f;
  if (r.z < 0) r.z = any, w.z = 0.0f;
  if (r.w < 0) r.w = any, w.w = 0.0f;
  *row = r;
  *wa = w;
}

// acc (this lane's channel pairs) += sum over the head-row's samples of
// sum_k (w_k a) v_k. vbase points at the lane's channel slice of pixel 0 of
// the head's value map; lp / wp at the head-row's locations / weights; row /
// wa at the group's staging slots. Every lane of the warp must call it (it
// syncs the warp), live = false for a lane group without an item.
// kSubst: the staged corners outside their level are substituted
// (substitute_outside_corners) and every corner is loaded.
template <typename T, int G, int kBytes, int kChunk = MSDA_FWD_CHUNK, bool kSubst = false>
__device__ __forceinline__ void gather_head_row(const Level* levels, LevelOf level, int samples, bool live,
                                                const T* vbase, int row_stride, const T* lp, const T* wp, int sub,
                                                int4* row, float4* wa, float2 (&acc)[Slice<T, kBytes>::kPairs]) {
  using S = Slice<T, kBytes>;
  constexpr int kPairs = S::kPairs, kWords = kBytes / 4;
  constexpr int C = FwdSlots<G, kChunk>::kSamples;
#pragma unroll
  for (int i = 0; i < kPairs; ++i) acc[i] = make_float2(0.0f, 0.0f);
  for (int s0 = 0; s0 < samples; s0 += C) {
#pragma unroll
    for (int i = sub; i < C; i += G) {
      stage_sample(levels, level, samples, live, s0 + i, lp, wp, row + i, wa + i);
      if constexpr (kSubst) substitute_outside_corners(row + i, wa + i);
    }
    __syncwarp();
#pragma unroll kFwdUnroll
    for (int i = 0; i < C; ++i) {
      const int4 r4 = row[i];
      const float4 w4 = wa[i];
      const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
      const float was[4] = {w4.x, w4.y, w4.z, w4.w};
      Words<kWords> raw[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if constexpr (kSubst)
          raw[k] = ldg_words<kBytes>(vbase + static_cast<int64_t>(rows[k]) * row_stride);
        else
          raw[k] = rows[k] >= 0 ? ldg_words<kBytes>(vbase + static_cast<int64_t>(rows[k]) * row_stride)
                                : zero_words<kWords>();
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
#if MSDA_FWD_PACKED
        const float2 w2 = make_float2(was[k], was[k]);
#pragma unroll
        for (int q = 0; q < kPairs; ++q) acc[q] = ffma2(w2, S::pair(raw[k], q), acc[q]);
#else
#pragma unroll
        for (int q = 0; q < kPairs; ++q) {
          const float2 v = S::pair(raw[k], q);
          acc[q].x = fmaf(was[k], v.x, acc[q].x);
          acc[q].y = fmaf(was[k], v.y, acc[q].y);
        }
#endif
      }
    }
    __syncwarp();
  }
}

template <typename T, int G, int kBytes, int kChunk>
__global__ void __launch_bounds__(kCtaThreads, MSDA_FWD_MINBLOCKS) forward_vec_kernel(
    Dims d, const T* __restrict__ value, const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts,
    const T* __restrict__ loc, const T* __restrict__ weight, T* __restrict__ out, const int* __restrict__ order) {
  using S = Slice<T, kBytes>;
  constexpr int kCh = S::kChannels, kPairs = S::kPairs;
  constexpr int kGroups = kCtaThreads / G;
  using Slots = FwdSlots<G, kChunk>;
  extern __shared__ Level levels[];
  __shared__ int4 s_row[kGroups * Slots::kPerGroup];
  __shared__ float4 s_wa[kGroups * Slots::kPerGroup];
  stage_levels(levels, shapes, starts, d);

  const int sub = threadIdx.x % G;
  const int base = (threadIdx.x / G) * Slots::kPerGroup;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int row_stride = d.heads * d.channels;  // elements between neighbouring pixels
  const int samples = d.levels * d.points;

  // Whole warps take the same number of trips (the trip count depends only on
  // the warp's first item), so the warp-wide syncs are convergent.
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kGroups;
  for (int64_t slot = static_cast<int64_t>(blockIdx.x) * kGroups + threadIdx.x / G;
       slot - (threadIdx.x % 32) / G < items; slot += stride) {
    const bool live = slot < items;
    const int64_t item = order ? order[live ? slot : items - 1] : (live ? slot : items - 1);
    const ImageHead ih = image_head(item, d, items < (int64_t{1} << 31));
    const int h = ih.h;
    const int64_t b = ih.b;
    const T* vbase = value + (b * d.spatial_size) * row_stride + h * d.channels + sub * kCh;
    float2 acc[kPairs];
    const T* lp = loc + item * samples * 2;
    const T* wp = weight + item * samples;
    // substituting needs a row 0 to fall back on (an empty value map has none);
    // it measured faster for bf16 only (c4 forward 2.49 -> 2.40 ms; c1 fp32
    // 0.190 -> 0.198 ms)
    bool exact = !(MSDA_FWD_SUBST && sizeof(T) == 2) || d.spatial_size == 0;
    if (!exact) {
      gather_head_row<T, G, kBytes, kChunk, true>(levels, level_of(d), samples, live, vbase, row_stride, lp, wp, sub,
                                                  s_row + base, s_wa + base, acc);
      exact = __any_sync(0xffffffffu, live && !finite_pairs(acc));  // warp-uniform, rare
    }
    if (exact)
      gather_head_row<T, G, kBytes, kChunk>(levels, level_of(d), samples, live, vbase, row_stride, lp, wp, sub,
                                            s_row + base, s_wa + base, acc);
    if (live) store_slice<T, kBytes>(out + item * d.channels + sub * kCh, acc);
  }
}

// BEVFormer spatial cross-attention, forward fused with the rebatch scatter
// and the camera-count normalisation, for one camera: for every batch entry
// b, rebatched query q < valid_len of camera cam and head h,
//   slots[b, index[q], h, :] += msda(b * cams + cam, q, h) / count[b, index[q]]
// (read-modify-write in the storage dtype: index holds distinct BEV queries,
// so no two items of a launch share a slot row). Locations / weights are the
// rebatched (B * cams, max_len, Hh, L, P[, 2]) tensors; an index outside
// [0, num_query) leaves its rows untouched.
template <typename T, int G>
__global__ void __launch_bounds__(kCtaThreads) scatter_div_vec_kernel(
    Dims d, SlotDims sd, const T* __restrict__ value, const int64_t* __restrict__ shapes,
    const int64_t* __restrict__ starts, const T* __restrict__ loc, const T* __restrict__ weight,
    const int64_t* __restrict__ index, const T* __restrict__ count, T* __restrict__ slots) {
  using S = Slice<T, 16>;
  constexpr int kCh = S::kChannels, kPairs = S::kPairs;
  constexpr int kGroups = kCtaThreads / G;
  extern __shared__ Level levels[];
  __shared__ int4 s_row[kGroups * FwdSlots<G>::kPerGroup];
  __shared__ float4 s_wa[kGroups * FwdSlots<G>::kPerGroup];
  stage_levels(levels, shapes, starts, d);

  const int sub = threadIdx.x % G;
  const int base = (threadIdx.x / G) * FwdSlots<G>::kPerGroup;
  const int64_t items = static_cast<int64_t>(sd.batch) * sd.valid_len * d.heads;
  const int row_stride = d.heads * d.channels;
  const int samples = d.levels * d.points;

  const int64_t stride = static_cast<int64_t>(gridDim.x) * kGroups;
  for (int64_t slot = static_cast<int64_t>(blockIdx.x) * kGroups + threadIdx.x / G;
       slot - (threadIdx.x % 32) / G < items; slot += stride) {
    const bool live = slot < items;
    const int64_t item = live ? slot : items - 1;
    const int h = static_cast<int>(item % d.heads);
    const int64_t bq = item / d.heads;
    const int64_t q = bq % sd.valid_len;
    const int64_t b = bq / sd.valid_len;
    const int64_t image = b * sd.cams + sd.cam;
    const int64_t lrow = (image * d.queries + q) * d.heads + h;  // rebatched (image, q, h) row
    const T* vbase = value + (image * d.spatial_size) * row_stride + h * d.channels + sub * kCh;
    float2 acc[kPairs];
    const T* lp = loc + lrow * samples * 2;
    const T* wp = weight + lrow * samples;
    // substituted out-of-level corners as in forward_vec_kernel (bf16 only)
    bool exact = !(MSDA_FWD_SUBST && sizeof(T) == 2) || d.spatial_size == 0;
    if (!exact) {
      gather_head_row<T, G, 16, MSDA_FWD_CHUNK, true>(levels, level_of(d), samples, live, vbase, row_stride, lp, wp, sub,
                                                      s_row + base, s_wa + base, acc);
      exact = __any_sync(0xffffffffu, live && !finite_pairs(acc));
    }
    if (exact)
      gather_head_row<T, G, 16>(levels, level_of(d), samples, live, vbase, row_stride, lp, wp, sub, s_row + base,
                                s_wa + base, acc);
    const int64_t bev = index[q];
    if (live && bev >= 0 && bev < sd.num_query) {
      const int64_t srow = b * sd.num_query + bev;
      const float inv = 1.0f / to_f32(count[srow]);
      T* dst = slots + (srow * d.heads + h) * d.channels + sub * kCh;
      float f[kCh];
      Vec16<T>::unpack(*reinterpret_cast<const uint4*>(dst), f);
#pragma unroll
      for (int q2 = 0; q2 < kPairs; ++q2) {
        f[2 * q2] += acc[q2].x * inv;
        f[2 * q2 + 1] += acc[q2].y * inv;
      }
      st16(dst, Vec16<T>::pack(f));
    }
  }
}

// Any D: one thread per output channel.
template <typename T>
__global__ void __launch_bounds__(256) forward_scalar_kernel(Dims d, const T* __restrict__ value,
                                                             const int64_t* __restrict__ shapes,
                                                             const int64_t* __restrict__ starts,
                                                             const T* __restrict__ loc, const T* __restrict__ weight,
                                                             T* __restrict__ out) {
  extern __shared__ Level levels[];
  stage_levels(levels, shapes, starts, d);
  const int64_t total = static_cast<int64_t>(d.batch) * d.queries * d.heads * d.channels;
  const int row_stride = d.heads * d.channels;
  const int samples = d.levels * d.points;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c_ = static_cast<int>(idx % d.channels);
    const int64_t item = idx / d.channels;
    const int h = static_cast<int>(item % d.heads);
    const int64_t b = item / (static_cast<int64_t>(d.queries) * d.heads);
    const T* vbase = value + (b * d.spatial_size) * row_stride + h * d.channels + c_;
    const T* lp = loc + item * samples * 2;
    const T* wp = weight + item * samples;
    float acc = 0.0f;
    for (int l = 0; l < d.levels; ++l) {
      const Level lv = levels[l];
      for (int p = 0; p < d.points; ++p) {
        const int s = l * d.points + p;
        const float x = to_f32(lp[2 * s]), y = to_f32(lp[2 * s + 1]);
        const float a = to_f32(wp[s]);
        Corners c;
        if (!corners(lv, x, y, c)) continue;
        float bil = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (c.row[k] >= 0) bil += c.w[k] * to_f32(vbase[static_cast<int64_t>(c.row[k]) * row_stride]);
        acc = fmaf(bil, a, acc);
      }
    }
    out[idx] = from_f32<T>(acc);
  }
}

template <typename T, int G, int kBytes>
static cudaError_t launch_forward_vec(const Dims& d, const Args& a, cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t groups_per_cta = kCtaThreads / G;
  const int64_t blocks = (items + groups_per_cta - 1) / groups_per_cta;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  // head-rows of at most 4 samples (single-level cases) stage 4 at a time
  auto kernel = d.levels * d.points <= 4 ? forward_vec_kernel<T, G, kBytes, 4>
                                         : forward_vec_kernel<T, G, kBytes, MSDA_FWD_CHUNK>;
  kernel<<<grid, kCtaThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<T*>(a.out), a.order);
  return cudaGetLastError();
}

template <typename T, int kBytes>
static cudaError_t launch_forward_lanes(int g, const Dims& d, const Args& a, cudaStream_t stream) {
  switch (g) {
    case 1: return launch_forward_vec<T, 1, kBytes>(d, a, stream);
    case 2: return launch_forward_vec<T, 2, kBytes>(d, a, stream);
    case 4: return launch_forward_vec<T, 4, kBytes>(d, a, stream);
    case 8: return launch_forward_vec<T, 8, kBytes>(d, a, stream);
    case 16: return launch_forward_vec<T, 16, kBytes>(d, a, stream);
    case 32: return launch_forward_vec<T, 32, kBytes>(d, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_forward_t(const Dims& d, const Args& a, cudaStream_t stream) {
  if constexpr (sizeof(T) == 2) {
    bool staged = false;
    const cudaError_t e = launch_forward_staged(d, a, stream, &staged);
    if (staged || e != cudaSuccess) return e;
  }
  constexpr int kWide = sizeof(T) == 2 ? MSDA_FWD_LANE_BYTES_BF16 : MSDA_FWD_LANE_BYTES_F32;
  if constexpr (kWide == 32) {
    if (const int g = vec_lanes(d.channels, sizeof(T), 32, a)) return launch_forward_lanes<T, 32>(g, d, a, stream);
  }
  if (const int g = vec_group(d.channels, sizeof(T), a)) return launch_forward_lanes<T, 16>(g, d, a, stream);
  const int64_t total = static_cast<int64_t>(d.batch) * d.queries * d.heads * d.channels;
  const int64_t blocks = (total + kCtaThreads - 1) / kCtaThreads;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  forward_scalar_kernel<T><<<grid, kCtaThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<T*>(a.out));
  return cudaGetLastError();
}

template <typename T, int G>
static cudaError_t launch_scatter_div_vec(const Dims& d, const SlotDims& sd, const Args& a, const int64_t* index,
                                         const void* count, void* slots, cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(sd.batch) * sd.valid_len * d.heads;
  const int64_t groups_per_cta = kCtaThreads / G;
  const int64_t blocks = (items + groups_per_cta - 1) / groups_per_cta;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  scatter_div_vec_kernel<T, G><<<grid, kCtaThreads, level_smem(d), stream>>>(
      d, sd, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), index, static_cast<const T*>(count), static_cast<T*>(slots));
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_scatter_div_t(const Dims& d, const SlotDims& sd, const Args& a, const int64_t* index,
                                       const void* count, void* slots, cudaStream_t stream) {
  Args probe = a;
  probe.out = slots;  // the slot rows are read and written in 16-byte lane slices
  switch (vec_group(d.channels, sizeof(T), probe)) {
    case 1: return launch_scatter_div_vec<T, 1>(d, sd, a, index, count, slots, stream);
    case 2: return launch_scatter_div_vec<T, 2>(d, sd, a, index, count, slots, stream);
    case 4: return launch_scatter_div_vec<T, 4>(d, sd, a, index, count, slots, stream);
    case 8: return launch_scatter_div_vec<T, 8>(d, sd, a, index, count, slots, stream);
    case 16: return launch_scatter_div_vec<T, 16>(d, sd, a, index, count, slots, stream);
    case 32: return launch_scatter_div_vec<T, 32>(d, sd, a, index, count, slots, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_scatter_div(DType dtype, const Dims& d, const SlotDims& sd, const Args& a, const int64_t* index,
                               const void* count, void* slots, cudaStream_t stream) {
  if (sd.batch == 0 || sd.valid_len == 0 || d.heads == 0) return cudaSuccess;
  return dtype == DType::kBF16 ? launch_scatter_div_t<__nv_bfloat16>(d, sd, a, index, count, slots, stream)
                               : launch_scatter_div_t<float>(d, sd, a, index, count, slots, stream);
}

cudaError_t launch_forward_rowwise(DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0 || d.channels == 0) return cudaSuccess;
  return dtype == DType::kBF16 ? launch_forward_t<__nv_bfloat16>(d, a, stream) : launch_forward_t<float>(d, a, stream);
}

}  // namespace msda
