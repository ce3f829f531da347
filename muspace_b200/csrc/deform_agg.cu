// SparseDrive deformable aggregation on sm_100a.
//
//   output[b, a, c] = sum over (pt, cam) with sampling_location in (0, 1)^2,
//                     sum over scales s of
//                     weights[b, a, pt, cam, s, group(c)] * bilinear(map(cam, s), loc)[c]
//
// with bilinear sampling at h = y * H - 0.5, w = x * W - 0.5 and corners
// outside the map read as zero. Replaces the kernels of
// csrc/deformable_aggregation/deformable_aggregation_musa.mu: the "opt" pair
// (292-429), one thread per (b, a, pt, cam, scale, channel) with an fp32
// atomicAdd into the output and index math through six fast divisions, and
// the "base" pair (158-290).
//
// B200 design (vector kernels). One warp owns one (b, anchor) row of C
// channels; lane l holds the 16-byte channel slices l, l + 32, ... so each
// corner gather is C * 4 contiguous bytes per warp (1 KB for C = 256). The warp
// compacts the row's in-image (pt, cam) pairs with a ballot, then stages the
// geometry of 32 (pair, scale) samples at a time in shared memory (one sample
// per lane: four corner rows, four bilinear weights, the group weights), and
// every lane walks the staged samples gathering its slices. The forward keeps
// the row in registers and stores it once: no atomics. The backward, whose
// outputs are all per (pt, cam), gives a warp one camera's pairs of the row,
// (b, cam, anchor) items with anchors fastest, so that the resident warps share
// one camera's maps and their gradients in L2. It forms per
// corner the dot of grad_output with the gathered slice (4 per lane and
// sample), from which a shuffle reduction over the lanes of a group gives the
// weight gradient and a reduction over the warp, once per pair, the location
// gradient; feature gradients leave as red.global.add.v4.f32 of whole 16-byte
// slices. The scalar kernels below cover every other shape and serve the
// "base" entry points.
#include "deform_agg.h"

// 1: the forward also runs camera-major, each (b, cam, anchor) warp adding its
// camera's partial row into the zero-filled output with vector REDs (the
// summation order over cameras then varies between runs, as in the
// reference's atomicAdd kernels); 0: one warp per (b, anchor) row, stored once.
#ifndef DA_FWD_CAM_MAJOR
#define DA_FWD_CAM_MAJOR 1
#endif
// 1: the backward runs camera-major (below); 0: one warp per (b, anchor) row.
#ifndef DA_BWD_CAM_MAJOR
#define DA_BWD_CAM_MAJOR 1
#endif

// CTAs per SM the backward's register budget is sized for (7: 72 registers,
// measured 2 % faster than 6 or 8; 0: left to the compiler).
#ifndef DA_BWD_MINBLOCKS
#define DA_BWD_MINBLOCKS 7
#endif
#if DA_BWD_MINBLOCKS > 0
#define DA_BWD_BOUNDS __launch_bounds__(kThreads, DA_BWD_MINBLOCKS)
#else
#define DA_BWD_BOUNDS __launch_bounds__(kThreads)
#endif

namespace da {
namespace {

constexpr int kWarps = 4;  // anchor rows per CTA of the vector kernels
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxGroups = 8;  // the reference's MAX_GROUPS

struct Map {
  int h, w, start;
};

// Stage the (H, W, start) table of every camera and scale. A map whose rows
// would leave [0, num_feat) is emptied, so a malformed table cannot make a
// kernel touch memory outside the feature tensor.
__device__ __forceinline__ void stage_maps(Map* maps, const int* shape, const int* start, const Dims& d) {
  for (int i = threadIdx.x; i < d.cams * d.scales; i += blockDim.x) {
    const int h = shape[2 * i], w = shape[2 * i + 1], s = start[i];
    const bool ok = h > 0 && w > 0 && s >= 0 && static_cast<int64_t>(h) * w + s <= d.num_feat;
    maps[i] = ok ? Map{h, w, s} : Map{0, 0, 0};
  }
  __syncthreads();
}

// One bilinear sample in the reference's arithmetic
// (deformable_aggregation_musa.mu:36-90): corner rows inside the feature
// tensor (-1 outside the map) and the weights hh*hw, hh*lw, lh*hw, lh*lw.
struct Geo {
  int row[4];
  float w[4];
  float lh, lw, hh, hw;
};

__device__ __forceinline__ void geometry(const Map& m, float loc_w, float loc_h, Geo& g) {
  const float h_im = __fsub_rn(__fmul_rn(loc_h, static_cast<float>(m.h)), 0.5f);
  const float w_im = __fsub_rn(__fmul_rn(loc_w, static_cast<float>(m.w)), 0.5f);
  const float hf = floorf(h_im), wf = floorf(w_im);
  const int h_low = static_cast<int>(hf), w_low = static_cast<int>(wf);
  g.lh = __fsub_rn(h_im, hf);
  g.lw = __fsub_rn(w_im, wf);
  g.hh = __fsub_rn(1.0f, g.lh);
  g.hw = __fsub_rn(1.0f, g.lw);
  // (0, 1) locations keep h_low in [-1, H - 1] and w_low in [-1, W - 1]
  const bool h0 = h_low >= 0 && h_low < m.h, h1 = h_low + 1 >= 0 && h_low + 1 < m.h;
  const bool w0 = w_low >= 0 && w_low < m.w, w1 = w_low + 1 >= 0 && w_low + 1 < m.w;
  const int base = m.start + h_low * m.w + w_low;
  g.row[0] = (h0 && w0) ? base : -1;
  g.row[1] = (h0 && w1) ? base + 1 : -1;
  g.row[2] = (h1 && w0) ? base + m.w : -1;
  g.row[3] = (h1 && w1) ? base + m.w + 1 : -1;
  g.w[0] = __fmul_rn(g.hh, g.hw);
  g.w[1] = __fmul_rn(g.hh, g.lw);
  g.w[2] = __fmul_rn(g.lh, g.hw);
  g.w[3] = __fmul_rn(g.lh, g.lw);
}

__device__ __forceinline__ bool inside(float2 l) { return l.x > 0.0f && l.x < 1.0f && l.y > 0.0f && l.y < 1.0f; }

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ void red4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// Per-warp staging of 32 (pair, scale) samples.
struct Stage {
  int pair[32];
  float2 loc[32];
  int4 row[32];
  float4 bil[32];
  float4 geo[32];  // lh, lw, W, H (backward)
  float wg[32][kMaxGroups];
};

// Compacts the in-image pairs among p = first + i * step, i in [i0, min(i0 + 32,
// count)), of a row into st.pair / st.loc; returns how many there are. Lanes
// of out-of-image pairs call on_outside(p) (the backward zeroes their
// gradients there).
template <typename F>
__device__ __forceinline__ int compact_pairs(const float* loc_row, int first, int step, int i0, int count,
                                             int d_scales, Stage& st, F&& on_outside) {
  const int lane = threadIdx.x % 32;
  const int i = i0 + lane;
  const int p = first + i * step;
  float2 l = make_float2(0.0f, 0.0f);
  bool act = false;
  if (i < count) {
    l = __ldg(reinterpret_cast<const float2*>(loc_row) + p);
    act = inside(l) && d_scales > 0;  // without scales an in-image pair contributes nothing either
    if (!act) on_outside(p);
  }
  const unsigned mask = __ballot_sync(0xffffffffu, act);
  if (act) {
    const int pos = __popc(mask & ((1u << lane) - 1u));
    st.pair[pos] = p;
    st.loc[pos] = l;
  }
  __syncwarp();
  return __popc(mask);
}

// Lane q of the warp stages sample q0 + q of the compacted list (pair-major,
// scale fastest).
__device__ __forceinline__ void stage_sample(const Dims& d, const Map* maps, const float* w_row, int q0, int total,
                                             Stage& st) {
  const int lane = threadIdx.x % 32;
  const int q = q0 + lane;
  if (q < total) {
    const int a = q / d.scales, s = q - a * d.scales;
    const int pair = st.pair[a];
    const float2 l = st.loc[a];
    const Map m = maps[(pair % d.cams) * d.scales + s];
    Geo g;
    geometry(m, l.x, l.y, g);
    st.row[lane] = make_int4(g.row[0], g.row[1], g.row[2], g.row[3]);
    st.bil[lane] = make_float4(g.w[0], g.w[1], g.w[2], g.w[3]);
    st.geo[lane] = make_float4(g.lh, g.lw, static_cast<float>(m.w), static_cast<float>(m.h));
    const float* wp = w_row + (static_cast<int64_t>(pair) * d.scales + s) * d.groups;
    for (int i = 0; i < d.groups; ++i) st.wg[lane][i] = __ldg(wp + i);
  }
  __syncwarp();
}

template <int kRounds>
__global__ void __launch_bounds__(kThreads) forward_vec(Dims d, const float* __restrict__ feat,
                                                        const int* __restrict__ shape, const int* __restrict__ start,
                                                        const float* __restrict__ loc,
                                                        const float* __restrict__ weights, float* __restrict__ out) {
  extern __shared__ Map maps[];
  __shared__ Stage stage[kWarps];
  stage_maps(maps, shape, start, d);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  Stage& st = stage[warp];
  const int pairs = d.pts * d.cams;
#if DA_FWD_CAM_MAJOR
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (item >= static_cast<int64_t>(d.batch) * d.cams * d.anchors) return;  // whole warp
  const int64_t bc = item / d.anchors;
  const int cam = static_cast<int>(bc % d.cams);
  const int64_t b = bc / d.cams;
  const int64_t row = b * d.anchors + (item - bc * d.anchors);
  const int first = cam, step = d.cams, count = d.pts;
  bool any = false;
#else
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (row >= static_cast<int64_t>(d.batch) * d.anchors) return;  // whole warp
  const int64_t b = row / d.anchors;
  const int first = 0, step = 1, count = pairs;
#endif
  const int slices = d.channels / 4;
  const int per_group = d.channels / d.groups;
  const float* fb = feat + b * d.num_feat * static_cast<int64_t>(d.channels);
  const float* loc_row = loc + row * pairs * 2;
  const float* w_row = weights + row * pairs * static_cast<int64_t>(d.scales) * d.groups;

  float4 acc[kRounds];
#pragma unroll
  for (int r = 0; r < kRounds; ++r) acc[r] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);

  for (int p0 = 0; p0 < count; p0 += 32) {
    const int n = compact_pairs(loc_row, first, step, p0, count, d.scales, st, [](int) {});
#if DA_FWD_CAM_MAJOR
    any |= n > 0;
#endif
    const int total = n * d.scales;
    for (int q0 = 0; q0 < total; q0 += 32) {
      stage_sample(d, maps, w_row, q0, total, st);
      const int count = total - q0 < 32 ? total - q0 : 32;
      for (int i = 0; i < count; ++i) {
        const int4 r4 = st.row[i];
        const float4 b4 = st.bil[i];
        const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
        const float bil[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int r = 0; r < kRounds; ++r) {
          const int slice = lane + 32 * r;
          if (slice >= slices) continue;
          const float wg = st.wg[i][(slice * 4) / per_group];
          float4 v[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            v[k] = rows[k] >= 0 ? ldg4(fb + static_cast<int64_t>(rows[k]) * d.channels + slice * 4)
                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          // sampled = w1 v1 + w2 v2 + w3 v3 + w4 v4, then output += sampled * weight
          const float sx = bil[0] * v[0].x + bil[1] * v[1].x + bil[2] * v[2].x + bil[3] * v[3].x;
          const float sy = bil[0] * v[0].y + bil[1] * v[1].y + bil[2] * v[2].y + bil[3] * v[3].y;
          const float sz = bil[0] * v[0].z + bil[1] * v[1].z + bil[2] * v[2].z + bil[3] * v[3].z;
          const float sw = bil[0] * v[0].w + bil[1] * v[1].w + bil[2] * v[2].w + bil[3] * v[3].w;
          acc[r].x = fmaf(sx, wg, acc[r].x);
          acc[r].y = fmaf(sy, wg, acc[r].y);
          acc[r].z = fmaf(sz, wg, acc[r].z);
          acc[r].w = fmaf(sw, wg, acc[r].w);
        }
      }
      __syncwarp();  // the next staging overwrites the slots read above
    }
  }
#if DA_FWD_CAM_MAJOR
  if (!any) return;  // warp-uniform: no in-image pair of this camera
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int slice = lane + 32 * r;
    if (slice < slices) red4(out + row * d.channels + slice * 4, acc[r].x, acc[r].y, acc[r].z, acc[r].w);
  }
#else
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int slice = lane + 32 * r;
    if (slice < slices) *reinterpret_cast<float4*>(out + row * d.channels + slice * 4) = acc[r];
  }
#endif
}

// Sum over aligned groups of `width` lanes (a power of two).
__device__ __forceinline__ float lanes_sum(float v, int width) {
  for (int m = width / 2; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

template <int kRounds>
__global__ void DA_BWD_BOUNDS backward_vec(Dims d, const float* __restrict__ feat,
                                                         const int* __restrict__ shape, const int* __restrict__ start,
                                                         const float* __restrict__ loc,
                                                         const float* __restrict__ weights,
                                                         const float* __restrict__ grad_out,
                                                         float* __restrict__ grad_feat, float* __restrict__ grad_loc,
                                                         float* __restrict__ grad_weights) {
  extern __shared__ Map maps[];
  __shared__ Stage stage[kWarps];
  stage_maps(maps, shape, start, d);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // item = (b, cam, anchor), anchors fastest: the warps resident at one time
  // work on one or two cameras' maps of one batch element, whose features and
  // feature gradients (2 x 15 MB at the production shapes) stay in L2, where a
  // warp per (b, anchor) spread them over all six cameras of several elements.
  Stage& st = stage[warp];
  const int pairs = d.pts * d.cams;
#if DA_BWD_CAM_MAJOR
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (item >= static_cast<int64_t>(d.batch) * d.cams * d.anchors) return;  // whole warp
  const int64_t bc = item / d.anchors;
  const int cam = static_cast<int>(bc % d.cams);
  const int64_t b = bc / d.cams;
  const int64_t row = b * d.anchors + (item - bc * d.anchors);
  const int first = cam, step = d.cams, count = d.pts;  // this camera's pairs pt * cams + cam
#else
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (row >= static_cast<int64_t>(d.batch) * d.anchors) return;  // whole warp
  const int64_t b = row / d.anchors;
  const int first = 0, step = 1, count = pairs;
#endif
  const int slices = d.channels / 4;
  const int per_group = d.channels / d.groups;
  const int group_lanes = per_group / 4;  // lanes holding one group's channels (a power of two)
  const float* fb = feat + b * d.num_feat * static_cast<int64_t>(d.channels);
  float* gfb = grad_feat + b * d.num_feat * static_cast<int64_t>(d.channels);
  const float* loc_row = loc + row * pairs * 2;
  const int64_t w_per_pair = static_cast<int64_t>(d.scales) * d.groups;
  const float* w_row = weights + row * pairs * w_per_pair;
  float* gw_row = grad_weights + row * pairs * w_per_pair;
  float* gl_row = grad_loc + row * pairs * 2;

  float4 g[kRounds];
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int slice = lane + 32 * r;
    g[r] = slice < slices ? ldg4(grad_out + row * d.channels + slice * 4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }

  float lx = 0.0f, ly = 0.0f;  // this lane's share of the current pair's location gradient
  for (int p0 = 0; p0 < count; p0 += 32) {
    const int n = compact_pairs(loc_row, first, step, p0, count, d.scales, st, [&](int p) {
      *reinterpret_cast<float2*>(gl_row + 2 * p) = make_float2(0.0f, 0.0f);
      for (int64_t i = 0; i < w_per_pair; ++i) gw_row[p * w_per_pair + i] = 0.0f;
    });
    const int total = n * d.scales;
    for (int q0 = 0; q0 < total; q0 += 32) {
      stage_sample(d, maps, w_row, q0, total, st);
      const int count = total - q0 < 32 ? total - q0 : 32;
      for (int i = 0; i < count; ++i) {
        const int q = q0 + i;
        const int a = q / d.scales, s = q - a * d.scales;
        const int4 r4 = st.row[i];
        const float4 b4 = st.bil[i];
        const float4 geo = st.geo[i];
        const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
        const float bil[4] = {b4.x, b4.y, b4.z, b4.w};
        const float lh = geo.x, lw = geo.y, hh = 1.0f - lh, hw = 1.0f - lw;
        float x = 0.0f, y = 0.0f;
#pragma unroll
        for (int r = 0; r < kRounds; ++r) {
          const int slice = lane + 32 * r;
          float part = 0.0f;  // sum over this lane's channels of g_c * sampled_c
          if (slice < slices) {
            const float wg = st.wg[i][(slice * 4) / per_group];
            float dot[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float4 v = rows[k] >= 0 ? ldg4(fb + static_cast<int64_t>(rows[k]) * d.channels + slice * 4)
                                            : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
              dot[k] = g[r].x * v.x + g[r].y * v.y + g[r].z * v.z + g[r].w * v.w;
            }
            part = bil[0] * dot[0] + bil[1] * dot[1] + bil[2] * dot[2] + bil[3] * dot[3];
            x += wg * (hh * (dot[1] - dot[0]) + lh * (dot[3] - dot[2]));
            y += wg * (hw * (dot[2] - dot[0]) + lw * (dot[3] - dot[1]));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (rows[k] < 0) continue;
              const float c = bil[k] * wg;
              red4(gfb + static_cast<int64_t>(rows[k]) * d.channels + slice * 4, c * g[r].x, c * g[r].y,
                   c * g[r].z, c * g[r].w);
            }
          }
          // weight gradient of the groups this round covers
          part = lanes_sum(part, group_lanes);
          if (slice < slices && lane % group_lanes == 0)
            gw_row[st.pair[a] * w_per_pair + s * d.groups + (slice * 4) / per_group] = part;
        }
        lx += geo.z * x;  // W
        ly += geo.w * y;  // H
        if (s == d.scales - 1) {
          const float sx = lanes_sum(lx, 32), sy = lanes_sum(ly, 32);
          if (lane == 0) *reinterpret_cast<float2*>(gl_row + 2 * st.pair[a]) = make_float2(sx, sy);
          lx = ly = 0.0f;
        }
      }
      __syncwarp();
    }
  }
}

// ---------------------------------------------------------------------------
// scalar kernels ("base" entry points and every shape the vector kernels skip)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) forward_scalar(Dims d, const float* __restrict__ feat,
                                                      const int* __restrict__ shape, const int* __restrict__ start,
                                                      const float* __restrict__ loc, const float* __restrict__ weights,
                                                      float* __restrict__ out) {
  extern __shared__ Map maps[];
  stage_maps(maps, shape, start, d);
  const int64_t total = static_cast<int64_t>(d.batch) * d.anchors * d.channels;
  const int pairs = d.pts * d.cams;
  const int per_group = d.channels / d.groups;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % d.channels);
    const int64_t row = idx / d.channels;
    const int64_t b = row / d.anchors;
    const float* fb = feat + b * d.num_feat * static_cast<int64_t>(d.channels) + c;
    float acc = 0.0f;
    for (int p = 0; p < pairs; ++p) {
      const float2 l = reinterpret_cast<const float2*>(loc)[row * pairs + p];
      if (!inside(l)) continue;
      for (int s = 0; s < d.scales; ++s) {
        Geo g;
        geometry(maps[(p % d.cams) * d.scales + s], l.x, l.y, g);
        float sampled = 0.0f;
        for (int k = 0; k < 4; ++k)
          if (g.row[k] >= 0) sampled += g.w[k] * fb[static_cast<int64_t>(g.row[k]) * d.channels];
        acc = fmaf(sampled, weights[((row * pairs + p) * d.scales + s) * d.groups + c / per_group], acc);
      }
    }
    out[idx] = acc;
  }
}

// One thread per (b, anchor, pt, cam), as the reference's gradient kernel.
__global__ void __launch_bounds__(256) backward_scalar(Dims d, const float* __restrict__ feat,
                                                       const int* __restrict__ shape, const int* __restrict__ start,
                                                       const float* __restrict__ loc, const float* __restrict__ weights,
                                                       const float* __restrict__ grad_out,
                                                       float* __restrict__ grad_feat, float* __restrict__ grad_loc,
                                                       float* __restrict__ grad_weights) {
  extern __shared__ Map maps[];
  stage_maps(maps, shape, start, d);
  const int pairs = d.pts * d.cams;
  const int64_t total = static_cast<int64_t>(d.batch) * d.anchors * pairs;
  const int per_group = d.channels / d.groups;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = idx / pairs;
    const int p = static_cast<int>(idx % pairs);
    const int64_t b = row / d.anchors;
    const float2 l = reinterpret_cast<const float2*>(loc)[idx];
    float* gw = grad_weights + idx * d.scales * d.groups;
    if (!inside(l)) {
      reinterpret_cast<float2*>(grad_loc)[idx] = make_float2(0.0f, 0.0f);
      for (int i = 0; i < d.scales * d.groups; ++i) gw[i] = 0.0f;
      continue;
    }
    const float* fb = feat + b * d.num_feat * static_cast<int64_t>(d.channels);
    float* gfb = grad_feat + b * d.num_feat * static_cast<int64_t>(d.channels);
    const float* go = grad_out + row * d.channels;
    float gx = 0.0f, gy = 0.0f;
    for (int s = 0; s < d.scales; ++s) {
      const Map m = maps[(p % d.cams) * d.scales + s];
      Geo g;
      geometry(m, l.x, l.y, g);
      const float* wg = weights + (idx * d.scales + s) * d.groups;
      float local[kMaxGroups] = {0.0f};
      for (int c = 0; c < d.channels; ++c) {
        const int grp = c / per_group;
        const float top = go[c] * wg[grp];
        float v[4];
        for (int k = 0; k < 4; ++k) {
          v[k] = g.row[k] >= 0 ? fb[static_cast<int64_t>(g.row[k]) * d.channels + c] : 0.0f;
          if (g.row[k] >= 0) atomicAdd(gfb + static_cast<int64_t>(g.row[k]) * d.channels + c, g.w[k] * top);
        }
        local[grp] += go[c] * (g.w[0] * v[0] + g.w[1] * v[1] + g.w[2] * v[2] + g.w[3] * v[3]);
        gx += static_cast<float>(m.w) * (g.hh * (v[1] - v[0]) + g.lh * (v[3] - v[2])) * top;
        gy += static_cast<float>(m.h) * (g.hw * (v[2] - v[0]) + g.lw * (v[3] - v[1])) * top;
      }
      for (int i = 0; i < d.groups; ++i) gw[s * d.groups + i] = local[i];
    }
    reinterpret_cast<float2*>(grad_loc)[idx] = make_float2(gx, gy);
  }
}

size_t map_smem(const Dims& d) { return sizeof(Map) * static_cast<size_t>(d.cams * d.scales > 0 ? d.cams * d.scales : 1); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Rounds of 32 lane slices per row, or 0 when the vector kernels do not apply.
int vec_rounds(const Dims& d, const Args& a, bool backward) {
  if (d.channels <= 0 || d.channels % 4 != 0 || d.channels > 512) return 0;
  const int per_group = d.channels / d.groups;
  if (per_group % 4 != 0) return 0;
  const int lanes = per_group / 4;
  if (lanes > 32 || (lanes & (lanes - 1)) != 0) return 0;
  if (!aligned16(a.feat) || (reinterpret_cast<uintptr_t>(a.loc) & 7u) != 0) return 0;
  if (backward ? (!aligned16(a.grad_out) || !aligned16(a.grad_feat) || (reinterpret_cast<uintptr_t>(a.grad_loc) & 7u))
               : !aligned16(a.out))
    return 0;
  const int slices = d.channels / 4;
  return slices <= 32 ? 1 : slices <= 64 ? 2 : 4;
}

int scalar_grid(int64_t work) {
  const int64_t blocks = (work + 255) / 256;
  return static_cast<int>(blocks < (1LL << 30) ? blocks : (1LL << 30));
}

}  // namespace

cudaError_t forward(const Dims& d, const Args& a, bool optimized, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(d.batch) * d.anchors;
  if (rows == 0 || d.channels == 0) return cudaSuccess;
  const int rounds = optimized ? vec_rounds(d, a, false) : 0;
  const size_t smem = map_smem(d);
  if (rounds) {
#if DA_FWD_CAM_MAJOR
    const cudaError_t zero =
        cudaMemsetAsync(a.out, 0, static_cast<size_t>(rows) * d.channels * sizeof(float), stream);
    if (zero != cudaSuccess) return zero;
    const int64_t items = rows * d.cams;
    if (items == 0) return cudaSuccess;
#else
    const int64_t items = rows;
#endif
    const int grid = static_cast<int>((items + kWarps - 1) / kWarps);
    switch (rounds) {
      case 1: forward_vec<1><<<grid, kThreads, smem, stream>>>(d, a.feat, a.shape, a.start, a.loc, a.weights, a.out); break;
      case 2: forward_vec<2><<<grid, kThreads, smem, stream>>>(d, a.feat, a.shape, a.start, a.loc, a.weights, a.out); break;
      default: forward_vec<4><<<grid, kThreads, smem, stream>>>(d, a.feat, a.shape, a.start, a.loc, a.weights, a.out); break;
    }
  } else {
    forward_scalar<<<scalar_grid(rows * d.channels), 256, smem, stream>>>(d, a.feat, a.shape, a.start, a.loc,
                                                                          a.weights, a.out);
  }
  return cudaGetLastError();
}

cudaError_t backward(const Dims& d, const Args& a, bool optimized, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(d.batch) * d.anchors;
  if (rows == 0) return cudaSuccess;
  const int rounds = optimized ? vec_rounds(d, a, true) : 0;
  const size_t smem = map_smem(d);
  if (rounds) {
#if DA_BWD_CAM_MAJOR
    const int64_t items = rows * d.cams;
    if (items == 0) return cudaSuccess;  // no cameras: nothing to write either
#else
    const int64_t items = rows;
#endif
    const int grid = static_cast<int>((items + kWarps - 1) / kWarps);
    switch (rounds) {
      case 1: backward_vec<1><<<grid, kThreads, smem, stream>>>(d, a.feat, a.shape, a.start, a.loc, a.weights, a.grad_out, a.grad_feat, a.grad_loc, a.grad_weights); break;
      case 2: backward_vec<2><<<grid, kThreads, smem, stream>>>(d, a.feat, a.shape, a.start, a.loc, a.weights, a.grad_out, a.grad_feat, a.grad_loc, a.grad_weights); break;
      default: backward_vec<4><<<grid, kThreads, smem, stream>>>(d, a.feat, a.shape, a.start, a.loc, a.weights, a.grad_out, a.grad_feat, a.grad_loc, a.grad_weights); break;
    }
  } else {
    backward_scalar<<<scalar_grid(rows * d.pts * d.cams), 256, smem, stream>>>(
        d, a.feat, a.shape, a.start, a.loc, a.weights, a.grad_out, a.grad_feat, a.grad_loc, a.grad_weights);
  }
  return cudaGetLastError();
}

}  // namespace da
