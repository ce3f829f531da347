// FlashSCA (flash_bevpool_sca) forward and backward on sm_100a.
//
// out[b, y, x, c] = (1 / visible cameras) * sum over the (camera, height)
//   pairs whose projection of the cell centre lands in the image, the levels
//   and the points of head(c), of weight * bilinear(level map, base + offset)[c]
// with base = (u / W_img * w - 0.5, v / H_img * h - 0.5), zero padding and
// non-finite feature values read as 0.
//
// Replaces csrc/flashbev/flash_bevpool_sca_musa.mu, which runs one thread per
// output channel: every thread re-projects the cell into every camera twice
// (visibility, then sampling) and recomputes every sample's geometry, and the
// backward adds offset and weight gradients with one atomic per channel.
//
// B200 design. A work item is one (b, cell, head): G = (C / heads) / 4 lanes,
// each holding a 16-byte slice of the head's channels. The group projects the
// cell into all cameras once (one (camera, height) pair per lane and round),
// compacts the landing pairs with a ballot and counts the visible cameras from
// the same bits. Samples (pair, level, point) are then taken in chunks: the
// lane at sub = i * G / C computes sample i's geometry once and stages its
// corner rows and bilinear-times-attention weights in shared memory, and every
// lane gathers its slice of the four corners (one 16-byte load each). The
// backward forms per corner the dot of the lane's grad_output slice with the
// gathered slice, reduces the four dots over the group with a transpose
// reduction, and one lane per sample adds the offset and weight gradients (one
// atomic per sample and component instead of one per channel); value
// gradients leave as red.global.add.v4.f32. The backward stages 8 samples at
// a time in level-major order (one level's samples of every landing height
// together) and first folds repeated corner rows of the chunk into their first
// occurrence, which removes 23 % of the RED payload at BEVFormer-base sizes.
#include "flash_sca.h"
#include "msda_device.cuh"

namespace fsca {
namespace {

using msda::Words;

struct Map {
  int h, w, start;
};

__device__ __forceinline__ float sanitize(float v) { return fabsf(v) <= 3.402823466e+38f ? v : 0.0f; }

// One row of the projection: p[0] x + p[1] y + p[2] z + p[3], left to right.
__device__ __forceinline__ float dot_row(const float* p, float x, float y, float z) {
  return __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(p[0], x), __fmul_rn(p[1], y)), __fmul_rn(p[2], z)), p[3]);
}

// The reference's projection test (flashbev.py:100-113; kernel 17-24): depth
// must be positive, u = row0 / max(depth, eps), v = row1 / max(depth, eps),
// and the point must land in [0, W) x [0, H).
__device__ __forceinline__ bool project(const float* p, float x, float y, float z, float eps, float img_h,
                                        float img_w, float& u, float& v) {
  const float depth = dot_row(p + 8, x, y, z);
  if (!(depth > 0.0f)) return false;
  const float safe = fmaxf(depth, eps);
  u = __fdiv_rn(dot_row(p, x, y, z), safe);
  v = __fdiv_rn(dot_row(p + 4, x, y, z), safe);
  return u >= 0.0f && u < img_w && v >= 0.0f && v < img_h;
}

template <int G>
struct Shape {
  static constexpr int kThreads = G >= 8 ? 256 : 32 * G;
  static constexpr int kGroups = kThreads / G;
  static constexpr int kChunk = G < 4 ? G : 4;  // samples per dot round of the backward
  // samples staged per chunk (the backward folds them and takes its dots in rounds of kChunk)
  static constexpr int kBwdChunk = G < 8 ? kChunk : 8;
  static constexpr int kBwdStager = G / kBwdChunk;
  static constexpr int kSlots = kBwdChunk + 1;  // + padding against bank conflicts between groups
  static constexpr int kHashSlots = kBwdChunk >= 8 ? 64 : (kBwdChunk >= 4 ? 32 : (kBwdChunk >= 2 ? 16 : 8));
};

// Per-group shared memory.
template <int G>
struct GroupSmem {
  int pair[kMaxPairs];
  float2 uv[kMaxPairs];  // projection / image size
  int4 row[Shape<G>::kSlots];
  float4 wa[Shape<G>::kSlots];   // w_k * a of each corner; in the backward, once a round's REDs are out, its dots
  float4 geo[Shape<G>::kSlots];  // du, dv, attention weight, entry (int bits)
  alignas(16) int hash[Shape<G>::kHashSlots];  // the backward's row fold
};

struct Cell {
  float x, y, z0, sz;
};

// Projects the cell into every (camera, height) pair (pair = cam * gz + iz),
// compacts the landing ones into s.pair / s.uv and returns how many there
// are; visible = cameras with at least one landing height. All lanes of the
// warp call it.
template <int G>
__device__ __forceinline__ int land_pairs(const Dims& d, const float* proj_b, const Cell& c, float eps, float img_h,
                                          float img_w, bool live, int sub, GroupSmem<G>& s, int& visible) {
  const int lane = threadIdx.x % 32;
  const int first = lane - sub;
  const unsigned group_bits = G == 32 ? 0xffffffffu : ((1u << G) - 1u) << first;
  const int pairs = d.cams * d.gz;
  int n = 0;
  uint64_t lands = 0;
  for (int k0 = 0; k0 < pairs; k0 += G) {
    const int pr = k0 + sub;
    bool ok = false;
    float u = 0.0f, v = 0.0f;
    if (live && pr < pairs) {
      const int cam = pr / d.gz, iz = pr - cam * d.gz;
      const float z = __fadd_rn(c.z0, __fmul_rn(static_cast<float>(iz) + 0.5f, c.sz));
      ok = project(proj_b + cam * 12, c.x, c.y, z, eps, img_h, img_w, u, v);
    }
    const unsigned rel = (__ballot_sync(0xffffffffu, ok) & group_bits) >> first;
    if (ok) {
      const int pos = n + __popc(rel & ((1u << sub) - 1u));
      s.pair[pos] = pr;
      // the projection normalised to the image, as each sample's base needs it
      s.uv[pos] = make_float2(__fdiv_rn(u, img_w), __fdiv_rn(v, img_h));
    }
    lands |= static_cast<uint64_t>(rel) << k0;
    n += __popc(rel);
  }
  visible = 0;
  const uint64_t heights = d.gz >= 64 ? ~0ull : ((1ull << d.gz) - 1ull);
  for (int cam = 0; cam < d.cams; ++cam) visible += ((lands >> (cam * d.gz)) & heights) != 0;
  __syncwarp();
  return n;
}

// Lane `i`-th stager stages sample s of the item (pair-major, then level, then
// point; or level-major): four corner rows in the (cams * S) plane of the batch entry (-1 =
// outside the level), bilinear weights times attention, and (du, dv, weight,
// entry) for the gradients.
// Head, cell (x, y) and batch entry of item (b, gy, gx, heads order): 32-bit
// divisions when every item index of the call fits 31 bits (idx32), else
// 64-bit ones.
struct ItemCell {
  int head, ix, iy;
  int64_t cell, b;
};
__device__ __forceinline__ ItemCell item_cell(int64_t it, const Dims& d, bool idx32) {
  if (idx32) {
    const uint32_t i = static_cast<uint32_t>(it);
    const uint32_t cell = i / static_cast<uint32_t>(d.heads);
    const uint32_t row = cell / static_cast<uint32_t>(d.gx);
    return ItemCell{static_cast<int>(i - cell * static_cast<uint32_t>(d.heads)),
                    static_cast<int>(cell - row * static_cast<uint32_t>(d.gx)),
                    static_cast<int>(row % static_cast<uint32_t>(d.gy)), cell, row / static_cast<uint32_t>(d.gy)};
  }
  const int64_t cell = it / d.heads;
  return ItemCell{static_cast<int>(it % d.heads), static_cast<int>(cell % d.gx),
                  static_cast<int>((cell / d.gx) % d.gy), cell, cell / (static_cast<int64_t>(d.gx) * d.gy)};
}

// floor(x / div): a multiply-high by magic = ceil(2^32 / div) when the caller
// set one (exact for its range of x), else a division.
__device__ __forceinline__ int div_by(int x, int div, uint32_t magic) {
  return magic ? static_cast<int>(__umulhi(static_cast<uint32_t>(x), magic)) : x / div;
}

// level_magic: ceil(2^32 / per_level) for the level-major order, or 0.
template <int G, bool kLevelMajor = false>
__device__ __forceinline__ void stage(const Dims& d, const Map* maps, const float* off_item, const float* w_item,
                                      int s, int samples, int slot, GroupSmem<G>& sm, uint32_t level_magic = 0) {
  int4 r = make_int4(-1, -1, -1, -1);
  float4 wa = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float4 geo = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (s < samples) {
    int pi, level, point;
    if (kLevelMajor) {  // level, then pair, then point: one level's samples of every height together
      const int per_level = samples / d.levels;  // landing pairs * points
      level = div_by(s, per_level, level_magic);
      const int rem = s - level * per_level;
      pi = div_by(rem, d.points, d.points_magic);
      point = rem - pi * d.points;
    } else {
      const int lp = d.levels * d.points;
      pi = div_by(s, lp, d.lp_magic);
      const int rem = s - pi * lp;
      level = div_by(rem, d.points, d.points_magic);
      point = rem - level * d.points;
    }
    const int pr = sm.pair[pi];
    const int cam = pr / d.gz, iz = pr - cam * d.gz;
    const float2 uv = sm.uv[pi];
    const Map m = maps[level];
    const int e = (level * d.points + point) * d.gz + iz;  // entry inside the (cell, head) block
    const float2 off = *reinterpret_cast<const float2*>(off_item + 2 * e);
    const float weight = w_item[e];
    const float bu = __fsub_rn(__fmul_rn(uv.x, static_cast<float>(m.w)), 0.5f);
    const float bv = __fsub_rn(__fmul_rn(uv.y, static_cast<float>(m.h)), 0.5f);
    const float su = __fadd_rn(bu, off.x), sv = __fadd_rn(bv, off.y);
    const float fu = floorf(su), fv = floorf(sv);
    // finite samples only (a non-finite offset samples nothing, as its corners fail every bound)
    if (fabsf(fu) < 1e9f && fabsf(fv) < 1e9f && m.w > 0) {
      const int u0 = static_cast<int>(fu), v0 = static_cast<int>(fv);
      const float du = __fsub_rn(su, fu), dv = __fsub_rn(sv, fv);
      const float hu = __fsub_rn(1.0f, du), hv = __fsub_rn(1.0f, dv);
      const bool u0ok = u0 >= 0 && u0 < m.w, u1ok = u0 + 1 >= 0 && u0 + 1 < m.w;
      const bool v0ok = v0 >= 0 && v0 < m.h, v1ok = v0 + 1 >= 0 && v0 + 1 < m.h;
      // rows only for in-level corners (the indices of the others may be far outside int range)
      const int plane = cam * d.stride_n + m.start;
      const auto row = [&](bool ok, int uu, int vv) { return ok ? plane + vv * m.w + uu : -1; };
      // corner order: (u0, v0), (u0, v1), (u1, v0), (u1, v1), as f00, f01, f10, f11
      r = make_int4(row(u0ok && v0ok, u0, v0), row(u0ok && v1ok, u0, v0 + 1), row(u1ok && v0ok, u0 + 1, v0),
                    row(u1ok && v1ok, u0 + 1, v0 + 1));
      wa = make_float4(__fmul_rn(__fmul_rn(hu, hv), weight), __fmul_rn(__fmul_rn(hu, dv), weight),
                       __fmul_rn(__fmul_rn(du, hv), weight), __fmul_rn(__fmul_rn(du, dv), weight));
      geo = make_float4(du, dv, weight, __int_as_float(static_cast<int>(e)));
    } else {
      geo = make_float4(0.0f, 0.0f, weight, __int_as_float(static_cast<int>(e)));
    }
  }
  sm.row[slot] = r;
  sm.wa[slot] = wa;
  sm.geo[slot] = geo;
}

__device__ __forceinline__ void stage_maps(Map* maps, const int* shapes, const int* starts, const Dims& d) {
  for (int l = threadIdx.x; l < d.levels; l += blockDim.x) {
    const int h = shapes[2 * l], w = shapes[2 * l + 1], s = starts[l];
    const bool ok = h > 0 && w > 0 && s >= 0 && static_cast<int64_t>(h) * w + s <= d.stride_n;
    maps[l] = ok ? Map{h, w, s} : Map{0, 0, 0};
  }
  __syncthreads();
}

__device__ __forceinline__ float4 gather_raw(const float* p, int row, int channels) {
  if (row < 0) return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  return __ldg(reinterpret_cast<const float4*>(p + static_cast<int64_t>(row) * channels));
}

__device__ __forceinline__ float4 sanitize(float4 v) {
  return make_float4(sanitize(v.x), sanitize(v.y), sanitize(v.z), sanitize(v.w));
}

__device__ __forceinline__ float4 gather(const float* p, int row, int channels) {
  return sanitize(gather_raw(p, row, channels));
}

// Zero where the feature value was not finite: the reference replaces such
// values by a constant before sampling, so they receive no gradient.
__device__ __forceinline__ float keep(float raw, float grad) { return fabsf(raw) <= 3.402823466e+38f ? grad : 0.0f; }

// Samples the forward stages per round: 1 = one per lane round of the
// backward (Shape::kBwdChunk: every lane of a group stages one), 0 = the dot
// round size (Shape::kChunk: half the lanes stage).
#ifndef FSCA_FWD_WIDE_CHUNK
#define FSCA_FWD_WIDE_CHUNK 1
#endif
#define FSCA_FWD_CHUNK_OF(G) (FSCA_FWD_WIDE_CHUNK ? Shape<G>::kBwdChunk : Shape<G>::kChunk)

// One item's sum over its samples: sum_k wa_k * value(row_k) for the lane's
// slice, staging FSCA_FWD_CHUNK_OF(G) samples at a time. kSanitize reads a non-finite value
// as 0. All lanes of the warp call it with the warp's common trip count.
template <int G, bool kSanitize>
__device__ __forceinline__ float4 sum_item(const Dims& d, const Map* maps, const float* off_item, const float* w_item,
                                           int trips, int samples, int sub, const float* vb, GroupSmem<G>& sm) {
  constexpr int Cs = FSCA_FWD_CHUNK_OF(G);
  constexpr int kStager = G / Cs;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int s0 = 0; s0 < trips; s0 += Cs) {
    if (sub % kStager == 0) {
      const int i = sub / kStager;
      stage<G>(d, maps, off_item, w_item, s0 + i, samples, i, sm);
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < Cs; ++i) {
      const int4 r4 = sm.row[i];
      const float4 w4 = sm.wa[i];
      const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
      const float wa[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 v = kSanitize ? gather(vb, rows[k], d.channels) : gather_raw(vb, rows[k], d.channels);
        acc.x = fmaf(wa[k], v.x, acc.x);
        acc.y = fmaf(wa[k], v.y, acc.y);
        acc.z = fmaf(wa[k], v.z, acc.z);
        acc.w = fmaf(wa[k], v.w, acc.w);
      }
    }
    __syncwarp();
  }
  return acc;
}

// CTAs per SM the register budgets are sized for (0: left to the compiler).
#ifndef FSCA_FWD_MINBLOCKS
#define FSCA_FWD_MINBLOCKS 4
#endif
// (backward at 4: 64 registers, 4 CTAs/SM; 1.371 -> 1.266 ms at BEVFormer-base
// sizes against the compiler's own 80 registers)
#ifndef FSCA_BWD_MINBLOCKS
#define FSCA_BWD_MINBLOCKS 4
#endif
// 1: fold repeated corner rows of a staged chunk before the backward's REDs.
#ifndef FSCA_BWD_FOLD
#define FSCA_BWD_FOLD 1
#endif
// 1: the fold goes through a per-group hash table (msda::fold_rows_hashed)
// instead of a scan over all lower entries.
#ifndef FSCA_BWD_HASH_FOLD
#define FSCA_BWD_HASH_FOLD 1
#endif
// 1: the backward's REDs are predicated instead of branched around.
#ifndef FSCA_BWD_PRED_RED
#define FSCA_BWD_PRED_RED 1
#endif
#if FSCA_FWD_MINBLOCKS > 0
#define FSCA_FWD_BOUNDS(G) __launch_bounds__(Shape<G>::kThreads, FSCA_FWD_MINBLOCKS)
#else
#define FSCA_FWD_BOUNDS(G) __launch_bounds__(Shape<G>::kThreads)
#endif
#if FSCA_BWD_MINBLOCKS > 0
#define FSCA_BWD_BOUNDS(G) __launch_bounds__(Shape<G>::kThreads, FSCA_BWD_MINBLOCKS)
#else
#define FSCA_BWD_BOUNDS(G) __launch_bounds__(Shape<G>::kThreads)
#endif

template <int G>
__global__ void FSCA_FWD_BOUNDS(G) forward_kernel(Dims d, Grid grid, float eps,
                                                                     const float* __restrict__ value,
                                                                     const float* __restrict__ proj,
                                                                     const int* __restrict__ shapes,
                                                                     const int* __restrict__ starts,
                                                                     const int* __restrict__ image_size,
                                                                     const float* __restrict__ offsets,
                                                                     const float* __restrict__ weights,
                                                                     float* __restrict__ out) {
  using Sh = Shape<G>;
  __shared__ Map maps[kMaxLevels];
  __shared__ GroupSmem<G> smem[Sh::kGroups];
  stage_maps(maps, shapes, starts, d);
  const int sub = threadIdx.x % G, group = threadIdx.x / G;
  GroupSmem<G>& sm = smem[group];
  const float img_h = static_cast<float>(image_size[0]), img_w = static_cast<float>(image_size[1]);
  const int64_t items = static_cast<int64_t>(d.batch) * d.gy * d.gx * d.heads;
  const int per_head = d.channels / d.heads;
  const int block = d.levels * d.points * d.gz;  // offset / weight entries per (cell, head)

  const int64_t stride = static_cast<int64_t>(gridDim.x) * Sh::kGroups;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * Sh::kGroups + group;
       item - (threadIdx.x % 32) / G < items; item += stride) {
    const bool live = item < items;
    const int64_t it = live ? item : items - 1;
    const ItemCell ic = item_cell(it, d, items < (int64_t{1} << 31));
    const int head = ic.head, ix = ic.ix, iy = ic.iy;
    const int64_t cell = ic.cell, b = ic.b;
    const Cell c{__fadd_rn(grid.xmin, __fmul_rn(static_cast<float>(ix) + 0.5f, grid.sx)),
                 __fadd_rn(grid.ymin, __fmul_rn(static_cast<float>(iy) + 0.5f, grid.sy)), grid.zmin, grid.sz};
    int visible = 0;
    const int n = land_pairs<G>(d, proj + b * d.cams * 12, c, eps, img_h, img_w, live, sub, sm, visible);
    const int samples = n * d.levels * d.points;
    // groups of a warp land in different numbers of pairs: every group runs the
    // warp's longest sample loop (extra slots stage empty samples), so the warp
    // syncs below stay convergent
    const int trips = static_cast<int>(__reduce_max_sync(0xffffffffu, static_cast<unsigned>(samples)));
    const float* vb = value + b * d.cams * static_cast<int64_t>(d.stride_n) * d.channels + head * per_head + sub * 4;
    const float* off_item = offsets + it * block * 2;
    const float* w_item = weights + it * block;
    // Gathers read raw values; a non-finite feature value (or an overflowing
    // sum) leaves the lane's sum non-finite, and then every group of the warp
    // (the staging syncs need the whole warp) sums its item again with each
    // gathered value read as 0 when it is not finite, the reference's
    // _sanitize_value. Finite inputs never pay for the test per value.
    float4 acc = sum_item<G, false>(d, maps, off_item, w_item, trips, samples, sub, vb, sm);
    const bool finite = fabsf(acc.x) <= 3.402823466e+38f && fabsf(acc.y) <= 3.402823466e+38f &&
                        fabsf(acc.z) <= 3.402823466e+38f && fabsf(acc.w) <= 3.402823466e+38f;
    if (__any_sync(0xffffffffu, live && !finite))
      acc = sum_item<G, true>(d, maps, off_item, w_item, trips, samples, sub, vb, sm);
    if (live) {
      const float inv = visible > 0 ? __fdiv_rn(1.0f, static_cast<float>(visible)) : 0.0f;
      *reinterpret_cast<float4*>(out + cell * d.channels + head * per_head + sub * 4) =
          make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
  }
}

template <int G>
__global__ void FSCA_BWD_BOUNDS(G) backward_kernel(
    Dims d, float eps, const float* __restrict__ roi, const float* __restrict__ value,
    const float* __restrict__ proj, const int* __restrict__ shapes, const int* __restrict__ starts,
    const int* __restrict__ image_size, const float* __restrict__ offsets, const float* __restrict__ weights,
    const float* __restrict__ grad_out, float* __restrict__ grad_value, float* __restrict__ grad_offsets,
    float* __restrict__ grad_weights) {
  using Sh = Shape<G>;
  constexpr int C = Sh::kChunk;      // samples per dot round
  constexpr int Cs = Sh::kBwdChunk;  // samples per staged chunk
  __shared__ Map maps[kMaxLevels];
  __shared__ GroupSmem<G> smem[Sh::kGroups];
  stage_maps(maps, shapes, starts, d);
  const int sub = threadIdx.x % G, group = threadIdx.x / G;
  GroupSmem<G>& sm = smem[group];
  const float img_h = static_cast<float>(image_size[0]), img_w = static_cast<float>(image_size[1]);
  // the reference's backward grid: size = (max - min) / g from the roi tensor
  const Grid grid{__fdiv_rn(__fsub_rn(roi[1], roi[0]), static_cast<float>(d.gx)),
                  __fdiv_rn(__fsub_rn(roi[3], roi[2]), static_cast<float>(d.gy)),
                  __fdiv_rn(__fsub_rn(roi[5], roi[4]), static_cast<float>(d.gz)), roi[0], roi[2], roi[4]};
  const int64_t items = static_cast<int64_t>(d.batch) * d.gy * d.gx * d.heads;
  const int per_head = d.channels / d.heads;
  const int block = d.levels * d.points * d.gz;

  const int64_t stride = static_cast<int64_t>(gridDim.x) * Sh::kGroups;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * Sh::kGroups + group;
       item - (threadIdx.x % 32) / G < items; item += stride) {
    const bool live = item < items;
    const int64_t it = live ? item : items - 1;
    // 64-bit split in the backward: the 32-bit one measured slower here (1.239 -> 1.249 ms)
    const ItemCell ic = item_cell(it, d, false);
    const int head = ic.head, ix = ic.ix, iy = ic.iy;
    const int64_t cell = ic.cell, b = ic.b;
    const Cell c{__fadd_rn(grid.xmin, __fmul_rn(static_cast<float>(ix) + 0.5f, grid.sx)),
                 __fadd_rn(grid.ymin, __fmul_rn(static_cast<float>(iy) + 0.5f, grid.sy)), grid.zmin, grid.sz};
    int visible = 0;
    const int n = land_pairs<G>(d, proj + b * d.cams * 12, c, eps, img_h, img_w, live, sub, sm, visible);
    const int samples = n * d.levels * d.points;
    const int trips = static_cast<int>(__reduce_max_sync(0xffffffffu, static_cast<unsigned>(samples)));  // see forward
    // the level of a sample in level-major order by a multiply-high (one division per item)
    const int per_level = n * d.points;
    const uint32_t level_magic =
        per_level > 1 && static_cast<uint64_t>(samples) * per_level < (uint64_t{1} << 32) ? 0xffffffffu / per_level + 1 : 0;
    const int64_t plane = b * d.cams * static_cast<int64_t>(d.stride_n) * d.channels + head * per_head + sub * 4;
    const float* vb = value + plane;
    float* gvb = grad_value + plane;
    const float* off_item = offsets + it * block * 2;
    const float* w_item = weights + it * block;
    float* goff_item = grad_offsets + it * block * 2;
    float* gw_item = grad_weights + it * block;
    const float inv = visible > 0 ? __fdiv_rn(1.0f, static_cast<float>(visible)) : 0.0f;
    float4 g = *reinterpret_cast<const float4*>(grad_out + cell * d.channels + head * per_head + sub * 4);
    g = make_float4(g.x * inv, g.y * inv, g.z * inv, g.w * inv);  // grad * inv_count per channel

    for (int s0 = 0; s0 < trips; s0 += Cs) {
      if (sub % Sh::kBwdStager == 0) {
        const int i = sub / Sh::kBwdStager;
        stage<G, true>(d, maps, off_item, w_item, s0 + i, samples, i, sm, level_magic);
      }
      __syncwarp();
      // samples of one level around the heights of a camera share corner rows
      // (at the coarse levels most of them): each row's w * a is summed into
      // its first occurrence in the chunk and only those rows are sent
#if FSCA_BWD_FOLD && FSCA_BWD_HASH_FOLD
      msda::fold_rows_hashed<G, 4 * Cs, Sh::kHashSlots>(reinterpret_cast<const int*>(sm.row),
                                                       reinterpret_cast<float*>(sm.wa), sm.hash, sub);
#elif FSCA_BWD_FOLD
      msda::fold_repeated_rows<G, 4 * Cs>(reinterpret_cast<const int*>(sm.row),
                                          reinterpret_cast<float*>(sm.wa), sub);
#endif
#pragma unroll 1
      for (int c0 = 0; c0 < Cs; c0 += C) {
        float t[C][4];
#pragma unroll
        for (int i = 0; i < C; ++i) {
          const int4 r4 = sm.row[c0 + i];
          const float4 w4 = sm.wa[c0 + i];
          const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
          const float wa[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 raw = gather_raw(vb, rows[k], d.channels);
            float dot = g.x * raw.x + g.y * raw.y + g.z * raw.z + g.w * raw.w;
            float4 pay = make_float4(wa[k] * g.x, wa[k] * g.y, wa[k] * g.z, wa[k] * g.w);
            // the partial dot is finite unless a value of the slice is not (or a
            // product overflows); only then are the values tested one by one
            if (!(fabsf(dot) <= 3.402823466e+38f)) {
              const float4 v = sanitize(raw);
              dot = g.x * v.x + g.y * v.y + g.z * v.z + g.w * v.w;
              pay = make_float4(keep(raw.x, pay.x), keep(raw.y, pay.y), keep(raw.z, pay.z), keep(raw.w, pay.w));
            }
            t[i][k] = dot;
#if FSCA_BWD_PRED_RED
            msda::red_add_v4_if(rows[k] >= 0 && wa[k] != 0.0f,
                                gvb + static_cast<int64_t>(rows[k] >= 0 ? rows[k] : 0) * d.channels, pay.x, pay.y,
                                pay.z, pay.w);
#else
            if (rows[k] >= 0 && wa[k] != 0.0f)
              msda::red_add_v4(gvb + static_cast<int64_t>(rows[k]) * d.channels, pay.x, pay.y, pay.z, pay.w);
#endif
          }
        }
        msda::reduce_to_stagers<G, C>(t, sub);
        __syncwarp();  // the round's w * a slots are read; they take its dots
        if (sub % (G / C) == 0) sm.wa[c0 + sub / (G / C)] = make_float4(t[0][0], t[0][1], t[0][2], t[0][3]);
      }
      __syncwarp();
      // offset / weight gradients of the chunk: every stager lane takes its own
      // sample (the whole chunk in one pass of the warp)
      if (sub % Sh::kBwdStager == 0) {
        const int i = sub / Sh::kBwdStager;
        if (live && s0 + i < samples) {
          const float4 geo = sm.geo[i];
          const float du = geo.x, dv = geo.y, weight = geo.z;
          const int e = __float_as_int(geo.w);
          const float4 tt = sm.wa[i];  // f00, f01, f10, f11 dots
          const float hu = 1.0f - du, hv = 1.0f - dv;
          const float ds_du = hv * (tt.z - tt.x) + dv * (tt.w - tt.y);
          const float ds_dv = hu * (tt.y - tt.x) + du * (tt.w - tt.z);
          atomicAdd(goff_item + 2 * e, weight * ds_du);
          atomicAdd(goff_item + 2 * e + 1, weight * ds_dv);
          atomicAdd(gw_item + e, hu * hv * tt.x + hu * dv * tt.y + du * hv * tt.z + du * dv * tt.w);
        }
      }
      __syncwarp();
    }
  }
}

template <int G>
cudaError_t launch_forward(const Dims& d, const Grid& g, float eps, const Args& a, cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(d.batch) * d.gy * d.gx * d.heads;
  const int64_t blocks = (items + Shape<G>::kGroups - 1) / Shape<G>::kGroups;
  forward_kernel<G><<<static_cast<int>(blocks < (1LL << 30) ? blocks : (1LL << 30)), Shape<G>::kThreads, 0,
                      stream>>>(d, g, eps, a.value, a.projection, a.shapes, a.starts, a.image_size, a.offsets,
                                a.weights, a.out);
  return cudaGetLastError();
}

template <int G>
cudaError_t launch_backward(const Dims& d, float eps, const Args& a, cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(d.batch) * d.gy * d.gx * d.heads;
  const int64_t blocks = (items + Shape<G>::kGroups - 1) / Shape<G>::kGroups;
  backward_kernel<G><<<static_cast<int>(blocks < (1LL << 30) ? blocks : (1LL << 30)), Shape<G>::kThreads, 0,
                       stream>>>(d, eps, a.roi, a.value, a.projection, a.shapes, a.starts, a.image_size,
                                 a.offsets, a.weights, a.grad_out, a.grad_value, a.grad_offsets, a.grad_weights);
  return cudaGetLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int lanes_per_head(const Dims& d, const Args& a, bool backward) {
  if (d.heads <= 0 || d.channels % d.heads != 0) return 0;
  const int per_head = d.channels / d.heads;
  if (per_head % 4 != 0) return 0;
  const int g = per_head / 4;
  if (g != 1 && g != 2 && g != 4 && g != 8 && g != 16 && g != 32) return 0;
  if (!aligned16(a.value) || (reinterpret_cast<uintptr_t>(a.offsets) & 7u) != 0) return 0;
  if (backward ? (!aligned16(a.grad_out) || !aligned16(a.grad_value)) : !aligned16(a.out)) return 0;
  return g;
}

cudaError_t forward(const Dims& d, const Grid& g, float eps, const Args& a, cudaStream_t stream) {
  if (static_cast<int64_t>(d.batch) * d.gy * d.gx * d.heads == 0) return cudaSuccess;
  switch (lanes_per_head(d, a, false)) {
    case 1: return launch_forward<1>(d, g, eps, a, stream);
    case 2: return launch_forward<2>(d, g, eps, a, stream);
    case 4: return launch_forward<4>(d, g, eps, a, stream);
    case 8: return launch_forward<8>(d, g, eps, a, stream);
    case 16: return launch_forward<16>(d, g, eps, a, stream);
    case 32: return launch_forward<32>(d, g, eps, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t backward(const Dims& d, float eps, const Args& a, cudaStream_t stream) {
  if (static_cast<int64_t>(d.batch) * d.gy * d.gx * d.heads == 0) return cudaSuccess;
  switch (lanes_per_head(d, a, true)) {
    case 1: return launch_backward<1>(d, eps, a, stream);
    case 2: return launch_backward<2>(d, eps, a, stream);
    case 4: return launch_backward<4>(d, eps, a, stream);
    case 8: return launch_backward<8>(d, eps, a, stream);
    case 16: return launch_backward<16>(d, eps, a, stream);
    case 32: return launch_backward<32>(d, eps, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fsca
