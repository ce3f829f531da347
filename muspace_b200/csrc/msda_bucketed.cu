// grad_value for the MSDA backward, and the dispatch of both directions.
//
// Why. A BEVFormer-base SCA call (6 cameras, 10000 queries, 8 heads, 4 levels x
// 8 points) has 15 M samples. Scattering their 61 M corners one by one into
// grad_value (fp32, 128 bytes per corner and head) sends 7.6 GB of RED payload
// to L2, whose reduction rate on B200 (~5-6 TB/s) then bounds the backward far
// above the HBM time of the whole call. But a head-row's samples cluster
// around one image position across all levels, and head-rows that sample near
// each other hit the same pixels, most of all on the coarse levels.
//
// Bucketing. Every head-row (b, q, h) gets the key (b, h, tile): tile is the
// cell of a kTiles x kTiles grid over the normalised image holding the mean of
// its level-0 sampling locations. A counting sort (count, scan, scatter) lists
// head-row ids bucket by bucket in `order` (scratch); one CTA runs one bucket.
//
// Scatter. Each level gets a small pixel grid around the bucket's tile. The
// CTA stages its samples chunk by chunk, sorts the (sample, corner) entries
// that fall in the grid by pixel (counting sort in shared memory), and lets
// workers sum each pixel's run of entries in registers: one vector RED per
// pixel and chunk instead of one per sample corner (about 5x less RED traffic
// on BEVFormer-like sampling). Corners outside the grid RED directly.
//
// The backward is then: the row-wise kernel computing grad_loc / grad_w only
// (msda_backward.cu, full occupancy, no REDs) + this scatter. The forward is
// the row-wise kernel.
#include <algorithm>

#include "msda_device.cuh"

namespace msda {
namespace {

// Tuning constants; the MSDA_* macros let a build sweep them.
#ifndef MSDA_TILES
#define MSDA_TILES 10
#endif
#ifndef MSDA_MARGIN
#define MSDA_MARGIN 0.03f
#endif
constexpr int kTiles = MSDA_TILES;       // bucket grid per image: kTiles x kTiles
constexpr float kMargin = MSDA_MARGIN;   // normalised margin of a scatter grid around its tile
constexpr int kMaxLevels = 16;           // level table entries staged per CTA
constexpr int kThreads = 256;
constexpr int kMaxCells = 1280;          // scatter grid pixels per CTA (all levels)

struct Rect {    // scatter grid of one level
  int x0, y0;    // level pixel of grid pixel (0, 0)
  int gw, gh;    // grid extent in pixels (cells: gw - 1 by gh - 1)
  int base;      // first grid pixel of the level in the CTA's grid
};


struct BucketPlan {
  int* keys;    // [items]
  int* order;   // [items]
  int* count;   // [buckets]
  int* offset;  // [buckets + 1]
  int* cursor;  // [buckets]
  int buckets;
};

__device__ __forceinline__ int tile_of(float u) {
  const float t = floorf(u * static_cast<float>(kTiles));  // NaN -> tile 0
  return t >= 0.0f ? (t < static_cast<float>(kTiles) ? static_cast<int>(t) : kTiles - 1) : 0;
}

// ---------------------------------------------------------------------------
// bucketing: count, scan, scatter
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) bucket_count_kernel(Dims d, const T* __restrict__ loc, int* __restrict__ keys,
                                                           int* __restrict__ count) {
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int samples = d.levels * d.points;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < items;
       item += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const T* lp = loc + item * samples * 2;
    float sx = 0.0f, sy = 0.0f;
    for (int p = 0; p < d.points; ++p) {
      const float2 xy = load_loc(lp + 2 * p);
      sx += xy.x;
      sy += xy.y;
    }
    const float inv = 1.0f / static_cast<float>(d.points);
    const int h = static_cast<int>(item % d.heads);
    const int b = static_cast<int>(item / (static_cast<int64_t>(d.queries) * d.heads));
    const int key = ((b * d.heads + h) * kTiles + tile_of(sy * inv)) * kTiles + tile_of(sx * inv);
    keys[item] = key;
    atomicAdd(count + key, 1);
  }
}

// Exclusive scan of count[] into offset[] and cursor[] (one CTA of 1024).
__global__ void __launch_bounds__(1024) bucket_scan_kernel(const int* __restrict__ count, int* __restrict__ offset,
                                                           int* __restrict__ cursor, int buckets) {
  __shared__ int warp_sums[32];
  const int per = (buckets + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * per;
  const int hi = min(lo + per, buckets);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += count[i];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < static_cast<int>(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  int run = (warp > 0 ? warp_sums[warp - 1] : 0) + incl - local;
  for (int i = lo; i < hi; ++i) {
    offset[i] = run;
    cursor[i] = run;
    run += count[i];
  }
  if (threadIdx.x == blockDim.x - 1) offset[buckets] = run;
}

__global__ void __launch_bounds__(256) bucket_scatter_kernel(int64_t items, const int* __restrict__ keys,
                                                             int* __restrict__ cursor, int* __restrict__ order) {
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < items;
       item += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int pos = atomicAdd(cursor + keys[item], 1);
    order[pos] = static_cast<int>(item);
  }
}

// ---------------------------------------------------------------------------
// CTA set-up
// ---------------------------------------------------------------------------
__device__ __forceinline__ void stage_level_table(const Dims& d, const int64_t* shapes, const int64_t* starts,
                                                  Level* levels) {
  for (int l = threadIdx.x; l < d.levels; l += blockDim.x) {
    const int64_t hh = shapes[2 * l], ww = shapes[2 * l + 1], ss = starts[l];
    const bool ok =
        hh > 0 && ww > 0 && ss >= 0 && hh <= (1 << 24) && ww <= (1 << 24) && ss + hh * ww <= d.spatial_size;
    levels[l] = Level{ok ? static_cast<int>(hh) : 0, ok ? static_cast<int>(ww) : 0, ok ? static_cast<int>(ss) : 0};
  }
}

// Cells a location in [u0, u1] can fall in: floor(u * size - 0.5), clipped to
// [-1, size - 1] (cell -1 has its right / lower corners in the level).
__device__ __forceinline__ void cell_span(float u0, float u1, int size, int& lo, int& hi) {
  const float fs = static_cast<float>(size);
  lo = max(-1, static_cast<int>(floorf(u0 * fs - 0.5f)));
  hi = min(size - 1, static_cast<int>(floorf(u1 * fs - 0.5f)));
}

// Thread 0: grid of every level, coarsest first, within kMaxCells pixels; a
// level that does not fit keeps fewer rows (its other samples scatter
// directly).
__device__ void plan_grids(const Level* levels, Rect* rects, int n_levels, int tx, int ty) {
  const float t = 1.0f / static_cast<float>(kTiles);
  const float u0 = tx * t - kMargin, u1 = (tx + 1) * t + kMargin;
  const float v0 = ty * t - kMargin, v1 = (ty + 1) * t + kMargin;
  int used = 0;
  for (int l = n_levels - 1; l >= 0; --l) {
    Rect r{0, 0, 0, 0, used};
    if (levels[l].width > 0 && levels[l].height > 0) {
      int cx0, cx1, cy0, cy1;
      cell_span(u0, u1, levels[l].width, cx0, cx1);
      cell_span(v0, v1, levels[l].height, cy0, cy1);
      if (cx1 >= cx0 && cy1 >= cy0) {
        r.x0 = cx0;
        r.y0 = cy0;
        r.gw = cx1 - cx0 + 2;  // pixels cx0 .. cx1 + 1
        r.gh = cy1 - cy0 + 2;
        const int left = kMaxCells - used;
        if (r.gw * r.gh > left) r.gh = r.gw > 0 ? left / r.gw : 0;
        if (r.gh < 2) r.gw = r.gh = 0;
      }
    }
    rects[l] = r;
    used += r.gw * r.gh;
  }
}

// ---------------------------------------------------------------------------
// grad_value scatter
// ---------------------------------------------------------------------------
// Per chunk of up to kSampleCap samples of the bucket:
//   (1) one thread per sample stages its corner weights w_k * a, a validity
//       mask, and either its grid cell (footprint inside the level's grid) or
//       the pixel of its corner (y0, x0) (footprint leaves the grid); each
//       valid corner inside the grid counts one entry for its grid pixel;
//       the chunk's grad_out rows are copied to shared memory in fp32;
//   (2) exclusive scan of the per-pixel counts;
//   (3) one thread per sample places its entries (w_k * a, head-row) at
//       their pixel's slot: the entries are now sorted by grid pixel;
//   (4) workers of D/8 lanes take equal slices of the sorted entries; a run of
//       one pixel is summed in registers (fp32x2 FMAs on 8 channels per lane)
//       and leaves as two full-sector vector REDs;
//   (5) corners of samples outside the grid RED directly.
constexpr int kSampleCap = 1024;  // samples staged per chunk
constexpr int kItemCap = 64;      // head-rows per chunk

struct Staged {
  float4 wa;  // w_k * a for the corners (y0, x0), (y0, x1), (y1, x0), (y1, x1)
  int where;  // grid cell, or the pixel of corner (y0, x0) when `flags` has kOutside
  int flags;  // head-row in chunk | level << 8 | corner-valid mask << 12 | kOutside
};
constexpr int kOutside = 1 << 16;

// Scatter workers: D/8 lanes, 8 fp32 channels each; lane sl owns channels
// [4 sl, 4 sl + 4) and [D/2 + 4 sl, D/2 + 4 sl + 4), so each of a worker's two
// REDs writes 2D contiguous bytes (whole 32-byte sectors).
template <int D>
struct ScatterLayout {
  static constexpr int kLanes = D / 8;
  static constexpr int kWorkers = kThreads / kLanes;
  __device__ __forceinline__ static void accumulate(const float* grow, int sl, float w, float2* acc) {
    const float4 a = *reinterpret_cast<const float4*>(grow + 4 * sl);
    const float4 c = *reinterpret_cast<const float4*>(grow + D / 2 + 4 * sl);
    const float2 w2 = make_float2(w, w);
    acc[0] = ffma2(make_float2(a.x, a.y), w2, acc[0]);
    acc[1] = ffma2(make_float2(a.z, a.w), w2, acc[1]);
    acc[2] = ffma2(make_float2(c.x, c.y), w2, acc[2]);
    acc[3] = ffma2(make_float2(c.z, c.w), w2, acc[3]);
  }
  __device__ __forceinline__ static void red(float* gline, int pixel, int row_stride, int sl, float2* acc) {
    float* dst = gline + static_cast<int64_t>(pixel) * row_stride;
    red_add_v4(dst + 4 * sl, acc[0].x, acc[0].y, acc[1].x, acc[1].y);
    red_add_v4(dst + D / 2 + 4 * sl, acc[2].x, acc[2].y, acc[3].x, acc[3].y);
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.0f, 0.0f);
  }
};

// Exclusive scan of in[0, n) into out[0, n] by the whole CTA (scratch: 32 ints).
__device__ __forceinline__ void block_exclusive_scan(const int* in, int* out, int n, int* scratch) {
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * per, hi = min(lo + per, n);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += in[i];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  int run = incl - local;
  for (int w = 0; w < warp; ++w) run += scratch[w];
  for (int i = lo; i < hi; ++i) {
    out[i] = run;
    run += in[i];
  }
  if (threadIdx.x == blockDim.x - 1) out[n] = run;
  __syncthreads();
}

template <int D>
struct ScatterSmem {
  Level* levels;
  Rect* rects;
  Staged* staged;          // [kSampleCap]
  float* ent_w;            // [4 kSampleCap]
  unsigned short* ent_il;  // [4 kSampleCap]
  unsigned short* outside; // [kSampleCap]
  int* pix_count;          // [kMaxCells]: entries per grid pixel, then the placement cursor
  int* pix_start;          // [kMaxCells + 16]
  int* pix_global;         // [kMaxCells]: pixel of the batch's map, -1 outside the level
  int* scalars;            // [64]: [0] outside count, [32..63] scan scratch
  float* gstage;           // [kItemCap][D]
  static constexpr size_t kBytes = 512 + sizeof(Staged) * kSampleCap + 4 * kSampleCap * (sizeof(float) + 2) +
                                   2 * kSampleCap + (3 * kMaxCells + 16) * sizeof(int) + 64 * sizeof(int) +
                                   kItemCap * D * sizeof(float);
  __device__ explicit ScatterSmem(unsigned char* base) {
    levels = reinterpret_cast<Level*>(base);
    rects = reinterpret_cast<Rect*>(base + sizeof(Level) * kMaxLevels);
    staged = reinterpret_cast<Staged*>(base + 512);
    ent_w = reinterpret_cast<float*>(staged + kSampleCap);
    gstage = ent_w + 4 * kSampleCap;
    pix_count = reinterpret_cast<int*>(gstage + kItemCap * D);
    pix_start = pix_count + kMaxCells;
    pix_global = pix_start + kMaxCells + 16;
    scalars = pix_global + kMaxCells;
    ent_il = reinterpret_cast<unsigned short*>(scalars + 64);
    outside = ent_il + 4 * kSampleCap;
  }
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 3) scatter_bucketed_kernel(
    Dims d, const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts, const T* __restrict__ loc,
    const T* __restrict__ weight, const T* __restrict__ grad_out, float* __restrict__ grad_value,
    const int* __restrict__ order, const int* __restrict__ offset) {
  using S = ScatterLayout<D>;
  using V = Vec16<T>;
  constexpr int kVec = V::kLanes;
  extern __shared__ __align__(16) unsigned char smem[];
  ScatterSmem<D> sm(smem);

  const int key = blockIdx.x;
  const int begin = offset[key], end = offset[key + 1];
  if (begin == end) return;  // the whole CTA leaves together
  stage_level_table(d, shapes, starts, sm.levels);
  __syncthreads();
  const int tx = key % kTiles, ty = (key / kTiles) % kTiles, bh = key / (kTiles * kTiles);
  const int h = bh % d.heads, b = bh / d.heads;
  if (threadIdx.x == 0) plan_grids(sm.levels, sm.rects, d.levels, tx, ty);
  __syncthreads();
  int cells = 0;
  for (int l = 0; l < d.levels; ++l) {
    const Rect r = sm.rects[l];
    const Level lv = sm.levels[l];
    for (int gy = threadIdx.x / 32; gy < r.gh; gy += kThreads / 32)
      for (int gx = threadIdx.x % 32; gx < r.gw; gx += 32) {
        const int px = r.x0 + gx, py = r.y0 + gy;
        sm.pix_global[r.base + gy * r.gw + gx] =
            (px >= 0 && px < lv.width && py >= 0 && py < lv.height) ? lv.start + py * lv.width + px : -1;
      }
    cells = max(cells, r.base + r.gw * r.gh);
  }

  const int row_stride = d.heads * d.channels;
  const int samples = d.levels * d.points;
  float* gline = grad_value + (static_cast<int64_t>(b) * d.spatial_size) * row_stride + h * d.channels;
  const int worker = threadIdx.x / S::kLanes, sl = threadIdx.x % S::kLanes;
  const int chunk = min(kItemCap, kSampleCap / samples);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per_pass = samples <= 32 ? 32 / samples : 1;  // head-rows a warp stages per pass
  const int lane_item = samples <= 32 ? lane / samples : 0;
  const int lane_s = samples <= 32 ? lane - lane_item * samples : lane;

  for (int first = begin; first < end; first += chunk) {
    const int n = min(chunk, end - first);
    for (int i = threadIdx.x; i < cells; i += blockDim.x) sm.pix_count[i] = 0;
    if (threadIdx.x == 0) sm.scalars[0] = 0;
    __syncthreads();
    // (1) staging and per-pixel counts
    if (lane_item < per_pass) {
      for (int il = warp * per_pass + lane_item; il < n; il += (kThreads / 32) * per_pass) {
        const int64_t item = order[first + il];
        for (int s = lane_s; s < samples; s += 32) {
          const int l = s / d.points;
          const Level lv = sm.levels[l];
          const float2 xy = load_loc(loc + (item * samples + s) * 2);
          const float a = to_f32(weight[item * samples + s]);
          const float fh = static_cast<float>(lv.height), fw = static_cast<float>(lv.width);
          const float y = unnormalize(xy.y, 0.5f * fh);
          const float x = unnormalize(xy.x, 0.5f * fw);
          Staged st{make_float4(0.0f, 0.0f, 0.0f, 0.0f), 0, il | (l << 8)};
          if (y > -2.0f && x > -2.0f && y < fh + 1.0f && x < fw + 1.0f) {
            const float yf = floorf(y), xf = floorf(x);
            const int y0 = static_cast<int>(yf), x0 = static_cast<int>(xf);
            const float lh = __fsub_rn(y, yf), lw = __fsub_rn(x, xf);
            const float hh = __fsub_rn(1.0f, lh), hw = __fsub_rn(1.0f, lw);
            const bool x0ok = x0 >= 0 && x0 < lv.width, x1ok = x0 + 1 < lv.width;
            const bool y0ok = y0 >= 0 && y0 < lv.height, y1ok = y0 + 1 < lv.height;
            const int mask = (y0ok && x0ok ? 1 : 0) | (y0ok && x1ok && x0 + 1 >= 0 ? 2 : 0) |
                             (y1ok && x0ok && y0 + 1 >= 0 ? 4 : 0) | (y1ok && x1ok && x0 + 1 >= 0 && y0 + 1 >= 0 ? 8 : 0);
            st.wa = make_float4(__fmul_rn(hh, hw) * a, __fmul_rn(hh, lw) * a, __fmul_rn(lh, hw) * a,
                                __fmul_rn(lh, lw) * a);
            const Rect r = sm.rects[l];
            const int gx = x0 - r.x0, gy = y0 - r.y0;
            if (gx >= 0 && gy >= 0 && gx < r.gw - 1 && gy < r.gh - 1) {
              st.where = r.base + gy * r.gw + gx;
              st.flags |= mask << 12;
              if (mask & 1) atomicAdd(sm.pix_count + st.where, 1);
              if (mask & 2) atomicAdd(sm.pix_count + st.where + 1, 1);
              if (mask & 4) atomicAdd(sm.pix_count + st.where + r.gw, 1);
              if (mask & 8) atomicAdd(sm.pix_count + st.where + r.gw + 1, 1);
            } else if (mask) {
              st.where = lv.start + y0 * lv.width + x0;
              st.flags |= (mask << 12) | kOutside;
              sm.outside[atomicAdd(sm.scalars, 1)] = static_cast<unsigned short>(il * samples + s);
            }
          }
          sm.staged[il * samples + s] = st;
        }
      }
    }
    for (int i = threadIdx.x; i < n * (D / kVec); i += blockDim.x) {
      const int il = i / (D / kVec), part = i % (D / kVec);
      float f[kVec];
      V::unpack(__ldg(reinterpret_cast<const uint4*>(grad_out + static_cast<int64_t>(order[first + il]) * d.channels) +
                      part),
                f);
#pragma unroll
      for (int v = 0; v < kVec; v += 4)
        *reinterpret_cast<float4*>(sm.gstage + il * D + part * kVec + v) = make_float4(f[v], f[v + 1], f[v + 2], f[v + 3]);
    }
    __syncthreads();
    // (2) pixel offsets
    block_exclusive_scan(sm.pix_count, sm.pix_start, cells, sm.scalars + 32);
    for (int i = threadIdx.x; i < cells; i += blockDim.x) sm.pix_count[i] = sm.pix_start[i];
    __syncthreads();
    // (3) entries sorted by grid pixel
    for (int j = threadIdx.x; j < n * samples; j += blockDim.x) {
      const Staged st = sm.staged[j];
      if (st.flags & kOutside) continue;
      const int mask = (st.flags >> 12) & 15;
      if (!mask) continue;
      const int gw = sm.rects[(st.flags >> 8) & 15].gw;
      const unsigned short il = static_cast<unsigned short>(st.flags & 255);
      const float w4[4] = {st.wa.x, st.wa.y, st.wa.z, st.wa.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (!(mask & (1 << k))) continue;
        const int pos = atomicAdd(sm.pix_count + st.where + (k >> 1) * gw + (k & 1), 1);
        sm.ent_w[pos] = w4[k];
        sm.ent_il[pos] = il;
      }
    }
    __syncthreads();
    // (4) equal slices of the sorted entries; one RED per pixel run
    {
      const int total = sm.pix_start[cells];
      const int per = (total + S::kWorkers - 1) / S::kWorkers;
      int e = min(total, worker * per);
      const int e1 = min(total, e + per);
      if (e < e1) {
        int lo = 0, hi = cells;  // the pixel whose range holds e: last start <= e
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (sm.pix_start[mid] <= e) lo = mid; else hi = mid;
        }
        int pixel = lo;
        float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                         make_float2(0.0f, 0.0f)};
        while (e < e1) {
          const int stop = min(e1, sm.pix_start[pixel + 1]);
#pragma unroll 4
          for (; e < stop; ++e) S::accumulate(sm.gstage + sm.ent_il[e] * D, sl, sm.ent_w[e], acc);
          S::red(gline, sm.pix_global[pixel], row_stride, sl, acc);
          while (e < e1 && e >= sm.pix_start[pixel + 1]) ++pixel;  // skip to the next non-empty pixel
        }
      }
    }
    // (5) corners of samples outside the grid
    const int n_out = sm.scalars[0];
    for (int t = worker; t < n_out * 4; t += S::kWorkers) {
      const Staged st = sm.staged[sm.outside[t >> 2]];
      const int k = t & 3;
      if (!((st.flags >> 12) & (1 << k))) continue;
      const int width = sm.levels[(st.flags >> 8) & 15].width;
      float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                       make_float2(0.0f, 0.0f)};
      S::accumulate(sm.gstage + (st.flags & 255) * D, sl, reinterpret_cast<const float*>(&st.wa)[k], acc);
      S::red(gline, st.where + (k >> 1) * width + (k & 1), row_stride, sl, acc);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Whether the bucketed grad_value scatter applies (else the row-wise backward
// scatters its own corners).
bool scatter_applies(DType dtype, const Dims& d, const Args& a) {
  const size_t elem = dtype == DType::kBF16 ? 2 : 4;
  if (vec_group(d.channels, elem, a) == 0) return false;  // the row-wise dot kernel must be the vector one
  if (d.channels != 16 && d.channels != 32 && d.channels != 64 && d.channels != 128) return false;
  if (d.levels < 1 || d.levels > kMaxLevels) return false;
  const int samples = d.levels * d.points;
  if (samples < 1 || samples > kSampleCap) return false;
  const int64_t buckets = static_cast<int64_t>(d.batch) * d.heads * kTiles * kTiles;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  return buckets < (1LL << 30) && items < (1LL << 31) - 1;
}

size_t plan_bytes(const Dims& d) {
  const size_t items = static_cast<size_t>(d.batch) * d.queries * d.heads;
  const size_t buckets = static_cast<size_t>(d.batch) * d.heads * kTiles * kTiles;
  return (2 * items + 3 * buckets + 1) * sizeof(int);
}

BucketPlan carve(void* scratch, const Dims& d) {
  const size_t items = static_cast<size_t>(d.batch) * d.queries * d.heads;
  const int buckets = d.batch * d.heads * kTiles * kTiles;
  int* p = static_cast<int*>(scratch);
  BucketPlan plan;
  plan.keys = p;
  plan.order = p + items;
  plan.count = plan.order + items;
  plan.offset = plan.count + buckets;
  plan.cursor = plan.offset + buckets + 1;
  plan.buckets = buckets;
  return plan;
}

template <typename T>
cudaError_t bucketize(const Dims& d, const Args& a, const BucketPlan& plan, cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  cudaError_t err = cudaMemsetAsync(plan.count, 0, sizeof(int) * plan.buckets, stream);
  if (err != cudaSuccess) return err;
  const int grid = static_cast<int>(std::min<int64_t>((items + 255) / 256, grid_cap()));
  bucket_count_kernel<T><<<grid, 256, 0, stream>>>(d, static_cast<const T*>(a.loc), plan.keys, plan.count);
  bucket_scan_kernel<<<1, 1024, 0, stream>>>(plan.count, plan.offset, plan.cursor, plan.buckets);
  bucket_scatter_kernel<<<grid, 256, 0, stream>>>(items, plan.keys, plan.cursor, plan.order);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_scatter(const Dims& d, const Args& a, const BucketPlan& plan, cudaStream_t stream) {
  auto kernel = scatter_bucketed_kernel<T, D>;
  constexpr size_t smem = ScatterSmem<D>::kBytes;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);  // room for 3 CTAs
  if (err != cudaSuccess) return err;
  kernel<<<plan.buckets, kThreads, smem, stream>>>(d, a.shapes, a.starts, static_cast<const T*>(a.loc),
                                                    static_cast<const T*>(a.weight),
                                                    static_cast<const T*>(a.grad_out), a.grad_value, plan.order,
                                                    plan.offset);
  return cudaGetLastError();
}

// Backward = row-wise dot products (grad_loc, grad_w) + bucketed grad_value scatter.
template <typename T>
cudaError_t split_backward(DType dtype, const Dims& d, const Args& a, const BucketPlan& plan, cudaStream_t stream) {
  Args dots = a;
  dots.skip_grad_value = true;
  cudaError_t err = launch_backward_rowwise(dtype, d, dots, stream);
  if (err != cudaSuccess) return err;
  err = bucketize<T>(d, a, plan, stream);
  if (err != cudaSuccess) return err;
  switch (d.channels) {
    case 16: return launch_scatter<T, 16>(d, a, plan, stream);
    case 32: return launch_scatter<T, 32>(d, a, plan, stream);
    case 64: return launch_scatter<T, 64>(d, a, plan, stream);
    default: return launch_scatter<T, 128>(d, a, plan, stream);
  }
}

cudaError_t backward_with_plan(DType dtype, const Dims& d, const Args& a, void* scratch, cudaStream_t stream) {
  const BucketPlan plan = carve(scratch, d);
  return dtype == DType::kBF16 ? split_backward<__nv_bfloat16>(dtype, d, a, plan, stream)
                               : split_backward<float>(dtype, d, a, plan, stream);
}

}  // namespace

cudaError_t launch_forward(DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0 || d.channels == 0) return cudaSuccess;
  return launch_forward_rowwise(dtype, d, a, stream);
}

#ifndef MSDA_BUCKETED_BACKWARD
#define MSDA_BUCKETED_BACKWARD 0
#endif

// The fused row-wise backward (gathers, dot products and corner REDs in one
// pass) measures faster than dot products + bucketed scatter on every
// configuration so far, so it is the default. MSDA_BUCKETED_BACKWARD=1 builds
// the split form, with its bucket plan from the stream-ordered allocator.
cudaError_t launch_backward(DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0) return cudaSuccess;
  if (MSDA_BUCKETED_BACKWARD && scatter_applies(dtype, d, a)) {
    void* scratch = nullptr;
    if (cudaMallocAsync(&scratch, plan_bytes(d), stream) == cudaSuccess) {
      const cudaError_t err = backward_with_plan(dtype, d, a, scratch, stream);
      const cudaError_t ferr = cudaFreeAsync(scratch, stream);
      return err != cudaSuccess ? err : ferr;
    }
    (void)cudaGetLastError();  // clear the allocation failure
  }
  return launch_backward_rowwise(dtype, d, a, stream);
}

size_t backward_scratch_bytes(DType dtype, const Dims& d, const Args& a) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0) return 0;
  return scatter_applies(dtype, d, a) ? plan_bytes(d) : 0;
}

cudaError_t launch_backward_on_scratch(DType dtype, const Dims& d, const Args& a, void* scratch, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0) return cudaSuccess;
  if (!scatter_applies(dtype, d, a)) return launch_backward_rowwise(dtype, d, a, stream);
  return backward_with_plan(dtype, d, a, scratch, stream);
}

}  // namespace msda
