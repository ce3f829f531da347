// Bucketed MSDA: head-rows grouped by where they sample; per-sample geometry
// staged once in shared memory; the backward's grad_value scatter combined
// per bilinear cell before it reaches L2.
//
// Why. A BEVFormer-base SCA call (6 cameras, 10000 queries, 8 heads, 4 levels x
// 8 points) makes 15 M samples = 61 M corner gathers of 64 bytes and, in the
// backward, 61 M corner scatters of 128 bytes (fp32). Scattered one by one the
// backward is bound by the L2 reduction rate (~6 TB/s of RED payload on B200),
// far above the HBM time of the whole call. But a head-row's samples cluster
// around one image position across all levels, and head-rows of neighbouring
// positions hit the same pixels, especially on the coarse levels.
//
// Bucketing. Every head-row (b, q, h) gets the key (b, h, tile): tile is the
// cell of a kTiles x kTiles grid over the normalised image holding the mean of
// its level-0 sampling locations. A counting sort (count, scan, scatter) lists
// head-row ids bucket by bucket in `order`; one CTA runs one bucket.
//
// Staging. A CTA walks its bucket in chunks of up to kMetaCap samples. For each
// sample one thread computes the geometry once (grid_sample's unnormalisation,
// corner pixels, bilinear weights times the attention weight) into SampleMeta;
// lane groups then run the head-rows against the staged samples: corner reads
// (through L1, which holds the bucket's neighbourhood), unpack, FMA.
//
// Backward scatter. Each level of a bucket gets a small pixel grid around its
// tile. A chunk's samples whose 2x2 corner footprint lies in the grid are
// counting-sorted by cell; each grid pixel then sums the contributions of the
// four cells touching it (weight x grad_out row, in registers) and issues one
// full-line vector RED. Samples outside the grid scatter their corners
// directly. The L2 sees one RED per touched pixel per chunk instead of one per
// sample corner.
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
#ifndef MSDA_FORWARD_BUCKETED
#define MSDA_FORWARD_BUCKETED 0
#endif
constexpr int kTiles = MSDA_TILES;       // bucket grid per image: kTiles x kTiles
constexpr float kMargin = MSDA_MARGIN;   // normalised margin of a scatter grid around its tile
constexpr int kMaxLevels = 16;           // level table entries staged per CTA
constexpr int kThreads = 256;
constexpr int kMetaCap = 1024;           // staged samples per chunk
constexpr int kMaxCells = 2048;          // scatter grid pixels per CTA (all levels)

struct Rect {    // scatter grid of one level
  int x0, y0;    // level pixel of grid pixel (0, 0)
  int gw, gh;    // grid extent in pixels (cells: gw - 1 by gh - 1)
  int base;      // first grid pixel of the level in the CTA's grid
};

struct SampleMeta {
  int4 pix;      // corner pixel (start + y * W + x) in the batch's map, -1 outside the level
  float4 wa;     // bilinear weight * attention weight per corner
};
// Corner order is (y0, x0), (y0, x1), (y1, x0), (y1, x1).

struct SampleAux {  // backward only
  float lh, lw, a;
  int slot;         // head-row in the chunk | level << 8 | (grid cell + 1) << 12; cell + 1 == 0: not in the grid
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
// staging
// ---------------------------------------------------------------------------
template <bool kBackward>
__device__ __forceinline__ void stage_sample(const Level& lv, const Rect* r, float loc_x, float loc_y, float a,
                                             SampleMeta& m, int& cell, float& lh_out, float& lw_out) {
  const float fh = static_cast<float>(lv.height), fw = static_cast<float>(lv.width);
  const float y = unnormalize(loc_y, 0.5f * fh);
  const float x = unnormalize(loc_x, 0.5f * fw);
  cell = -1;
  if (!(y > -2.0f && x > -2.0f && y < fh + 1.0f && x < fw + 1.0f)) {
    m.pix = make_int4(-1, -1, -1, -1);
    m.wa = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    lh_out = lw_out = 0.0f;
    return;
  }
  const float yf = floorf(y), xf = floorf(x);
  const int y0 = static_cast<int>(yf), x0 = static_cast<int>(xf);
  const float lh = __fsub_rn(y, yf), lw = __fsub_rn(x, xf);
  const float hh = __fsub_rn(1.0f, lh), hw = __fsub_rn(1.0f, lw);
  const bool x0ok = x0 >= 0 && x0 < lv.width, x1ok = x0 + 1 >= 0 && x0 + 1 < lv.width;
  const bool y0ok = y0 >= 0 && y0 < lv.height, y1ok = y0 + 1 >= 0 && y0 + 1 < lv.height;
  const int p00 = lv.start + y0 * lv.width + x0;
  m.pix = make_int4(y0ok && x0ok ? p00 : -1, y0ok && x1ok ? p00 + 1 : -1, y1ok && x0ok ? p00 + lv.width : -1,
                    y1ok && x1ok ? p00 + lv.width + 1 : -1);
  m.wa = make_float4(__fmul_rn(hh, hw) * a, __fmul_rn(hh, lw) * a, __fmul_rn(lh, hw) * a, __fmul_rn(lh, lw) * a);
  lh_out = lh;
  lw_out = lw;
  if (kBackward) {
    const int gx = x0 - r->x0, gy = y0 - r->y0;
    if (gx >= 0 && gy >= 0 && gx < r->gw - 1 && gy < r->gh - 1) cell = r->base + gy * r->gw + gx;
  }
}

// Stage every sample of head-rows order[first .. first + n); a warp takes
// whole head-rows (several per pass when they have <= 32 samples).
template <typename T, bool kBackward>
__device__ __forceinline__ void stage_chunk(const Dims& d, const Level* levels, const Rect* rects, const T* loc,
                                            const T* weight, const int* order, int first, int n, SampleMeta* meta,
                                            SampleAux* aux, int* pix_count, unsigned short* outside,
                                            int* n_outside) {
  const int samples = d.levels * d.points;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int per_pass = samples <= 32 ? 32 / samples : 1;
  const int lane_item = samples <= 32 ? lane / samples : 0;
  const int lane_s = samples <= 32 ? lane - lane_item * samples : lane;
  if (lane_item >= per_pass) return;
  for (int il = warp * per_pass + lane_item; il < n; il += nwarps * per_pass) {
    const int64_t item = order[first + il];
    for (int s = lane_s; s < samples; s += 32) {
      const int l = s / d.points;
      const float2 xy = load_loc(loc + (item * samples + s) * 2);
      const float a = to_f32(weight[item * samples + s]);
      const int j = il * samples + s;
      int cell;
      float lh, lw;
      stage_sample<kBackward>(levels[l], kBackward ? rects + l : nullptr, xy.x, xy.y, a, meta[j], cell, lh, lw);
      if (kBackward) {
        aux[j] = SampleAux{lh, lw, a, il | (l << 8) | ((cell + 1) << 12)};
        const int4 pix = meta[j].pix;
        if (cell >= 0) {
          const int gw = rects[l].gw;
          if (pix.x >= 0) atomicAdd(pix_count + cell, 1);
          if (pix.y >= 0) atomicAdd(pix_count + cell + 1, 1);
          if (pix.z >= 0) atomicAdd(pix_count + cell + gw, 1);
          if (pix.w >= 0) atomicAdd(pix_count + cell + gw + 1, 1);
        } else if (pix.x >= 0 || pix.y >= 0 || pix.z >= 0 || pix.w >= 0) {
          outside[atomicAdd(n_outside, 1)] = static_cast<unsigned short>(j);
        }
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 corner_row(const T* vlane, int pix, int row_stride) {
  return pix >= 0 ? ldg16(vlane + static_cast<int64_t>(pix) * row_stride) : make_uint4(0, 0, 0, 0);
}

// Lane layout shared by both kernels: a group of 2 * LPC lanes per head-row;
// lane (col, sub) holds 16 bytes (LPC per corner row) of corner column col.
template <typename T, int LPC>
struct Layout {
  static constexpr int kVec = 16 / static_cast<int>(sizeof(T));
  static constexpr int kD = LPC * kVec;
  static constexpr int kGroup = 2 * LPC;
  static constexpr int kGroups = kThreads / kGroup;
  __host__ __device__ static int items_per_chunk(int samples) {
    const int cap = kMetaCap / samples;
    return cap < kGroups * 8 ? cap : kGroups * 8;
  }
};

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <typename T, int LPC>
__global__ void __launch_bounds__(kThreads, 3) forward_bucketed_kernel(
    Dims d, const T* __restrict__ value, const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts,
    const T* __restrict__ loc, const T* __restrict__ weight, T* __restrict__ out, const int* __restrict__ order,
    const int* __restrict__ offset) {
  using L = Layout<T, LPC>;
  using V = Vec16<T>;
  constexpr int kVec = L::kVec, kGroup = L::kGroup;
  __shared__ Level levels[kMaxLevels];
  __shared__ SampleMeta meta[kMetaCap];
  const int key = blockIdx.x;
  const int begin = offset[key], end = offset[key + 1];
  if (begin == end) return;  // the whole CTA leaves together
  stage_level_table(d, shapes, starts, levels);
  __syncthreads();
  const int bh = key / (kTiles * kTiles), h = bh % d.heads, b = bh / d.heads;
  const int row_stride = d.heads * d.channels;
  const int samples = d.levels * d.points;
  const int lane_g = threadIdx.x % kGroup, col = lane_g / LPC, sub = lane_g % LPC;
  const T* vlane = value + (static_cast<int64_t>(b) * d.spatial_size) * row_stride + h * d.channels + sub * kVec;
  const int chunk = L::items_per_chunk(samples);
  // groups walk the chunk warp by warp: equal trip counts keep the shuffles convergent
  const int warp_first = (threadIdx.x / 32) * (32 / kGroup), in_warp = (threadIdx.x % 32) / kGroup;
  for (int first = begin; first < end; first += chunk) {
    const int n = min(chunk, end - first);
    stage_chunk<T, false>(d, levels, nullptr, loc, weight, order, first, n, meta, nullptr, nullptr, nullptr, nullptr);
    __syncthreads();
    for (int base = warp_first; base < n; base += L::kGroups) {
      const bool live = base + in_warp < n;
      const int il = live ? base + in_warp : n - 1;
      const SampleMeta* m = meta + il * samples;
      float acc[kVec];
#pragma unroll
      for (int i = 0; i < kVec; ++i) acc[i] = 0.0f;
#pragma unroll 4
      for (int s = 0; s < samples; ++s) {
        const int4 pix = m[s].pix;
        const float4 wa = m[s].wa;
        float v0[kVec], v1[kVec];
        V::unpack(corner_row(vlane, col ? pix.y : pix.x, row_stride), v0);
        V::unpack(corner_row(vlane, col ? pix.w : pix.z, row_stride), v1);
        const float w0 = col ? wa.y : wa.x, w1 = col ? wa.w : wa.z;
#pragma unroll
        for (int i = 0; i < kVec; ++i) acc[i] = fmaf(w1, v1[i], fmaf(w0, v0[i], acc[i]));
      }
#pragma unroll
      for (int i = 0; i < kVec; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], LPC, kGroup);
      if (live && col == 0) st16(out + static_cast<int64_t>(order[first + il]) * d.channels + sub * kVec, V::pack(acc));
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
// Per chunk: (1) stage samples, count grid cells, list samples outside the
// grids; copy the chunk's grad_out rows to shared memory in fp32. (2) lane
// groups run the head-rows: corner reads and the partial dot products
// T_k = sum_c g_c v_k,c, from which grad_w = sum_k w_k T_k,
// grad_x = W a (hh (T_01 - T_00) + lh (T_11 - T_10)),
// grad_y = H a (hw (T_10 - T_00) + lw (T_11 - T_01)). (3) scan the cell
// counts and sort the grid samples by cell. (4) every grid pixel sums
// wa_k * g over the samples of the four cells around it and issues one RED;
// then the samples outside the grids RED their corners one by one.
// Scatter workers of the backward: D/8 lanes per worker, 8 fp32 channels
// each; lane sl owns channels [4 sl, 4 sl + 4) and [D/2 + 4 sl, D/2 + 4 sl + 4),
// so each of the two REDs of a worker writes D*2 contiguous bytes (whole
// 32-byte sectors).
template <int D>
struct ScatterLayout {
  static constexpr int kLanes = D / 8;
  static constexpr int kWorkers = kThreads / kLanes;
  __device__ __forceinline__ static void accumulate(const float* grow, int sl, float2 w, float2* acc) {
    const float4 a = *reinterpret_cast<const float4*>(grow + 4 * sl);
    const float4 c = *reinterpret_cast<const float4*>(grow + D / 2 + 4 * sl);
    acc[0] = ffma2(make_float2(a.x, a.y), w, acc[0]);
    acc[1] = ffma2(make_float2(a.z, a.w), w, acc[1]);
    acc[2] = ffma2(make_float2(c.x, c.y), w, acc[2]);
    acc[3] = ffma2(make_float2(c.z, c.w), w, acc[3]);
  }
  __device__ __forceinline__ static void red(float* gline, int pixel, int row_stride, int sl, float2* acc) {
    if (pixel >= 0) {
      float* dst = gline + static_cast<int64_t>(pixel) * row_stride;
      red_add_v4(dst + 4 * sl, acc[0].x, acc[0].y, acc[1].x, acc[1].y);
      red_add_v4(dst + D / 2 + 4 * sl, acc[2].x, acc[2].y, acc[3].x, acc[3].y);
    }
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

// Shared-memory layout of the backward kernel.
template <typename T, int LPC>
struct BackwardSmem {
  Level* levels;
  Rect* rects;
  SampleMeta* meta;
  SampleAux* aux;
  int* pix_count;    // [kMaxCells]: entries per grid pixel, then the placement cursor
  int* pix_start;    // [kMaxCells + 1]
  int* pix_global;   // [kMaxCells]
  unsigned short* entries;  // [4 kMetaCap]: sample | corner << 10, sorted by grid pixel
  unsigned short* outside;  // [kMetaCap]: samples whose footprint leaves the grid
  int* scalars;             // [64]: [0] outside count, [1..32] scan scratch
  float* gstage;            // [items per chunk][D] grad_out rows in fp32
  static size_t bytes(int samples) {
    return 512 + static_cast<size_t>(kMetaCap) * (sizeof(SampleMeta) + sizeof(SampleAux)) +
           (3 * kMaxCells + 16) * sizeof(int) + 5 * kMetaCap * sizeof(unsigned short) + 64 * sizeof(int) +
           static_cast<size_t>(Layout<T, LPC>::items_per_chunk(samples)) * Layout<T, LPC>::kD * sizeof(float);
  }
  __device__ explicit BackwardSmem(unsigned char* base) {
    levels = reinterpret_cast<Level*>(base);
    rects = reinterpret_cast<Rect*>(base + sizeof(Level) * kMaxLevels);
    meta = reinterpret_cast<SampleMeta*>(base + 512);
    aux = reinterpret_cast<SampleAux*>(meta + kMetaCap);
    pix_count = reinterpret_cast<int*>(aux + kMetaCap);
    pix_start = pix_count + kMaxCells;
    pix_global = pix_start + kMaxCells + 16;
    entries = reinterpret_cast<unsigned short*>(pix_global + kMaxCells);
    outside = entries + 4 * kMetaCap;
    scalars = reinterpret_cast<int*>(outside + kMetaCap);
    gstage = reinterpret_cast<float*>(scalars + 64);
  }
};

template <typename T, int LPC>
__global__ void __launch_bounds__(kThreads, 2) backward_bucketed_kernel(
    Dims d, const T* __restrict__ value, const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts,
    const T* __restrict__ loc, const T* __restrict__ weight, const T* __restrict__ grad_out,
    float* __restrict__ grad_value, float* __restrict__ grad_loc, float* __restrict__ grad_weight,
    const int* __restrict__ order, const int* __restrict__ offset) {
  using L = Layout<T, LPC>;
  using V = Vec16<T>;
  using S = ScatterLayout<L::kD>;
  constexpr int kVec = L::kVec, kGroup = L::kGroup, kD = L::kD;
  extern __shared__ __align__(16) unsigned char smem[];
  BackwardSmem<T, LPC> sm(smem);

  const int key = blockIdx.x;
  const int begin = offset[key], end = offset[key + 1];
  if (begin == end) return;
  stage_level_table(d, shapes, starts, sm.levels);
  __syncthreads();
  const int tx = key % kTiles, ty = (key / kTiles) % kTiles, bh = key / (kTiles * kTiles);
  const int h = bh % d.heads, b = bh / d.heads;
  if (threadIdx.x == 0) plan_grids(sm.levels, sm.rects, d.levels, tx, ty);
  __syncthreads();
  // grid pixel -> pixel of the batch's map (-1 outside the level)
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
  const int lane_g = threadIdx.x % kGroup, col = lane_g / LPC, sub = lane_g % LPC;
  const int64_t head0 = (static_cast<int64_t>(b) * d.spatial_size) * row_stride + h * d.channels;
  const T* vlane = value + head0 + sub * kVec;
  const int chunk = L::items_per_chunk(samples);
  const int warp_first = (threadIdx.x / 32) * (32 / kGroup), in_warp = (threadIdx.x % 32) / kGroup;
  // scatter workers: S::kLanes lanes per worker, lane sl owns channels [4 sl, 4 sl + 4) and [D/2 + 4 sl, ...)
  const int worker = threadIdx.x / S::kLanes, sl = threadIdx.x % S::kLanes;
  float* gline = grad_value + head0;

  for (int first = begin; first < end; first += chunk) {
    const int n = min(chunk, end - first);
    for (int i = threadIdx.x; i < cells; i += blockDim.x) sm.pix_count[i] = 0;
    if (threadIdx.x == 0) sm.scalars[0] = 0;
    __syncthreads();
    // (1) staging, per-pixel entry counts, and the chunk's grad_out rows in fp32
    stage_chunk<T, true>(d, sm.levels, sm.rects, loc, weight, order, first, n, sm.meta, sm.aux, sm.pix_count,
                         sm.outside, sm.scalars);
    for (int i = threadIdx.x; i < n * LPC; i += blockDim.x) {
      const int il = i / LPC, part = i % LPC;
      float f[kVec];
      V::unpack(__ldg(reinterpret_cast<const uint4*>(grad_out + static_cast<int64_t>(order[first + il]) * d.channels) +
                      part),
                f);
#pragma unroll
      for (int v = 0; v < kVec; v += 4)
        *reinterpret_cast<float4*>(sm.gstage + il * kD + part * kVec + v) = make_float4(f[v], f[v + 1], f[v + 2], f[v + 3]);
    }
    __syncthreads();
    // (2) corner reads and the dot products T_k = sum_c g_c v_k,c, one head-row per group
    for (int base = warp_first; base < n; base += L::kGroups) {
      const bool live = base + in_warp < n;
      const int il = live ? base + in_warp : n - 1;
      const int64_t item = order[first + il];
      float2 g2[kVec / 2];
#pragma unroll
      for (int v = 0; v < kVec; v += 4) {
        const float4 q = *reinterpret_cast<const float4*>(sm.gstage + il * kD + sub * kVec + v);
        g2[v / 2] = make_float2(q.x, q.y);
        g2[v / 2 + 1] = make_float2(q.z, q.w);
      }
      const SampleMeta* m = sm.meta + il * samples;
      const SampleAux* ax = sm.aux + il * samples;
      int s = 0;
      for (int l = 0; l < d.levels; ++l) {
        const float fw = static_cast<float>(sm.levels[l].width), fh = static_cast<float>(sm.levels[l].height);
#pragma unroll 2
        for (int p = 0; p < d.points; ++p, ++s) {
          const int4 pix = m[s].pix;
          const uint4 r0 = corner_row(vlane, col ? pix.y : pix.x, row_stride);
          const uint4 r1 = corner_row(vlane, col ? pix.w : pix.z, row_stride);
          float2 a0 = make_float2(0.0f, 0.0f), a1 = make_float2(0.0f, 0.0f);
          const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w}, w1[4] = {r1.x, r1.y, r1.z, r1.w};
#pragma unroll
          for (int i = 0; i < kVec / 2; ++i) {
            const float2 v0 = sizeof(T) == 2 ? bf16x2_to_float2(w0[i])
                                             : make_float2(__uint_as_float(w0[2 * i]), __uint_as_float(w0[2 * i + 1]));
            const float2 v1 = sizeof(T) == 2 ? bf16x2_to_float2(w1[i])
                                             : make_float2(__uint_as_float(w1[2 * i]), __uint_as_float(w1[2 * i + 1]));
            a0 = ffma2(g2[i], v0, a0);
            a1 = ffma2(g2[i], v1, a1);
          }
          float t0 = a0.x + a0.y, t1 = a1.x + a1.y;
#pragma unroll
          for (int mask = 1; mask < LPC; mask <<= 1) {
            t0 += __shfl_xor_sync(0xffffffffu, t0, mask, kGroup);
            t1 += __shfl_xor_sync(0xffffffffu, t1, mask, kGroup);
          }
          const float u0 = __shfl_xor_sync(0xffffffffu, t0, LPC, kGroup);
          const float u1 = __shfl_xor_sync(0xffffffffu, t1, LPC, kGroup);
          if (live && lane_g == 0) {  // lane 0 is column 0: T_00 = t0, T_01 = u0, T_10 = t1, T_11 = u1
            const SampleAux q = ax[s];
            const float hh = 1.0f - q.lh, hw = 1.0f - q.lw;
            const int64_t so = item * samples + s;
            grad_weight[so] = hh * hw * t0 + hh * q.lw * u0 + q.lh * hw * t1 + q.lh * q.lw * u1;
            *reinterpret_cast<float2*>(grad_loc + 2 * so) = make_float2(
                fw * q.a * (hh * (u0 - t0) + q.lh * (u1 - t1)), fh * q.a * (hw * (t1 - t0) + q.lw * (u1 - u0)));
          }
        }
      }
    }
    // (3) entries (sample, corner) sorted by grid pixel: scan the counts, then place
    block_exclusive_scan(sm.pix_count, sm.pix_start, cells, sm.scalars + 1);
    for (int i = threadIdx.x; i < cells; i += blockDim.x) sm.pix_count[i] = sm.pix_start[i];  // placement cursor
    __syncthreads();
    for (int j = threadIdx.x; j < n * samples; j += blockDim.x) {
      const int slot = sm.aux[j].slot;
      const int cell = (slot >> 12) - 1;
      if (cell < 0) continue;
      const int gw = sm.rects[(slot >> 8) & 15].gw;
      const int4 pix = sm.meta[j].pix;
      const int pk[4] = {pix.x, pix.y, pix.z, pix.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (pk[k] >= 0) sm.entries[atomicAdd(sm.pix_count + cell + (k >> 1) * gw + (k & 1), 1)] =
                            static_cast<unsigned short>(j | (k << 10));
    }
    __syncthreads();
    // (4a) equal slices of the pixel-sorted entries: runs of one pixel sum in
    // registers and leave with one RED
    {
      const int total = sm.pix_start[cells];
      const int per = (total + S::kWorkers - 1) / S::kWorkers;
      const int e0 = min(total, worker * per), e1 = min(total, e0 + per);
      if (e0 < e1) {
        int lo = 0, hi = cells;  // last pixel whose start <= e0
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (sm.pix_start[mid] <= e0) lo = mid; else hi = mid;
        }
        int pixel = lo, next = sm.pix_start[pixel + 1];
        bool pending = false;
        float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                         make_float2(0.0f, 0.0f)};
        for (int e = e0; e < e1; ++e) {
          while (e >= next) {  // the run of `pixel` ended; empty pixels in between send nothing
            if (pending) S::red(gline, sm.pix_global[pixel], row_stride, sl, acc);
            pending = false;
            ++pixel;
            next = sm.pix_start[pixel + 1];
          }
          const int ent = sm.entries[e];
          const int j = ent & 1023, k = ent >> 10;
          const float w = reinterpret_cast<const float*>(&sm.meta[j].wa)[k];
          S::accumulate(sm.gstage + (sm.aux[j].slot & 255) * kD, sl, make_float2(w, w), acc);
          pending = true;
        }
        if (pending) S::red(gline, sm.pix_global[pixel], row_stride, sl, acc);
      }
    }
    // (4b) samples outside the grids: every in-level corner directly
    const int n_out = sm.scalars[0];
    for (int e = worker; e < n_out * 4; e += S::kWorkers) {
      const int j = sm.outside[e >> 2], k = e & 3;
      const int pix = reinterpret_cast<const int*>(&sm.meta[j].pix)[k];
      if (pix < 0) continue;
      const float w = reinterpret_cast<const float*>(&sm.meta[j].wa)[k];
      float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                       make_float2(0.0f, 0.0f)};
      S::accumulate(sm.gstage + (sm.aux[j].slot & 255) * kD, sl, make_float2(w, w), acc);
      S::red(gline, pix, row_stride, sl, acc);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Lanes per corner row for the bucketed kernels, or 0 when they do not apply.
int bucketed_lanes(const Dims& d, size_t elem, const Args& a) {
  const int g = vec_group(d.channels, elem, a);
  if (g != 2 && g != 4 && g != 8 && g != 16) return 0;
  if (d.channels % 4 != 0 || d.channels / 4 > 2 * g) return 0;  // one fp32 line within a group
  if (d.levels < 1 || d.levels > kMaxLevels) return 0;
  const int samples = d.levels * d.points;
  if (samples < 1 || samples > kMetaCap) return 0;
  const int64_t buckets = static_cast<int64_t>(d.batch) * d.heads * kTiles * kTiles;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  if (buckets >= (1LL << 30) || items >= (1LL << 31) - 1) return 0;
  return g;
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


template <typename T, int LPC>
cudaError_t launch_bucketed(bool forward, const Dims& d, const Args& a, const BucketPlan& plan, cudaStream_t stream) {
  if (forward) {
    forward_bucketed_kernel<T, LPC><<<plan.buckets, kThreads, 0, stream>>>(
        d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
        static_cast<const T*>(a.weight), static_cast<T*>(a.out), plan.order, plan.offset);
    return cudaGetLastError();
  }
  const size_t smem = BackwardSmem<T, LPC>::bytes(d.levels * d.points);
  auto kernel = backward_bucketed_kernel<T, LPC>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  kernel<<<plan.buckets, kThreads, smem, stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<const T*>(a.grad_out), a.grad_value, a.grad_loc, a.grad_weight,
      plan.order, plan.offset);
  return cudaGetLastError();
}

template <typename T>
cudaError_t run_bucketed(bool forward, const Dims& d, const Args& a, int lpc, const BucketPlan& plan,
                         cudaStream_t stream) {
  cudaError_t err = bucketize<T>(d, a, plan, stream);
  if (err != cudaSuccess) return err;
  switch (lpc) {
    case 2: return launch_bucketed<T, 2>(forward, d, a, plan, stream);
    case 4: return launch_bucketed<T, 4>(forward, d, a, plan, stream);
    case 8: return launch_bucketed<T, 8>(forward, d, a, plan, stream);
    default: return launch_bucketed<T, 16>(forward, d, a, plan, stream);
  }
}

// Scratch comes from the stream-ordered allocator (cudaMallocAsync) and goes
// back to it right after the launches; a failed allocation falls back to the
// row-wise kernels, which need no scratch.
cudaError_t dispatch(bool forward, DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  const size_t elem = dtype == DType::kBF16 ? 2 : 4;
#if MSDA_FORWARD_BUCKETED
  const int lpc = bucketed_lanes(d, elem, a);
#else
  const int lpc = forward ? 0 : bucketed_lanes(d, elem, a);
#endif
  if (lpc != 0) {
    void* scratch = nullptr;
    if (cudaMallocAsync(&scratch, plan_bytes(d), stream) == cudaSuccess) {
      const BucketPlan plan = carve(scratch, d);
      cudaError_t err = dtype == DType::kBF16 ? run_bucketed<__nv_bfloat16>(forward, d, a, lpc, plan, stream)
                                              : run_bucketed<float>(forward, d, a, lpc, plan, stream);
      const cudaError_t ferr = cudaFreeAsync(scratch, stream);
      return err != cudaSuccess ? err : ferr;
    }
    (void)cudaGetLastError();  // clear the allocation failure
  }
  return forward ? launch_forward_rowwise(dtype, d, a, stream) : launch_backward_rowwise(dtype, d, a, stream);
}

}  // namespace

cudaError_t launch_forward(DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0 || d.channels == 0) return cudaSuccess;
  return dispatch(true, dtype, d, a, stream);
}

cudaError_t launch_backward(DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0) return cudaSuccess;
  return dispatch(false, dtype, d, a, stream);
}

size_t backward_scratch_bytes(DType dtype, const Dims& d, const Args& a) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0) return 0;
  return bucketed_lanes(d, dtype == DType::kBF16 ? 2 : 4, a) != 0 ? plan_bytes(d) : 0;
}

cudaError_t launch_backward_on_scratch(DType dtype, const Dims& d, const Args& a, void* scratch, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0) return cudaSuccess;
  const int lpc = bucketed_lanes(d, dtype == DType::kBF16 ? 2 : 4, a);
  if (lpc == 0) return launch_backward_rowwise(dtype, d, a, stream);
  const BucketPlan plan = carve(scratch, d);
  return dtype == DType::kBF16 ? run_bucketed<__nv_bfloat16>(false, d, a, lpc, plan, stream)
                               : run_bucketed<float>(false, d, a, lpc, plan, stream);
}

}  // namespace msda
