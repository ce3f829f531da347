// MSDA forward for bf16 value maps with D = 32, with the smallest levels of
// each head staged in shared memory by tiled TMA copies (sm_100a).
//
// The row-wise forward (msda_forward.cu) gathers every corner row of every
// sample from L2 through the load/store units, and that path bounds it. In
// BEVFormer's spatial cross-attention the two coarsest levels (29 x 50 and
// 15 x 25 pixels) take half of every head-row's samples but hold 1825
// pixels: one head's rows of them are 117 KB of bf16, gathered from L2 tens
// of thousands of times per camera.
//
// Here a CTA of 1024 threads owns one (image, head) and a tile of its
// queries. It selects on the device, from the level table (the shapes are
// device data), the smallest levels whose rows fit kStageRows, and copies
// that head's 64-byte rows of them into shared memory with
// cp.async.bulk.tensor.2d: 64-row boxes over the value map viewed as
// [B * Lin rows, Hh * D columns], all completing on one mbarrier. The
// corners of those levels are then read from shared memory, and the other
// levels keep the row-wise path: staged geometry per 8-sample chunk, 4 lanes
// x 16 bytes per head-row, packed fp32 FMAs in the row-wise kernel's order
// (so both kernels give bit-identical rows), out-of-level corners replaced
// by an in-level row with weight 0, and an exact re-sum of a head-row that
// comes out non-finite. A thread waits for the copies (bounded) only before
// its first staged sample, so they overlap the first head-row's other
// levels. A wait that gives up is counted in g_stage_wait_timeouts, and that
// thread reads the staged rows from global memory instead.
//
// Replaces the same reference kernels as the row-wise forward
// (csrc/ms_deformable_attn/ms_deform_attn_musa_kernel.muh:243-417).
#include <cuda.h>  // CUtensorMap and its enums only: the encoder comes from cudaGetDriverEntryPoint

#include <atomic>
#include <cstdlib>

#include "msda_device.cuh"

// Measured slower than the row-wise forward on B200 (c2 0.427 vs 0.305 ms,
// c4 2.98 vs 2.35 ms): the forward is bound by instruction issue as much as by
// L1TEX, a shared-memory gather costs the same instruction as the global one
// it replaces, and one 197 KB CTA per (image, head, tile) spreads the CTAs in
// flight over more value maps than L2 holds. So it is opt-in: a call takes it
// only while the environment variable MUSPACE_FWD_STAGED is "1" (read on every
// call), or always in builds with -DMSDA_FWD_STAGED=1.
#ifndef MSDA_FWD_STAGED
#define MSDA_FWD_STAGED 0
#endif

namespace msda {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kStThreads = 1024;
constexpr int kStLanes = 4;                       // lanes per head-row: 32 bf16 channels = 4 x 16 bytes
constexpr int kStGroups = kStThreads / kStLanes;  // head-rows in flight per CTA
constexpr int kStChunk = 8;                       // samples whose geometry is staged at once
constexpr int kStPerGroup = kStChunk + 1;         // geometry slots per group (+1 spreads the groups' banks)
constexpr int kStRowBytes = 64;                   // one head's 32 bf16 channels of one pixel
constexpr int kStBoxRows = 64;                    // rows per TMA box
constexpr int kStageRows = 1920;                  // staged rows per CTA (120 KB)
constexpr int kStSelectLevels = 16;               // levels the device-side selection looks at
constexpr int kStWaitLimit = 1 << 16;             // mbarrier polls before a wait gives up

__device__ unsigned int g_stage_wait_timeouts = 0;

struct TileGrid {
  int tiles;         // query tiles per (image, head)
  int tile_queries;  // queries per tile (the last tile may hold fewer, never none)
};

size_t staged_smem_bytes(int levels) {
  return 128 + static_cast<size_t>(kStageRows) * kStRowBytes +
         static_cast<size_t>(kStGroups) * kStPerGroup * (sizeof(int4) + sizeof(float4)) +
         static_cast<size_t>(levels > 0 ? levels : 1) * (sizeof(Level) + sizeof(int));
}

__device__ __forceinline__ uint32_t shared_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void copy_barrier_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void copy_barrier_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Polls the copy barrier's phase 0 at most kStWaitLimit times; false when
// the copies have not all landed by then.
__device__ __forceinline__ bool copy_barrier_wait(uint32_t bar) {
  for (int i = 0; i < kStWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(bar)
        : "memory");
    if (done) return true;
  }
  return false;
}

// One box of kStBoxRows value rows (this head's 32 channels of consecutive
// pixels) into shared memory at dst; x = h * 32 (64h bytes, a multiple of
// 16), y = the first pixel's row in the [B * Lin] view.
__device__ __forceinline__ void copy_rows(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared rows a staged level of px pixels occupies: px rounded up to even
// (every box then starts on a 128-byte boundary), at least one box.
__device__ __forceinline__ int staged_rows_of(int64_t px) {
  const int64_t even = (px + 1) & ~static_cast<int64_t>(1);
  return static_cast<int>(even > kStBoxRows ? even : kStBoxRows);
}

// Picks the staged levels, smallest first, while their rows fit kStageRows:
// stage_row[l] = the level's first shared row, -1 = not staged. Returns the
// rows used. One thread; every CTA computes the same selection.
__device__ int select_staged_levels(const Level* levels, int num_levels, int* stage_row) {
  for (int l = 0; l < num_levels; ++l) stage_row[l] = -1;
  const int n = num_levels < kStSelectLevels ? num_levels : kStSelectLevels;
  int used = 0;
  for (;;) {
    int best = -1;
    int64_t best_px = 0;
    for (int l = 0; l < n; ++l) {
      const int64_t px = static_cast<int64_t>(levels[l].height) * levels[l].width;
      if (stage_row[l] < 0 && px > 0 && (best < 0 || px < best_px)) best = l, best_px = px;
    }
    if (best < 0 || best_px > kStageRows) break;
    const int rows = staged_rows_of(best_px);
    if (used + rows > kStageRows) break;
    stage_row[best] = used;
    used += rows;
  }
  return used;
}

// Warp 0: arms the barrier with the bytes of every box, then its lanes issue
// the boxes. Box k of a level starts at row min(64 k, rows - 64) of it, so
// the boxes cover exactly the level's shared rows (the last two may overlap
// and then write the same bytes); rows past the level read the next pixels,
// or zeros past the end of the value map.
__device__ __forceinline__ void issue_stage_copies(const CUtensorMap* map, const Level* levels, const int* stage_row,
                                                   int num_levels, int row0, int col, uint32_t stage, uint32_t bar) {
  const int lane = threadIdx.x & 31;
  uint32_t bytes = 0;
  for (int l = 0; l < num_levels; ++l) {
    if (stage_row[l] < 0) continue;
    const int rows = staged_rows_of(static_cast<int64_t>(levels[l].height) * levels[l].width);
    bytes += static_cast<uint32_t>((rows + kStBoxRows - 1) / kStBoxRows) * kStBoxRows * kStRowBytes;
  }
  if (lane == 0) copy_barrier_expect(bar, bytes);
  __syncwarp();
  int n = 0;
  for (int l = 0; l < num_levels; ++l) {
    if (stage_row[l] < 0) continue;
    const int rows = staged_rows_of(static_cast<int64_t>(levels[l].height) * levels[l].width);
    for (int k = 0; k * kStBoxRows < rows; ++k, ++n) {
      if (n % 32 != lane) continue;
      const int r = k * kStBoxRows < rows - kStBoxRows ? k * kStBoxRows : rows - kStBoxRows;
      copy_rows(stage + static_cast<uint32_t>(stage_row[l] + r) * kStRowBytes, map, col, row0 + levels[l].start + r,
                bar);
    }
  }
}

// Sample s of a head-row, like stage_sample, into the group's slots; the
// corners of a staged level are stored as shared rows. kSubst: every corner
// outside its level (and every corner of a sample past the last) takes an
// in-level corner of the same sample, else the level's first pixel (pixel 0
// past the last level), with weight 0, so all four can be loaded.
template <bool kSubst>
__device__ __forceinline__ void stage_staged_sample(const Level* levels, const int* stage_row, LevelOf level, int samples,
                                                    bool live, int s, const bf16* lp, const bf16* wp, int4* row_slot,
                                                    float4* wa_slot) {
  int r[4] = {-1, -1, -1, -1};
  float w[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int first = 0, shift = 0;
  bool staged = false;
  if (s < samples) {
    const int l = level(s);
    const Level lv = levels[l];
    const int sr = stage_row[l];
    first = lv.start;
    staged = sr >= 0;
    shift = sr - lv.start;
    if (live) {
      const float2 xy = load_loc(lp + 2 * s);
      const float a = to_f32(wp[s]);
      Corners c;
      if (corners(lv, xy.x, xy.y, c)) {
#pragma unroll
        for (int k = 0; k < 4; ++k) r[k] = c.row[k], w[k] = c.w[k] * a;
      }
    }
  }
  if constexpr (kSubst) {
    const int any = r[0] >= 0 ? r[0] : r[1] >= 0 ? r[1] : r[2] >= 0 ? r[2] : r[3] >= 0 ? r[3] : first;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (r[k] < 0) r[k] = any, w[k] = 0.0f;
  }
  if (staged) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (r[k] >= 0) r[k] += shift;
  }
  *row_slot = make_int4(r[0], r[1], r[2], r[3]);
  *wa_slot = make_float4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ Words<4> lds_words(const unsigned char* p) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  Words<4> r;
  r.w[0] = v.x, r.w[1] = v.y, r.w[2] = v.z, r.w[3] = v.w;
  return r;
}

// acc (this lane's 4 channel pairs) = the head-row's sum over its samples.
// lane_stage points at this lane's 16 bytes of shared row 0; wait_state is
// the thread's copy state (0 not waited yet, 1 landed, 2 gave up). Every lane
// of the warp calls it (it syncs the warp).
template <bool kSubst>
__device__ __forceinline__ void gather_staged_row(const Level* levels, const int* stage_row, int num_levels,
                                                  LevelOf level, int samples, bool live, const bf16* vbase,
                                                  int row_stride, const unsigned char* lane_stage, uint32_t bar,
                                                  int& wait_state, const bf16* lp, const bf16* wp, int sub, int4* row,
                                                  float4* wa, float2 (&acc)[4]) {
  using S = Slice<bf16, 16>;
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.0f, 0.0f);
  int lvl = 0, lvl_end = level.points;
  int cur_sr = stage_row[0];
  int cur_shift = cur_sr - levels[0].start;
  for (int s0 = 0; s0 < samples; s0 += kStChunk) {
#pragma unroll
    for (int i = sub; i < kStChunk; i += kStLanes)
      stage_staged_sample<kSubst>(levels, stage_row, level, samples, live, s0 + i, lp, wp, row + i, wa + i);
    __syncwarp();
    for (int i = 0; i < kStChunk; ++i) {
      const int s = s0 + i;
      if (s >= lvl_end && lvl + 1 < num_levels) {  // warp-uniform: every group is at sample s
        ++lvl;
        lvl_end += level.points;
        cur_sr = stage_row[lvl];
        cur_shift = cur_sr - levels[lvl].start;
      }
      const bool st = s < samples && cur_sr >= 0;
      if (st && wait_state == 0) {
        wait_state = copy_barrier_wait(bar) ? 1 : 2;
        if (wait_state == 2) atomicAdd(&g_stage_wait_timeouts, 1u);
      }
      const int4 r4 = row[i];
      const float4 w4 = wa[i];
      const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
      const float was[4] = {w4.x, w4.y, w4.z, w4.w};
      Words<4> raw[4];
      if (st && wait_state == 1) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          raw[k] = (kSubst || rows[k] >= 0) ? lds_words(lane_stage + rows[k] * kStRowBytes) : zero_words<4>();
      } else {
        const int adj = st ? -cur_shift : 0;  // a staged row read from global memory after a given-up wait
#pragma unroll
        for (int k = 0; k < 4; ++k)
          raw[k] = (kSubst || rows[k] >= 0)
                       ? ldg_words<16>(vbase + static_cast<int64_t>(rows[k] + adj) * row_stride)
                       : zero_words<4>();
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 w2 = make_float2(was[k], was[k]);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = ffma2(w2, S::pair(raw[k], q), acc[q]);
      }
    }
    __syncwarp();
  }
}

}  // namespace

__global__ void __launch_bounds__(kStThreads, 1)
    forward_staged_kernel(const __grid_constant__ CUtensorMap map, Dims d, TileGrid tg, const bf16* __restrict__ value,
                          const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts,
                          const bf16* __restrict__ loc, const bf16* __restrict__ weight, bf16* __restrict__ out) {
  extern __shared__ unsigned char st_smem[];
  __shared__ __align__(8) uint64_t s_bar;
  __shared__ int s_staged_rows;

  unsigned char* stage = st_smem + ((128u - (shared_addr(st_smem) & 127u)) & 127u);
  int4* s_row = reinterpret_cast<int4*>(stage + kStageRows * kStRowBytes);
  float4* s_wa = reinterpret_cast<float4*>(s_row + kStGroups * kStPerGroup);
  Level* levels = reinterpret_cast<Level*>(s_wa + kStGroups * kStPerGroup);
  int* stage_row = reinterpret_cast<int*>(levels + d.levels);
  const uint32_t bar = shared_addr(&s_bar);

  const int h = static_cast<int>(blockIdx.x % d.heads);
  const int tile = static_cast<int>((blockIdx.x / d.heads) % tg.tiles);
  const int b = static_cast<int>(blockIdx.x / (static_cast<unsigned>(d.heads) * tg.tiles));
  if (threadIdx.x == 0) copy_barrier_init(bar);
  stage_levels(levels, shapes, starts, d);  // ends with a CTA barrier
  if (threadIdx.x == 0) s_staged_rows = select_staged_levels(levels, d.levels, stage_row);
  __syncthreads();
  const int staged_rows = s_staged_rows;
  if (threadIdx.x < 32 && staged_rows > 0)
    issue_stage_copies(&map, levels, stage_row, d.levels, b * d.spatial_size, h * 32, shared_addr(stage), bar);

  const int q0 = tile * tg.tile_queries;
  const int n = d.queries - q0 < tg.tile_queries ? d.queries - q0 : tg.tile_queries;
  const int grp = threadIdx.x / kStLanes, sub = threadIdx.x % kStLanes;
  const int in_warp = (threadIdx.x % 32) / kStLanes;  // the group's index inside its warp
  const int row_stride = d.heads * 32;
  const int samples = d.levels * d.points;
  const bf16* vbase = value + static_cast<int64_t>(b) * d.spatial_size * row_stride + h * 32 + sub * 8;
  const unsigned char* lane_stage = stage + sub * 16;
  int4* row = s_row + grp * kStPerGroup;
  float4* wa = s_wa + grp * kStPerGroup;
  int wait_state = staged_rows > 0 ? 0 : 1;
  // whole warps take the same number of trips (set by the warp's first group)
  for (int j = grp; j - in_warp < n; j += kStGroups) {
    const bool live = j < n;
    const int64_t item = (static_cast<int64_t>(b) * d.queries + q0 + (live ? j : n - 1)) * d.heads + h;
    const bf16* lp = loc + item * samples * 2;
    const bf16* wp = weight + item * samples;
    float2 acc[4];
    gather_staged_row<true>(levels, stage_row, d.levels, level_of(d), samples, live, vbase, row_stride, lane_stage, bar,
                            wait_state, lp, wp, sub, row, wa, acc);
    if (__any_sync(0xffffffffu, live && !finite_pairs(acc)))  // warp-uniform, rare
      gather_staged_row<false>(levels, stage_row, d.levels, level_of(d), samples, live, vbase, row_stride, lane_stage,
                               bar, wait_state, lp, wp, sub, row, wa, acc);
    if (live) store_slice<bf16, 16>(out + item * 32 + sub * 8, acc);
  }
  // no copy may still be landing in this CTA's shared memory when it exits
  if (threadIdx.x == 0 && staged_rows > 0 && wait_state != 1 && !copy_barrier_wait(bar))
    atomicAdd(&g_stage_wait_timeouts, 1u);
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn tensor_map_encoder() {
  static const EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Query tiles per (image, head): the count that minimises waves x rounds
// (a CTA per SM; a round = one head-row per group), fewest tiles on a tie.
TileGrid choose_tiles(int64_t pairs, int queries, int sms) {
  struct Memo {
    int64_t pairs = -1;
    int queries = -1, sms = -1;
    TileGrid tg{1, 1};
  };
  static thread_local Memo memo;
  if (memo.pairs == pairs && memo.queries == queries && memo.sms == sms) return memo.tg;
  TileGrid best{1, queries};
  int64_t best_cost = -1;
  const int max_tiles = queries / (kStGroups / 2) > 1 ? queries / (kStGroups / 2) : 1;
  for (int t = 1; t <= max_tiles; ++t) {
    const int qt = (queries + t - 1) / t;
    const int tiles = (queries + qt - 1) / qt;  // no empty tile
    if (tiles != t) continue;
    const int64_t waves = (pairs * tiles + sms - 1) / sms;
    const int64_t rounds = (qt + kStGroups - 1) / kStGroups;
    const int64_t cost = waves * (8 * rounds + 1);  // + about an eighth of a round to stage a CTA's levels
    if (best_cost < 0 || cost < best_cost) best_cost = cost, best = TileGrid{tiles, qt};
  }
  memo.pairs = pairs, memo.queries = queries, memo.sms = sms, memo.tg = best;
  return best;
}

std::atomic<size_t> g_smem_set[64];  // dynamic shared memory the kernel is opened to, per device

}  // namespace

unsigned int staged_wait_timeouts() {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_stage_wait_timeouts, sizeof(v)) != cudaSuccess) return ~0u;
  return v;
}

// The staged forward when the call suits it (bf16, D = 32, natural order,
// enough head-rows to fill the GPU with 4-round CTAs, some level that can
// fit); *used = false leaves the call to the row-wise kernels.
cudaError_t launch_forward_staged(const Dims& d, const Args& a, cudaStream_t stream, bool* used) {
  *used = false;
  if (!MSDA_FWD_STAGED) {
    const char* on = std::getenv("MUSPACE_FWD_STAGED");
    if (!on || on[0] != '1' || on[1] != '\0') return cudaSuccess;
  }
  if (d.channels != 32 || d.heads <= 0 || d.levels <= 0 || d.points <= 0 || d.spatial_size <= 0 || d.batch <= 0 ||
      d.queries <= 0 || a.order != nullptr)
    return cudaSuccess;
  if (d.levels == 1 && d.spatial_size > kStageRows) return cudaSuccess;  // nothing could be staged
  if (!aligned16(a.value) || !aligned16(a.out) || (reinterpret_cast<uintptr_t>(a.loc) & 3u) != 0) return cudaSuccess;
  if (static_cast<int64_t>(d.batch) * d.spatial_size + kStageRows >= (int64_t{1} << 31)) return cudaSuccess;
  int dev = 0, sms = 0, smem_max = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaSuccess;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return cudaSuccess;
  const int64_t pairs = static_cast<int64_t>(d.batch) * d.heads;
  if (pairs * d.queries < static_cast<int64_t>(sms) * kStGroups * 4) return cudaSuccess;
  const size_t smem = staged_smem_bytes(d.levels);
  if (smem + 64 > static_cast<size_t>(smem_max)) return cudaSuccess;
  const EncodeTiledFn encode = tensor_map_encoder();
  if (!encode) return cudaSuccess;

  CUtensorMap map;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.heads) * 32,
                              static_cast<cuuint64_t>(d.batch) * static_cast<cuuint64_t>(d.spatial_size)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(d.heads) * 32 * sizeof(bf16)};
  const cuuint32_t box[2] = {32, kStBoxRows};
  const cuuint32_t elem[2] = {1, 1};
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.value), dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaSuccess;

  const TileGrid tg = choose_tiles(pairs, d.queries, sms);
  const int64_t blocks = pairs * tg.tiles;
  if (blocks > 0x7fffffffLL) return cudaSuccess;
  if (g_smem_set[dev].load(std::memory_order_relaxed) < smem) {
    const cudaError_t e =
        cudaFuncSetAttribute(forward_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    g_smem_set[dev].store(smem, std::memory_order_relaxed);
  }
  *used = true;
  forward_staged_kernel<<<static_cast<unsigned>(blocks), kStThreads, smem, stream>>>(
      map, d, tg, static_cast<const bf16*>(a.value), a.shapes, a.starts, static_cast<const bf16*>(a.loc),
      static_cast<const bf16*>(a.weight), static_cast<bf16*>(a.out));
  return cudaGetLastError();
}

}  // namespace msda
