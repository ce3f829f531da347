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
// corner's whole 128-byte fp32 grad_value line). The head-row's samples are
// taken in chunks of Cs = min(G, 8) (4 for head-rows of at most 4 samples):
//  1. stage: the lane at sub = i * G / Cs computes the geometry of chunk
//     sample i once and stages its four corner rows, w_k * a and
//     (lh, lw, W a, H a) in shared memory;
//  2. fold: the chunk's 4 Cs (corner row, w_k * a) entries are merged by row
//     (samples of one head-row cluster, so at coarse levels most corners
//     repeat: on BEVFormer-like locations 117 corner rows per head-row shrink
//     to 72); a repeated row's w_k * a moves to its first occurrence;
//  3. per sample: every lane gathers its slice of the four corners, forms the
//     corner dots T_k = sum_c g_c v_k,c over its channels (packed fp32x2
//     FMAs) and sends (sum of w_k * a) * g for each first-occurrence row with
//     red.global.add.v4.f32; after every round of Cd samples (4 for bf16, 2
//     for fp32) a transpose reduction hands one lane per sample the four T_k,
//     which it puts in shared memory;
//  4. after the rounds every stager lane writes its own sample's
//       grad_w = sum_k w_k T_k,
//       grad_x = W a (hh (T_1 - T_0) + lh (T_3 - T_2)),
//       grad_y = H a (hw (T_2 - T_0) + lw (T_3 - T_1))
//     (the whole chunk in one pass of the warp, contiguous stores).
// That is backward_vec_kernel. For bf16 D = 16 / 32 (every BEVFormer shape)
// backward_pair_kernel runs instead: the
// same stage and fold, then a lane pair forms one sample's dots (no transpose
// reduction) and every lane sends 4-channel fp32 REDs (description above the
// kernel).
#include "msda_device.cuh"

namespace msda {

#ifndef MSDA_BWD_CHUNK_F32
#define MSDA_BWD_CHUNK_F32 2
#endif
#ifndef MSDA_BWD_MINBLOCKS_F32
#define MSDA_BWD_MINBLOCKS_F32 4
#endif
#ifndef MSDA_BWD_MINBLOCKS_BF16
#define MSDA_BWD_MINBLOCKS_BF16 4
#endif
#ifndef MSDA_BWD_PAIR
#define MSDA_BWD_PAIR 1
#endif
#ifndef MSDA_BWD_MIXED_FMA
#define MSDA_BWD_MIXED_FMA 1
#endif
#ifndef MSDA_BWD_DEDUP
#define MSDA_BWD_DEDUP 1
#endif
// 1: repeated corner rows fold through a per-group hash table in shared
// memory (fold_rows_hashed) instead of a scan over all lower entries.
#ifndef MSDA_BWD_HASH_FOLD
#define MSDA_BWD_HASH_FOLD 1
#endif
// 1: the REDs of the lane-pair kernel are predicated instead of branched
// around (a warp's four groups disagree on which entries need one).
#ifndef MSDA_BWD_PRED_RED
#define MSDA_BWD_PRED_RED 1
#endif
// 1: bf16 D = 32 forms a sample's dots with four lanes (one 16-byte chunk of
// each corner row per lane) instead of a lane pair (two chunks per lane).
#ifndef MSDA_BWD_QUAD
#define MSDA_BWD_QUAD 1
#endif
// 1: for head-rows of at most 4 samples with one 16-byte chunk per lane (all
// four corners in flight) the first dot pass's gathers are issued before the
// row fold (c3 backward 0.275 -> 0.262 ms, bevformer-1l bf16 0.269 -> 0.262;
// with four passes per chunk, as at c4, it measured 0.5-1 % slower).
#ifndef MSDA_BWD_PREFETCH
#define MSDA_BWD_PREFETCH 1
#endif
// 1: the lane-pair kernel also takes bf16 head-rows of at most 4 samples.
#ifndef MSDA_PAIR_SHORT
#define MSDA_PAIR_SHORT 1
#endif
// Samples per dot round (their partial dots live in registers: 4 per sample)
// and CTAs per SM the register budget is sized for; measured on B200 (fp32
// D = 32: rounds of 2 at 3 CTAs/SM beat rounds of 4 at 2 or 3; 4 CTAs/SM at
// 64 registers beat 3 for fp32 D = 32 and bf16 8-byte lanes by 2-3 %).
template <typename T>
constexpr int kChunk = sizeof(T) == 2 ? 4 : MSDA_BWD_CHUNK_F32;
template <typename T, int kBytes>
constexpr int kMinBlocks = sizeof(T) == 2 ? (kBytes == 8 ? MSDA_BWD_MINBLOCKS_BF16 : 2) : MSDA_BWD_MINBLOCKS_F32;

// kScatter = false computes grad_loc / grad_w only; grad_value then comes from
// the bucketed scatter kernel (msda_bucketed.cu).
template <typename T, int G, int kBytes, int kStageMax, bool kScatter>
__global__ void __launch_bounds__(kCtaThreads, kMinBlocks<T, kBytes>) backward_vec_kernel(
    Dims d, const T* __restrict__ value, const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts,
    const T* __restrict__ loc, const T* __restrict__ weight, const T* __restrict__ grad_out,
    float* __restrict__ grad_value, float* __restrict__ grad_loc, float* __restrict__ grad_weight,
    const int* __restrict__ order) {
  using S = Slice<T, kBytes>;
  constexpr int kCh = S::kChannels, kPairs = S::kPairs, kWords = kBytes / 4;
  constexpr int Cs = G < kStageMax ? G : kStageMax;       // samples staged per chunk
  constexpr int kStage = G / Cs;                           // stager lanes: sub % kStage == 0
  constexpr int Cd = Cs < kChunk<T> ? Cs : kChunk<T>;      // samples per dot round
  constexpr int kFin = G / Cd;                             // finishing lanes: sub % kFin == 0
  constexpr int kGroups = kCtaThreads / G;
  // Each group's Cs slots plus one of padding, so the groups of a warp reading
  // their slot i at once hit different shared-memory banks.
  constexpr int kSlots = Cs + 1;
  extern __shared__ Level levels[];
  __shared__ int4 s_row[kGroups * kSlots];
  __shared__ float4 s_wa[kGroups * kSlots];
  __shared__ float4 s_geo[kGroups * kSlots];
  __shared__ float4 s_dots[kGroups * kSlots];
  stage_levels(levels, shapes, starts, d);

  const int sub = threadIdx.x % G;
  const int base = (threadIdx.x / G) * kSlots;  // the group's slots are base .. base + Cs - 1
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
    const ImageHead ih = image_head(it, d, items < (int64_t{1} << 31));
    const int h = ih.h;
    const int64_t b = ih.b;
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

    for (int s0 = 0; s0 < samples; s0 += Cs) {
      // 1. stage, with the geometry of the gradient formula: (lh, lw, W a, H a),
      // lh = -1 for a sample with no corner inside its level
      if (sub % kStage == 0) {
        const int i = sub / kStage;
        float4 geo = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float2 wh = make_float2(0.0f, 0.0f);
        const bool valid =
            stage_sample(levels, level_of(d), samples, live, s0 + i, lp, wp, s_row + base + i, s_wa + base + i, &geo, &wh);
        s_geo[base + i] =
            valid ? make_float4(geo.x, geo.y, wh.x * geo.z, wh.y * geo.z) : make_float4(-1.0f, 0.0f, 0.0f, 0.0f);
      }
      __syncwarp();
#if MSDA_BWD_DEDUP
      // 2. one RED per distinct corner row of the chunk
      if constexpr (kScatter)
        fold_repeated_rows<G, 4 * Cs>(reinterpret_cast<const int*>(s_row + base),
                                      reinterpret_cast<float*>(s_wa + base), sub);
#endif
      // 3. per sample: gathers, corner dots, the sample's REDs; per round the
      // dots reach their sample's finishing lane
#pragma unroll
      for (int r = 0; r < Cs / Cd; ++r) {
        float t[Cd][4];
#pragma unroll
        for (int i = 0; i < Cd; ++i) {
          const int4 r4 = s_row[base + r * Cd + i];
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
            const float4 w4 = s_wa[base + r * Cd + i];
            const float wa[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (rows[k] >= 0 && wa[k] != 0.0f)
                scatter_slice<kPairs>(gbase + static_cast<int64_t>(rows[k]) * row_stride, wa[k], g2);
          }
        }
        reduce_to_stagers<G, Cd>(t, sub);
        if (sub % kFin == 0) s_dots[base + r * Cd + sub / kFin] = make_float4(t[0][0], t[0][1], t[0][2], t[0][3]);
      }
      __syncwarp();
      // 4. grad_w / grad_loc of the chunk: every stager lane takes its own
      // sample (the whole chunk in one pass of the warp)
      if (sub % kStage == 0) {
        const int i = sub / kStage;
        const int s = s0 + i;
        if (live && s < samples) {
          const float4 geo = s_geo[base + i];
          const float4 t = s_dots[base + i];
          float gw = 0.0f, gx = 0.0f, gy = 0.0f;
          if (geo.x >= 0.0f) {
            const float lh = geo.x, lw = geo.y;
            const float hh = __fsub_rn(1.0f, lh), hw = __fsub_rn(1.0f, lw);
            gw = __fmul_rn(hh, hw) * t.x + __fmul_rn(hh, lw) * t.y + __fmul_rn(lh, hw) * t.z + __fmul_rn(lh, lw) * t.w;
            gx = geo.z * (hh * (t.y - t.x) + lh * (t.w - t.z));
            gy = geo.w * (hw * (t.z - t.x) + lw * (t.w - t.y));
          }
          const int64_t so = it * samples + s;
          grad_weight[so] = gw;
          *reinterpret_cast<float2*>(grad_loc + 2 * so) = make_float2(gx, gy);
        }
      }
      __syncwarp();  // the next chunk's staging overwrites the slots read above
    }
  }
}

// Backward with the work of a sample split two ways. kCPL = 16-byte chunks of
// the head-row each lane of a pair holds (the row has 2 kCPL chunks), and
// G = D / 4 lanes per head-row (each owning a 4-channel fp32 slice of the
// gradients). Per chunk of Cs staged samples:
//  - stage / fold as in backward_vec_kernel;
//  - dots: a lane pair owns a sample, lane h of the pair holding chunks h,
//    h + 2, ... (so the pair's first loads fill whole 32-byte sectors); it
//    gathers those chunks of the four corners, forms the corner dots with its
//    grad_output chunks, xor shuffles complete them, and lane 0 of the pair
//    (or quad, kLPS = 4) puts them in shared memory: no transpose reduction;
//  - REDs: every lane sends its 4-channel slice of (sum of w_k a) * g for each
//    first-occurrence corner row (whole 128-byte lines per group for D = 32);
//  - grad_w / grad_loc as in backward_vec_kernel, once per chunk by the stager
//    lanes.

// CTAs per SM the lane-pair kernel's register budget is sized for (4: 64
// registers, 32 resident warps; 8.60 -> 8.06 ms for the c4 backward against 3).
#ifndef MSDA_PAIR_MINBLOCKS
#define MSDA_PAIR_MINBLOCKS 4
#endif

template <typename T, int kCPL, int kStageMax, bool kScatter, int kLPS = 2>
__global__ void __launch_bounds__(kCtaThreads, MSDA_PAIR_MINBLOCKS) backward_pair_kernel(
    Dims d, const T* __restrict__ value, const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts,
    const T* __restrict__ loc, const T* __restrict__ weight, const T* __restrict__ grad_out,
    float* __restrict__ grad_value, float* __restrict__ grad_loc, float* __restrict__ grad_weight,
    const int* __restrict__ order) {
  using Sh = PairShape<T, kCPL, kLPS>;
  using S16 = Slice<T, 16>;
  constexpr int G = Sh::G;
  constexpr int Cs = G < kStageMax ? G : kStageMax;  // samples staged per chunk
  constexpr int kStage = G / Cs;                     // stager lanes: sub % kStage == 0
  constexpr int kPerPass = G / kLPS;                  // samples whose dots run at once
  // every lane's sample of a pass exists (i < Cs), so the full-warp shuffles of
  // the dots below are reached by all lanes
  static_assert(kPerPass <= Cs && Cs % kPerPass == 0, "a pass's samples must lie inside the staged chunk");
  constexpr int kPasses = Cs / kPerPass > 0 ? Cs / kPerPass : 1;
  constexpr int kGroups = kCtaThreads / G;
  constexpr int kSlots = Cs + 1;
  constexpr int kHashSlots = 8 * Cs;  // >= 2 * (4 Cs entries), a power of two
  extern __shared__ Level levels[];
  __shared__ int4 s_row[kGroups * kSlots];
  __shared__ float4 s_wa[kGroups * kSlots];
  __shared__ float4 s_geo[kGroups * kSlots];
  __shared__ float4 s_dots[kGroups * kSlots];
  __shared__ __align__(16) int s_hash[MSDA_BWD_HASH_FOLD ? kGroups * kHashSlots : 4];
  stage_levels(levels, shapes, starts, d);

  const int sub = threadIdx.x % G;
  const int lq = sub % kLPS, member = sub / kLPS;  // lane of the sample's lanes, sample within the pass
  const int base = (threadIdx.x / G) * kSlots;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int row_stride = d.heads * d.channels;
  const int samples = d.levels * d.points;

  const int64_t stride = static_cast<int64_t>(gridDim.x) * kGroups;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * kGroups + threadIdx.x / G;
       item - (threadIdx.x % 32) / G < items; item += stride) {
    const bool live = item < items;
    const int64_t slot = live ? item : items - 1;
    const int64_t it = order ? order[slot] : slot;
    const ImageHead ih = image_head(it, d, items < (int64_t{1} << 31));
    const int h = ih.h;
    const int64_t b = ih.b;
    const int64_t head0 = (b * d.spatial_size) * row_stride + h * d.channels;
    const T* vrow = value + head0;
    float* gbase = grad_value + head0 + sub * 4;
    const T* lp = loc + it * samples * 2;
    const T* wp = weight + it * samples;
    const T* grow = grad_out + it * d.channels;

    // grad_output in the dot layout (chunks lq, lq + kLPS, ...) and as this
    // lane's 4-channel slice for the REDs
    // bf16 with the mixed-precision FMA keeps grad_output as raw words
    constexpr bool kMixed = sizeof(T) == 2 && MSDA_BWD_MIXED_FMA;
    float2 ga[kCPL][Sh::kPairs16];
    Words<4> graw[kCPL];
    {
      const uint64_t policy = evict_first_policy();
#pragma unroll
      for (int j = 0; j < kCPL; ++j) {
        graw[j] = ld_stream_words<16>(grow + (j * kLPS + lq) * Sh::kPer16, policy);
        if constexpr (!kMixed) {
#pragma unroll
          for (int q = 0; q < Sh::kPairs16; ++q) ga[j][q] = S16::pair(graw[j], q);
        }
      }
    }
    float2 gr[2];
    {
      const Words<4 * static_cast<int>(sizeof(T)) / 4> w =
          ld_stream_words<4 * static_cast<int>(sizeof(T))>(grow + 4 * sub, evict_first_policy());
      gr[0] = Slice<T, 4 * sizeof(T)>::pair(w, 0);
      gr[1] = Slice<T, 4 * sizeof(T)>::pair(w, 1);
    }

    for (int s0 = 0; s0 < samples; s0 += Cs) {
      if (sub % kStage == 0) {
        // geometry for the gradient formula: (lh, lw, W a, H a), lh = -1 for
        // a sample with no corner inside its level
        const int i = sub / kStage;
        float4 geo = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float2 wh = make_float2(0.0f, 0.0f);
        const bool valid =
            stage_sample(levels, level_of(d), samples, live, s0 + i, lp, wp, s_row + base + i, s_wa + base + i, &geo, &wh);
        s_geo[base + i] =
            valid ? make_float4(geo.x, geo.y, wh.x * geo.z, wh.y * geo.z) : make_float4(-1.0f, 0.0f, 0.0f, 0.0f);
      }
      __syncwarp();
      // REDs of pass p's samples by every lane's slice
      auto pass_reds = [&](int p) {
        if constexpr (kScatter) {
#pragma unroll
          for (int m = 0; m < kPerPass; ++m) {
            const int i2 = p * kPerPass + m;
            if (i2 >= Cs) break;
            const int4 r4 = s_row[base + i2];
            const float4 w4 = s_wa[base + i2];
            const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
            const float wa[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
#if MSDA_BWD_PRED_RED
              const float2 w2 = make_float2(wa[k], wa[k]);
              const float2 lo = fmul2(w2, gr[0]), hi = fmul2(w2, gr[1]);
              red_add_v4_if(rows[k] >= 0 && wa[k] != 0.0f,
                            gbase + static_cast<int64_t>(rows[k] >= 0 ? rows[k] : 0) * row_stride, lo.x, lo.y,
                            hi.x, hi.y);
#else
              if (rows[k] >= 0 && wa[k] != 0.0f)
                scatter_slice<2>(gbase + static_cast<int64_t>(rows[k]) * row_stride, wa[k], gr);
#endif
            }
          }
        }
      };
      if constexpr (kCPL == 1 && kStageMax == 4 && MSDA_BWD_PREFETCH) {
        // head-rows of at most 4 samples, all four corners in flight: the first
        // of the chunk's two passes has its gathers issued before the fold, so
        // their latency hides behind its shared-memory work
        auto gather_corners = [&](int i, Words<4> (&raw)[4]) {
          const int4 r4 = s_row[base + i];
          const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
          for (int k = 0; k < 4; ++k)
            raw[k] = rows[k] >= 0 ? ldg_words<16>(vrow + static_cast<int64_t>(rows[k]) * row_stride + lq * Sh::kPer16)
                                  : zero_words<4>();
        };
        auto dots = [&](int i, const Words<4> (&raw)[4]) {
          float t[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float2 acc = make_float2(0.0f, 0.0f);
            if constexpr (kMixed) {
#pragma unroll
              for (int q = 0; q < 4; ++q) acc = fma_bf16x2_f32(graw[0].w[q], raw[k].w[q], acc);
            } else {
#pragma unroll
              for (int q = 0; q < Sh::kPairs16; ++q) acc = ffma2(ga[0][q], S16::pair(raw[k], q), acc);
            }
            t[k] = acc.x + acc.y;
          }
#pragma unroll
          for (int m = 1; m < kLPS; m <<= 1)
#pragma unroll
            for (int k = 0; k < 4; ++k) t[k] += __shfl_xor_sync(0xffffffffu, t[k], m);
          if (lq == 0) s_dots[base + i] = make_float4(t[0], t[1], t[2], t[3]);
        };
        Words<4> first[4];
        if (member < Cs) gather_corners(member, first);
#if MSDA_BWD_DEDUP
        if constexpr (kScatter) {
#if MSDA_BWD_HASH_FOLD
          fold_rows_hashed<G, 4 * Cs, kHashSlots>(reinterpret_cast<const int*>(s_row + base),
                                                  reinterpret_cast<float*>(s_wa + base),
                                                  s_hash + (threadIdx.x / G) * kHashSlots, sub);
#else
          fold_repeated_rows<G, 4 * Cs>(reinterpret_cast<const int*>(s_row + base),
                                        reinterpret_cast<float*>(s_wa + base), sub);
#endif
        }
#endif
        if (member < Cs) dots(member, first);
        pass_reds(0);
#pragma unroll 1
        for (int p = 1; p < kPasses; ++p) {
          const int i = p * kPerPass + member;
          if (i < Cs) {
            Words<4> raw[4];
            gather_corners(i, raw);
            dots(i, raw);
          }
          pass_reds(p);
        }
      } else {
#if MSDA_BWD_DEDUP
        if constexpr (kScatter) {
#if MSDA_BWD_HASH_FOLD
          fold_rows_hashed<G, 4 * Cs, kHashSlots>(reinterpret_cast<const int*>(s_row + base),
                                                  reinterpret_cast<float*>(s_wa + base),
                                                  s_hash + (threadIdx.x / G) * kHashSlots, sub);
#else
          fold_repeated_rows<G, 4 * Cs>(reinterpret_cast<const int*>(s_row + base),
                                        reinterpret_cast<float*>(s_wa + base), sub);
#endif
        }
#endif
#pragma unroll 1
        for (int p = 0; p < kPasses; ++p) {
          // dots of sample i by the pair
          const int i = p * kPerPass + member;
          if (i < Cs) {
            const int4 r4 = s_row[base + i];
            const int rows[4] = {r4.x, r4.y, r4.z, r4.w};
            float t[4];
#pragma unroll
            for (int k0 = 0; k0 < 4; k0 += Sh::kCornersInFlight) {
              Words<4> raw[Sh::kCornersInFlight][kCPL];
#pragma unroll
              for (int kk = 0; kk < Sh::kCornersInFlight; ++kk) {
                const int row = rows[k0 + kk];
#pragma unroll
                for (int j = 0; j < kCPL; ++j)
                  raw[kk][j] = row >= 0 ? ldg_words<16>(vrow + static_cast<int64_t>(row) * row_stride +
                                                        (j * kLPS + lq) * Sh::kPer16)
                                        : zero_words<4>();
              }
#pragma unroll
              for (int kk = 0; kk < Sh::kCornersInFlight; ++kk) {
                float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int j = 0; j < kCPL; ++j) {
                  if constexpr (kMixed) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc = fma_bf16x2_f32(graw[j].w[q], raw[kk][j].w[q], acc);
                  } else {
#pragma unroll
                    for (int q = 0; q < Sh::kPairs16; ++q) acc = ffma2(ga[j][q], S16::pair(raw[kk][j], q), acc);
                  }
                }
                t[k0 + kk] = acc.x + acc.y;
              }
            }
#pragma unroll
            for (int m = 1; m < kLPS; m <<= 1)
#pragma unroll
              for (int k = 0; k < 4; ++k) t[k] += __shfl_xor_sync(0xffffffffu, t[k], m);
            if (lq == 0) s_dots[base + i] = make_float4(t[0], t[1], t[2], t[3]);
          }
          pass_reds(p);
        }
      }
      __syncwarp();
      // grad_w / grad_loc of the chunk: every stager lane takes its own sample
      // (the whole chunk in one pass of the warp; the group's stores cover
      // contiguous runs of grad_w and grad_loc)
      if (sub % kStage == 0) {
        const int i = sub / kStage;
        const int s = s0 + i;
        if (live && s < samples) {
          const float4 geo = s_geo[base + i];
          const float4 t = s_dots[base + i];
          float gw = 0.0f, gx = 0.0f, gy = 0.0f;
          if (geo.x >= 0.0f) {
            const float lh = geo.x, lw = geo.y;
            const float hh = __fsub_rn(1.0f, lh), hw = __fsub_rn(1.0f, lw);
            gw = __fmul_rn(hh, hw) * t.x + __fmul_rn(hh, lw) * t.y + __fmul_rn(lh, hw) * t.z + __fmul_rn(lh, lw) * t.w;
            gx = geo.z * (hh * (t.y - t.x) + lh * (t.w - t.z));
            gy = geo.w * (hw * (t.z - t.x) + lw * (t.w - t.y));
          }
          const int64_t so = it * samples + s;
          grad_weight[so] = gw;
          *reinterpret_cast<float2*>(grad_loc + 2 * so) = make_float2(gx, gy);
        }
      }
      __syncwarp();  // the next chunk's staging overwrites the slots read above
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
            if (grad_value != nullptr) {  // null: grad_loc / grad_w only
#pragma unroll
              for (int k = 0; k < 4; ++k)
                if (c.row[k] >= 0)
                  atomicAdd(grad_value + vrow0 + static_cast<int64_t>(c.row[k]) * row_stride + ch, c.w[k] * a * gc);
            }
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
  // head-rows of at most 4 samples (single-level cases) stage 4 at a time
  const bool short_rows = d.levels * d.points <= 4;
  auto kernel = short_rows ? (a.skip_grad_value ? backward_vec_kernel<T, G, kBytes, 4, false>
                                                : backward_vec_kernel<T, G, kBytes, 4, true>)
                           : (a.skip_grad_value ? backward_vec_kernel<T, G, kBytes, 8, false>
                                                : backward_vec_kernel<T, G, kBytes, 8, true>);
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

template <typename T, int kCPL, int kLPS = 2>
static cudaError_t launch_backward_pair(const Dims& d, const Args& a, cudaStream_t stream) {
  constexpr int G = PairShape<T, kCPL, kLPS>::G;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t groups_per_cta = kCtaThreads / G;
  const int64_t blocks = (items + groups_per_cta - 1) / groups_per_cta;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  const bool short_rows = d.levels * d.points <= 4;
  auto kernel = short_rows ? (a.skip_grad_value ? backward_pair_kernel<T, kCPL, 4, false, kLPS>
                                                : backward_pair_kernel<T, kCPL, 4, true, kLPS>)
                           : (a.skip_grad_value ? backward_pair_kernel<T, kCPL, 8, false, kLPS>
                                                : backward_pair_kernel<T, kCPL, 8, true, kLPS>);
  kernel<<<grid, kCtaThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<const T*>(a.grad_out), a.grad_value, a.grad_loc, a.grad_weight,
      a.order);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_backward_t(const Dims& d, const Args& a, cudaStream_t stream) {
#if MSDA_BWD_PAIR
  // The lane-pair kernel where it measured faster on B200: bf16 rows of 2 or 4
  // chunks of 16 bytes (D = 16, 32) (c2 / c4: backward 1.18 -> 1.11 ms /
  // 9.38 -> 8.81 ms; at 4 CTAs/SM also single-level rows of 4 samples: c3
  // 0.287 -> 0.277 ms, bevformer-1l bf16 0.331 -> 0.325 ms). fp32 rows (4
  // chunks per lane, one corner in flight) ran slower than backward_vec_kernel.
  if constexpr (sizeof(T) == 2) {
    if ((MSDA_PAIR_SHORT || d.levels * d.points > 4) && vec_lanes(d.channels, sizeof(T), 16, a) != 0 &&
        vec_lanes(d.channels, 4, 16, a) != 0) {
      switch (d.channels * static_cast<int>(sizeof(T)) / 32) {
        case 1: return launch_backward_pair<T, 1>(d, a, stream);
        case 2:
          // D = 32: four lanes of one 16-byte chunk each per sample (a gather instruction
          // reads 64 bytes of each row it touches), or two lanes of two chunks
          return MSDA_BWD_QUAD ? launch_backward_pair<T, 1, 4>(d, a, stream) : launch_backward_pair<T, 2>(d, a, stream);
        default: break;
      }
    }
  }
#endif
  // bf16: 8-byte lanes (4 channels, whole-line REDs) up to D = 128, 16-byte
  // lanes for D = 256; fp32: 16-byte lanes (4 channels).
  if constexpr (sizeof(T) == 2) {
    if (const int g = vec_lanes(d.channels, sizeof(T), 8, a)) return launch_backward_lanes<T, 8>(g, d, a, stream);
    if (vec_lanes(d.channels, sizeof(T), 16, a) == 32) return launch_backward_vec<T, 32, 16>(d, a, stream);
  } else {
    if (const int g = vec_lanes(d.channels, sizeof(T), 16, a)) return launch_backward_lanes<T, 16>(g, d, a, stream);
  }
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t blocks = (items + kCtaThreads - 1) / kCtaThreads;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  backward_scalar_kernel<T><<<grid, kCtaThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<const T*>(a.grad_out), a.skip_grad_value ? nullptr : a.grad_value,
      a.grad_loc, a.grad_weight);
  return cudaGetLastError();
}

cudaError_t launch_backward_rowwise(DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0) return cudaSuccess;
  return dtype == DType::kBF16 ? launch_backward_t<__nv_bfloat16>(d, a, stream)
                               : launch_backward_t<float>(d, a, stream);
}

}  // namespace msda
