// Device-side building blocks of the B200 MSDA kernels.
//
// Layouts (row-major, contiguous), as muSPACE's MSDA operator defines them
// (mu_space/ops/multi_scale_deformable_attn.py:26-58):
//   value               (B, Lin, Hh, D)      storage dtype T (float or bf16)
//   sampling_locations  (B, Lq, Hh, L, P, 2) T, last dim (x = width, y = height)
//   attention_weights   (B, Lq, Hh, L, P)    T
//   output / grad_out   (B, Lq, Hh*D)        T
//   grad_value          (B, Lin, Hh, D)      fp32, accumulated
//   grad_loc / grad_w   like loc / weights   fp32, written
// All arithmetic (geometry, bilinear weights, sums) is fp32 whatever T is.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "msda_kernels.h"

namespace msda {

// ---------------------------------------------------------------------------
// storage-dtype helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// A (x, y) location pair widened to fp32.
__device__ __forceinline__ float2 load_loc(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }
__device__ __forceinline__ float2 load_loc(const __nv_bfloat16* p) {
  const uint32_t u = __ldg(reinterpret_cast<const unsigned int*>(p));
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

// 16 bytes of channels <-> fp32 registers.
template <typename T>
struct Vec16;

template <>
struct Vec16<float> {
  static constexpr int kLanes = 4;
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    f[0] = __uint_as_float(r.x);
    f[1] = __uint_as_float(r.y);
    f[2] = __uint_as_float(r.z);
    f[3] = __uint_as_float(r.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};

template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int kLanes = 8;
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// ---------------------------------------------------------------------------
// lane slices: kBytes of one head-row's channels per lane
// ---------------------------------------------------------------------------
// A head-row of D channels is split over G = D * sizeof(T) / kBytes lanes.
// Slice<T, kBytes> loads a lane's bytes and widens them to fp32 channel pairs
// (kPairs float2; channel 2i in .x, 2i+1 in .y).
template <int kWords>
struct Words {
  uint32_t w[kWords];
};

template <int kBytes>
__device__ __forceinline__ Words<kBytes / 4> ldg_words(const void* p) {
  Words<kBytes / 4> r;
  if constexpr (kBytes == 32) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    r.w[0] = a.x, r.w[1] = a.y, r.w[2] = a.z, r.w[3] = a.w;
    r.w[4] = b.x, r.w[5] = b.y, r.w[6] = b.z, r.w[7] = b.w;
  } else if constexpr (kBytes == 16) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    r.w[0] = v.x, r.w[1] = v.y, r.w[2] = v.z, r.w[3] = v.w;
  } else {
    static_assert(kBytes == 8, "lane slices are 8, 16 or 32 bytes");
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    r.w[0] = v.x, r.w[1] = v.y;
  }
  return r;
}

template <typename T, int kBytes>
struct Slice {
  static constexpr int kChannels = kBytes / static_cast<int>(sizeof(T));
  static constexpr int kPairs = kChannels / 2;
  __device__ __forceinline__ static float2 pair(const Words<kBytes / 4>& r, int i) {
    if constexpr (sizeof(T) == 2) {
      return make_float2(__uint_as_float(r.w[i] << 16), __uint_as_float(r.w[i] & 0xffff0000u));
    } else {
      return make_float2(__uint_as_float(r.w[2 * i]), __uint_as_float(r.w[2 * i + 1]));
    }
  }
};

// Zero-filled words for a corner outside the level.
template <int kWords>
__device__ __forceinline__ Words<kWords> zero_words() {
  Words<kWords> r;
#pragma unroll
  for (int i = 0; i < kWords; ++i) r.w[i] = 0u;
  return r;
}

// Streaming read of data used exactly once (locations, weights, grad_out):
// do not keep it in L1, and let L2 evict it first so the value maps stay.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t policy;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

__device__ __forceinline__ uint4 ld_stream16(const void* p, uint64_t policy) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(policy));
  return r;
}

__device__ __forceinline__ uint2 ld_stream8(const void* p, uint64_t policy) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p), "l"(policy));
  return r;
}

template <int kBytes>
__device__ __forceinline__ Words<kBytes / 4> ld_stream_words(const void* p, uint64_t policy) {
  Words<kBytes / 4> r;
  if constexpr (kBytes == 16) {
    const uint4 v = ld_stream16(p, policy);
    r.w[0] = v.x, r.w[1] = v.y, r.w[2] = v.z, r.w[3] = v.w;
  } else {
    const uint2 v = ld_stream8(p, policy);
    r.w[0] = v.x, r.w[1] = v.y;
  }
  return r;
}

__device__ __forceinline__ void st16(void* p, const uint4& v) { *reinterpret_cast<uint4*>(p) = v; }

// Two independent fp32 FMAs in one instruction (sm_100 fma.rn.f32x2); each
// lane rounds exactly like fmaf. 1: through the compiler's own sm_100
// intrinsic (__ffma2_rn / __fmul2_rn), which it schedules and allocates
// registers for; 0: inline PTX.
#ifndef MSDA_NATIVE_F2
#define MSDA_NATIVE_F2 1
#endif
union F2 {
  float2 f;
  unsigned long long u;
};
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
#if MSDA_NATIVE_F2
  return __ffma2_rn(a, b, c);
#else
  F2 x, y, z, r;
  x.f = a;
  y.f = b;
  z.f = c;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.u) : "l"(x.u), "l"(y.u), "l"(z.u));
  return r.f;
#endif
}
// acc.x += lo(g) * lo(v), acc.y += hi(g) * hi(v) for two words of two bf16
// channels each, in fp32 (sm_100 mixed-precision FMA: the bf16 x bf16 product
// is exact in fp32, so this equals unpacking both words and using fmaf).
__device__ __forceinline__ float2 fma_bf16x2_f32(uint32_t g, uint32_t v, float2 acc) {
  asm("{\n .reg .b16 gl, gh, vl, vh;\n mov.b32 {gl, gh}, %2;\n mov.b32 {vl, vh}, %3;\n"
      " fma.rn.f32.bf16 %0, gl, vl, %0;\n fma.rn.f32.bf16 %1, gh, vh, %1;\n}"
      : "+f"(acc.x), "+f"(acc.y)
      : "r"(g), "r"(v));
  return acc;
}

// A 32-bit word of two bf16 channels as (low channel, high channel) in fp32.
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Vector reduction into fp32 global memory (no return value -> RED, not ATOM).
// No "memory" clobber: the kernels never read the gradient buffers they
// reduce into, so loads of other tensors may move across a RED (the compiler
// can then keep several samples' corner gathers in flight).
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d));
}
// The same RED under a predicate (no branch: lanes of a warp that disagree on
// `on` do not split the warp).
__device__ __forceinline__ void red_add_v4_if(bool on, float* p, float a, float b, float c, float d) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.u32 q, %5, 0;\n @q red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n}" ::"l"(p),
      "f"(a), "f"(b), "f"(c), "f"(d), "r"(static_cast<unsigned>(on)));
}

// Whether every channel pair of acc is finite.
template <int kPairs>
__device__ __forceinline__ bool finite_pairs(const float2 (&acc)[kPairs]) {
  bool ok = true;
#pragma unroll
  for (int q = 0; q < kPairs; ++q) ok = ok && fabsf(acc[q].x) <= 3.402823466e+38f && fabsf(acc[q].y) <= 3.402823466e+38f;
  return ok;
}

// Stores a lane's kBytes slice of channels (fp32 pairs) in the storage dtype.
template <typename T, int kBytes>
__device__ __forceinline__ void store_slice(T* dst, const float2 (&acc)[Slice<T, kBytes>::kPairs]) {
  constexpr int kPer16 = 16 / static_cast<int>(sizeof(T));  // channels per 16 bytes
#pragma unroll
  for (int h = 0; h < kBytes / 16; ++h) {
    float f[kPer16];
#pragma unroll
    for (int q = 0; q < kPer16 / 2; ++q) f[2 * q] = acc[h * kPer16 / 2 + q].x, f[2 * q + 1] = acc[h * kPer16 / 2 + q].y;
    st16(dst + h * kPer16, Vec16<T>::pack(f));
  }
}

// ---------------------------------------------------------------------------
// level table
// ---------------------------------------------------------------------------
// Stage the (H, W, start) table in shared memory. A level whose rows would fall
// outside [0, Lin) is emptied (H = W = 0), so a malformed table can never make
// a kernel read or write outside the value / grad_value buffers.
__device__ __forceinline__ void stage_levels(Level* table, const int64_t* shapes, const int64_t* starts,
                                             const Dims& d) {
  for (int l = threadIdx.x; l < d.levels; l += blockDim.x) {
    const int64_t h = shapes[2 * l], w = shapes[2 * l + 1], s = starts[l];
    const bool ok = h > 0 && w > 0 && s >= 0 && h <= (1 << 24) && w <= (1 << 24) && s + h * w <= d.spatial_size;
    table[l].height = ok ? static_cast<int>(h) : 0;
    table[l].width = ok ? static_cast<int>(w) : 0;
    table[l].start = ok ? static_cast<int>(s) : 0;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// sampling geometry
// ---------------------------------------------------------------------------
// grid_sample(align_corners=False) maps a location in [0, 1] to a pixel
// coordinate as ((2 * loc - 1) + 1) * (size / 2) - 0.5, every step rounded to
// fp32 on its own; the _rn intrinsics keep the compiler from fusing steps, so
// the four corners and their weights equal the reference's bit for bit.
__device__ __forceinline__ float unnormalize(float loc, float half_size) {
  const float g = __fsub_rn(__fmul_rn(2.0f, loc), 1.0f);
  return __fsub_rn(__fmul_rn(__fadd_rn(g, 1.0f), half_size), 0.5f);
}

// One bilinear sample: the four corner rows (pixel index inside the batch's
// value map, or -1 when the corner is outside the level) and their weights.
struct Corners {
  int row[4];  // pixel index, -1 = zero padding
  float w[4];  // bilinear weights hh*hw, hh*lw, lh*hw, lh*lw
  float lh, lw, hh, hw;
};

// Returns false when no corner can be inside the level (or the coordinate is
// not finite); the sample then contributes nothing and has zero gradients.
__device__ __forceinline__ bool corners(const Level& lv, float loc_x, float loc_y, Corners& c) {
  const float fh = static_cast<float>(lv.height), fw = static_cast<float>(lv.width);
  const float y = unnormalize(loc_y, 0.5f * fh);
  const float x = unnormalize(loc_x, 0.5f * fw);
  if (!(y > -2.0f && x > -2.0f && y < fh + 1.0f && x < fw + 1.0f)) return false;
  const float yf = floorf(y), xf = floorf(x);
  const int y0 = static_cast<int>(yf), x0 = static_cast<int>(xf);
  c.lh = __fsub_rn(y, yf);
  c.lw = __fsub_rn(x, xf);
  c.hh = __fsub_rn(1.0f, c.lh);
  c.hw = __fsub_rn(1.0f, c.lw);
  const bool y0ok = y0 >= 0 && y0 < lv.height, y1ok = y0 + 1 >= 0 && y0 + 1 < lv.height;
  const bool x0ok = x0 >= 0 && x0 < lv.width, x1ok = x0 + 1 >= 0 && x0 + 1 < lv.width;
  const int base = lv.start + y0 * lv.width + x0;
  c.row[0] = (y0ok && x0ok) ? base : -1;
  c.row[1] = (y0ok && x1ok) ? base + 1 : -1;
  c.row[2] = (y1ok && x0ok) ? base + lv.width : -1;
  c.row[3] = (y1ok && x1ok) ? base + lv.width + 1 : -1;
  c.w[0] = __fmul_rn(c.hh, c.hw);
  c.w[1] = __fmul_rn(c.hh, c.lw);
  c.w[2] = __fmul_rn(c.lh, c.hw);
  c.w[3] = __fmul_rn(c.lh, c.lw);
  return true;
}

// ---------------------------------------------------------------------------
// staged sample geometry (row-wise vector kernels)
// ---------------------------------------------------------------------------
// Threads per CTA of the row-wise vector kernels (their shared staging arrays
// have one slot per thread).
constexpr int kCtaThreads = 256;

// The G lanes of a group take the samples of a head-row in chunks of
// kSamples = min(G, kMax); the lane at sub = i * kStagerStride computes the
// geometry of sample i of the chunk for the whole group.
template <int G, int kMax>
struct Chunk {
  static constexpr int kSamples = G < kMax ? G : kMax;
  static constexpr int kStagerStride = G / kSamples;
};

// The level of sample s of a head-row (samples are level-major, `points` per
// level): a multiply-high by Dims::points_magic when the host set one, else a
// division.
struct LevelOf {
  int points;
  uint32_t magic;
  __device__ __forceinline__ int operator()(int s) const {
    return magic ? static_cast<int>(__umulhi(static_cast<uint32_t>(s), magic)) : s / points;
  }
};
__device__ __forceinline__ LevelOf level_of(const Dims& d) { return LevelOf{d.points, d.points_magic}; }

// Image and head of head-row `item` ((b, q, h) order, heads fastest): 32-bit
// divisions when every head-row index of the call fits 31 bits (idx32; every
// realistic call), else the 64-bit ones.
struct ImageHead {
  int64_t b;
  int h;
};
__device__ __forceinline__ ImageHead image_head(int64_t item, const Dims& d, bool idx32) {
  if (idx32) {
    const uint32_t i = static_cast<uint32_t>(item);
    return ImageHead{static_cast<int64_t>(i / static_cast<uint32_t>(d.queries * d.heads)),
                     static_cast<int>(i % static_cast<uint32_t>(d.heads))};
  }
  return ImageHead{item / (static_cast<int64_t>(d.queries) * d.heads), static_cast<int>(item % d.heads)};
}

// Computes sample s of a head-row (locations lp, weights wp) and stores its
// four corner rows (-1 = outside the level, or no sample) and w_k * a in the
// caller's shared slots. Returns whether the sample has a corner inside its
// level, and, when geo is given, stores (lh, lw, a, 1) there for a valid
// sample (the caller zeroes it), for the gradient formulas; when wh is given
// too, the level's (W, H) as floats.
template <typename T>
__device__ __forceinline__ bool stage_sample(const Level* levels, LevelOf level, int samples, bool live, int s,
                                             const T* lp, const T* wp, int4* row_slot, float4* wa_slot,
                                             float4* geo = nullptr, float2* wh = nullptr) {
  int4 r = make_int4(-1, -1, -1, -1);
  float4 wa = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  bool valid = false;
  if (live && s < samples) {
    const Level lv = levels[level(s)];
    const float2 xy = load_loc(lp + 2 * s);
    const float a = to_f32(wp[s]);
    Corners c;
    valid = corners(lv, xy.x, xy.y, c);
    if (valid) {
      r = make_int4(c.row[0], c.row[1], c.row[2], c.row[3]);
      wa = make_float4(c.w[0] * a, c.w[1] * a, c.w[2] * a, c.w[3] * a);
      if (geo) *geo = make_float4(c.lh, c.lw, a, 1.0f);
      if (wh) *wh = make_float2(static_cast<float>(lv.width), static_cast<float>(lv.height));
    }
  }
  *row_slot = r;
  *wa_slot = wa;
  return valid;
}

// Folds repeated corner rows of a chunk's kEnt staged (row, wa) entries into
// their first occurrence: an entry whose row already appears at a lower
// index adds its wa to that entry (shared-memory atomic) and its own wa
// becomes 0, so a RED is due exactly for the entries with row >= 0 and
// wa != 0. Rows are left as they are (the gathers still need them). Lane sub
// of the group owns entries sub, sub + G, ...
template <int G, int kEnt>
__device__ __forceinline__ void fold_repeated_rows(const int* row, float* wa, int sub) {
  static_assert(kEnt % 4 == 0, "entries come in whole samples");
  constexpr int kPer = (kEnt + G - 1) / G;
  int mine[kPer], target[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = sub + j * G;
    mine[j] = e < kEnt ? row[e] : -1;
    target[j] = -1;
  }
  // earliest lower-index entry with the same row; only entries below
  // (j + 1) * G can precede entry j, so the scan stops there
#pragma unroll
  for (int e4 = 0; e4 < ((kPer - 1) * G + G < kEnt ? (kPer - 1) * G + G : kEnt); e4 += 4) {
    const int4 r4 = *reinterpret_cast<const int4*>(row + e4);
    const int rs[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e2 = e4 + u;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (e2 >= (j + 1) * G) continue;  // never below entry j
        const bool before = e2 < j * G || e2 < sub + j * G;
        if (before && target[j] < 0 && rs[u] == mine[j] && mine[j] >= 0) target[j] = e2;
      }
    }
  }
  float moved[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = sub + j * G;
    moved[j] = (target[j] >= 0) ? wa[e] : 0.0f;
  }
  __syncwarp();  // every lane has read the wa it moves before any entry changes
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (target[j] >= 0) {
      atomicAdd(wa + target[j], moved[j]);
      wa[sub + j * G] = 0.0f;
    }
  }
  __syncwarp();
}

// The same fold through a per-group hash table in shared memory (kSlots ints,
// a power of two >= 2 kEnt): every entry with a RED due claims its row's slot
// with a compare-and-swap; an entry that finds the slot held by an entry of
// the same row moves its wa there, one that finds another row (a hash
// collision) keeps its own RED. The owner of a row is whichever entry claimed
// it first, so the fold costs a few instructions per entry instead of a scan
// over all lower entries. Movers are never owners, so no entry is read while
// another lane adds into it.
template <int G, int kEnt, int kSlots>
__device__ __forceinline__ void fold_rows_hashed(const int* row, float* wa, int* table, int sub) {
  static_assert((kSlots & (kSlots - 1)) == 0 && kSlots >= 2 * kEnt, "table: a power of two, at least twice the entries");
  constexpr int kPer = (kEnt + G - 1) / G;
  constexpr int kShift = 32 - __builtin_ctz(kSlots);
#pragma unroll
  for (int t = sub * 4; t < kSlots; t += G * 4) *reinterpret_cast<int4*>(table + t) = make_int4(-1, -1, -1, -1);
  __syncwarp();
  int owner[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = sub + j * G;
    owner[j] = e;
    if (e < kEnt) {
      const int r = row[e];
      if (r >= 0 && wa[e] != 0.0f) {
        const int slot = static_cast<int>((static_cast<uint32_t>(r) * 2654435761u) >> kShift);
        const int held = atomicCAS(table + slot, -1, e);
        if (held >= 0 && row[held] == r) owner[j] = held;
      }
    }
  }
  __syncwarp();  // every claim is settled before any wa moves
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = sub + j * G;
    if (owner[j] != e) {
      atomicAdd(wa + owner[j], wa[e]);
      wa[e] = 0.0f;
    }
  }
  __syncwarp();
}

// Lane layout of the lane-pair / lane-quad backward kernels (msda_backward.cu):
// a head-row of D channels is kLPS x kCPL 16-byte chunks; a sample's dots are
// formed by kLPS lanes, lane q holding chunks q, q + kLPS, ... of the corner
// rows, and G = D / 4 lanes per head-row each own a 4-channel fp32 slice of
// the gradients.
template <typename T, int kCPL, int kLPS = 2>
struct PairShape {
  static constexpr int kPer16 = 16 / static_cast<int>(sizeof(T));  // channels per 16-byte chunk
  static constexpr int kChannels = kLPS * kCPL * kPer16;           // D
  static constexpr int G = kChannels / 4;                          // lanes per head-row
  static constexpr int kPairs16 = kPer16 / 2;                      // fp32 pairs per chunk
#ifndef MSDA_PAIR_CORNERS
#define MSDA_PAIR_CORNERS 1
#endif
  // corner gathers issued together (register budget: kCPL * 4 words each; at
  // 64 registers one corner at a time measured fastest for D = 32)
  static constexpr int kCornersInFlight = kCPL == 1 ? 4 : (kCPL == 2 ? MSDA_PAIR_CORNERS : 1);
};

// ---------------------------------------------------------------------------
// lane-group reductions and gradient scatter
// ---------------------------------------------------------------------------
// Sum over the G lanes of a group (G a power of two <= 32, groups aligned).
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int m = G / 2; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m, G);
  return v;
}

// Which fp32 channels a lane scatters into grad_value. A vector RED moves 16
// bytes per lane, and the L2 processes reductions per 32-byte sector, so one
// RED instruction of the group should cover whole sectors. With fp32 storage
// the lane's load slice (4 channels, lanes side by side) already does. With
// bf16 storage a lane loads 8 channels (16 bytes), which are 32 bytes of fp32:
// scattering them itself would touch every sector with two half-filled REDs.
// Instead lane j scatters channels [4j, 4j+4) and [4G+4j, 4G+4j+4), so each
// RED instruction of the group fills 16G contiguous bytes.
template <typename T, int G>
struct RedSlice {
  __device__ __forceinline__ static void load(const T*, int, const float* g, float* gr) {
#pragma unroll
    for (int i = 0; i < Vec16<T>::kLanes; ++i) gr[i] = g[i];
  }
  __device__ __forceinline__ static void scatter(float* head_row, int sub, float wa, const float* gr) {
    float* dst = head_row + sub * 4;
    red_add_v4(dst, wa * gr[0], wa * gr[1], wa * gr[2], wa * gr[3]);
  }
};

template <int G>
struct RedSlice<__nv_bfloat16, G> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* grow, int sub, const float*, float* gr) {
    const uint2 lo = __ldg(reinterpret_cast<const uint2*>(grow + 4 * sub));
    const uint2 hi = __ldg(reinterpret_cast<const uint2*>(grow + 4 * G + 4 * sub));
    const uint32_t w[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      gr[2 * i] = __uint_as_float(w[i] << 16);
      gr[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static void scatter(float* head_row, int sub, float wa, const float* gr) {
    red_add_v4(head_row + 4 * sub, wa * gr[0], wa * gr[1], wa * gr[2], wa * gr[3]);
    red_add_v4(head_row + 4 * G + 4 * sub, wa * gr[4], wa * gr[5], wa * gr[6], wa * gr[7]);
  }
};

// t[C][4] holds a lane's partial corner dots for the C samples of a chunk.
// Sums them over the G lanes of the group so that every lane with
// sub / (G / C) == i ends with sample i's totals in t[0]: first log2(C)
// halving exchanges over the high lane bits (a lane keeps half of the samples
// it holds and sends the other half to its xor partner, 4 values each), then
// plain butterflies over the remaining low bits.
template <int G, int C, int M = G / 2, int N = C>
__device__ __forceinline__ void reduce_to_stagers(float (&t)[C][4], int sub) {
  if constexpr (M >= 1) {
    if constexpr (N > 1) {
      const bool upper = (sub & M) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float send = upper ? t[i][k] : t[i + N / 2][k];
          const float keep = upper ? t[i + N / 2][k] : t[i][k];
          t[i][k] = keep + __shfl_xor_sync(0xffffffffu, send, M);
        }
      }
      reduce_to_stagers<G, C, M / 2, N / 2>(t, sub);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) t[0][k] += __shfl_xor_sync(0xffffffffu, t[0][k], M);
      reduce_to_stagers<G, C, M / 2, 1>(t, sub);
    }
  }
}

// Two fp32 products in one instruction (sm_100 mul.rn.f32x2).
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
#if MSDA_NATIVE_F2
  return __fmul2_rn(a, b);
#else
  F2 x, y, r;
  x.f = a;
  y.f = b;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.u) : "l"(x.u), "l"(y.u));
  return r.f;
#endif
}

// grad_value[corner row] += wa * g over a lane's own channel slice
// (kPairs * 2 fp32 channels, 16-byte aligned): one vector RED per 4 channels.
template <int kPairs>
__device__ __forceinline__ void scatter_slice(float* dst, float wa, const float2 (&g2)[kPairs]) {
  const float2 w2 = make_float2(wa, wa);
#pragma unroll
  for (int q = 0; q < kPairs / 2; ++q) {
    const float2 lo = fmul2(w2, g2[2 * q]), hi = fmul2(w2, g2[2 * q + 1]);
    red_add_v4(dst + 4 * q, lo.x, lo.y, hi.x, hi.y);
  }
}

}  // namespace msda
