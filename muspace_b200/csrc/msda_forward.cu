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
// one 16-byte load per lane, 64 / 128 contiguous bytes per group. Locations
// and weights are read by the group's lanes together (one broadcast
// transaction) and the point loop is unrolled so several samples' corner
// loads are in flight per thread. Items are ordered batch-major, so at any
// moment the CTAs in flight gather from one or two cameras' value maps, which
// stay resident in L2. Any other D takes the scalar kernel below.
#include "msda_device.cuh"

namespace msda {

template <typename T, int G>
__global__ void __launch_bounds__(256) forward_vec_kernel(Dims d, const T* __restrict__ value,
                                                          const int64_t* __restrict__ shapes,
                                                          const int64_t* __restrict__ starts,
                                                          const T* __restrict__ loc, const T* __restrict__ weight,
                                                          T* __restrict__ out, const int* __restrict__ order) {
  using V = Vec16<T>;
  constexpr int kVec = V::kLanes;
  extern __shared__ Level levels[];
  stage_levels(levels, shapes, starts, d);

  const int sub = threadIdx.x % G;
  const int groups_per_cta = blockDim.x / G;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int row_stride = d.heads * d.channels;  // elements between neighbouring pixels
  const int samples = d.levels * d.points;

  for (int64_t slot = static_cast<int64_t>(blockIdx.x) * groups_per_cta + threadIdx.x / G; slot < items;
       slot += static_cast<int64_t>(gridDim.x) * groups_per_cta) {
    const int64_t item = order ? order[slot] : slot;
    const int h = static_cast<int>(item % d.heads);
    const int64_t b = item / (static_cast<int64_t>(d.queries) * d.heads);
    const T* vbase = value + (b * d.spatial_size) * row_stride + h * d.channels + sub * kVec;
    const T* lp = loc + item * samples * 2;
    const T* wp = weight + item * samples;

    float acc[kVec];
#pragma unroll
    for (int i = 0; i < kVec; ++i) acc[i] = 0.0f;

    for (int l = 0; l < d.levels; ++l) {
      const Level lv = levels[l];
#pragma unroll 4
      for (int p = 0; p < d.points; ++p) {
        const int s = l * d.points + p;
        const float2 xy = load_loc(lp + 2 * s);
        const float a = to_f32(wp[s]);
        Corners c;
        if (!corners(lv, xy.x, xy.y, c)) continue;
        uint4 raw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          raw[k] = c.row[k] >= 0 ? ldg16(vbase + static_cast<int64_t>(c.row[k]) * row_stride) : make_uint4(0, 0, 0, 0);
        float v[4][kVec];
#pragma unroll
        for (int k = 0; k < 4; ++k) V::unpack(raw[k], v[k]);
#pragma unroll
        for (int i = 0; i < kVec; ++i) {
          const float bil = c.w[0] * v[0][i] + c.w[1] * v[1][i] + c.w[2] * v[2][i] + c.w[3] * v[3][i];
          acc[i] = fmaf(bil, a, acc[i]);
        }
      }
    }
    st16(out + item * d.channels + sub * kVec, V::pack(acc));
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

template <typename T, int G>
static cudaError_t launch_forward_vec(const Dims& d, const Args& a, cudaStream_t stream) {
  constexpr int kThreads = 256;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t groups_per_cta = kThreads / G;
  const int64_t blocks = (items + groups_per_cta - 1) / groups_per_cta;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  forward_vec_kernel<T, G><<<grid, kThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<T*>(a.out), a.order);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_forward_t(const Dims& d, const Args& a, cudaStream_t stream) {
  const int g = vec_group(d.channels, sizeof(T), a);
  switch (g) {
    case 1: return launch_forward_vec<T, 1>(d, a, stream);
    case 2: return launch_forward_vec<T, 2>(d, a, stream);
    case 4: return launch_forward_vec<T, 4>(d, a, stream);
    case 8: return launch_forward_vec<T, 8>(d, a, stream);
    case 16: return launch_forward_vec<T, 16>(d, a, stream);
    case 32: return launch_forward_vec<T, 32>(d, a, stream);
    default: break;
  }
  constexpr int kThreads = 256;
  const int64_t total = static_cast<int64_t>(d.batch) * d.queries * d.heads * d.channels;
  const int64_t blocks = (total + kThreads - 1) / kThreads;
  const int grid = static_cast<int>(blocks < grid_cap() ? blocks : grid_cap());
  forward_scalar_kernel<T><<<grid, kThreads, level_smem(d), stream>>>(
      d, static_cast<const T*>(a.value), a.shapes, a.starts, static_cast<const T*>(a.loc),
      static_cast<const T*>(a.weight), static_cast<T*>(a.out));
  return cudaGetLastError();
}

cudaError_t launch_forward_rowwise(DType dtype, const Dims& d, const Args& a, cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0 || d.channels == 0) return cudaSuccess;
  return dtype == DType::kBF16 ? launch_forward_t<__nv_bfloat16>(d, a, stream) : launch_forward_t<float>(d, a, stream);
}

}  // namespace msda
