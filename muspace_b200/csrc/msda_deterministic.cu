// Deterministic MSDA backward: grad_value summed in 64-bit fixed point.
//
// The default backward adds every sample's corner contributions w_k * a * g
// into the fp32 grad_value with vector REDs, so the order of the additions,
// and with it the last bits of grad_value, changes from run to run (the
// reference's atomicAdd kernels behave the same). This path makes grad_value
// bit-reproducible with integer arithmetic instead of a destination sort:
//   0. one pass takes max |grad_output| and max |attention_weights|, which
//      bound every contribution (w_k <= 1);
//   1. the row-wise backward writes grad_loc / grad_w (each by one lane, in a
//      fixed order, as in the default path) without touching grad_value;
//   2. every contribution, converted to a 64-bit integer at a power-of-two
//      scale derived from that bound, is added into a 64-bit accumulator per
//      grad_value element; integer addition is associative, so the sums do not
//      depend on the order in which the additions land;
//   3. each accumulator is converted back once and added into grad_value.
// The scale leaves headroom for every sample of a (batch, head) landing on one
// element, so no sum can overflow. A contribution is kept to 2^-(61 - headroom)
// of the bound, finer than fp32 resolution for all but contributions far below
// the largest one; the result is the exactly rounded sum of the fp32
// contributions to that resolution. When grad_output or the weights hold a
// non-finite value, step 2 adds the fp32 contributions into grad_value
// directly (the non-finite elements are the same in any order).
#include "msda_device.cuh"

namespace msda {
namespace {

constexpr size_t kHeaderBytes = 256;  // two words of maxima, padded to keep the accumulators aligned

// Largest |x| of two tensors as float bits (for x >= 0 the unsigned order of
// the bits is the float order, with NaN above inf).
template <typename T>
__global__ void __launch_bounds__(256) max_abs_kernel(const T* __restrict__ g, int64_t ng, const T* __restrict__ w,
                                                     int64_t nw, unsigned* __restrict__ header) {
  unsigned mg = 0u, mw = 0u;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < ng; i += stride)
    mg = max(mg, __float_as_uint(fabsf(to_f32(g[i]))));
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nw; i += stride)
    mw = max(mw, __float_as_uint(fabsf(to_f32(w[i]))));
  mg = __reduce_max_sync(0xffffffffu, mg);
  mw = __reduce_max_sync(0xffffffffu, mw);
  if (threadIdx.x % 32 == 0) {
    atomicMax(header, mg);
    atomicMax(header + 1, mw);
  }
}

struct FixedPoint {
  bool finite;
  double scale;
};

// The scale of step 2: contributions are bounded by s = max|g| * max|a|, and
// s * scale < 2^(62 - headroom_bits) (frexp: s < 2^e).
__device__ __forceinline__ FixedPoint fixed_point(const unsigned* header, int headroom_bits) {
  const float mg = __uint_as_float(header[0]), mw = __uint_as_float(header[1]);
  FixedPoint f;
  f.finite = isfinite(mg) && isfinite(mw);
  const double s = static_cast<double>(mg) * static_cast<double>(mw);
  int e = 0;
  frexp(s, &e);
  f.scale = s > 0.0 ? ldexp(1.0, 62 - headroom_bits - e) : 1.0;
  return f;
}

// Step 2: one warp per head-row (b, q, h). Lane i computes the geometry of
// sample s0 + i once; the pass's corner entries (4 per sample) go to shared
// memory, repeated corner rows are chained to their first claimer through a
// per-warp hash table, and the warp then walks the claimers with lanes over
// the channels: each lane converts every contribution of a claimer's chain
// to fixed point exactly as it would alone, sums them in a register (integer
// sums are exact, so the result is the same bits as one atomic per entry)
// and issues one atomic per distinct row.
constexpr int kDetWarps = 8;             // 256 threads
constexpr int kDetEntries = 4 * 32;      // corner entries of one 32-sample pass
constexpr int kDetTable = 2 * kDetEntries;

template <typename T>
__global__ void __launch_bounds__(256) fixed_point_scatter_kernel(
    Dims d, const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts, const T* __restrict__ loc,
    const T* __restrict__ weight, const T* __restrict__ grad_out, const unsigned* __restrict__ header,
    int headroom_bits, unsigned long long* __restrict__ acc, float* __restrict__ grad_value) {
  extern __shared__ Level levels[];
  __shared__ int s_table[kDetWarps][kDetTable];
  __shared__ int s_row[kDetWarps][kDetEntries];
  __shared__ float s_wa[kDetWarps][kDetEntries];
  __shared__ int s_next[kDetWarps][kDetEntries];  // claimer: chain head; repeat: next repeat (-1 ends)
  stage_levels(levels, shapes, starts, d);
  const FixedPoint fp = fixed_point(header, headroom_bits);
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int* table = s_table[warp];
  int* erow = s_row[warp];
  float* ewa = s_wa[warp];
  int* enext = s_next[warp];
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t row_stride = static_cast<int64_t>(d.heads) * d.channels;
  const int samples = d.levels * d.points;
  const LevelOf level = level_of(d);
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + warp; item < items; item += warps) {
    const int h = static_cast<int>(item % d.heads);
    const int64_t b = item / (static_cast<int64_t>(d.queries) * d.heads);
    const int64_t head0 = b * d.spatial_size * row_stride + static_cast<int64_t>(h) * d.channels;
    for (int s0 = 0; s0 < samples; s0 += 32) {
      int row[4] = {-1, -1, -1, -1};
      float wa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (s0 + lane < samples) {
        const int64_t so = item * samples + s0 + lane;
        const float2 xy = load_loc(loc + 2 * so);
        const float a = to_f32(weight[so]);
        Corners c;
        if (corners(levels[level(s0 + lane)], xy.x, xy.y, c)) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            row[k] = c.row[k];
            wa[k] = c.w[k] * a;
          }
        }
      }
      const int n = samples - s0 < 32 ? samples - s0 : 32;
      __syncwarp();  // the previous pass has finished reading the entries
#pragma unroll
      for (int t = lane; t < kDetTable; t += 32) table[t] = -1;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        erow[4 * lane + k] = row[k];
        ewa[4 * lane + k] = wa[k];
        enext[4 * lane + k] = -1;
      }
      __syncwarp();
      // claims: the first entry to take a row's slot owns the row; an entry
      // finding its row's slot taken by another row stays on its own
      int owner[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = 4 * lane + k;
        owner[k] = e;
        if (row[k] >= 0) {
          const int slot = static_cast<int>((static_cast<uint32_t>(row[k]) * 2654435761u) >> 24);  // 256 slots
          const int held = atomicCAS(table + slot, -1, e);
          if (held >= 0 && erow[held] == row[k]) owner[k] = held;
        }
      }
      __syncwarp();
      // repeats join their owner's chain (owners are never repeats, so a
      // repeat's own link is written by it alone)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = 4 * lane + k;
        if (owner[k] != e) {
          enext[e] = atomicExch(enext + owner[k], e);
          erow[e] = -2;  // reached through its owner
        }
      }
      __syncwarp();
      for (int c0 = 0; c0 < d.channels; c0 += 32) {
        const int ch = c0 + lane;
        const bool active = ch < d.channels;
        const float gc = active ? to_f32(grad_out[item * d.channels + ch]) : 0.0f;
        for (int e = 0; e < 4 * n; ++e) {
          const int r = erow[e];
          if (r < 0) continue;  // outside the level, no sample, or a repeat (warp-uniform)
          if (fp.finite) {
            const auto fixed = [&](float contribution) -> long long {
              return __double2ll_rn(static_cast<double>(contribution) * fp.scale);
            };
            long long sum = fixed(ewa[e] * gc);
            for (int x = enext[e]; x >= 0; x = enext[x]) sum += fixed(ewa[x] * gc);
            if (active)
              atomicAdd(acc + head0 + static_cast<int64_t>(r) * row_stride + ch, static_cast<unsigned long long>(sum));
          } else {
            float sum = ewa[e] * gc;
            for (int x = enext[e]; x >= 0; x = enext[x]) sum += ewa[x] * gc;
            if (active) atomicAdd(grad_value + head0 + static_cast<int64_t>(r) * row_stride + ch, sum);
          }
        }
      }
    }
  }
}

// Step 3: grad_value += acc / scale, one writer per element.
__global__ void __launch_bounds__(256) fixed_point_finish_kernel(int64_t n, const unsigned long long* __restrict__ acc,
                                                                 const unsigned* __restrict__ header,
                                                                 int headroom_bits, float* __restrict__ grad_value) {
  const FixedPoint fp = fixed_point(header, headroom_bits);
  if (!fp.finite) return;
  const double inv = 1.0 / fp.scale;  // a power of two: exact
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    grad_value[i] += static_cast<float>(static_cast<double>(static_cast<long long>(acc[i])) * inv);
}

int grid_for(int64_t threads) {
  const int64_t blocks = (threads + 255) / 256;
  return static_cast<int>(blocks < 148 * 64 ? (blocks > 0 ? blocks : 1) : 148 * 64);
}

// Most contributions one grad_value element can receive: every sample of a
// (batch, head) landing on it (a sample's four corners are distinct pixels).
int headroom_bits(const Dims& d) {
  const int64_t most = static_cast<int64_t>(d.queries) * d.levels * d.points;
  int bits = 1;
  while (bits < 62 && (int64_t{1} << bits) < most) ++bits;
  return bits + 1;
}

template <typename T>
cudaError_t launch_t(const Dims& d, const Args& a, void* workspace, cudaStream_t stream) {
  const int64_t n_value = static_cast<int64_t>(d.batch) * d.spatial_size * d.heads * d.channels;
  auto* header = static_cast<unsigned*>(workspace);
  auto* acc = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(workspace) + kHeaderBytes);
  cudaError_t err = cudaMemsetAsync(workspace, 0, deterministic_workspace_bytes(d), stream);
  if (err != cudaSuccess) return err;
  const int64_t items = static_cast<int64_t>(d.batch) * d.queries * d.heads;
  const int64_t n_grad = items * d.channels;
  const int64_t n_weight = items * d.levels * d.points;
  max_abs_kernel<T><<<grid_for(n_grad > n_weight ? n_grad : n_weight), 256, 0, stream>>>(
      static_cast<const T*>(a.grad_out), n_grad, static_cast<const T*>(a.weight), n_weight, header);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  Args dots = a;
  dots.skip_grad_value = true;
  if ((err = launch_backward_rowwise(sizeof(T) == 2 ? DType::kBF16 : DType::kF32, d, dots, stream)) != cudaSuccess)
    return err;
  const int bits = headroom_bits(d);
  fixed_point_scatter_kernel<T><<<grid_for(items * 32), 256, level_smem(d), stream>>>(
      d, a.shapes, a.starts, static_cast<const T*>(a.loc), static_cast<const T*>(a.weight),
      static_cast<const T*>(a.grad_out), header, bits, acc, a.grad_value);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  fixed_point_finish_kernel<<<grid_for(n_value), 256, 0, stream>>>(n_value, acc, header, bits, a.grad_value);
  return cudaGetLastError();
}

}  // namespace

size_t deterministic_workspace_bytes(const Dims& d) {
  return kHeaderBytes + static_cast<size_t>(d.batch) * d.spatial_size * d.heads * d.channels * sizeof(uint64_t);
}

cudaError_t launch_backward_deterministic(DType dtype, const Dims& d, const Args& a, void* workspace,
                                          cudaStream_t stream) {
  if (d.batch == 0 || d.queries == 0 || d.heads == 0 || d.channels == 0) return cudaSuccess;
  return dtype == DType::kBF16 ? launch_t<__nv_bfloat16>(d, a, workspace, stream)
                               : launch_t<float>(d, a, workspace, stream);
}

}  // namespace msda
