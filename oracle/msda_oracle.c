/*
 * MSDA CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A scalar, single-threaded C restatement of muSPACE's multi-scale deformable
 * attention forward and backward. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py load this file (through oracle/msda_oracle.py);
 * the product library never links or calls it.
 *
 * What it restates (paths inside the muSPACE tree):
 *   - sampling geometry: the grid_sample unnormalisation the reference's
 *       PyTorch path runs (mu_space/ops/multi_scale_deformable_attn.py:35,42-48):
 *       g = 2 * loc - 1, then x = (g + 1) * (W / 2) - 0.5, every step rounded to
 *       fp32 separately (no contraction). For loc >= 0.25 this equals the MUSA
 *       kernel's loc * W - 0.5 (ms_deform_attn_musa_kernel.muh:282-283) bit for
 *       bit; below it the extra rounding of (2 * loc - 1) + 1 can move x by one
 *       ulp, which only matters for the one-sided derivative at an integer x.
 *     The MUSA kernel also skips a sample unless -1 < y < H and -1 < x < W
 *       (ms_deform_attn_musa_kernel.muh:286); grid_sample has no such test. The
 *       two agree on every output and on every gradient except at exactly
 *       x == -1 or y == -1, where grid_sample keeps the derivative of the
 *       in-bounds corner row. This oracle follows grid_sample; it only skips
 *       samples whose four corners are all outside (x <= -2, x >= W + 1, ...)
 *       and non-finite coordinates, which changes no result.
 *   - per-corner zeroing outside [0, H-1] x [0, W-1] and the bilinear weights:
 *       ms_deform_attn_musa_kernel.muh:49-90
 *   - the backward formulas (grad_value scatter, grad_attn = g . val,
 *     grad_loc = (W * sum gw * g * a, H * sum gh * g * a)):
 *       ms_deform_attn_musa_kernel.muh:93-166
 *   - tensor layouts value (B, Lin, Hh, D), loc (B, Lq, Hh, L, P, 2) with the
 *     last dim (x, y), weight (B, Lq, Hh, L, P), out (B, Lq, Hh * D):
 *       mu_space/ops/multi_scale_deformable_attn.py:26-58
 * The PyTorch grid_sample formulation of mu_space/ops/multi_scale_deformable_attn.py:26-58
 * (align_corners=False, zero padding) computes the same function; the golden
 * vectors under tests/golden/ come from that function and pin this oracle.
 *
 * Geometry is evaluated in fp32 step by step as grid_sample does (so a
 * bfloat16 location is widened first and never rounded again); every sum is
 * accumulated in double so the oracle carries no accumulation-order noise.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

typedef struct {
  int64_t batch, spatial_size, heads, channels, levels, queries, points;
} oracle_dims;

/* grid_sample's align_corners=False unnormalisation of a [0, 1] location.
 * volatile stores force one fp32 rounding per step. */
static float unnormalize(float loc, int64_t size) {
  volatile float g = 2.0f * loc;
  g = g - 1.0f;
  volatile float t = g + 1.0f;
  volatile float s = t * ((float)size * 0.5f);
  return s - 0.5f;
}

/* One sample's corner table: value row offsets (or -1) and bilinear weights. */
typedef struct {
  int64_t row[4];
  double wt[4];
  float lh, lw, hh, hw;
  int valid;
} corners_t;

static void sample_corners(const oracle_dims *d, const int64_t *shapes, const int64_t *start, int64_t b,
                           int64_t lvl, float loc_x, float loc_y, corners_t *c) {
  const int64_t H = shapes[2 * lvl], W = shapes[2 * lvl + 1];
  const float h_im = unnormalize(loc_y, H);
  const float w_im = unnormalize(loc_x, W);
  c->valid = (h_im > -2.0f && w_im > -2.0f && h_im < (float)H + 1.0f && w_im < (float)W + 1.0f);
  for (int k = 0; k < 4; ++k) {
    c->row[k] = -1;
    c->wt[k] = 0.0;
  }
  if (!c->valid) return;
  const int64_t h_low = (int64_t)floorf(h_im), w_low = (int64_t)floorf(w_im);
  const float lh = h_im - (float)h_low, lw = w_im - (float)w_low;
  const float hh = 1.0f - lh, hw = 1.0f - lw;
  c->lh = lh;
  c->lw = lw;
  c->hh = hh;
  c->hw = hw;
  const int64_t ys[4] = {h_low, h_low, h_low + 1, h_low + 1};
  const int64_t xs[4] = {w_low, w_low + 1, w_low, w_low + 1};
  const double ws[4] = {(double)hh * hw, (double)hh * lw, (double)lh * hw, (double)lh * lw};
  const int64_t base = b * d->spatial_size + start[lvl];
  for (int k = 0; k < 4; ++k) {
    if (ys[k] >= 0 && xs[k] >= 0 && ys[k] <= H - 1 && xs[k] <= W - 1) {
      c->row[k] = base + ys[k] * W + xs[k];
      c->wt[k] = ws[k];
    }
  }
}

void msda_oracle_forward(const oracle_dims *d, const float *value, const int64_t *shapes, const int64_t *start,
                         const float *loc, const float *weight, float *out) {
  const int64_t Hh = d->heads, D = d->channels, L = d->levels, P = d->points;
  for (int64_t b = 0; b < d->batch; ++b)
    for (int64_t q = 0; q < d->queries; ++q)
      for (int64_t h = 0; h < Hh; ++h) {
        const int64_t item = (b * d->queries + q) * Hh + h;
        for (int64_t c = 0; c < D; ++c) {
          double acc = 0.0;
          for (int64_t l = 0; l < L; ++l)
            for (int64_t p = 0; p < P; ++p) {
              const int64_t s = (item * L + l) * P + p;
              corners_t cr;
              sample_corners(d, shapes, start, b, l, loc[2 * s], loc[2 * s + 1], &cr);
              if (!cr.valid) continue;
              double v = 0.0;
              for (int k = 0; k < 4; ++k)
                if (cr.row[k] >= 0) v += cr.wt[k] * (double)value[(cr.row[k] * Hh + h) * D + c];
              acc += v * (double)weight[s];
            }
          out[item * D + c] = (float)acc;
        }
      }
}

/* grad_value is ACCUMULATED into (the caller zeroes it, as the reference FFI
 * requires); grad_loc and grad_weight are written. */
void msda_oracle_backward(const oracle_dims *d, const float *value, const int64_t *shapes, const int64_t *start,
                          const float *loc, const float *weight, const float *grad_out, double *grad_value,
                          float *grad_loc, float *grad_weight) {
  const int64_t Hh = d->heads, D = d->channels, L = d->levels, P = d->points;
  for (int64_t b = 0; b < d->batch; ++b)
    for (int64_t q = 0; q < d->queries; ++q)
      for (int64_t h = 0; h < Hh; ++h) {
        const int64_t item = (b * d->queries + q) * Hh + h;
        const float *g = grad_out + item * D;
        for (int64_t l = 0; l < L; ++l) {
          const int64_t H = shapes[2 * l], W = shapes[2 * l + 1];
          for (int64_t p = 0; p < P; ++p) {
            const int64_t s = (item * L + l) * P + p;
            const double a = (double)weight[s];
            corners_t cr;
            sample_corners(d, shapes, start, b, l, loc[2 * s], loc[2 * s + 1], &cr);
            double g_attn = 0.0, g_x = 0.0, g_y = 0.0;
            if (cr.valid) {
              /* d(bilinear)/d(w_im) and d/d(h_im) per corner, same signs as
               * ms_deform_attn_musa_kernel.muh:130-160 */
              const double dx[4] = {-(double)cr.hh, (double)cr.hh, -(double)cr.lh, (double)cr.lh};
              const double dy[4] = {-(double)cr.hw, -(double)cr.lw, (double)cr.hw, (double)cr.lw};
              for (int64_t c = 0; c < D; ++c) {
                const double gc = (double)g[c];
                double val = 0.0, gx = 0.0, gy = 0.0;
                for (int k = 0; k < 4; ++k) {
                  if (cr.row[k] < 0) continue;
                  const int64_t off = (cr.row[k] * Hh + h) * D + c;
                  const double v = (double)value[off];
                  val += cr.wt[k] * v;
                  gx += dx[k] * v;
                  gy += dy[k] * v;
                  grad_value[off] += cr.wt[k] * gc * a;
                }
                g_attn += gc * val;
                g_x += gc * gx;
                g_y += gc * gy;
              }
            }
            grad_weight[s] = (float)g_attn;
            grad_loc[2 * s] = (float)((double)W * g_x * a);
            grad_loc[2 * s + 1] = (float)((double)H * g_y * a);
          }
        }
      }
}
