/* Oracle (test infrastructure only): the elastic field composed with the
 * affine that follows it into one grid_sample grid.  This is an extension
 * with no counterpart in the reference, which resamples twice
 * (batchaug/pytorch/geometric/elastic.py:101-125, then
 * batchaug/compose.py:71-110).  The composed mapping, restated op by op:
 *
 *   u   = unnormalise(theta . base(p)), affine_grid with align_corners=False
 *         (the bmm as x*t0, fused y and z terms, then the translation) and
 *         ((g + 1) * N - 1) * 0.5 per axis;
 *   uc  = u clamped to [0, N-1] (NaN -> 0);
 *   out = trilinear(field, uc) + (u - uc) / half,  half = max((N-1)/2, 1e-6),
 *         interpolating x, then y, then z as a*(1-f) + b*f;
 *   elements without the affine: out = field; elements without the field:
 *   field = the identity grid of the elastic convention,
 *   linspace(-(N-1)/2, (N-1)/2, N) / half.
 * Compiled with -ffp-contract=off; fmaf marks the fused steps. */
#include <math.h>
#include <stdint.h>

float ora_linspace(float start, float end, int64_t i, int64_t n);
float ora_base_coord(int64_t i, int64_t n, int align_corners);

static float ident_coord(int64_t q, int64_t n) {
  const float half_lo = ((float)n - 1.0f) / 2.0f;
  const float c0 = ora_linspace(-half_lo, half_lo, q, n);
  return c0 / (half_lo < 1e-6f ? 1e-6f : half_lo);
}

static float field_at(const float* field, int has_field, int64_t b, int64_t H, int64_t W,
                      int64_t D, int64_t z, int64_t y, int64_t x, int r) {
  if (has_field) return field[((b * H + z) * W * D + y * D + x) * 3 + r];
  const int64_t q = r == 0 ? x : (r == 1 ? y : z);
  const int64_t n = r == 0 ? D : (r == 1 ? W : H);
  return ident_coord(q, n);
}

static float lerp_rn(float a, float b, float g, float f) { return a * g + b * f; }

void ora_compose_field(const float* field, const float* theta, const uint8_t* mask_field,
                       const uint8_t* mask_affine, int64_t B, int64_t H, int64_t W, int64_t D,
                       float* out) {
  const int64_t n[3] = {D, W, H};
  for (int64_t b = 0; b < B; ++b) {
    const int hf = mask_field == 0 || mask_field[b] != 0;
    const int ha = mask_affine == 0 || mask_affine[b] != 0;
    const float* t = theta + b * 12;
    for (int64_t h = 0; h < H; ++h)
      for (int64_t w = 0; w < W; ++w)
        for (int64_t d = 0; d < D; ++d) {
          float* o = out + ((b * H + h) * W * D + w * D + d) * 3;
          if (!ha) {
            for (int r = 0; r < 3; ++r) o[r] = field_at(field, hf, b, H, W, D, h, w, d, r);
            continue;
          }
          const float bx = ora_base_coord(d, D, 0), by = ora_base_coord(w, W, 0),
                      bz = ora_base_coord(h, H, 0);
          float u[3], uc[3], f[3], g1[3];
          int64_t i0[3], i1[3];
          for (int r = 0; r < 3; ++r) {
            const float g = fmaf(bz, t[r * 4 + 2], fmaf(by, t[r * 4 + 1], bx * t[r * 4])) + t[r * 4 + 3];
            u[r] = ((g + 1.0f) * (float)n[r] - 1.0f) * 0.5f;
            const float hi = (float)(n[r] - 1);
            uc[r] = isnan(u[r]) ? 0.0f : fminf(fmaxf(u[r], 0.0f), hi);
            i0[r] = (int64_t)floorf(uc[r]);
            i1[r] = i0[r] + 1 < n[r] ? i0[r] + 1 : i0[r];
            f[r] = uc[r] - (float)i0[r];
            g1[r] = 1.0f - f[r];
          }
          for (int r = 0; r < 3; ++r) {
#define FA(z, y, x) field_at(field, hf, b, H, W, D, z, y, x, r)
            const float c00 = lerp_rn(FA(i0[2], i0[1], i0[0]), FA(i0[2], i0[1], i1[0]), g1[0], f[0]);
            const float c01 = lerp_rn(FA(i0[2], i1[1], i0[0]), FA(i0[2], i1[1], i1[0]), g1[0], f[0]);
            const float c10 = lerp_rn(FA(i1[2], i0[1], i0[0]), FA(i1[2], i0[1], i1[0]), g1[0], f[0]);
            const float c11 = lerp_rn(FA(i1[2], i1[1], i0[0]), FA(i1[2], i1[1], i1[0]), g1[0], f[0]);
#undef FA
            const float c0 = lerp_rn(c00, c01, g1[1], f[1]);
            const float c1 = lerp_rn(c10, c11, g1[1], f[1]);
            const float fi = lerp_rn(c0, c1, g1[2], f[2]);
            const float half_lo = ((float)n[r] - 1.0f) / 2.0f;
            const float half = half_lo < 1e-6f ? 1e-6f : half_lo;
            o[r] = fi + (u[r] - uc[r]) / half;
          }
        }
  }
}
