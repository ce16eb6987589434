/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of the batchaug hot path (reference PyTorch backend,
 * halleewong/batchaug) used as the parity checker for the CUDA kernels of
 * batchaug_b200 and as the timed CPU baseline in bench.py.  Nothing in the
 * product path links or calls this file: only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference leg load liboracle_ba.so.
 *
 * The reference's arithmetic lives in PyTorch (third-party dependency,
 * installed version torch 2.11.0; the reference pins only torch>=2.0 in
 * pyproject.toml:14).  The published algorithms restated here are:
 *   - torch.linspace (symmetric two-sided formula, one fused rounding),
 *   - F.affine_grid  (base grid linspace_from_neg_one, then bmm with theta),
 *   - F.grid_sample  (5-D, bilinear=trilinear / nearest, zeros / border /
 *                     reflection padding, align_corners False / True),
 * and the batchaug wrappers around them:
 *   - batchaug/pytorch/geometric/affine.py:154-195  monai_affine_to_theta
 *   - batchaug/compose.py:71-110                    Compose._materialize
 *   - batchaug/pytorch/geometric/affine.py:284-317  RandAffine.apply
 *   - batchaug/pytorch/geometric/elastic.py:101-125 Rand3DElastic.apply
 *
 * Floating-point contract: this file is compiled with -ffp-contract=off so
 * every multiply and add rounds separately, exactly like torch's scalar CPU
 * grid sampler.  Where torch's CPU path fuses (MKL's bmm in affine_grid,
 * linspace) the oracle calls fmaf() explicitly.  The orderings were pinned
 * against torch 2.11 CPU outputs (tests/golden).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORA_F32 0
#define ORA_BF16 1

#define ORA_BILINEAR 0
#define ORA_NEAREST 1

#define ORA_PAD_ZEROS 0
#define ORA_PAD_BORDER 1
#define ORA_PAD_REFLECTION 2

#define ORA_XFORM_AFFINE 0 /* MONAI-convention (B,4,4) affine */
#define ORA_XFORM_THETA 1  /* affine_grid theta, rows of 4, row stride 4 */
#define ORA_XFORM_GRID 2   /* grid_sample grid (B,H,W,D,3), xyz order */

/* ------------------------------------------------------------------ */
/* bfloat16 storage: round-to-nearest-even as c10::BFloat16 does.     */
/* ------------------------------------------------------------------ */
static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if (f != f) return (uint16_t)0x7FC0; /* canonical NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

float ora_bf16_round(float f) { return bf16_to_f32(f32_to_bf16(f)); }

void ora_bf16_from_f32(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = f32_to_bf16(src[i]);
}

void ora_bf16_to_f32(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = bf16_to_f32(src[i]);
}

static inline float load_elem(const void* p, int dtype, int64_t i) {
  return dtype == ORA_BF16 ? bf16_to_f32(((const uint16_t*)p)[i]) : ((const float*)p)[i];
}

static inline void store_elem(void* p, int dtype, int64_t i, float v) {
  if (dtype == ORA_BF16)
    ((uint16_t*)p)[i] = f32_to_bf16(v);
  else
    ((float*)p)[i] = v;
}

/* ------------------------------------------------------------------ */
/* torch.linspace(-1, 1, N)[i]: step = fl(2/(N-1)); the first half is */
/* fma(step, i, -1), the second half fma(-step, N-1-i, 1).            */
/* ------------------------------------------------------------------ */
float ora_linspace_m1p1(int64_t i, int64_t n) {
  if (n == 1) return -1.0f;
  float step = 2.0f / (float)(n - 1);
  if (i < n / 2) return fmaf(step, (float)i, -1.0f);
  return fmaf(-step, (float)(n - 1 - i), 1.0f);
}

/* affine_grid's linspace_from_neg_one: 0 for a single step; otherwise the
 * linspace, scaled by (N-1)/N when align_corners is false (one multiply,
 * one divide, each rounded). */
float ora_base_coord(int64_t i, int64_t n, int align_corners) {
  if (n <= 1) return 0.0f;
  float r = ora_linspace_m1p1(i, n);
  if (!align_corners) r = (r * (float)(n - 1)) / (float)n;
  return r;
}

/* monai_affine_to_theta (affine.py:154-195): theta = P @ S_norm @ A @ S_inv @ P
 * with P swapping axes 0 and 2.  Every product of the chain has one nonzero
 * term, so theta[i][j] = fl(fl(sn[p(i)] * A[p(i)][p(j)]) * si[p(j)]). */
void ora_affine_to_theta(const float* affine, int64_t batch, int64_t h, int64_t w, int64_t d,
                         float* theta /* (B,3,4) */) {
  const int perm[4] = {2, 1, 0, 3};
  float sn[4], si[4];
  sn[0] = (float)(2.0 / (double)h);
  sn[1] = (float)(2.0 / (double)w);
  sn[2] = (float)(2.0 / (double)d);
  sn[3] = 1.0f;
  si[0] = (float)((double)h / 2.0);
  si[1] = (float)((double)w / 2.0);
  si[2] = (float)((double)d / 2.0);
  si[3] = 1.0f;
  for (int64_t b = 0; b < batch; ++b) {
    const float* a = affine + b * 16;
    float* t = theta + b * 12;
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 4; ++j) {
        int pi = perm[i], pj = perm[j];
        float v = sn[pi] * a[pi * 4 + pj];
        t[i * 4 + j] = v * si[pj];
      }
  }
}

/* ------------------------------------------------------------------ */
/* grid_sample coordinate helpers (restated from the published         */
/* algorithm of torch's GridSampler: unnormalize, clip, reflect).      */
/* ------------------------------------------------------------------ */
static inline float unnormalize(float coord, int64_t size, int align_corners) {
  if (align_corners) return ((coord + 1.0f) / 2.0f) * (float)(size - 1);
  return ((coord + 1.0f) * (float)size - 1.0f) / 2.0f;
}

static inline float clip_coord(float in, int64_t size) {
  /* std::min(size-1, std::max(in, 0)): std::max(a,b) is (a<b)?b:a and
   * std::min(a,b) is (b<a)?b:a, so a NaN coordinate clips to size-1. */
  float lo = (in < 0.0f) ? 0.0f : in;
  float hi = (float)(size - 1);
  return (lo < hi) ? lo : hi;
}

static inline float reflect_coord(float in, int64_t twice_low, int64_t twice_high) {
  if (twice_low == twice_high) return 0.0f;
  float mn = (float)twice_low / 2.0f;
  float span = (float)(twice_high - twice_low) / 2.0f;
  in = fabsf(in - mn);
  float extra = fmodf(in, span);
  int flips = (int)floorf(in / span);
  if (flips % 2 == 0) return extra + mn;
  return span - extra + mn;
}

static inline float source_index(float coord, int64_t size, int padding, int align_corners) {
  coord = unnormalize(coord, size, align_corners);
  if (padding == ORA_PAD_BORDER) {
    coord = clip_coord(coord, size);
  } else if (padding == ORA_PAD_REFLECTION) {
    if (align_corners)
      coord = reflect_coord(coord, 0, 2 * (size - 1));
    else
      coord = reflect_coord(coord, -1, 2 * size - 1);
    coord = clip_coord(coord, size);
  }
  return coord;
}

static inline int inb(int64_t z, int64_t y, int64_t x, int64_t nz, int64_t ny, int64_t nx) {
  return z >= 0 && z < nz && y >= 0 && y < ny && x >= 0 && x < nx;
}

/* One output voxel of grid_sample for every channel of one element.
 * ix indexes D (last dim), iy indexes W, iz indexes H. */
static void sample_voxel(const void* src, void* dst, int dtype, int64_t C, int64_t H, int64_t W,
                         int64_t D, int64_t src_b_off, int64_t out_idx, float gx, float gy, float gz,
                         int mode, int padding, int align_corners) {
  const int64_t hwd = H * W * D;
  float ix = source_index(gx, D, padding, align_corners);
  float iy = source_index(gy, W, padding, align_corners);
  float iz = source_index(gz, H, padding, align_corners);
  if (mode == ORA_NEAREST) {
    int64_t xn = (int64_t)nearbyintf(ix);
    int64_t yn = (int64_t)nearbyintf(iy);
    int64_t zn = (int64_t)nearbyintf(iz);
    int ok = inb(zn, yn, xn, H, W, D);
    for (int64_t c = 0; c < C; ++c) {
      float v = ok ? load_elem(src, dtype, src_b_off + c * hwd + (zn * W + yn) * D + xn) : 0.0f;
      store_elem(dst, dtype, src_b_off + c * hwd + out_idx, v);
    }
    return;
  }
  int64_t x0 = (int64_t)floorf(ix), y0 = (int64_t)floorf(iy), z0 = (int64_t)floorf(iz);
  int64_t x1 = x0 + 1, y1 = y0 + 1, z1 = z0 + 1;
  /* distances as torch writes them: (corner_int - coord) / (coord - corner_int) */
  float wx0 = (float)x1 - ix, wx1 = ix - (float)x0;
  float wy0 = (float)y1 - iy, wy1 = iy - (float)y0;
  float wz0 = (float)z1 - iz, wz1 = iz - (float)z0;
  float tnw = wx0 * wy0 * wz0;
  float tne = wx1 * wy0 * wz0;
  float tsw = wx0 * wy1 * wz0;
  float tse = wx1 * wy1 * wz0;
  float bnw = wx0 * wy0 * wz1;
  float bne = wx1 * wy0 * wz1;
  float bsw = wx0 * wy1 * wz1;
  float bse = wx1 * wy1 * wz1;
  const int64_t cz[8] = {z0, z0, z0, z0, z1, z1, z1, z1};
  const int64_t cy[8] = {y0, y0, y1, y1, y0, y0, y1, y1};
  const int64_t cx[8] = {x0, x1, x0, x1, x0, x1, x0, x1};
  const float cw[8] = {tnw, tne, tsw, tse, bnw, bne, bsw, bse};
  for (int64_t c = 0; c < C; ++c) {
    const int64_t cb = src_b_off + c * hwd;
    float out = 0.0f;
    for (int k = 0; k < 8; ++k)
      if (inb(cz[k], cy[k], cx[k], H, W, D))
        out += load_elem(src, dtype, cb + (cz[k] * W + cy[k]) * D + cx[k]) * cw[k];
    store_elem(dst, dtype, cb + out_idx, out);
  }
}

/* Resample a (B,C,H,W,D) tensor: the fused materialisation of a lazily
 * composed geometric group (compose.py:71-110) or one eager geometric
 * apply (affine.py:284-317, elastic.py:101-125).  Output voxels of masked-out
 * elements copy the input (torch.where(mask, result, tensor)).
 * xform_kind: ORA_XFORM_AFFINE -> MONAI affine (B,4,4), converted with
 *             monai_affine_to_theta; ORA_XFORM_THETA -> theta rows (B,3|4,4)
 *             with xform_stride floats per element; ORA_XFORM_GRID -> grid
 *             (B,H,W,D,3).  Returns 0 on success, 1 on bad arguments. */
int ora_resample3d(const void* src, void* dst, int dtype, int64_t B, int64_t C, int64_t H,
                   int64_t W, int64_t D, int xform_kind, const float* xform, int64_t xform_stride,
                   int mode, int padding, int align_corners, const uint8_t* mask, int nthreads) {
  if (!src || !dst || !xform || B < 0 || C < 0 || H <= 0 || W <= 0 || D <= 0) return 1;
  if (dtype != ORA_F32 && dtype != ORA_BF16) return 1;
  const int64_t hwd = H * W * D;
  float* theta = NULL;
  if (xform_kind == ORA_XFORM_AFFINE) {
    theta = (float*)malloc(sizeof(float) * 12 * (B > 0 ? B : 1));
    ora_affine_to_theta(xform, B, H, W, D, theta);
  }
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t z = 0; z < H; ++z) {
      const int64_t boff = b * C * hwd;
      if (mask && !mask[b]) {
        for (int64_t c = 0; c < C; ++c) {
          int64_t base = boff + c * hwd + z * W * D;
          if (dtype == ORA_BF16)
            memcpy((uint16_t*)dst + base, (const uint16_t*)src + base, sizeof(uint16_t) * W * D);
          else
            memcpy((float*)dst + base, (const float*)src + base, sizeof(float) * W * D);
        }
        continue;
      }
      const float* th = NULL;
      if (xform_kind == ORA_XFORM_AFFINE) th = theta + b * 12;
      if (xform_kind == ORA_XFORM_THETA) th = xform + b * xform_stride;
      float bz = ora_base_coord(z, H, align_corners);
      for (int64_t y = 0; y < W; ++y) {
        float by = ora_base_coord(y, W, align_corners);
        for (int64_t x = 0; x < D; ++x) {
          const int64_t out_idx = (z * W + y) * D + x;
          float gx, gy, gz;
          if (xform_kind == ORA_XFORM_GRID) {
            const float* g = xform + (b * hwd + out_idx) * 3;
            gx = g[0];
            gy = g[1];
            gz = g[2];
          } else {
            float bx = ora_base_coord(x, D, align_corners);
            /* affine_grid's bmm, as MKL accumulates it: x*t0 rounded, then
             * fused y and z terms, then the translation. */
            gx = fmaf(bz, th[2], fmaf(by, th[1], bx * th[0])) + th[3];
            gy = fmaf(bz, th[6], fmaf(by, th[5], bx * th[4])) + th[7];
            gz = fmaf(bz, th[10], fmaf(by, th[9], bx * th[8])) + th[11];
          }
          sample_voxel(src, dst, dtype, C, H, W, D, boff, out_idx, gx, gy, gz, mode, padding,
                       align_corners);
        }
      }
    }
  }
  free(theta);
  return 0;
}

/* The affine_grid grid itself (B,H,W,D,3), used to pin the coordinate
 * restatement against F.affine_grid. */
void ora_affine_grid(const float* theta, int64_t theta_stride, int64_t B, int64_t H, int64_t W,
                     int64_t D, int align_corners, float* grid) {
  for (int64_t b = 0; b < B; ++b) {
    const float* th = theta + b * theta_stride;
    for (int64_t z = 0; z < H; ++z) {
      float bz = ora_base_coord(z, H, align_corners);
      for (int64_t y = 0; y < W; ++y) {
        float by = ora_base_coord(y, W, align_corners);
        for (int64_t x = 0; x < D; ++x) {
          float bx = ora_base_coord(x, D, align_corners);
          float* g = grid + ((b * H + z) * W * D + y * D + x) * 3;
          g[0] = fmaf(bz, th[2], fmaf(by, th[1], bx * th[0])) + th[3];
          g[1] = fmaf(bz, th[6], fmaf(by, th[5], bx * th[4])) + th[7];
          g[2] = fmaf(bz, th[10], fmaf(by, th[9], bx * th[8])) + th[11];
        }
      }
    }
  }
}
