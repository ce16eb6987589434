/* Oracle (test infrastructure only): RandSimulateLowResolution,
 * batchaug/pytorch/intensity/resolution.py:74-118, restated from torch's CPU
 * F.interpolate arithmetic for 5-D inputs as pinned against outputs of the
 * reference itself (tests/golden/lowres_*.npz, bit-exact for every
 * downsample/upsample mode pair in fp32 and bf16):
 *
 *   target size per axis  max(1, rint(float(s) * zoom))            (:84-92)
 *   down = interpolate(x, target, downsample_mode), cast to dtype   (:105-108)
 *   up   = interpolate(down, shape, upsample_mode), cast to dtype   (:110-113)
 *
 * Per-axis maps (output index o, input size n, output size m):
 *   nearest        i = min(floor(o * s), n-1),          s = float(n)/m
 *   nearest-exact  i = min(floor((o + 0.5f) * s), n-1)
 *   trilinear      src = fma(s, o + 0.5f, -0.5f) clamped at 0 (align_corners:
 *                  s = (n-1)/(m-1), src = s*o); i0 = min(floor(src), n-1),
 *                  i1 = i0 + (i0 < n-1), l1 = clamp(src - i0, 0, 1),
 *                  l0 = 1 - l1, both held in the dtype (bf16: l1 rounded,
 *                  then l0 = bf16(1 - l1)); equal sizes copy
 *   area           box [floor(o*n/m), ceil((o+1)*n/m)), sum in the dtype
 *                  (each add rounded), then / kh / kw / kd, each rounded
 * Trilinear nests H (outer), W, D (inner), each level fma(t0, w0, t1 * w1)
 * in fp32; nearest modes equal sizes are the identity.  Compiled with
 * -ffp-contract=off; fmaf marks the fused steps. */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORA_BF16 1
float ora_bf16_round(float f);

enum { LR_NEAREST = 0, LR_NEAREST_EXACT = 1, LR_TRILINEAR = 2, LR_AREA = 3 };

static inline float rnd(int dtype, float v) { return dtype == ORA_BF16 ? ora_bf16_round(v) : v; }

static inline float ldv(const void* p, int dtype, int64_t i) {
  if (dtype == ORA_BF16) {
    uint32_t u = (uint32_t)((const uint16_t*)p)[i] << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
  }
  return ((const float*)p)[i];
}

static inline void stv(void* p, int dtype, int64_t i, float v) {
  if (dtype == ORA_BF16) {
    float r = ora_bf16_round(v);
    uint32_t u;
    memcpy(&u, &r, 4);
    ((uint16_t*)p)[i] = (uint16_t)(u >> 16);
  } else {
    ((float*)p)[i] = v;
  }
}

typedef struct {
  int64_t i0, i1;  /* linear taps (nearest: i0 = i1) */
  float l0, l1;
  int64_t a, e;    /* area box [a, e) */
} axmap;

static void axis_map(int mode, int align, int64_t n, int64_t m, int64_t o, int dtype, axmap* r) {
  r->a = (o * n) / m;
  r->e = ((o + 1) * n + m - 1) / m;
  if (mode == LR_NEAREST || mode == LR_NEAREST_EXACT) {
    int64_t i = o;
    if (n != m) {
      const float s = (float)n / (float)m;
      const float p = mode == LR_NEAREST ? (float)o * s : ((float)o + 0.5f) * s;
      i = (int64_t)floorf(p);
      if (i > n - 1) i = n - 1;
    }
    r->i0 = r->i1 = i;
    r->l0 = 1.0f;
    r->l1 = 0.0f;
    return;
  }
  if (mode == LR_TRILINEAR) {
    if (n == m) {
      r->i0 = r->i1 = o;
      r->l0 = 1.0f;
      r->l1 = 0.0f;
      return;
    }
    float src;
    if (align) {
      const float s = m > 1 ? (float)(n - 1) / (float)(m - 1) : 0.0f;
      src = s * (float)o;
    } else {
      const float s = (float)n / (float)m;
      src = fmaf(s, (float)o + 0.5f, -0.5f);
      if (src < 0.0f) src = 0.0f;
    }
    int64_t i0 = (int64_t)floorf(src);
    if (i0 > n - 1) i0 = n - 1;
    float l1 = src - (float)i0;
    l1 = l1 < 0.0f ? 0.0f : (l1 > 1.0f ? 1.0f : l1);
    l1 = rnd(dtype, l1);
    r->i0 = i0;
    r->i1 = i0 + (i0 < n - 1 ? 1 : 0);
    r->l1 = l1;
    r->l0 = rnd(dtype, 1.0f - l1);
  }
}

/* One interpolate of x (C, n0,n1,n2) to (C, m0,m1,m2), result cast to dtype. */
static void interp(const void* x, void* out, int dtype, int64_t C, const int64_t* n,
                   const int64_t* m, int mode, int align) {
  axmap* mp[3];
  for (int ax = 0; ax < 3; ++ax) {
    mp[ax] = (axmap*)malloc(sizeof(axmap) * (size_t)m[ax]);
    for (int64_t o = 0; o < m[ax]; ++o) axis_map(mode, align, n[ax], m[ax], o, dtype, &mp[ax][o]);
  }
  const int64_t nin = n[0] * n[1] * n[2], nout = m[0] * m[1] * m[2];
  for (int64_t c = 0; c < C; ++c)
    for (int64_t h = 0; h < m[0]; ++h)
      for (int64_t w = 0; w < m[1]; ++w)
        for (int64_t d = 0; d < m[2]; ++d) {
          const axmap *A = &mp[0][h], *Bm = &mp[1][w], *D = &mp[2][d];
          const int64_t base = c * nin;
          float v;
          if (mode == LR_AREA) {
            float acc = 0.0f;
            for (int64_t a = A->a; a < A->e; ++a)
              for (int64_t b = Bm->a; b < Bm->e; ++b)
                for (int64_t e = D->a; e < D->e; ++e)
                  acc = rnd(dtype, acc + ldv(x, dtype, base + (a * n[1] + b) * n[2] + e));
            acc = rnd(dtype, acc / (float)(A->e - A->a));
            acc = rnd(dtype, acc / (float)(Bm->e - Bm->a));
            v = acc / (float)(D->e - D->a);
          } else if (mode == LR_TRILINEAR) {
            float th[2];
            for (int ih = 0; ih < 2; ++ih) {
              const int64_t hh = ih ? A->i1 : A->i0;
              float tw[2];
              for (int iw = 0; iw < 2; ++iw) {
                const int64_t ww = iw ? Bm->i1 : Bm->i0;
                const int64_t row = base + (hh * n[1] + ww) * n[2];
                const float x0 = ldv(x, dtype, row + D->i0), x1 = ldv(x, dtype, row + D->i1);
                tw[iw] = fmaf(x0, D->l0, x1 * D->l1);
              }
              th[ih] = fmaf(tw[0], Bm->l0, tw[1] * Bm->l1);
            }
            v = fmaf(th[0], A->l0, th[1] * A->l1);
          } else {
            v = ldv(x, dtype, base + (A->i0 * n[1] + Bm->i0) * n[2] + D->i0);
          }
          stv(out, dtype, c * nout + (h * m[1] + w) * m[2] + d, v);
        }
  for (int ax = 0; ax < 3; ++ax) free(mp[ax]);
}

/* resolution.py:74-118 for a (B, C, H, W, D) batch; zoom (B,) fp32; mask
 * (B,) or NULL; masked-out elements are copied.  Returns 1 for a bad mode. */
int ora_lowres(const void* x, void* out, int dtype, int64_t B, int64_t C, int64_t H, int64_t W,
               int64_t D, const float* zoom, const uint8_t* mask, int down_mode, int up_mode,
               int align_corners, int nthreads) {
  if (down_mode < 0 || down_mode > 3 || up_mode < 0 || up_mode > 3) return 1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  const int64_t S[3] = {H, W, D};
  const int64_t per = C * H * W * D;
  const size_t esz = dtype == ORA_BF16 ? 2 : 4;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic)
#endif
  for (int64_t b = 0; b < B; ++b) {
    const char* xb = (const char*)x + (size_t)(b * per) * esz;
    char* ob = (char*)out + (size_t)(b * per) * esz;
    if (mask && !mask[b]) {
      memcpy(ob, xb, (size_t)per * esz);
      continue;
    }
    int64_t t[3];
    for (int ax = 0; ax < 3; ++ax) {
      const int64_t v = (int64_t)nearbyintf((float)S[ax] * zoom[b]);
      t[ax] = v < 1 ? 1 : v;
    }
    void* down = malloc((size_t)(C * t[0] * t[1] * t[2]) * esz);
    interp(xb, down, dtype, C, S, t, down_mode, down_mode == LR_TRILINEAR ? align_corners : 0);
    interp(down, ob, dtype, C, t, S, up_mode, up_mode == LR_TRILINEAR ? align_corners : 0);
    free(down);
  }
  return 0;
}
