/*
 * CPU ORACLE — test infrastructure only (see oracle.c for the contract).
 *
 * Restates the reference PyTorch backend's intensity chain and Gaussian
 * smoothing, op by op and in the tensor's own dtype, because the reference
 * rounds every intermediate to that dtype (bf16 tensors: one bf16 rounding
 * per torch op, each op computed in fp32).
 *
 *   batchaug/pytorch/intensity/noise.py:48-66        RandGaussianNoise
 *   batchaug/pytorch/intensity/contrast.py:35-68     ScaleIntensity.apply
 *   batchaug/pytorch/intensity/contrast.py:116-131   RandAdjustContrast.apply
 *   batchaug/pytorch/intensity/scale_shift.py:51-56  RandScaleIntensity.apply
 *   batchaug/pytorch/intensity/scale_shift.py:106-113 RandShiftIntensity.apply
 *   batchaug/pytorch/intensity/bias_field.py:8-53,99-112 RandBiasField
 *   batchaug/pytorch/intensity/smooth.py:9-34        gaussian_1d_batch
 *   batchaug/pytorch/intensity/smooth.py:37-88       separable_gaussian_conv3d
 *   batchaug/pytorch/geometric/elastic.py:37-99      Rand3DElastic.sample_params
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

float ora_bf16_round(float f);
float ora_linspace_m1p1(int64_t i, int64_t n);

static inline float rnd(int dtype, float v) { return dtype == ORA_BF16 ? ora_bf16_round(v) : v; }

static inline float ld(const void* p, int dtype, int64_t i) {
  if (dtype == ORA_BF16) {
    uint32_t u = ((uint32_t)((const uint16_t*)p)[i]) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
  }
  return ((const float*)p)[i];
}

static inline void st(void* p, int dtype, int64_t i, float v) {
  if (dtype == ORA_BF16) {
    float r = ora_bf16_round(v);
    uint32_t u;
    memcpy(&u, &r, 4);
    ((uint16_t*)p)[i] = (uint16_t)(u >> 16);
  } else {
    ((float*)p)[i] = v;
  }
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
}

/* torch.linspace(start, end, n)[i] (general range, fused rounding). */
float ora_linspace(float start, float end, int64_t i, int64_t n) {
  if (n == 1) return start;
  float step = (end - start) / (float)(n - 1);
  if (i < n / 2) return fmaf(step, (float)i, start);
  return fmaf(-step, (float)(n - 1 - i), end);
}

/* min/max of each contiguous group; a NaN anywhere makes both NaN, as
 * torch.min/max do. */
void ora_minmax(const void* x, int dtype, int64_t n_groups, int64_t group_size, float* mins,
                float* maxs, int nthreads) {
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t g = 0; g < n_groups; ++g) {
    float mn = INFINITY, mx = -INFINITY;
    int nan = 0;
    for (int64_t i = 0; i < group_size; ++i) {
      float v = ld(x, dtype, g * group_size + i);
      if (v != v) nan = 1;
      if (v < mn) mn = v;
      if (v > mx) mx = v;
    }
    mins[g] = nan ? NAN : mn;
    maxs[g] = nan ? NAN : mx;
  }
}

/* noise.py:62-66: tensor + noise.to(dt) * mask.to(dt), every op in dt. */
void ora_noise_add(const void* x, void* out, int dtype, const float* noise, const uint8_t* mask,
                   int64_t B, int64_t n_per_b, int nthreads) {
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < n_per_b; ++i) {
      int64_t k = b * n_per_b + i;
      float m = (mask == NULL || mask[b]) ? 1.0f : 0.0f;
      float nz = rnd(dtype, noise[k]);
      float nm = rnd(dtype, nz * m);
      st(out, dtype, k, ld(x, dtype, k) + nm);
    }
}

/* contrast.py:116-131: per-element min/max over all channels, gamma in
 * fp32, one cast back; masked elements keep the input. */
void ora_adjust_contrast(const void* x, void* out, int dtype, const float* gamma,
                         const uint8_t* mask, int64_t B, int64_t n_per_b, int nthreads) {
  float* mins = (float*)malloc(sizeof(float) * (B > 0 ? B : 1));
  float* maxs = (float*)malloc(sizeof(float) * (B > 0 ? B : 1));
  ora_minmax(x, dtype, B, n_per_b, mins, maxs, nthreads);
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < n_per_b; ++i) {
      int64_t k = b * n_per_b + i;
      float v = ld(x, dtype, k);
      if (mask && !mask[b]) {
        st(out, dtype, k, v);
        continue;
      }
      float rng = maxs[b] - mins[b];
      float nrm = (v - mins[b]) / (rng + 1e-7f);
      nrm = (nrm < 0.0f) ? 0.0f : nrm;
      float r = powf(nrm, gamma[b]) * rng + mins[b];
      st(out, dtype, k, r);
    }
  free(mins);
  free(maxs);
}

/* scale_shift.py:51-56: tensor * (1 + factor.to(dt)), every op in dt. */
void ora_rand_scale(const void* x, void* out, int dtype, const float* factor, const uint8_t* mask,
                    int64_t B, int64_t n_per_b, int nthreads) {
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < n_per_b; ++i) {
      int64_t k = b * n_per_b + i;
      float v = ld(x, dtype, k);
      if (mask && !mask[b]) {
        st(out, dtype, k, v);
        continue;
      }
      float s = rnd(dtype, 1.0f + rnd(dtype, factor[b]));
      st(out, dtype, k, v * s);
    }
}

/* scale_shift.py:106-113: tensor + offset.to(dt), optional clamp to [0,1]. */
void ora_rand_shift(const void* x, void* out, int dtype, const float* offset, const uint8_t* mask,
                    int safe, int64_t B, int64_t n_per_b, int nthreads) {
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < n_per_b; ++i) {
      int64_t k = b * n_per_b + i;
      float v = ld(x, dtype, k);
      if (mask && !mask[b]) {
        st(out, dtype, k, v);
        continue;
      }
      float r = rnd(dtype, v + rnd(dtype, offset[b]));
      if (safe) r = (r < 0.0f) ? 0.0f : ((r > 1.0f) ? 1.0f : r);
      st(out, dtype, k, r);
    }
}

/* contrast.py:35-68: ScaleIntensity in the tensor dtype.
 * flags bit0: minv given, bit1: maxv given, bit2: channel_wise,
 * bit3: factor given (then out = x * (1 + factor)). */
void ora_scale_intensity(const void* x, void* out, int dtype, int64_t B, int64_t C,
                         int64_t n_spatial, double minv, double maxv, double factor, int flags,
                         int nthreads) {
  const int has_min = flags & 1, has_max = (flags >> 1) & 1, chw = (flags >> 2) & 1;
  const int has_factor = (flags >> 3) & 1;
  const int64_t n = B * C * n_spatial;
  if (has_factor) {
    float s = (float)(1.0 + factor);
    for (int64_t k = 0; k < n; ++k) st(out, dtype, k, ld(x, dtype, k) * s);
    return;
  }
  if (!has_min && !has_max) {
    for (int64_t k = 0; k < n; ++k) st(out, dtype, k, ld(x, dtype, k));
    return;
  }
  const int64_t n_groups = chw ? B * C : B;
  const int64_t gsize = chw ? n_spatial : C * n_spatial;
  float* mins = (float*)malloc(sizeof(float) * (n_groups > 0 ? n_groups : 1));
  float* maxs = (float*)malloc(sizeof(float) * (n_groups > 0 ? n_groups : 1));
  ora_minmax(x, dtype, n_groups, gsize, mins, maxs, nthreads);
  const float span = (float)(maxv - minv);
  const float fminv = (float)minv;
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t g = 0; g < n_groups; ++g)
    for (int64_t i = 0; i < gsize; ++i) {
      int64_t k = g * gsize + i;
      float v = ld(x, dtype, k);
      float denom = rnd(dtype, maxs[g] - mins[g]);
      int is_const = denom == 0.0f;
      if (is_const) denom = 1.0f;
      float nrm = rnd(dtype, rnd(dtype, v - mins[g]) / denom);
      float r = nrm;
      if (has_min && has_max) r = rnd(dtype, rnd(dtype, nrm * span) + fminv);
      if (has_min && is_const) r = rnd(dtype, v * fminv);
      st(out, dtype, k, r);
    }
  free(mins);
  free(maxs);
}

/* Legendre values L_0..L_deg at one coordinate with the reference's
 * recurrence p_n = ((2n-1) * c * p_{n-1} - (n-1) * p_{n-2}) / n. */
static void legendre(float c, int deg, float* p) {
  p[0] = 1.0f;
  if (deg >= 1) p[1] = c;
  for (int n = 2; n <= deg; ++n) {
    float a = ((float)(2 * n - 1) * c) * p[n - 1];
    float s = (float)(n - 1) * p[n - 2];
    p[n] = (a - s) / (float)n;
  }
}

/* bias_field.py:8-53 and :99-112.  Triplets (i,j,k), i+j+k <= degree, in
 * the reference's nested-loop order; the einsum over coefficients is the
 * fused chain torch's CPU mm produces. */
int ora_bias_field(const void* x, void* out, int dtype, const float* coeffs, const uint8_t* mask,
                   int64_t B, int64_t C, int64_t H, int64_t W, int64_t D, int degree, int nthreads) {
  if (degree < 1 || degree > 8) return 1;
  int tri[165][3];
  int nc = 0;
  for (int i = 0; i <= degree; ++i)
    for (int j = 0; j <= degree - i; ++j)
      for (int k = 0; k <= degree - i - j; ++k) {
        tri[nc][0] = i;
        tri[nc][1] = j;
        tri[nc][2] = k;
        ++nc;
      }
  const int64_t hwd = H * W * D;
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t b = 0; b < B; ++b)
    for (int64_t z = 0; z < H; ++z) {
      float lx[9], ly[9], lz[9];
      legendre(ora_linspace(-1.0f, 1.0f, z, H), degree, lx);
      for (int64_t y = 0; y < W; ++y) {
        legendre(ora_linspace(-1.0f, 1.0f, y, W), degree, ly);
        for (int64_t xi = 0; xi < D; ++xi) {
          legendre(ora_linspace(-1.0f, 1.0f, xi, D), degree, lz);
          const float* cb = coeffs + b * nc;
          float acc = 0.0f;
          for (int t = 0; t < nc; ++t) {
            float basis = (lx[tri[t][0]] * ly[tri[t][1]]) * lz[tri[t][2]];
            acc = (t == 0) ? cb[0] * basis : fmaf(cb[t], basis, acc);
          }
          float mult = expf(acc);
          int64_t s = (z * W + y) * D + xi;
          for (int64_t c = 0; c < C; ++c) {
            int64_t k = (b * C + c) * hwd + s;
            float v = ld(x, dtype, k);
            if (mask && !mask[b])
              st(out, dtype, k, v);
            else
              st(out, dtype, k, v * mult);
          }
        }
      }
    }
  return 0;
}

/* smooth.py:9-34: per-element erf-integrated taps, padded to the batch-max
 * tail.  Returns K (taps per element) and writes (B,K) into out when out
 * is not NULL. */
int64_t ora_gaussian_1d_batch(const float* sigmas, int64_t B, double truncated, float* out) {
  double max_sigma = 0.0;
  for (int64_t b = 0; b < B; ++b) {
    float s = sigmas[b] < 1e-6f ? 1e-6f : sigmas[b];
    if (b == 0 || (double)s > max_sigma) max_sigma = (double)s;
  }
  double t = max_sigma * truncated;
  int64_t tail = (int64_t)((t > 0.5 ? t : 0.5) + 0.5);
  int64_t K = 2 * tail + 1;
  if (!out) return K;
  for (int64_t b = 0; b < B; ++b) {
    float s = sigmas[b] < 1e-6f ? 1e-6f : sigmas[b];
    float tt = 0.70710678f / s;
    float* o = out + b * K;
    float sum = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
      float xk = (float)(k - tail);
      float v = 0.5f * (erff(tt * (xk + 0.5f)) - erff(tt * (xk - 0.5f)));
      o[k] = v < 0.0f ? 0.0f : v;
      sum += o[k];
    }
    for (int64_t k = 0; k < K; ++k) o[k] = o[k] / sum;
  }
  return K;
}

/* Source index of padded position q along an axis of length n, or -1 for a
 * zero tap: padding 0 = conv3d's implicit zeros, 1 = F.pad "reflect"
 * (mirror without repeating the edge), 2 = F.pad "replicate". */
static int64_t pad_index(int64_t q, int64_t n, int padding) {
  if (q >= 0 && q < n) return q;
  if (padding == 1) {
    if (n == 1) return 0;
    int64_t period = 2 * (n - 1);
    int64_t r = q % period;
    if (r < 0) r += period;
    return r < n ? r : period - r;
  }
  if (padding == 2) return q < 0 ? 0 : n - 1;
  return -1;
}

/* One padded 1-D correlation along `axis` (0=H,1=W,2=D) of an fp32
 * (B,C,H,W,D) array with per-element taps (B,K). */
static void conv_axis(const float* in, float* out, const float* taps, int64_t K, int64_t B,
                      int64_t C, int64_t H, int64_t W, int64_t D, int axis, int padding) {
  const int64_t pad = K / 2;
  const int64_t hwd = H * W * D;
  const int64_t n = axis == 0 ? H : (axis == 1 ? W : D);
  const int64_t stride = axis == 0 ? W * D : (axis == 1 ? D : 1);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t bc = 0; bc < B * C; ++bc)
    for (int64_t s = 0; s < hwd; ++s) {
      const int64_t b = bc / C;
      const float* w = taps + b * K;
      const int64_t pos = (s / stride) % n;
      const float* src = in + bc * hwd + s;
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        int64_t q = pad_index(pos + k - pad, n, padding);
        if (q < 0) continue;
        acc += src[(q - pos) * stride] * w[k];
      }
      out[bc * hwd + s] = acc;
    }
}

/* smooth.py:37-88: H pass, then W, then D, in fp32, result cast to dtype;
 * padding 0 = padding_mode None/"constant", 1 = "reflect", 2 = "replicate".
 * x and out may be the same buffer. */
void ora_separable_gauss(const void* x, void* out, int dtype, const float* kh, int64_t Kh,
                         const float* kw, int64_t Kw, const float* kd, int64_t Kd, int64_t B,
                         int64_t C, int64_t H, int64_t W, int64_t D, int padding, int nthreads) {
  set_threads(nthreads);
  const int64_t n = B * C * H * W * D;
  float* a = (float*)malloc(sizeof(float) * (n > 0 ? n : 1));
  float* t = (float*)malloc(sizeof(float) * (n > 0 ? n : 1));
  for (int64_t k = 0; k < n; ++k) a[k] = ld(x, dtype, k);
  conv_axis(a, t, kh, Kh, B, C, H, W, D, 0, padding);
  conv_axis(t, a, kw, Kw, B, C, H, W, D, 1, padding);
  conv_axis(a, t, kd, Kd, B, C, H, W, D, 2, padding);
  for (int64_t k = 0; k < n; ++k) st(out, dtype, k, t[k]);
  free(a);
  free(t);
}

/* elastic.py:43-99: turn a uniform draw u (B,3,H,W,D) in [0,1) into the
 * grid_sample grid (B,H,W,D,3): disp = smooth(u*2-1) * magnitude, plus the
 * MONAI centred grid, divided by (N-1)/2, reordered to (x=D, y=W, z=H). */
void ora_elastic_grid(const float* u, const float* taps, int64_t K, const float* magnitude,
                      int64_t B, int64_t H, int64_t W, int64_t D, float* grid, int nthreads) {
  set_threads(nthreads);
  const int64_t hwd = H * W * D;
  const int64_t n = B * 3 * hwd;
  float* a = (float*)malloc(sizeof(float) * (n > 0 ? n : 1));
  float* t = (float*)malloc(sizeof(float) * (n > 0 ? n : 1));
  for (int64_t k = 0; k < n; ++k) a[k] = u[k] * 2.0f - 1.0f;
  /* three components, each smoothed as its own (B,1,H,W,D) tensor */
  conv_axis(a, t, taps, K, B, 3, H, W, D, 0, 0);
  conv_axis(t, a, taps, K, B, 3, H, W, D, 1, 0);
  conv_axis(a, t, taps, K, B, 3, H, W, D, 2, 0);
  const int64_t sz[3] = {H, W, D};
  float half[3];
  for (int i = 0; i < 3; ++i) {
    half[i] = ((float)sz[i] - 1.0f) / 2.0f;
    if (half[i] < 1e-6f) half[i] = 1e-6f;
  }
  for (int64_t b = 0; b < B; ++b)
    for (int64_t z = 0; z < H; ++z)
      for (int64_t y = 0; y < W; ++y)
        for (int64_t x = 0; x < D; ++x) {
          const int64_t s = (z * W + y) * D + x;
          const int64_t idx[3] = {z, y, x};
          float* g = grid + (b * hwd + s) * 3;
          for (int comp = 0; comp < 3; ++comp) {
            float disp = t[(b * 3 + comp) * hwd + s] * magnitude[b];
            float c0 = ora_linspace(-((float)sz[comp] - 1.0f) / 2.0f,
                                    ((float)sz[comp] - 1.0f) / 2.0f, idx[comp], sz[comp]);
            float v = (c0 + disp) / half[comp];
            g[2 - comp] = v;
          }
        }
  free(a);
  free(t);
}

/* Per-group moments in double: sum, sum of squares and the count of nonzero
 * values (torch reduces float tensors with double accumulators on CPU). */
static void group_moments(const void* x, int dtype, int64_t n_groups, int64_t gsize, double* sum,
                          double* sumsq, int64_t* nnz, int nthreads) {
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t g = 0; g < n_groups; ++g) {
    double s = 0.0, ss = 0.0;
    int64_t nz = 0;
    for (int64_t i = 0; i < gsize; ++i) {
      const double v = (double)ld(x, dtype, g * gsize + i);
      s += v;
      ss += v * v;
      nz += v != 0.0;
    }
    sum[g] = s;
    sumsq[g] = ss;
    nnz[g] = nz;
  }
}

/* torch.std (unbiased) of n values from their sum and sum of squares. */
static float std_of(double s, double ss, int64_t n) {
  if (n < 2) return NAN;
  const double m = s / (double)n;
  double v = (ss - s * m) / (double)(n - 1);
  if (v < 0.0) v = 0.0;
  return (float)sqrt(v);
}

/* scale_shift.py:130-198: out = x + factor * std(x), std per element or per
 * channel (channel_wise); nonzero: std of the nonzero values when there are
 * at least two of them, else of all values.  fp32 arithmetic, one cast. */
void ora_std_shift(const void* x, void* out, int dtype, const float* factor, const uint8_t* mask,
                   int64_t B, int64_t C, int64_t n_spatial, int nonzero, int channel_wise,
                   int nthreads) {
  const int64_t n_groups = channel_wise ? B * C : B;
  const int64_t gsize = channel_wise ? n_spatial : C * n_spatial;
  const int64_t ng = n_groups > 0 ? n_groups : 1;
  double* s = (double*)malloc(sizeof(double) * ng);
  double* ss = (double*)malloc(sizeof(double) * ng);
  int64_t* nz = (int64_t*)malloc(sizeof(int64_t) * ng);
  group_moments(x, dtype, n_groups, gsize, s, ss, nz, nthreads);
  for (int64_t g = 0; g < n_groups; ++g) {
    const int64_t b = channel_wise ? g / C : g;
    float sd = (nonzero && nz[g] > 1) ? std_of(s[g], ss[g], nz[g]) : std_of(s[g], ss[g], gsize);
    const float shift = factor[b] * sd;
    for (int64_t i = 0; i < gsize; ++i) {
      const int64_t k = g * gsize + i;
      const float v = ld(x, dtype, k);
      st(out, dtype, k, (mask && !mask[b]) ? v : v + shift);
    }
  }
  free(s);
  free(ss);
  free(nz);
}

/* scale_shift.py:201-274: out = mean + (x - mean) * (1 + factor), mean per
 * element or per channel, fp32 arithmetic, one cast. */
void ora_fixed_mean(const void* x, void* out, int dtype, const float* factor, const uint8_t* mask,
                    int64_t B, int64_t C, int64_t n_spatial, int channel_wise, int nthreads) {
  const int64_t n_groups = channel_wise ? B * C : B;
  const int64_t gsize = channel_wise ? n_spatial : C * n_spatial;
  const int64_t ng = n_groups > 0 ? n_groups : 1;
  double* s = (double*)malloc(sizeof(double) * ng);
  double* ss = (double*)malloc(sizeof(double) * ng);
  int64_t* nz = (int64_t*)malloc(sizeof(int64_t) * ng);
  group_moments(x, dtype, n_groups, gsize, s, ss, nz, nthreads);
  for (int64_t g = 0; g < n_groups; ++g) {
    const int64_t b = channel_wise ? g / C : g;
    const float mean = (float)(s[g] / (double)gsize);
    const float f1 = 1.0f + factor[b];
    for (int64_t i = 0; i < gsize; ++i) {
      const int64_t k = g * gsize + i;
      const float v = ld(x, dtype, k);
      st(out, dtype, k, (mask && !mask[b]) ? v : mean + (v - mean) * f1);
    }
  }
  free(s);
  free(ss);
  free(nz);
}

/* noise.py:86-164: out = sqrt((x + n1)^2 + n2^2), n = mean + std * u with
 * u1, u2 ~ N(0,1) (injected), std per element (times std(x) over the element
 * when relative); fp32 arithmetic, one cast. */
void ora_rician(const void* x, void* out, int dtype, const float* u1, const float* u2,
                const float* noise_std, double mean, int relative, const uint8_t* mask, int64_t B,
                int64_t n_per_b, int nthreads) {
  const int64_t nb = B > 0 ? B : 1;
  double* s = (double*)malloc(sizeof(double) * nb);
  double* ss = (double*)malloc(sizeof(double) * nb);
  int64_t* nz = (int64_t*)malloc(sizeof(int64_t) * nb);
  if (relative) group_moments(x, dtype, B, n_per_b, s, ss, nz, nthreads);
  const float fm = (float)mean;
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < n_per_b; ++i) {
      const int64_t k = b * n_per_b + i;
      const float v = ld(x, dtype, k);
      if (mask && !mask[b]) {
        st(out, dtype, k, v);
        continue;
      }
      const float sd = relative ? noise_std[b] * std_of(s[b], ss[b], n_per_b) : noise_std[b];
      const float n1 = fm + sd * u1[k];
      const float n2 = fm + sd * u2[k];
      const float a = v + n1;
      st(out, dtype, k, sqrtf(a * a + n2 * n2));
    }
  free(s);
  free(ss);
  free(nz);
}

/* sharpen.py:117-136, after the two blurs: out = blurred + alpha * (blurred -
 * double_blurred), one op at a time in the tensor dtype (alpha cast to it
 * first); masked-out elements keep x.  bl and db hold the two blurs already
 * cast to the dtype. */
void ora_sharpen_combine(const void* bl, const void* db, const void* x, void* out, int dtype,
                         const float* alpha, const uint8_t* mask, int64_t B, int64_t n_per_b,
                         int nthreads) {
  set_threads(nthreads);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < n_per_b; ++i) {
      const int64_t k = b * n_per_b + i;
      if (mask && !mask[b]) {
        st(out, dtype, k, ld(x, dtype, k));
        continue;
      }
      const float a = rnd(dtype, alpha[b]);
      const float u = ld(bl, dtype, k);
      const float d = rnd(dtype, u - ld(db, dtype, k));
      const float t = rnd(dtype, a * d);
      st(out, dtype, k, u + t);
    }
}
