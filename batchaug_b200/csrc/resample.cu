// Fused 3-D resample: one kernel per Compose materialisation.
//
// Replaces batchaug/compose.py:71-110 (_materialize: monai_affine_to_theta,
// F.affine_grid, F.grid_sample on an fp32 copy, .to(dtype), torch.where) and
// the eager applies of RandAffine (affine.py:284-317), Rand3DElastic
// (elastic.py:101-125), RandZoom (zoom.py:90-121) and RandRotate90's
// non-square fallback (rotate90.py:100-112).
//
// Design (B200).  No grid tensor and no fp32 copy of the input reach HBM.
// A CTA covers a compact BD(D) x TY(W) x TZ(H) output brick of one element.
// Its prologue puts in shared memory everything that does not vary per voxel:
// the element's theta (derived from the MONAI affine when given one) and, for
// the brick's D positions, affine_grid's base coordinate times theta's first
// column — so the hot loop has no divisions.  Each thread then produces
// output voxels in pairs, carrying both voxels of a pair through Blackwell's
// packed fp32x2 arithmetic where that cannot change rounding (fma chains,
// add-only and multiply-only steps; a packed multiply followed by a packed add
// is contracted by the compiler, so those stay scalar), and for every key and
// channel gathers the 8 trilinear taps
// (1 for nearest) through the read-only cache: one base pointer and constant
// tap deltas when the footprint is inside the volume, per-tap bounds checks
// only near its faces.  Mode, padding and dtype are compile-time in the hot
// path (a uniform switch per key).  Masked-out elements take a plain copy.
//
// Arithmetic reproduces torch's CPU affine_grid and grid_sample bit for bit:
// the base grid is torch.linspace's two-sided fused formula scaled by
// (N-1)/N, the bmm with theta is the fused chain MKL produces, and the
// unnormalise / clip / reflect / trilinear steps round exactly where torch's
// scalar code rounds (this file is compiled with -fmad=false; fused or packed
// operations appear only where written explicitly).
#include <stdio.h>

#include "ba_common.cuh"

namespace ba {
namespace {

#ifndef BA_RS_TX
#define BA_RS_TX 8
#endif
#ifndef BA_RS_TY
#define BA_RS_TY 2
#endif
#ifndef BA_RS_TZ
#define BA_RS_TZ 8
#endif
#ifndef BA_RS_PAIRS
#define BA_RS_PAIRS 2
#endif
#ifndef BA_RS_NB
#define BA_RS_NB 4
#endif
#ifndef BA_RS_MINBLOCKS
#define BA_RS_MINBLOCKS 5
#endif

constexpr int TX = BA_RS_TX;         // threads along D
constexpr int TY = BA_RS_TY;         // threads along W
constexpr int TZ = BA_RS_TZ;         // threads along H
constexpr int PAIRS = BA_RS_PAIRS;   // voxel pairs per thread and brick, along D
constexpr int NB = BA_RS_NB;         // bricks per CTA, stacked along H
constexpr int BD = TX * 2 * PAIRS;   // brick extent along D
constexpr int NTHREADS = TX * TY * TZ;
static_assert(NTHREADS % 32 == 0, "whole warps");

struct KeyArgs {
  const void* src;
  void* dst;
  int32_t channels;
  int32_t dtype;
  int32_t mode;
  int32_t padding;
};

struct ResampleArgs {
  int64_t batch;
  int32_t H, W, D;
  int32_t xform_kind;
  int32_t align_corners;
  int32_t n_keys;
  const float* xform;
  int64_t xform_stride;
  const uint8_t* mask;
  float sn[3];  // fl32(2/H), fl32(2/W), fl32(2/D)
  float si[3];  // H/2, W/2, D/2
  KeyArgs keys[BA_MAX_KEYS];
};

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100), two voxels per instruction.  A packed
// multiply whose result feeds a packed add can come out fused into one fma
// even under -fmad=false, so packed multiplies are used only where no add
// follows (the weight products); multiply-then-add steps (unnormalise, the
// tap accumulation) are scalar __fmul_rn / __fadd_rn, which are never fused.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return __fadd2_rn(a, f2(-b.x, -b.y)); }
__device__ __forceinline__ float2 add2_down(float2 a, float2 b) { return __fadd2_rd(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }

// affine_grid's linspace_from_neg_one.
__device__ __forceinline__ float base_coord(int i, int n, int align_corners) {
  if (n <= 1) return 0.0f;
  const float step = 2.0f / (float)(n - 1);
  float r = linspace_at(-1.0f, 1.0f, step, i, n);
  if (!align_corners) r = (r * (float)(n - 1)) / (float)n;
  return r;
}

// grid_sampler_unnormalize for two voxels: align_corners ? ((c+1)/2)*(size-1)
// : ((c+1)*size-1)/2, where /2 is the exact *0.5.
template <bool ALIGN>
__device__ __forceinline__ float2 unnormalize2(float2 c, float size) {
  if (ALIGN) return mul2(mul2(add2(c, f2(1.0f)), f2(0.5f)), f2(size - 1.0f));
  return f2(__fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(c.x, 1.0f), size), 1.0f), 0.5f),
            __fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(c.y, 1.0f), size), 1.0f), 0.5f));
}

// std::min(size-1, std::max(in, 0)) with std's argument order: max keeps a
// NaN (max.NaN), then min turns it into size-1, as torch's clip does.
__device__ __forceinline__ float clip_coord(float in, float hi) {
  float lo;
  asm("max.NaN.f32 %0, %1, 0f00000000;" : "=f"(lo) : "f"(in));
  return fminf(lo, hi);
}

__device__ __forceinline__ float reflect_coord(float in, int twice_low, int twice_high) {
  if (twice_low == twice_high) return 0.0f;
  const float mn = (float)twice_low * 0.5f;
  const float span = (float)(twice_high - twice_low) * 0.5f;
  in = fabsf(in - mn);
  const float extra = fmodf(in, span);
  const int flips = (int)floorf(in / span);
  if ((flips & 1) == 0) return extra + mn;
  return span - extra + mn;
}

// Magnitude below which floor() is taken by rounding-mode addition: any
// coordinate at or beyond it is outside every supported volume, so the zeros
// padding maps it to -100 (out of bounds) like torch's sampler maps
// non-finite coordinates.
constexpr float COORD_LIMIT = 4194304.0f;  // 2^22

template <int PAD, bool ALIGN>
__device__ __forceinline__ float pad_coord(float c, int size) {
  if (PAD == BA_PAD_BORDER) {
    return clip_coord(c, (float)(size - 1));  // in [0, size-1] or NaN->size-1
  } else if (PAD == BA_PAD_REFLECTION) {
    c = ALIGN ? reflect_coord(c, 0, 2 * (size - 1)) : reflect_coord(c, -1, 2 * size - 1);
    return clip_coord(c, (float)(size - 1));
  }
  return (fabsf(c) < COORD_LIMIT) ? c : -100.0f;
}

template <int PAD, bool ALIGN>
__device__ __forceinline__ float2 pad2(float2 c, int size) {
  return f2(pad_coord<PAD, ALIGN>(c.x, size), pad_coord<PAD, ALIGN>(c.y, size));
}

// floor of two coordinates with |c| < 2^22: c + 1.5*2^23 rounded toward -inf
// is floor(c) + 1.5*2^23, an integer whose float bits hold floor(c).
struct Floor2 {
  float2 f;   // floor as floats
  int lo, hi; // floor as ints
};
__device__ __forceinline__ Floor2 floor2(float2 c) {
  constexpr float M = 12582912.0f;  // 1.5 * 2^23
  const float2 t = add2_down(c, f2(M));
  Floor2 r;
  r.f = sub2(t, f2(M));
  r.lo = __float_as_int(t.x) - 0x4B400000;
  r.hi = __float_as_int(t.y) - 0x4B400000;
  return r;
}

template <int DT>
__device__ __forceinline__ float ld(const void* base, int64_t i) {
  if (DT == BA_BF16) return bf16_bits_to_f32(__ldg((const uint16_t*)base + i));
  return __ldg((const float*)base + i);
}

template <int DT>
__device__ __forceinline__ void st(void* base, int64_t i, float v) {
  if (DT == BA_BF16)
    ((uint16_t*)base)[i] = f32_to_bf16_bits(v);
  else
    ((float*)base)[i] = v;
}

// The 8 tap values of one voxel with corner (x0, y0, z0), 0 for taps outside
// the volume, in torch's order tnw, tne, tsw, tse, bnw, bne, bsw, bse.
template <int DT>
__device__ __forceinline__ void taps8(const void* cbase, int x0, int y0, int z0, int H, int W,
                                      int D, bool interior, float* v) {
  const int dy = D, dz = W * D;
  if (interior) {
    const int o = (z0 * W + y0) * D + x0;
    v[0] = ld<DT>(cbase, o);
    v[1] = ld<DT>(cbase, o + 1);
    v[2] = ld<DT>(cbase, o + dy);
    v[3] = ld<DT>(cbase, o + dy + 1);
    v[4] = ld<DT>(cbase, o + dz);
    v[5] = ld<DT>(cbase, o + dz + 1);
    v[6] = ld<DT>(cbase, o + dz + dy);
    v[7] = ld<DT>(cbase, o + dz + dy + 1);
    return;
  }
  const bool vx0 = (unsigned)x0 < (unsigned)D, vx1 = (unsigned)(x0 + 1) < (unsigned)D;
  const bool vy0 = (unsigned)y0 < (unsigned)W, vy1 = (unsigned)(y0 + 1) < (unsigned)W;
  const bool vz0 = (unsigned)z0 < (unsigned)H, vz1 = (unsigned)(z0 + 1) < (unsigned)H;
  // unsigned arithmetic: offsets of out-of-bounds taps are never used
  const uint32_t o = ((uint32_t)z0 * (uint32_t)W + (uint32_t)y0) * (uint32_t)D + (uint32_t)x0;
  v[0] = (vz0 && vy0 && vx0) ? ld<DT>(cbase, o) : 0.0f;
  v[1] = (vz0 && vy0 && vx1) ? ld<DT>(cbase, o + 1u) : 0.0f;
  v[2] = (vz0 && vy1 && vx0) ? ld<DT>(cbase, o + dy) : 0.0f;
  v[3] = (vz0 && vy1 && vx1) ? ld<DT>(cbase, o + dy + 1u) : 0.0f;
  v[4] = (vz1 && vy0 && vx0) ? ld<DT>(cbase, o + dz) : 0.0f;
  v[5] = (vz1 && vy0 && vx1) ? ld<DT>(cbase, o + dz + 1u) : 0.0f;
  v[6] = (vz1 && vy1 && vx0) ? ld<DT>(cbase, o + dz + dy) : 0.0f;
  v[7] = (vz1 && vy1 && vx1) ? ld<DT>(cbase, o + dz + dy + 1u) : 0.0f;
}

// All channels of one key at a pair of output voxels (flat spatial indices
// sa, sb; sb is skipped when !has_b).  ix/iy/iz are the unnormalised source
// coordinates of the two voxels.
template <int MODE, int PAD, int DT, bool ALIGN>
__device__ __forceinline__ void sample_pair(const KeyArgs& k, int64_t b, int H, int W, int D,
                                            int hwd, float2 ix, float2 iy, float2 iz, int sa,
                                            int sb, bool has_b) {
  const float2 px = pad2<PAD, ALIGN>(ix, D);
  const float2 py = pad2<PAD, ALIGN>(iy, W);
  const float2 pz = pad2<PAD, ALIGN>(iz, H);
  const size_t esz = DT == BA_BF16 ? 2 : 4;
  const char* src_e = (const char*)k.src + (size_t)b * k.channels * hwd * esz;
  char* dst_e = (char*)k.dst + (size_t)b * k.channels * hwd * esz;
  if (MODE == BA_NEAREST) {
    // nearbyint (round half to even) in one conversion
    const int xa = __float2int_rn(px.x), ya = __float2int_rn(py.x), za = __float2int_rn(pz.x);
    const int xb = __float2int_rn(px.y), yb = __float2int_rn(py.y), zb = __float2int_rn(pz.y);
    const bool oka =
        (unsigned)xa < (unsigned)D && (unsigned)ya < (unsigned)W && (unsigned)za < (unsigned)H;
    const bool okb = has_b && (unsigned)xb < (unsigned)D && (unsigned)yb < (unsigned)W &&
                     (unsigned)zb < (unsigned)H;
    const int oa = oka ? (za * W + ya) * D + xa : 0;
    const int ob = okb ? (zb * W + yb) * D + xb : 0;
    for (int c = 0; c < k.channels; ++c) {
      const void* cs = src_e + (size_t)c * hwd * esz;
      void* cd = dst_e + (size_t)c * hwd * esz;
      const float va = oka ? ld<DT>(cs, oa) : 0.0f;
      const float vb = okb ? ld<DT>(cs, ob) : 0.0f;
      st<DT>(cd, sa, va);
      if (has_b) st<DT>(cd, sb, vb);
    }
    return;
  }
  // Trilinear: corner and the distances torch forms as (corner + 1 - coord)
  // and (coord - corner), then the weights as (x * y) * z products.
  const Floor2 fx = floor2(px), fy = floor2(py), fz = floor2(pz);
  const float2 one = f2(1.0f);
  const float2 wx1 = sub2(px, fx.f), wx0 = sub2(add2(fx.f, one), px);
  const float2 wy1 = sub2(py, fy.f), wy0 = sub2(add2(fy.f, one), py);
  const float2 wz1 = sub2(pz, fz.f), wz0 = sub2(add2(fz.f, one), pz);
  const float2 xy00 = mul2(wx0, wy0), xy10 = mul2(wx1, wy0);
  const float2 xy01 = mul2(wx0, wy1), xy11 = mul2(wx1, wy1);
  float2 w[8];
  w[0] = mul2(xy00, wz0);
  w[1] = mul2(xy10, wz0);
  w[2] = mul2(xy01, wz0);
  w[3] = mul2(xy11, wz0);
  w[4] = mul2(xy00, wz1);
  w[5] = mul2(xy10, wz1);
  w[6] = mul2(xy01, wz1);
  w[7] = mul2(xy11, wz1);
  const bool ia = (unsigned)fx.lo < (unsigned)(D - 1) && (unsigned)fy.lo < (unsigned)(W - 1) &&
                  (unsigned)fz.lo < (unsigned)(H - 1);
  const bool ib = (unsigned)fx.hi < (unsigned)(D - 1) && (unsigned)fy.hi < (unsigned)(W - 1) &&
                  (unsigned)fz.hi < (unsigned)(H - 1);
  // voxel b of a pair past the volume's end reuses voxel a's corner
  const int xb = has_b ? fx.hi : fx.lo, yb = has_b ? fy.hi : fy.lo, zb = has_b ? fz.hi : fz.lo;
  for (int c = 0; c < k.channels; ++c) {
    const void* cs = src_e + (size_t)c * hwd * esz;
    void* cd = dst_e + (size_t)c * hwd * esz;
    float va[8], vb[8];
    taps8<DT>(cs, fx.lo, fy.lo, fz.lo, H, W, D, ia, va);
    taps8<DT>(cs, xb, yb, zb, H, W, D, has_b ? ib : ia, vb);
    // out += v * w in torch's tap order
    float2 acc = f2(0.0f);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      acc.x = __fadd_rn(acc.x, __fmul_rn(va[t], w[t].x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(vb[t], w[t].y));
    }
    st<DT>(cd, sa, acc.x);
    if (has_b) st<DT>(cd, sb, acc.y);
  }
}

// A key's sampling spec as one compile-time code: (mode*3 + padding)*2 + dtype.
__host__ __device__ constexpr int spec_code(int mode, int pad, int dt) { return (mode * 3 + pad) * 2 + dt; }
__host__ __device__ constexpr int spec_mode(int s) { return s / 6; }
__host__ __device__ constexpr int spec_pad(int s) { return (s / 2) % 3; }
__host__ __device__ constexpr int spec_dt(int s) { return s % 2; }

template <int S, bool ALIGN>
__device__ __forceinline__ void sample_spec(const KeyArgs& k, int64_t b, int H, int W, int D,
                                            int hwd, float2 ix, float2 iy, float2 iz, int sa,
                                            int sb, bool has_b) {
  sample_pair<spec_mode(S), spec_pad(S), spec_dt(S), ALIGN>(k, b, H, W, D, hwd, ix, iy, iz, sa,
                                                             sb, has_b);
}

// The kernel samples key 0 with spec S0 and, when S1 >= 0, key 1 with spec
// S1 from the same coordinates; other key combinations are launched one key
// at a time.  CTA (x, y, z) covers NB bricks of BD(D) x TY(W) x TZ(H) output
// voxels of element z, stacked along H; the prologue (theta, base
// coordinates) is shared by the bricks.  A warp's 32 threads cover a
// TX x TY x (32 / (TX*TY)) block of voxels, which keeps the source rows one
// gather request touches few for rotated maps.
template <int S0, int S1>
__global__ void __launch_bounds__(NTHREADS, BA_RS_MINBLOCKS)
    resample3d_kernel(const __grid_constant__ ResampleArgs a) {
  const bool ALIGN = a.align_corners != 0;
  const int H = a.H, W = a.W, D = a.D;
  const int tiles_d = (D + BD - 1) / BD;
  const int tx = threadIdx.x % TX;
  const int ty = (threadIdx.x / TX) % TY;
  const int tz = threadIdx.x / (TX * TY);
  const int d_brick = (blockIdx.x % tiles_d) * BD;
  const int w_brick = (blockIdx.x / tiles_d) * TY;
  const int h_first = blockIdx.y * (TZ * NB);
  const int w = w_brick + ty;
  const int64_t b = blockIdx.z;
  const int hwd = H * W * D;
  const bool active = (a.mask == nullptr) || (a.mask[b] != 0);
  const bool affine = a.xform_kind != BA_XFORM_GRID;

  // Prologue: theta, then the base coordinates of the CTA's rows and
  // bx * theta[r][0] for the brick's D positions.
  __shared__ float s_theta[12];
  __shared__ float s_by[TY], s_bz[TZ * NB];
  __shared__ float2 s_px[3][PAIRS][TX];
  if (active && affine) {
    const int t = threadIdx.x;
    if (t < 12) {
      const int i = t / 4, j = t % 4;
      const float* x = a.xform + b * a.xform_stride;
      if (a.xform_kind == BA_XFORM_AFFINE) {
        // monai_affine_to_theta: theta = P S_norm A S_inv P, P swapping 0 and 2.
        const int pi = 2 - i, pj = (j == 3) ? 3 : 2 - j;
        const float s_j = (pj == 3) ? 1.0f : a.si[pj];
        s_theta[t] = (a.sn[pi] * x[pi * 4 + pj]) * s_j;
      } else {
        s_theta[t] = x[i * 4 + j];
      }
    }
    for (int q = t; q < TY + TZ * NB; q += NTHREADS) {
      if (q < TY)
        s_by[q] = base_coord(w_brick + q, W, ALIGN);
      else
        s_bz[q - TY] = base_coord(h_first + q - TY, H, ALIGN);
    }
    __syncthreads();
    if (t < BD) {
      // voxel j = 2p + q of lane x sits at d = d_brick + j*TX + x
      const int j = t / TX, x = t % TX;
      const int d = d_brick + t;  // t = j*TX + x
      const float bx = d < D ? base_coord(d, D, ALIGN) : 0.0f;
      const int p = j / 2, q = j % 2;
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        const float v = bx * s_theta[r * 4];
        float* slot = reinterpret_cast<float*>(&s_px[r][p][x]);
        slot[q] = v;
      }
    }
  }
  __syncthreads();
  if (w >= W) return;

  if (!active) {
    for (int nb = 0; nb < NB; ++nb) {
      const int h = h_first + nb * TZ + tz;
      if (h >= H) break;
      const int row = (h * W + w) * D;
      for (int j = 0; j < 2 * PAIRS; ++j) {
        const int d = d_brick + j * TX + tx;
        if (d >= D) break;
        for (int ki = 0; ki < a.n_keys; ++ki) {
          const KeyArgs& k = a.keys[ki];
          for (int c = 0; c < k.channels; ++c) {
            const int64_t i = (b * k.channels + c) * (int64_t)hwd + row + d;
            if (k.dtype == BA_BF16)
              ((uint16_t*)k.dst)[i] = __ldg((const uint16_t*)k.src + i);
            else
              ((float*)k.dst)[i] = __ldg((const float*)k.src + i);
          }
        }
      }
    }
    return;
  }

  float2 t1[3], t2[3], t3[3];
  float by = 0.0f;
  if (affine) {
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      t1[r] = f2(s_theta[r * 4 + 1]);
      t2[r] = f2(s_theta[r * 4 + 2]);
      t3[r] = f2(s_theta[r * 4 + 3]);
    }
    by = s_by[ty];
  }
  const float2 by2 = f2(by);
  const float fD = (float)D, fW = (float)W, fH = (float)H;
  for (int nb = 0; nb < NB; ++nb) {
    const int h = h_first + nb * TZ + tz;
    if (h >= H) break;
    const int row = (h * W + w) * D;
    const float2 bz2 = f2(affine ? s_bz[nb * TZ + tz] : 0.0f);
#pragma unroll
    for (int p = 0; p < PAIRS; ++p) {
      const int da = d_brick + (2 * p) * TX + tx, db = da + TX;
      if (da >= D) break;
      const bool has_b = db < D;
      float2 g[3];
      if (affine) {
        // affine_grid's bmm as MKL accumulates it: x*t0, then the fused y
        // and z terms, then the translation.
#pragma unroll
        for (int r = 0; r < 3; ++r)
          g[r] = add2(__ffma2_rn(bz2, t2[r], __ffma2_rn(by2, t1[r], s_px[r][p][tx])), t3[r]);
      } else {
        const float* ga = a.xform + (b * hwd + row + da) * 3;
        const float* gb = has_b ? ga + 3 * TX : ga;
#pragma unroll
        for (int r = 0; r < 3; ++r) g[r] = f2(__ldg(ga + r), __ldg(gb + r));
      }
      if (ALIGN) {
        const float2 ix = unnormalize2<true>(g[0], fD);
        const float2 iy = unnormalize2<true>(g[1], fW);
        const float2 iz = unnormalize2<true>(g[2], fH);
        sample_spec<S0, true>(a.keys[0], b, H, W, D, hwd, ix, iy, iz, row + da, row + db, has_b);
        if (S1 >= 0)
          sample_spec<(S1 < 0 ? 0 : S1), true>(a.keys[1], b, H, W, D, hwd, ix, iy, iz, row + da,
                                               row + db, has_b);
      } else {
        const float2 ix = unnormalize2<false>(g[0], fD);
        const float2 iy = unnormalize2<false>(g[1], fW);
        const float2 iz = unnormalize2<false>(g[2], fH);
        sample_spec<S0, false>(a.keys[0], b, H, W, D, hwd, ix, iy, iz, row + da, row + db, has_b);
        if (S1 >= 0)
          sample_spec<(S1 < 0 ? 0 : S1), false>(a.keys[1], b, H, W, D, hwd, ix, iy, iz, row + da,
                                                row + db, has_b);
      }
    }
  }
}

bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
  const char* pa = (const char*)a;
  const char* pb = (const char*)b;
  return pa < pb + nb && pb < pa + na;
}

}  // namespace
}  // namespace ba

extern "C" ba_status ba_resample3d(const ba_resample_desc* desc, ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(desc != nullptr, "ba_resample3d: desc is NULL");
  const ba_resample_desc& d = *desc;
  BA_REQUIRE(d.batch >= 0 && d.H > 0 && d.W > 0 && d.D > 0,
             "ba_resample3d: bad shape B=%lld H=%lld W=%lld D=%lld", (long long)d.batch,
             (long long)d.H, (long long)d.W, (long long)d.D);
  BA_REQUIRE(d.H * d.W * d.D < (int64_t)INT32_MAX / 2,
             "ba_resample3d: spatial size H*W*D=%lld exceeds the 2^30 limit",
             (long long)(d.H * d.W * d.D));
  BA_REQUIRE(d.batch <= 65535, "ba_resample3d: batch %lld exceeds 65535", (long long)d.batch);
  BA_REQUIRE(d.n_keys >= 1 && d.n_keys <= BA_MAX_KEYS, "ba_resample3d: n_keys=%d not in 1..%d",
             d.n_keys, BA_MAX_KEYS);
  BA_REQUIRE(d.xform_kind >= BA_XFORM_AFFINE && d.xform_kind <= BA_XFORM_GRID,
             "ba_resample3d: unknown xform_kind %d", d.xform_kind);
  BA_REQUIRE(d.xform != nullptr || d.batch == 0, "ba_resample3d: xform is NULL");
  if (d.xform_kind != BA_XFORM_GRID)
    BA_REQUIRE(d.xform_stride >= 12, "ba_resample3d: xform_stride %lld < 12",
               (long long)d.xform_stride);
  if (d.xform_kind == BA_XFORM_AFFINE)
    BA_REQUIRE(d.xform_stride >= 16, "ba_resample3d: AFFINE xform_stride %lld < 16",
               (long long)d.xform_stride);

  ResampleArgs a;
  memset(&a, 0, sizeof(a));
  a.batch = d.batch;
  a.H = (int32_t)d.H;
  a.W = (int32_t)d.W;
  a.D = (int32_t)d.D;
  a.xform_kind = d.xform_kind;
  a.align_corners = d.align_corners ? 1 : 0;
  a.n_keys = d.n_keys;
  a.xform = d.xform;
  a.xform_stride = d.xform_stride;
  a.mask = d.mask;
  a.sn[0] = (float)(2.0 / (double)d.H);
  a.sn[1] = (float)(2.0 / (double)d.W);
  a.sn[2] = (float)(2.0 / (double)d.D);
  a.si[0] = (float)((double)d.H / 2.0);
  a.si[1] = (float)((double)d.W / 2.0);
  a.si[2] = (float)((double)d.D / 2.0);

  const int64_t hwd = d.H * d.W * d.D;
  for (int i = 0; i < d.n_keys; ++i) {
    const ba_resample_key& k = d.keys[i];
    BA_REQUIRE(k.dtype == BA_F32 || k.dtype == BA_BF16, "ba_resample3d: key %d bad dtype %d", i,
               k.dtype);
    BA_REQUIRE(k.mode == BA_BILINEAR || k.mode == BA_NEAREST, "ba_resample3d: key %d bad mode %d",
               i, k.mode);
    BA_REQUIRE(k.padding >= BA_PAD_ZEROS && k.padding <= BA_PAD_REFLECTION,
               "ba_resample3d: key %d bad padding %d", i, k.padding);
    BA_REQUIRE(k.channels >= 0 && k.channels <= 65535, "ba_resample3d: key %d bad channels %lld",
               i, (long long)k.channels);
    const size_t esz = k.dtype == BA_BF16 ? 2 : 4;
    const size_t bytes = (size_t)(d.batch * k.channels * hwd) * esz;
    if (bytes == 0) continue;
    BA_REQUIRE(k.src != nullptr && k.dst != nullptr, "ba_resample3d: key %d has a NULL pointer", i);
    BA_REQUIRE(((uintptr_t)k.src % esz) == 0 && ((uintptr_t)k.dst % esz) == 0,
               "ba_resample3d: key %d pointers not aligned to the element size", i);
    BA_REQUIRE(!overlaps(k.src, bytes, k.dst, bytes),
               "ba_resample3d: key %d dst overlaps src (the resample is out of place)", i);
    a.keys[i].src = k.src;
    a.keys[i].dst = k.dst;
    a.keys[i].channels = (int32_t)k.channels;
    a.keys[i].dtype = k.dtype;
    a.keys[i].mode = k.mode;
    a.keys[i].padding = k.padding;
  }
  if (d.batch == 0) return BA_OK;

  const int tiles_d = (int)((d.D + BD - 1) / BD);
  const int64_t gx = (int64_t)tiles_d * ((d.W + TY - 1) / TY);
  const int64_t gy = (d.H + TZ * NB - 1) / (TZ * NB);
  BA_REQUIRE(gx <= INT32_MAX && gy <= 65535, "ba_resample3d: spatial extent too large");
  const dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)d.batch);
  const cudaStream_t st = (cudaStream_t)stream;
  auto code = [](const KeyArgs& k) { return spec_code(k.mode, k.padding, k.dtype); };
  // vol (bilinear) + seg (nearest) with one padding: one fused launch
  if (a.n_keys == 2) {
    KeyArgs k0 = a.keys[0], k1 = a.keys[1];
    if (k0.mode == BA_NEAREST && k1.mode == BA_BILINEAR) {
      a.keys[0] = k1;
      a.keys[1] = k0;
      k0 = a.keys[0];
      k1 = a.keys[1];
    }
    if (k0.mode == BA_BILINEAR && k1.mode == BA_NEAREST && k0.padding == k1.padding) {
      bool launched = true;
      switch (code(k0) * 16 + code(k1)) {
#define BA_PAIR(P, T0, T1)                                                                 \
  case spec_code(BA_BILINEAR, P, T0) * 16 + spec_code(BA_NEAREST, P, T1):                  \
    resample3d_kernel<spec_code(BA_BILINEAR, P, T0), spec_code(BA_NEAREST, P, T1)>         \
        <<<grid, NTHREADS, 0, st>>>(a);                                                    \
    break;
#define BA_PAIRS(P) BA_PAIR(P, 0, 0) BA_PAIR(P, 0, 1) BA_PAIR(P, 1, 0) BA_PAIR(P, 1, 1)
        BA_PAIRS(BA_PAD_ZEROS)
        BA_PAIRS(BA_PAD_BORDER)
        BA_PAIRS(BA_PAD_REFLECTION)
#undef BA_PAIRS
#undef BA_PAIR
        default:
          launched = false;
      }
      if (launched) return check_launch("ba_resample3d");
    }
  }
  // otherwise one launch per key, each with its own compile-time spec
  ResampleArgs one = a;
  one.n_keys = 1;
  for (int i = 0; i < a.n_keys; ++i) {
    one.keys[0] = a.keys[i];
    switch (code(one.keys[0])) {
#define BA_ONE(S)                                                      \
  case S:                                                              \
    resample3d_kernel<S, -1><<<grid, NTHREADS, 0, st>>>(one);          \
    break;
      BA_ONE(0) BA_ONE(1) BA_ONE(2) BA_ONE(3) BA_ONE(4) BA_ONE(5)
      BA_ONE(6) BA_ONE(7) BA_ONE(8) BA_ONE(9) BA_ONE(10) BA_ONE(11)
#undef BA_ONE
      default:
        break;
    }
    const ba_status s1 = check_launch("ba_resample3d");
    if (s1 != BA_OK) return s1;
  }
  return BA_OK;
}
