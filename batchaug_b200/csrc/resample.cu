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
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>

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
  int32_t* minmax;  // (B, channels, 2) min/max keys the fast kernel folds (or NULL)
};

// Elements per launch whose transform and mask ride in the kernel's
// parameters (BA_RESAMPLE_HOST_PARAMS): 16 floats and a mask byte each.
constexpr int RS_INLINE_B = 32;

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
  // elements b0 .. b0 + gridDim.z - 1 (the launch's blocks z, or y for the
  // grid kernel); with inline_params the affine / theta and mask of element
  // b are inl_xform[(b - b0) * xform_stride ..] and inl_mask[b - b0]
  int64_t b0;
  int32_t inline_params;
  float inl_xform[RS_INLINE_B * 16];
  uint8_t inl_mask[RS_INLINE_B];
};

__device__ __forceinline__ bool elem_active(const ResampleArgs& a, int64_t b) {
  if (a.inline_params) return a.inl_mask[b - a.b0] != 0;
  return a.mask == nullptr || a.mask[b] != 0;
}

// the element's affine / theta rows (AFFINE and THETA maps)
__device__ __forceinline__ const float* elem_xform(const ResampleArgs& a, int64_t b) {
  return a.inline_params ? a.inl_xform + (b - a.b0) * a.xform_stride : a.xform + b * a.xform_stride;
}

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100), two voxels per instruction.  A packed
// multiply whose result feeds a packed add can come out fused into one fma
// even under -fmad=false, so no packed multiply feeds a packed add where the
// fusion could change a result: the tap products are packed but summed with
// scalar __fadd_rn, and unnormalise is packed only for power-of-two sizes
// (where the product is exact); elsewhere it is scalar __fmul_rn / __fadd_rn.
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
// For a power-of-two size (c+1)*size is exact, so a fused multiply-subtract
// gives the same result: the packed form is safe.
__device__ __forceinline__ float2 unnormalize2_pow2(float2 c, float size) {
  return mul2(sub2(mul2(add2(c, f2(1.0f)), f2(size)), f2(1.0f)), f2(0.5f));
}

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
    // four channels' gathers in flight before their stores
    int c = 0;
    for (; c + 4 <= k.channels; c += 4) {
      float va[4], vb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const void* cs = src_e + (size_t)(c + j) * hwd * esz;
        va[j] = oka ? ld<DT>(cs, oa) : 0.0f;
        vb[j] = okb ? ld<DT>(cs, ob) : 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        void* cd = dst_e + (size_t)(c + j) * hwd * esz;
        st<DT>(cd, sa, va[j]);
        if (has_b) st<DT>(cd, sb, vb[j]);
      }
    }
    for (; c < k.channels; ++c) {
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
    // out += v * w in torch's tap order: products packed, sums scalar (a
    // packed product feeding a scalar add is never fused)
    float2 acc = f2(0.0f);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float2 pr = mul2(f2(va[t], vb[t]), w[t]);
      acc.x = __fadd_rn(acc.x, pr.x);
      acc.y = __fadd_rn(acc.y, pr.y);
    }
    st<DT>(cd, sa, acc.x);
    if (has_b) st<DT>(cd, sb, acc.y);
  }
}

// A nearest key's first (up to) four channels at a pair of output voxels,
// split into the gathers (nearest_begin) and the stores (nearest_end) so a
// kernel can issue the gathers, do other work while they are in flight, and
// store afterwards; channels past the fourth are gathered and stored in
// nearest_begin.  Coordinates, rounding and bounds are sample_pair's.
struct NearestPair {
  float va[4], vb[4];
};

template <int PAD, int DT, bool ALIGN>
__device__ __forceinline__ void nearest_begin(const KeyArgs& k, int64_t b, int H, int W, int D,
                                              int hwd, float2 ix, float2 iy, float2 iz, int sa,
                                              int sb, bool has_b, NearestPair& q) {
  const float2 px = pad2<PAD, ALIGN>(ix, D);
  const float2 py = pad2<PAD, ALIGN>(iy, W);
  const float2 pz = pad2<PAD, ALIGN>(iz, H);
  const size_t esz = DT == BA_BF16 ? 2 : 4;
  const char* src_e = (const char*)k.src + (size_t)b * k.channels * hwd * esz;
  const int xa = __float2int_rn(px.x), ya = __float2int_rn(py.x), za = __float2int_rn(pz.x);
  const int xb = __float2int_rn(px.y), yb = __float2int_rn(py.y), zb = __float2int_rn(pz.y);
  const bool oka =
      (unsigned)xa < (unsigned)D && (unsigned)ya < (unsigned)W && (unsigned)za < (unsigned)H;
  const bool okb = has_b && (unsigned)xb < (unsigned)D && (unsigned)yb < (unsigned)W &&
                   (unsigned)zb < (unsigned)H;
  const int oa = oka ? (za * W + ya) * D + xa : 0;
  const int ob = okb ? (zb * W + yb) * D + xb : 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const void* cs = src_e + (size_t)j * hwd * esz;
    q.va[j] = (j < k.channels && oka) ? ld<DT>(cs, oa) : 0.0f;
    q.vb[j] = (j < k.channels && okb) ? ld<DT>(cs, ob) : 0.0f;
  }
  char* dst_e = (char*)k.dst + (size_t)b * k.channels * hwd * esz;
  for (int c = 4; c < k.channels; ++c) {
    const void* cs = src_e + (size_t)c * hwd * esz;
    void* cd = dst_e + (size_t)c * hwd * esz;
    const float va = oka ? ld<DT>(cs, oa) : 0.0f;
    const float vb = okb ? ld<DT>(cs, ob) : 0.0f;
    st<DT>(cd, sa, va);
    if (has_b) st<DT>(cd, sb, vb);
  }
}

template <int DT>
__device__ __forceinline__ void nearest_end(const KeyArgs& k, int64_t b, int hwd, int sa, int sb,
                                            bool has_b, const NearestPair& q) {
  const size_t esz = DT == BA_BF16 ? 2 : 4;
  char* dst_e = (char*)k.dst + (size_t)b * k.channels * hwd * esz;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j >= k.channels) break;
    void* cd = dst_e + (size_t)j * hwd * esz;
    st<DT>(cd, sa, q.va[j]);
    if (has_b) st<DT>(cd, sb, q.vb[j]);
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
  const int64_t b = a.b0 + blockIdx.z;
  const int hwd = H * W * D;
  const bool active = elem_active(a, b);
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
      const float* x = elem_xform(a, b);
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
  const bool pD = (D & (D - 1)) == 0, pW = (W & (W - 1)) == 0, pH = (H & (H - 1)) == 0;
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
        const float2 ix = pD ? unnormalize2_pow2(g[0], fD) : unnormalize2<false>(g[0], fD);
        const float2 iy = pW ? unnormalize2_pow2(g[1], fW) : unnormalize2<false>(g[1], fW);
        const float2 iz = pH ? unnormalize2_pow2(g[2], fH) : unnormalize2<false>(g[2], fH);
        sample_spec<S0, false>(a.keys[0], b, H, W, D, hwd, ix, iy, iz, row + da, row + db, has_b);
        if (S1 >= 0)
          sample_spec<(S1 < 0 ? 0 : S1), false>(a.keys[1], b, H, W, D, hwd, ix, iy, iz, row + da,
                                                row + db, has_b);
      }
    }
  }
}

// ===========================================================================
// Staged resample: the source footprint of each output tile in shared memory.
//
// For affine maps (bilinear key, zeros or border padding) a CTA covers a
// 16(D) x 16(W) x 8(H) output tile.  Its prologue maps the tile's 8 corners
// to source voxels and takes their bounding box (the corner coordinates bound
// all others up to rounding, far below the 0.01-voxel slack used), and, when
// the box fits ST_MAX_FLOATS floats, copies it into shared memory with 16-byte
// cp.async copies (zero-filled outside the volume, which is exactly the value
// an out-of-bounds tap contributes).  The 8 taps of each voxel are then read
// from shared memory; a voxel whose footprint leaves the box (or a CTA whose
// box does not fit) gathers from global memory as resample3d_kernel does.
// Arithmetic is the same operation for operation, so results are identical.
// A second, nearest-mode key (the label map of a dict transform) is sampled
// from global memory with the same coordinates.
// ===========================================================================
#ifndef BA_ST_TW
#define BA_ST_TW 16
#endif
#ifndef BA_ST_TH
#define BA_ST_TH 8
#endif
#ifndef BA_ST_MAX_FLOATS
#define BA_ST_MAX_FLOATS 11264
#endif
#ifndef BA_ST_MINBLOCKS
#define BA_ST_MINBLOCKS 4
#endif
constexpr int ST_TD = 16, ST_TW = BA_ST_TW, ST_TH = BA_ST_TH;
constexpr int ST_THREADS = 128;
// 44 KB of staged source: five CTAs (with their static shared memory and the
// per-CTA reserve) fit in an SM's 228 KB; at 46-48 KB only four do
constexpr int ST_MAX_FLOATS = BA_ST_MAX_FLOATS;
#ifndef BA_FS_MAX_FLOATS
#define BA_FS_MAX_FLOATS 11264
#endif
// the largest box of one channel the fast kernel stages; a tile with a
// larger box gathers its taps from global memory.  Measured on B200: 8192,
// 6144 and 4096 floats are slower than 11264 on both a single-channel
// affine (more tiles gather) and a four-channel one, and so is a 14208-float
// limit with the shared memory a four-CTA instantiation leaves (staging
// 44-56 KB boxes costs more than gathering those tiles' taps)
#ifndef BA_FS_STAGE_FLOATS
#define BA_FS_STAGE_FLOATS BA_FS_MAX_FLOATS
#endif
static_assert(BA_FS_STAGE_FLOATS <= BA_FS_MAX_FLOATS, "a staged box must fit");
// the fast kernel re-checks its box with the padded pitches
constexpr int FS_MAX_SETUP_FLOATS = BA_FS_STAGE_FLOATS;
constexpr int ST_PW = ST_TW / 2, ST_PH = ST_TH / 8;
static_assert(ST_TW % 2 == 0 && ST_TH % 8 == 0, "tile covered by the thread layout");

template <int DT>
__device__ __forceinline__ float4 ld4(const void* base, int64_t i) {
  if (DT == BA_BF16) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>((const uint16_t*)base + i));
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
  }
  return __ldg(reinterpret_cast<const float4*>((const float*)base + i));
}


// Shared-memory state of a staged CTA: theta, the base coordinates of the
// tile's W and H positions, bx * theta[r][0] for its 16 D positions (packed
// as the thread layout pairs them), and the staged box.
struct StagedShared {
  float theta[12];
  float by[ST_TW], bz[ST_TH];
  float2 px[3][8];
  int lo[3], hi[3];
  int box[6];  // lx4, ly, lz, 16-byte chunks per row (0: not staged), ey, ez
};

// The reference's torch.where keeps a masked-out element: copy the tile, one
// 16-element D row per thread, 16-byte vectors where the row is whole and
// aligned.
__device__ __forceinline__ void staged_copy_masked(const ResampleArgs& a, int64_t b, int d0, int w0,
                                                   int h0, int hwd, int t) {
  static_assert(ST_TW * ST_TH == ST_THREADS, "one tile row per thread");
  const int H = a.H, W = a.W, D = a.D;
  const int w = w0 + t % ST_TW, h = h0 + t / ST_TW;
  if (w >= W || h >= H) return;
  const int n = min(ST_TD, D - d0);
  for (int ki = 0; ki < a.n_keys; ++ki) {
    const KeyArgs& kc = a.keys[ki];
    const int ke = kc.dtype == BA_BF16 ? 2 : 4;
    for (int c = 0; c < kc.channels; ++c) {
      const int64_t i0 = (b * kc.channels + c) * (int64_t)hwd + ((int64_t)h * W + w) * D + d0;
      const char* sp = (const char*)kc.src + i0 * ke;
      char* dp = (char*)kc.dst + i0 * ke;
      if (n == ST_TD && ((uintptr_t)sp % 16) == 0 && ((uintptr_t)dp % 16) == 0) {
        uint4 v[4];
        const int nv = ST_TD * ke / 16;  // 4 (fp32) or 2 (bf16)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q < nv) v[q] = __ldg(reinterpret_cast<const uint4*>(sp) + q);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q < nv) reinterpret_cast<uint4*>(dp)[q] = v[q];
      } else {
        for (int q = 0; q < n; ++q) {
          if (ke == 2)
            ((uint16_t*)dp)[q] = __ldg((const uint16_t*)sp + q);
          else
            ((float*)dp)[q] = __ldg((const float*)sp + q);
        }
      }
    }
  }
}

// Prologue of a staged CTA: theta, base coordinates, and the source box the
// tile's taps fall in.  The box is the corners' bounding box of the padded
// coordinates (every voxel's coordinate is within rounding, < 1e-3 voxel, of
// the affine image of its index, whose extremes are at the corners; the
// padding is monotone) with 0.01-voxel slack and one more voxel for the
// upper taps.  FAST pads as the fast kernel does (fast_pad: every tap of
// every voxel inside the box); otherwise as torch pads (voxels beyond
// [-1, size] fall outside the clipped box and gather from global memory).
template <int PAD>
__device__ __forceinline__ float fast_pad(float c, float size);

template <int PAD, bool FAST>
__device__ __forceinline__ void staged_setup(const ResampleArgs& a, int64_t b, int d0, int w0,
                                             int h0, bool ALIGN, int t, StagedShared& sh) {
  const int H = a.H, W = a.W, D = a.D;
  if (t < 12) {
    const int i = t / 4, j = t % 4;
    const float* x = elem_xform(a, b);
    if (a.xform_kind == BA_XFORM_AFFINE) {
      // monai_affine_to_theta: theta = P S_norm A S_inv P, P swapping 0 and 2.
      const int pi = 2 - i, pj = (j == 3) ? 3 : 2 - j;
      const float s_j = (pj == 3) ? 1.0f : a.si[pj];
      sh.theta[t] = (a.sn[pi] * x[pi * 4 + pj]) * s_j;
    } else {
      sh.theta[t] = x[i * 4 + j];
    }
  } else if (t >= 32 && t < 32 + ST_TW) {
    sh.by[t - 32] = base_coord(w0 + t - 32, W, ALIGN);
  } else if (t >= 64 && t < 64 + ST_TH) {
    sh.bz[t - 64] = base_coord(h0 + t - 64, H, ALIGN);
  } else if (t >= 96 && t < 99) {
    sh.lo[t - 96] = 0x7fffffff;
    sh.hi[t - 96] = -0x7fffffff;
  }
  __syncthreads();
  if (t < 16) {
    const int d = d0 + t;
    const float bx = d < D ? base_coord(d, D, ALIGN) : 0.0f;
    const int j = t & 7, q = t >> 3;
#pragma unroll
    for (int r = 0; r < 3; ++r) reinterpret_cast<float*>(&sh.px[r][j])[q] = bx * sh.theta[r * 4];
  } else if (t >= 32 && t < 40) {
    // bounding box of the tile's corners in source voxels
    const int c = t - 32;
    const int dc = (c & 1) ? min(d0 + ST_TD - 1, D - 1) : d0;
    const int wc = (c & 2) ? min(w0 + ST_TW - 1, W - 1) : w0;
    const int hc = (c & 4) ? min(h0 + ST_TH - 1, H - 1) : h0;
    const float bx = base_coord(dc, D, ALIGN), by = base_coord(wc, W, ALIGN),
                bz = base_coord(hc, H, ALIGN);
    const float sz[3] = {(float)D, (float)W, (float)H};
    const int isz[3] = {D, W, H};
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const float g = __fadd_rn(
          __fmaf_rn(bz, sh.theta[r * 4 + 2], __fmaf_rn(by, sh.theta[r * 4 + 1], bx * sh.theta[r * 4])),
          sh.theta[r * 4 + 3]);
      const float u = ALIGN ? __fmul_rn(__fmul_rn(__fadd_rn(g, 1.0f), 0.5f), sz[r] - 1.0f)
                            : __fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(g, 1.0f), sz[r]), 1.0f), 0.5f);
      const float p = FAST ? fast_pad<PAD>(u, sz[r])
                           : fminf(fmaxf(pad_coord<PAD, false>(u, isz[r]), -1.0e6f), 1.0e6f);
      atomicMin(&sh.lo[r], (int)floorf(p - 0.01f));
      atomicMax(&sh.hi[r], (int)floorf(p + 0.01f));
    }
  }
  __syncthreads();
  if (t == 0) {
    const int isz[3] = {D, W, H};
    int lo[3], hi[3];
    for (int r = 0; r < 3; ++r) {
      // FAST: the padded coordinates already lie in [-1, size]
      lo[r] = FAST ? sh.lo[r] : max(sh.lo[r], -1);
      hi[r] = FAST ? sh.hi[r] + 1 : min(sh.hi[r] + 1, isz[r]);  // + 1: the upper taps
    }
    const int lx4 = (lo[0] >= 0) ? (lo[0] & ~3) : -4;
    const int ex = ((hi[0] - lx4 + 1) + 3) & ~3;
    const int ey = hi[1] - lo[1] + 1, ez = hi[2] - lo[2] + 1;
    const bool ok = PAD != BA_PAD_REFLECTION && ex >= 4 && ey >= 2 && ez >= 2 &&
                    ex / 4 <= ST_THREADS &&
                    (int64_t)ex * ey * ez <= (FAST ? FS_MAX_SETUP_FLOATS : ST_MAX_FLOATS);
    sh.box[0] = lx4;
    sh.box[1] = lo[1];
    sh.box[2] = lo[2];
    sh.box[3] = ok ? ex / 4 : 0;
    sh.box[4] = ey;
    sh.box[5] = ez;
  }
  __syncthreads();
}

// Copy channel c's staged box into shared memory: 16-byte chunks, cp.async
// for fp32 (chunks outside the volume are zero-filled: source size 0),
// synchronous widening loads for bf16.  Ends with the block synchronised.
template <int DT>
__device__ __forceinline__ void stage_box(float4* s_dyn4, const char* src_c, int lx4, int ly,
                                          int lz, int nx4, int ey, int ez, int H, int W, int D,
                                          int t) {
  const int rows = ey * ez;
  const int rpp = ST_THREADS / nx4;  // rows per pass (nx4 <= ST_THREADS)
  const int lc = t % nx4;
  int row = t / nx4;
  int y = row % ey, z = row / ey;
  if (row < rpp) {
    for (; row < rows; row += rpp) {
      const int gy = ly + y, gz = lz + z, gx = lx4 + 4 * lc;
      const bool in = (unsigned)gy < (unsigned)W && (unsigned)gz < (unsigned)H && gx >= 0 && gx < D;
      const int64_t gi = in ? ((int64_t)gz * W + gy) * D + gx : 0;
      const unsigned sdst = (unsigned)__cvta_generic_to_shared(&s_dyn4[row * nx4 + lc]);
      if (DT == BA_F32) {
        const void* gsrc = (const float*)src_c + gi;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sdst), "l"(gsrc),
                     "r"(in ? 16 : 0) : "memory");
      } else {
        s_dyn4[row * nx4 + lc] = in ? ld4<DT>(src_c, gi) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      y += rpp;
      while (y >= ey) {
        y -= ey;
        ++z;
      }
    }
  }
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
}

template <int S0, int S1>
__global__ void __launch_bounds__(ST_THREADS, BA_ST_MINBLOCKS)
    resample3d_staged_kernel(const __grid_constant__ ResampleArgs a) {
  extern __shared__ float4 s_dyn4[];
  float* s_src = reinterpret_cast<float*>(s_dyn4);
  __shared__ StagedShared sh;
  constexpr int MODE = spec_mode(S0), PAD = spec_pad(S0), DT = spec_dt(S0);
  const bool ALIGN = a.align_corners != 0;
  const int H = a.H, W = a.W, D = a.D;
  const int tiles_d = (D + ST_TD - 1) / ST_TD;
  const int d0 = (blockIdx.x % tiles_d) * ST_TD;
  const int w0 = (blockIdx.x / tiles_d) * ST_TW;
  const int h0 = blockIdx.y * ST_TH;
  const int64_t b = a.b0 + blockIdx.z;
  const int hwd = H * W * D;
  const int t = threadIdx.x;
  const int tx = t & 7, ty = (t >> 3) & 1, tz = (t >> 4) & 1, wp = t >> 5;
  const KeyArgs& k = a.keys[0];
  const size_t esz = DT == BA_BF16 ? 2 : 4;
  if (!elem_active(a, b)) {
    staged_copy_masked(a, b, d0, w0, h0, hwd, t);
    return;
  }
  staged_setup<PAD, false>(a, b, d0, w0, h0, ALIGN, t, sh);
  const int lx4 = sh.box[0], ly = sh.box[1], lz = sh.box[2], nx4 = sh.box[3], ey = sh.box[4],
            ez = sh.box[5];
  const int ex = nx4 * 4;
  const bool staged = nx4 > 0;
  float2 t1[3], t2[3], t3[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    t1[r] = f2(sh.theta[r * 4 + 1]);
    t2[r] = f2(sh.theta[r * 4 + 2]);
    t3[r] = f2(sh.theta[r * 4 + 3]);
  }
  const float fD = (float)D, fW = (float)W, fH = (float)H;
  const bool pD = (D & (D - 1)) == 0, pW = (W & (W - 1)) == 0, pH = (H & (H - 1)) == 0;
  for (int c = 0; c < k.channels; ++c) {
    const char* src_c = (const char*)k.src + ((size_t)b * k.channels + c) * hwd * esz;
    char* dst_c = (char*)k.dst + ((size_t)b * k.channels + c) * hwd * esz;
    if (staged) stage_box<DT>(s_dyn4, src_c, lx4, ly, lz, nx4, ey, ez, H, W, D, t);
    for (int pp = 0; pp < ST_PW * ST_PH; ++pp) {
      const int pw = pp % ST_PW, ph = pp / ST_PW;
      const int h = h0 + tz + 2 * wp + 8 * ph;
      const float2 bz2 = f2(sh.bz[tz + 2 * wp + 8 * ph]);
      const int w = w0 + ty + 2 * pw;
      if (w >= W || h >= H) continue;
      const int da = d0 + tx, db = da + 8;
      if (da >= D) continue;
      const bool has_b = db < D;
      const float2 by2 = f2(sh.by[ty + 2 * pw]);
      float2 g[3];
#pragma unroll
      for (int r = 0; r < 3; ++r)
        g[r] = add2(__ffma2_rn(bz2, t2[r], __ffma2_rn(by2, t1[r], sh.px[r][tx])), t3[r]);
      float2 ix, iy, iz;
      if (ALIGN) {
        ix = unnormalize2<true>(g[0], fD);
        iy = unnormalize2<true>(g[1], fW);
        iz = unnormalize2<true>(g[2], fH);
      } else {
        ix = pD ? unnormalize2_pow2(g[0], fD) : unnormalize2<false>(g[0], fD);
        iy = pW ? unnormalize2_pow2(g[1], fW) : unnormalize2<false>(g[1], fW);
        iz = pH ? unnormalize2_pow2(g[2], fH) : unnormalize2<false>(g[2], fH);
      }
      const float2 px = ALIGN ? pad2<PAD, true>(ix, D) : pad2<PAD, false>(ix, D);
      const float2 py = ALIGN ? pad2<PAD, true>(iy, W) : pad2<PAD, false>(iy, W);
      const float2 pz = ALIGN ? pad2<PAD, true>(iz, H) : pad2<PAD, false>(iz, H);
      const int row = (h * W + w) * D;
      const Floor2 fx = floor2(px), fy = floor2(py), fz = floor2(pz);
      const float2 one = f2(1.0f);
      const float2 wx1 = sub2(px, fx.f), wx0 = sub2(add2(fx.f, one), px);
      const float2 wy1 = sub2(py, fy.f), wy0 = sub2(add2(fy.f, one), py);
      const float2 wz1 = sub2(pz, fz.f), wz0 = sub2(add2(fz.f, one), pz);
      const float2 xy00 = mul2(wx0, wy0), xy10 = mul2(wx1, wy0);
      const float2 xy01 = mul2(wx0, wy1), xy11 = mul2(wx1, wy1);
      float2 wt[8];
      wt[0] = mul2(xy00, wz0);
      wt[1] = mul2(xy10, wz0);
      wt[2] = mul2(xy01, wz0);
      wt[3] = mul2(xy11, wz0);
      wt[4] = mul2(xy00, wz1);
      wt[5] = mul2(xy10, wz1);
      wt[6] = mul2(xy01, wz1);
      wt[7] = mul2(xy11, wz1);
      float va[8], vb[8];
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int x0 = s ? (has_b ? fx.hi : fx.lo) : fx.lo;
        const int y0 = s ? (has_b ? fy.hi : fy.lo) : fy.lo;
        const int z0 = s ? (has_b ? fz.hi : fz.lo) : fz.lo;
        float* v = s ? vb : va;
        // all 8 taps inside the box: 0 <= x0 - lx4 and x0 + 1 - lx4 < ex, etc.
        const int ux = x0 - lx4, uy = y0 - ly, uz = z0 - lz;
        const bool inbox = staged && ux >= 0 && ux < ex - 1 && uy >= 0 && uy < ey - 1 &&
                           uz >= 0 && uz < ez - 1;
        if (inbox) {
          const int si = ((z0 - lz) * ey + (y0 - ly)) * ex + (x0 - lx4);
          const int pl = ey * ex;
          v[0] = s_src[si];
          v[1] = s_src[si + 1];
          v[2] = s_src[si + ex];
          v[3] = s_src[si + ex + 1];
          v[4] = s_src[si + pl];
          v[5] = s_src[si + pl + 1];
          v[6] = s_src[si + pl + ex];
          v[7] = s_src[si + pl + ex + 1];
        } else {
          const bool in_vol = (unsigned)x0 < (unsigned)(D - 1) && (unsigned)y0 < (unsigned)(W - 1) &&
                              (unsigned)z0 < (unsigned)(H - 1);
          taps8<DT>(src_c, x0, y0, z0, H, W, D, in_vol, v);
        }
      }
      if (S1 >= 0 && c == 0) {
        if (ALIGN)
          sample_spec<(S1 < 0 ? 0 : S1), true>(a.keys[1], b, H, W, D, hwd, ix, iy, iz, row + da,
                                               row + db, has_b);
        else
          sample_spec<(S1 < 0 ? 0 : S1), false>(a.keys[1], b, H, W, D, hwd, ix, iy, iz, row + da,
                                                row + db, has_b);
      }
      float2 acc = f2(0.0f);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        // products packed, sums scalar (never fused), in torch's tap order
        const float2 pr = mul2(f2(va[q], vb[q]), wt[q]);
        acc.x = __fadd_rn(acc.x, pr.x);
        acc.y = __fadd_rn(acc.y, pr.y);
      }
      st<DT>(dst_c, row + da, acc.x);
      if (has_b) st<DT>(dst_c, row + db, acc.y);
    }
    if (staged) __syncthreads();
  }
  (void)MODE;
}


// NaN-propagating min/max (PTX min.NaN / max.NaN): a NaN anywhere makes the
// running value NaN, as torch.min / torch.max propagate it.
__device__ __forceinline__ float rs_min_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float rs_max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// three-input forms (sm_100): one instruction folds a voxel pair
__device__ __forceinline__ float rs_min3_nan(float a, float b, float c) {
  float r;
  asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float rs_max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Block-wide min/max of the 128 threads' running (mn[i], mx[i]) for up to
// FS_FOLD_CH channels i < n, committed to channel i's (min, max) key pair at
// keys + 2 i with one atomic each (order-preserving int32 keys, NaN winning
// both: the intensity chain's statistics format).  One block exchange serves
// all n channels; every thread of the CTA calls it.
__device__ __forceinline__ void rs_commit_minmax_n(const float* mn, const float* mx, int n,
                                                   int32_t* keys) {
  constexpr int G = 4;  // FS_FOLD_CH
  __shared__ int32_t s_k[ST_THREADS / 32][2 * G];
  int32_t k[2 * G];
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const bool nan = (mn[i] != mn[i]) || (mx[i] != mx[i]);
    k[2 * i] = nan ? KEY_MIN_NAN : fkey(mn[i]);
    k[2 * i + 1] = nan ? KEY_MAX_NAN : fkey(mx[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < G; ++i) {
      k[2 * i] = min(k[2 * i], __shfl_xor_sync(0xFFFFFFFFu, k[2 * i], o));
      k[2 * i + 1] = max(k[2 * i + 1], __shfl_xor_sync(0xFFFFFFFFu, k[2 * i + 1], o));
    }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();  // an earlier commit's reads of s_k are done
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < 2 * G; ++i) s_k[warp][i] = k[i];
  __syncthreads();
  if (threadIdx.x < 2 * n) {
    const int i = threadIdx.x;  // (group i / 2, min or max)
    int32_t v = s_k[0][i];
    for (int w = 1; w < ST_THREADS / 32; ++w) v = (i & 1) ? max(v, s_k[w][i]) : min(v, s_k[w][i]);
    if ((i & 1) == 0 && v != fkey(INFINITY)) atomicMin(keys + i, v);
    if ((i & 1) == 1 && v != fkey(-INFINITY)) atomicMax(keys + i, v);
  }
}

// A masked-out element's tile when key 0 folds its min/max: the copy of
// staged_copy_masked (16-byte vectors where the row is whole and aligned),
// channel by channel, key 0's channels committed one at a time.
__device__ __forceinline__ void staged_copy_masked_fold(const ResampleArgs& a, int64_t b, int d0,
                                                        int w0, int h0, int hwd, int t) {
  const int H = a.H, W = a.W, D = a.D;
  const int w = w0 + t % ST_TW, h = h0 + t / ST_TW;
  const bool in = w < W && h < H;
  const int n = min(ST_TD, D - d0);
  for (int ki = 0; ki < a.n_keys; ++ki) {
    const KeyArgs& kc = a.keys[ki];
    const int ke = kc.dtype == BA_BF16 ? 2 : 4;
    const bool fold = ki == 0 && kc.minmax != nullptr;
    float gmn[4], gmx[4];  // the current group of 4 channels
    for (int c = 0; c < kc.channels; ++c) {
      float mn = INFINITY, mx = -INFINITY;
      if (in) {
        const int64_t i0 = (b * kc.channels + c) * (int64_t)hwd + ((int64_t)h * W + w) * D + d0;
        const char* sp = (const char*)kc.src + i0 * ke;
        char* dp = (char*)kc.dst + i0 * ke;
        if (n == ST_TD && ((uintptr_t)sp % 16) == 0 && ((uintptr_t)dp % 16) == 0) {
          uint4 v[4];
          const int nv = ST_TD * ke / 16;  // 4 (fp32) or 2 (bf16)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (q < nv) v[q] = __ldg(reinterpret_cast<const uint4*>(sp) + q);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (q < nv) reinterpret_cast<uint4*>(dp)[q] = v[q];
          if (fold) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (q >= nv) break;
              const uint32_t u[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
              for (int j = 0; j < 4; j += 2) {
                if (ke == 2) {
#pragma unroll
                  for (int e = j; e < j + 2; ++e) {
                    const float lo = __uint_as_float(u[e] << 16);
                    const float hi = __uint_as_float(u[e] & 0xFFFF0000u);
                    mn = rs_min3_nan(mn, lo, hi);
                    mx = rs_max3_nan(mx, lo, hi);
                  }
                } else {
                  const float x0 = __uint_as_float(u[j]), x1 = __uint_as_float(u[j + 1]);
                  mn = rs_min3_nan(mn, x0, x1);
                  mx = rs_max3_nan(mx, x0, x1);
                }
              }
            }
          }
        } else {
          for (int q = 0; q < n; ++q) {
            float v;
            if (ke == 2) {
              const uint16_t u = __ldg((const uint16_t*)sp + q);
              ((uint16_t*)dp)[q] = u;
              v = __uint_as_float((uint32_t)u << 16);
            } else {
              v = __ldg((const float*)sp + q);
              ((float*)dp)[q] = v;
            }
            mn = rs_min_nan(mn, v);
            mx = rs_max_nan(mx, v);
          }
        }
      }
      if (fold) {
        const int slot = c % 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (slot == 0) {
            gmn[i] = INFINITY;
            gmx[i] = -INFINITY;
          }
          if (i == slot) {
            gmn[i] = mn;
            gmx[i] = mx;
          }
        }
        if (slot == 3 || c + 1 == kc.channels)
          rs_commit_minmax_n(gmn, gmx, slot + 1, kc.minmax + 2 * (b * kc.channels + c - slot));
      }
    }
  }
}

// ===========================================================================
// Fast affine resample: the default for a bilinear key (zeros or border
// padding) of an affine map; BA_RESAMPLE_EXACT selects the kernels above.
// Tiles, thread layout, exact source coordinates and staging are
// resample3d_staged_kernel's; it differs in three ways:
//  * each coordinate is first clamped to the range its taps can need
//    (fast_pad): [-1, size] for zeros padding, where every tap outside the
//    volume reads the zero fill, and torch's [0, size - 1] clip for border.
//    The box staged from the clamped corners then holds every tap of the
//    tile, so there is no per-voxel containment test; the shared-memory
//    index is clamped to the box only to keep every access in bounds;
//  * trilinear interpolation is seven fused lerps a + t * (b - a) on voxel
//    pairs (fp32x2), against torch's eight rounded weight products and
//    sums: within 1e-5 (fp32) / 2 bf16 ulp of them.  Source coordinates are
//    the exact ones, so a nearest key sampled alongside stays bit-exact;
//  * a CTA whose box exceeds ST_MAX_FLOATS gathers its taps from global
//    memory (bounds-checked, zero outside the volume).
// ===========================================================================
template <int PAD>
__device__ __forceinline__ float fast_pad(float c, float size) {
  if (PAD == BA_PAD_BORDER) return clip_coord(c, size - 1.0f);
  return fminf(fmaxf(c, -1.0f), size);  // fmaxf(NaN, -1) = -1: a zero tap, as torch
}

__device__ __forceinline__ float2 lerp2(float2 a, float2 b, float2 t) {
  return __ffma2_rn(t, sub2(b, a), a);
}

// trilinear of the taps of two voxels (taps8 order) at fractions (fx, fy, fz)
__device__ __forceinline__ float2 trilerp2(const float* va, const float* vb, float2 fx, float2 fy,
                                           float2 fz) {
  const float2 c00 = lerp2(f2(va[0], vb[0]), f2(va[1], vb[1]), fx);
  const float2 c10 = lerp2(f2(va[2], vb[2]), f2(va[3], vb[3]), fx);
  const float2 c01 = lerp2(f2(va[4], vb[4]), f2(va[5], vb[5]), fx);
  const float2 c11 = lerp2(f2(va[6], vb[6]), f2(va[7], vb[7]), fx);
  return lerp2(lerp2(c00, c10, fy), lerp2(c01, c11, fy), fz);
}

constexpr int FS_MAX_FLOATS = BA_FS_MAX_FLOATS, FS_STAGE_FLOATS = BA_FS_STAGE_FLOATS;

// Copy the boxes of channels src_c, src_c + cstride, ... (nch of them) into
// shared memory, channel i at float offset i * box, rows of exp and planes of
// plp floats: 16-byte chunks, cp.async for fp32 (chunks outside the volume
// zero-filled: source size 0), synchronous widening loads for bf16.  Ends
// with the block synchronised.
template <int DT>
__device__ __forceinline__ void stage_box_pitched(float4* s_dyn4, const char* src_c,
                                                  size_t cstride, int nch, int box, int lx4,
                                                  int ly, int lz, int nx4, int ey, int ez, int exp,
                                                  int plp, int H, int W, int D, int t) {
  for (int ci = 0; ci < nch; ++ci, src_c += cstride, s_dyn4 += box / 4) {
  const int rows = ey * ez;
  const int rpp = ST_THREADS / nx4;  // rows per pass (nx4 <= ST_THREADS)
  const int lc = t % nx4;
  int row = t / nx4;
  int y = row % ey, z = row / ey;
  if (row < rpp) {
    for (; row < rows; row += rpp) {
      const int gy = ly + y, gz = lz + z, gx = lx4 + 4 * lc;
      const bool in = (unsigned)gy < (unsigned)W && (unsigned)gz < (unsigned)H && gx >= 0 && gx < D;
      const int64_t gi = in ? ((int64_t)gz * W + gy) * D + gx : 0;
      float4* sd = &s_dyn4[(z * plp + y * exp) / 4 + lc];
      if (DT == BA_F32) {
        const unsigned sdst = (unsigned)__cvta_generic_to_shared(sd);
        const void* gsrc = (const float*)src_c + gi;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sdst), "l"(gsrc),
                     "r"(in ? 16 : 0) : "memory");
      } else {
        *sd = in ? ld4<DT>(src_c, gi) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      y += rpp;
      while (y >= ey) {
        y -= ey;
        ++z;
      }
    }
  }
  }
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
}

// CTAs per SM the fast kernel's registers are bounded for.  Measured on
// B200: 5 (96 registers, a paired key's variants spilling) made a four-
// channel vol + seg affine 12 % slower than 4 (128) and left a one-channel
// one unchanged.
#ifndef BA_FS_MINBLOCKS
#define BA_FS_MINBLOCKS 4
#endif
#ifndef BA_FS_SEG_OVERLAP
#define BA_FS_SEG_OVERLAP 1
#endif
// channels staged side by side at most, when key 0 folds its min/max
constexpr int FS_FOLD_CH = 4;

// FOLD: key 0's minmax output is folded (only set for launches that ask)
template <int S0, int S1, bool FOLD>
__global__ void __launch_bounds__(ST_THREADS, BA_FS_MINBLOCKS)
    resample3d_fast_kernel(const __grid_constant__ ResampleArgs a) {
  extern __shared__ float4 s_dyn4[];
  const float* s_src = reinterpret_cast<const float*>(s_dyn4);
  __shared__ StagedShared sh;
  constexpr int PAD = spec_pad(S0), DT = spec_dt(S0);
  static_assert(spec_mode(S0) == BA_BILINEAR && PAD != BA_PAD_REFLECTION,
                "the fast kernel samples a bilinear key with zeros or border padding");
  const bool ALIGN = a.align_corners != 0;
  const int H = a.H, W = a.W, D = a.D;
  const int tiles_d = (D + ST_TD - 1) / ST_TD;
  const int d0 = (blockIdx.x % tiles_d) * ST_TD;
  const int w0 = (blockIdx.x / tiles_d) * ST_TW;
  const int h0 = blockIdx.y * ST_TH;
  const int64_t b = a.b0 + blockIdx.z;
  const int hwd = H * W * D;
  const int t = threadIdx.x;
  const int tx = t & 7, ty = (t >> 3) & 1, tz = (t >> 4) & 1, wp = t >> 5;
  const KeyArgs& k = a.keys[0];
  const size_t esz = DT == BA_BF16 ? 2 : 4;
  // key 0's per-(element, channel) min/max folded as the outputs are written
  const bool fold = FOLD && k.minmax != nullptr;
  if (!elem_active(a, b)) {
    if (fold)
      staged_copy_masked_fold(a, b, d0, w0, h0, hwd, t);
    else
      staged_copy_masked(a, b, d0, w0, h0, hwd, t);
    return;
  }
  staged_setup<PAD, true>(a, b, d0, w0, h0, ALIGN, t, sh);
  const int lx4 = sh.box[0], ly = sh.box[1], lz = sh.box[2], ey = sh.box[4], ez = sh.box[5];
  const int nx4 = sh.box[3];
  const int exp = nx4 * 4, plp = ey * exp, box = ez * plp;
  const bool staged = nx4 > 0 && box <= FS_STAGE_FLOATS;
  // channels staged together: as many as fit side by side, so each voxel's
  // coordinates serve every channel of a pass (at most FS_FOLD_CH of them
  // when folding min/max)
  int cstack = staged ? min(k.channels, FS_MAX_FLOATS / box) : 1;
  // folding: at most FS_FOLD_CH channels a pass, each with its own registers
  if (fold) cstack = min(cstack, FS_FOLD_CH);
  // a voxel's first tap, relative to the box: (z0 - lz) * plp + (y0 - ly) * exp
  // + x0 - lx4; clamped to [0, smax] so that even a wrong index stays inside
  const int s_off = -(lz * plp + ly * exp + lx4);
  const int smax = staged ? ez * plp - plp - exp - 2 : 0;
  float2 t1[3], t2[3], t3[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    t1[r] = f2(sh.theta[r * 4 + 1]);
    t2[r] = f2(sh.theta[r * 4 + 2]);
    t3[r] = f2(sh.theta[r * 4 + 3]);
  }
  const float fD = (float)D, fW = (float)W, fH = (float)H;
  const bool pD = (D & (D - 1)) == 0, pW = (W & (W - 1)) == 0, pH = (H & (H - 1)) == 0;
  const size_t cstride = (size_t)hwd * esz;
  // key 0's running min/max of this pass's channels, as stored (folding
  // only; indexed by compile-time channel numbers, so they stay in registers)
  float fmn[FS_FOLD_CH], fmx[FS_FOLD_CH];
  for (int c0 = 0; c0 < k.channels; c0 += cstack) {
#pragma unroll
    for (int i = 0; i < FS_FOLD_CH; ++i) {
      fmn[i] = INFINITY;
      fmx[i] = -INFINITY;
    }
    const int nch = min(cstack, k.channels - c0);
    const char* src_c = (const char*)k.src + ((size_t)b * k.channels + c0) * cstride;
    char* dst_c = (char*)k.dst + ((size_t)b * k.channels + c0) * cstride;
    if (staged)
      stage_box_pitched<DT>(s_dyn4, src_c, cstride, nch, box, lx4, ly, lz, nx4, ey, ez, exp, plp,
                            H, W, D, t);
    // channel ci's pair as stored, into its running min/max (ci a constant)
    auto fold_pair = [&](int ci, float2 r, bool has_b) {
      const float va = round_dt<DT>(r.x), vb = has_b ? round_dt<DT>(r.y) : va;
      fmn[ci] = rs_min3_nan(fmn[ci], va, vb);
      fmx[ci] = rs_max3_nan(fmx[ci], va, vb);
    };
    for (int pw = 0; pw < ST_PW; ++pw) {
      const int h = h0 + tz + 2 * wp;
      const int w = w0 + ty + 2 * pw;
      const int da = d0 + tx, db = da + 8;
      // every lane runs the iteration (the one-tap vote below is warp-wide);
      // a lane outside the volume computes but neither loads nor stores
      const bool valid = w < W && h < H && da < D;
      const bool has_b = db < D;
      const float2 bz2 = f2(sh.bz[tz + 2 * wp]);
      const float2 by2 = f2(sh.by[ty + 2 * pw]);
      float2 g[3];
#pragma unroll
      for (int r = 0; r < 3; ++r)
        g[r] = add2(__ffma2_rn(bz2, t2[r], __ffma2_rn(by2, t1[r], sh.px[r][tx])), t3[r]);
      float2 ix, iy, iz;
      if (ALIGN) {
        ix = unnormalize2<true>(g[0], fD);
        iy = unnormalize2<true>(g[1], fW);
        iz = unnormalize2<true>(g[2], fH);
      } else {
        ix = pD ? unnormalize2_pow2(g[0], fD) : unnormalize2<false>(g[0], fD);
        iy = pW ? unnormalize2_pow2(g[1], fW) : unnormalize2<false>(g[1], fW);
        iz = pH ? unnormalize2_pow2(g[2], fH) : unnormalize2<false>(g[2], fH);
      }
      const int row = (h * W + w) * D;
      // the paired nearest key (S1): its gathers issued now, stored after
      // this pair's interpolation, so their latency overlaps it
      constexpr int S1K = S1 < 0 ? 0 : S1;
      const bool seg = S1 >= 0 && c0 == 0 && valid;
      NearestPair nq;
      if (seg) {
        if (BA_FS_SEG_OVERLAP) {
          if (ALIGN)
            nearest_begin<spec_pad(S1K), spec_dt(S1K), true>(a.keys[1], b, H, W, D, hwd, ix, iy,
                                                             iz, row + da, row + db, has_b, nq);
          else
            nearest_begin<spec_pad(S1K), spec_dt(S1K), false>(a.keys[1], b, H, W, D, hwd, ix, iy,
                                                              iz, row + da, row + db, has_b, nq);
        } else if (ALIGN) {
          sample_spec<S1K, true>(a.keys[1], b, H, W, D, hwd, ix, iy, iz, row + da, row + db,
                                 has_b);
        } else {
          sample_spec<S1K, false>(a.keys[1], b, H, W, D, hwd, ix, iy, iz, row + da, row + db,
                                  has_b);
        }
      }
      const float2 px = f2(fast_pad<PAD>(ix.x, fD), fast_pad<PAD>(ix.y, fD));
      const float2 py = f2(fast_pad<PAD>(iy.x, fW), fast_pad<PAD>(iy.y, fW));
      const float2 pz = f2(fast_pad<PAD>(iz.x, fH), fast_pad<PAD>(iz.y, fH));
      const Floor2 fx = floor2(px), fy = floor2(py), fz = floor2(pz);
      const float2 wx = sub2(px, fx.f), wy = sub2(py, fy.f), wz = sub2(pz, fz.f);
      // voxel b of a pair past the volume's end reuses voxel a's corner
      const int xb = has_b ? fx.hi : fx.lo, yb = has_b ? fy.hi : fy.lo, zb = has_b ? fz.hi : fz.lo;
      if (staged) {
        const int sa = min(max(fz.lo * plp + fy.lo * exp + fx.lo + s_off, 0), smax);
        const int sb = min(max(zb * plp + yb * exp + xb + s_off, 0), smax);
        // every voxel of the warp on a source voxel centre (all fractions
        // zero: a flip or rot90 for ~88 % of warp iterations): the
        // interpolation is its one tap
        const bool centre = !valid || ((wx.x == 0.0f && wy.x == 0.0f && wz.x == 0.0f) &&
                                       (!has_b || (wx.y == 0.0f && wy.y == 0.0f && wz.y == 0.0f)));
        const bool one_tap = __all_sync(0xFFFFFFFFu, centre);
        // channel ci of the pass: interpolated from its staged box, stored
        auto chan = [&](int ci) -> float2 {
          const float* sc = s_src + ci * box;
          char* dst = dst_c + ci * cstride;
          float2 r;
          if (one_tap) {
            r = f2(sc[sa], sc[sb]);
          } else {
            float va[8], vb[8];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int si = q ? sb : sa;
              float* v = q ? vb : va;
              v[0] = sc[si];
              v[1] = sc[si + 1];
              v[2] = sc[si + exp];
              v[3] = sc[si + exp + 1];
              v[4] = sc[si + plp];
              v[5] = sc[si + plp + 1];
              v[6] = sc[si + plp + exp];
              v[7] = sc[si + plp + exp + 1];
            }
            r = trilerp2(va, vb, wx, wy, wz);
          }
          st<DT>(dst, row + da, r.x);
          if (has_b) st<DT>(dst, row + db, r.y);
          return r;
        };
        if (FOLD && fold) {
#pragma unroll
          for (int ci = 0; ci < FS_FOLD_CH; ++ci)
            if (valid && ci < nch) fold_pair(ci, chan(ci), has_b);
        } else {
          for (int ci = 0; valid && ci < nch; ++ci) chan(ci);
        }
      } else if (valid) {
        const bool ia = (unsigned)fx.lo < (unsigned)(D - 1) && (unsigned)fy.lo < (unsigned)(W - 1) &&
                        (unsigned)fz.lo < (unsigned)(H - 1);
        const bool ib = (unsigned)xb < (unsigned)(D - 1) && (unsigned)yb < (unsigned)(W - 1) &&
                        (unsigned)zb < (unsigned)(H - 1);
        float va[8], vb[8];
        taps8<DT>(src_c, fx.lo, fy.lo, fz.lo, H, W, D, ia, va);
        taps8<DT>(src_c, xb, yb, zb, H, W, D, ib, vb);
        const float2 r = trilerp2(va, vb, wx, wy, wz);
        st<DT>(dst_c, row + da, r.x);
        if (has_b) st<DT>(dst_c, row + db, r.y);
        if (fold) fold_pair(0, r, has_b);
      }
      if (BA_FS_SEG_OVERLAP && seg)
        nearest_end<spec_dt(S1K)>(a.keys[1], b, hwd, row + da, row + db, has_b, nq);
    }
    // the pass's channels complete: one block exchange commits them all
    if (fold) rs_commit_minmax_n(fmn, fmx, nch, k.minmax + 2 * (b * k.channels + c0));
    if (staged) __syncthreads();
  }
}

// ===========================================================================
// Signed-permutation resample: theta's 3x3 part holds one +-1 per row and
// column, and the source x (D) coordinate is driven by the output D index —
// flips, square-plane rot90s in the (H, W) plane and their products in a
// Compose.  Each source coordinate then depends on one output index only
// (the other terms of the affine_grid sum are exact zeros), so the kernel
// tabulates it per axis with the same arithmetic as the other kernels and
// copies rows as 16-byte (fp32) / 8-byte (bf16) vectors, forwards or
// reversed.  A coordinate a few ulp from an integer (torch's linspace base
// grid puts one position per axis there) takes the fast kernel's fused lerp
// from the neighbouring source voxel, fetched alongside the vector; the few
// rows off a centre along y or z lerp 2 or 4 source rows.  Nearest keys read
// the same voxels as the exact kernels and take this kernel in both modes.
// A warp covers R consecutive (h, w) rows of one element; a lane takes 4
// consecutive D positions.  D is a multiple of 4 and at most PM_MAX_D, rows
// 16-byte (fp32) / 8-byte (bf16) aligned.
// ===========================================================================
constexpr int PM_THREADS = 256;
constexpr int PM_WARPS = PM_THREADS / 32;
constexpr int PM_MAX_D = 1024;

struct PermAxis {
  int lo;      // floor of the coordinate clamped as the fast kernel clamps it
  float frac;  // its fractional part (0: on a voxel centre)
  int near;    // the nearest key's index, -1 outside the volume
};

template <int PAD>
__device__ __forceinline__ PermAxis perm_axis(float u, int size) {
  PermAxis r;
  const float p = fast_pad<PAD>(u, (float)size);
  const float f = floorf(p);
  r.lo = (int)f;
  r.frac = __fsub_rn(p, f);
  const int n = __float2int_rn(pad_coord<PAD, false>(u, size));
  r.near = (unsigned)n < (unsigned)size ? n : -1;
  return r;
}

// source coordinate along axis r for output index i along the axis that
// drives it: g = sign * base + t3 (the affine_grid sum's other terms are
// exact zeros), then grid_sampler_unnormalize
__device__ __forceinline__ float perm_coord(int i, int n_out, float sign, float t3, int size,
                                            bool align) {
  const float g = __fadd_rn(__fmul_rn(base_coord(i, n_out, align), sign), t3);
  return align ? __fmul_rn(__fmul_rn(__fadd_rn(g, 1.0f), 0.5f), (float)(size - 1))
               : __fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(g, 1.0f), (float)size), 1.0f), 0.5f);
}

template <int DT>
__device__ __forceinline__ void ld4v(const void* base, int64_t i, float* v) {
  if (DT == BA_BF16) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>((const uint16_t*)base + i));
    v[0] = __uint_as_float(u.x << 16);
    v[1] = __uint_as_float(u.x & 0xFFFF0000u);
    v[2] = __uint_as_float(u.y << 16);
    v[3] = __uint_as_float(u.y & 0xFFFF0000u);
  } else {
    const float4 f = __ldg(reinterpret_cast<const float4*>((const float*)base + i));
    v[0] = f.x;
    v[1] = f.y;
    v[2] = f.z;
    v[3] = f.w;
  }
}

template <int DT>
__device__ __forceinline__ void st4v(void* base, int64_t i, const float* v) {
  if (DT == BA_BF16) {
    uint2 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    *reinterpret_cast<uint2*>((uint16_t*)base + i) = u;
  } else {
    *reinterpret_cast<float4*>((float*)base + i) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// A voxel off a voxel centre (or on the volume's border): the fast kernel's
// lerps over its 8 taps, bounds-checked, zero outside the volume.  Rare, so
// kept out of line to leave the copy loop its registers.
template <int DT>
__device__ __noinline__ float perm_interp(const char* cs, PermAxis ax, PermAxis ay, PermAxis az,
                                          int H, int W, int D) {
  const int x0 = ax.lo, y0 = ay.lo, z0 = az.lo;
  float va[8];
  const bool interior = (unsigned)x0 < (unsigned)(D - 1) && (unsigned)y0 < (unsigned)(W - 1) &&
                        (unsigned)z0 < (unsigned)(H - 1);
  taps8<DT>(cs, x0, y0, z0, H, W, D, interior, va);
  return trilerp2(va, va, f2(ax.frac), f2(ay.frac), f2(az.frac)).x;
}

// The x side of a lane's 4 voxels (D positions d .. d+3 of a row): the
// aligned source chunk their nearest indices fill, forwards or reversed, and
// whether a bilinear lerp along x reaches the source voxel just before or
// just after that chunk.
struct PermX {
  int base;     // first source x of the chunk; -1 when the voxels do not fill one
  bool rev;     // reversed order (a flip along x)
  bool off;     // a voxel off a voxel centre along x
  bool need_l;  // a lerp reads source x base - 1
  bool need_r;  // a lerp reads source x base + 4
};

__device__ __forceinline__ PermX perm_x(const PermAxis* sx, int D) {
  PermX p;
  const int n0 = sx[0].near, n3 = sx[3].near;
  p.rev = n0 > n3;
  const int base = p.rev ? n3 : n0;
  bool ok = base >= 0 && (base & 3) == 0 && base + 3 < D;
  p.off = p.need_l = p.need_r = false;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const PermAxis ax = sx[j];
    ok = ok && ax.near == (p.rev ? base + 3 - j : base + j);
    if (ax.frac != 0.0f) {
      p.off = true;
      p.need_l = p.need_l || ax.lo < base;
      p.need_r = p.need_r || ax.lo + 1 > base + 3;
    }
  }
  p.base = ok ? base : -1;
  return p;
}

// One source row's chunk for a lane: 4 voxels as one vector plus, for x
// lerps, the voxels on either side (zero outside the volume); every load is
// issued before any use.
template <int DT>
__device__ __forceinline__ void perm_fetch(const char* cs, int64_t row, bool in, const PermX& px,
                                           int D, float* v, float& l, float& r) {
  if (in) {
    ld4v<DT>(cs, row + px.base, v);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = 0.0f;
  }
  l = (in && px.need_l && px.base > 0) ? ld<DT>(cs, row + px.base - 1) : 0.0f;
  r = (in && px.need_r && px.base + 4 < D) ? ld<DT>(cs, row + px.base + 4) : 0.0f;
}

__device__ __forceinline__ float pick6(const float (&w)[6], int i) {
  const float a = i == 0 ? w[0] : w[1];
  const float b = i == 2 ? w[2] : w[3];
  const float c = i == 4 ? w[4] : w[5];
  return i < 2 ? a : (i < 4 ? b : c);
}

// The 4 voxels in output order: the chunk's voxels, and the fast kernel's
// x lerp fma(f, hi - lo, lo) for the ones off a centre (trilerp2's lerps
// along y and z at fraction 0 return it unchanged).
template <bool LERP>
__device__ __forceinline__ void perm_xlerp(const float* v, float l, float r, const PermX& px,
                                           const PermAxis* sx, float* out) {
#pragma unroll
  for (int j = 0; j < 4; ++j) out[j] = px.rev ? v[3 - j] : v[j];
  if (LERP && px.off) {
    const float w[6] = {l, v[0], v[1], v[2], v[3], r};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const PermAxis ax = sx[j];
      if (ax.frac != 0.0f) {
        const int i = ax.lo - px.base + 1;  // 0 .. 4
        const float lo = pick6(w, i), hi = pick6(w, i + 1);
        out[j] = __fmaf_rn(ax.frac, __fsub_rn(hi, lo), lo);
      }
    }
  }
}

// Where a key's output row reads: its source row (nearest indices, or the
// floors for a bilinear key) and whether that row lies inside the volume.
template <int MODE>
__device__ __forceinline__ void perm_row(PermAxis ay, PermAxis az, int H, int W, int D,
                                         int64_t& row, bool& in) {
  const int yi = MODE == BA_NEAREST ? ay.near : ay.lo;
  const int zi = MODE == BA_NEAREST ? az.near : az.lo;
  in = (unsigned)yi < (unsigned)W && (unsigned)zi < (unsigned)H;
  row = ((int64_t)zi * W + yi) * D;
}

// The common case: rows on voxel centres along y and z (nearest keys always
// are), lanes whose voxels fill aligned source chunks.  R output rows of the
// warp and 4 / R channels at a time, both keys' loads issued before any
// store (a store could alias a later load as far as the compiler knows).
template <int S0, int S1, int R>
__device__ __forceinline__ void perm_rows_fast(const ResampleArgs& a, int64_t b, int H, int W,
                                               int D, int64_t orow0, int nr, int d, bool act,
                                               const PermX& px, const PermAxis* sy,
                                               const PermAxis* sz, const PermAxis* sx) {
  constexpr int CB = 4 / R;
  constexpr int M0 = spec_mode(S0), DT0 = spec_dt(S0);
  constexpr int S1K = S1 < 0 ? 0 : S1;
  constexpr int M1 = spec_mode(S1K), DT1 = spec_dt(S1K);
  const int64_t hwd = (int64_t)H * W * D;
  const KeyArgs& k0 = a.keys[0];
  const KeyArgs& k1 = a.keys[S1 >= 0 ? 1 : 0];
  const size_t e0 = DT0 == BA_BF16 ? 2 : 4, e1 = DT1 == BA_BF16 ? 2 : 4;
  int64_t src0[R], src1[R];
  bool in0[R], in1[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int rr = min(r, nr - 1);  // rows past the group's end repeat its last (not stored)
    perm_row<M0>(sy[rr], sz[rr], H, W, D, src0[r], in0[r]);
    in0[r] = in0[r] && act;
    if (S1 >= 0) {
      perm_row<M1>(sy[rr], sz[rr], H, W, D, src1[r], in1[r]);
      in1[r] = in1[r] && act;
    }
  }
  const int nc = max(k0.channels, S1 >= 0 ? k1.channels : 0);
  for (int c0 = 0; c0 < nc; c0 += CB) {
    float v0[4][4], l0[4], r0[4], v1[4][4];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        const int s = r * CB + j, c = c0 + j;
        perm_fetch<DT0>((const char*)k0.src + ((size_t)b * k0.channels + c) * hwd * e0, src0[r],
                        in0[r] && c < k0.channels, px, D, v0[s], l0[s], r0[s]);
        if (S1 >= 0) {
          float dl, dr;
          PermX p1 = px;
          p1.need_l = p1.need_r = false;
          perm_fetch<DT1>((const char*)k1.src + ((size_t)b * k1.channels + c) * hwd * e1, src1[r],
                          in1[r] && c < k1.channels, p1, D, v1[s], dl, dr);
        }
      }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        const int s = r * CB + j, c = c0 + j;
        if (!act || r >= nr) continue;
        const int64_t o = (orow0 + r) * D + d;
        float out[4];
        if (c < k0.channels) {
          perm_xlerp<M0 != BA_NEAREST>(v0[s], l0[s], r0[s], px, sx, out);
          st4v<DT0>((char*)k0.dst + ((size_t)b * k0.channels + c) * hwd * e0, o, out);
        }
        if (S1 >= 0 && c < k1.channels) {
          perm_xlerp<false>(v1[s], 0.0f, 0.0f, px, sx, out);
          st4v<DT1>((char*)k1.dst + ((size_t)b * k1.channels + c) * hwd * e1, o, out);
        }
      }
  }
}

// One key, one channel, one output row off voxel centres along y or z (a
// coordinate a few ulp from an integer: a few rows per volume), or lanes
// whose voxels do not fill aligned chunks: the 2 or 4 source rows around it
// fetched together, lerped along x, then along y and z as trilerp2 does.
template <int S>
__device__ __forceinline__ void perm_row_slow(const char* cs, char* cd, int H, int W, int D,
                                              int64_t o, bool act, bool xok, const PermX& px,
                                              PermAxis ay, PermAxis az, const PermAxis* sx) {
  constexpr int MODE = spec_mode(S), DT = spec_dt(S);
  float out[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (!xok) {
    if (act) {
      if (MODE == BA_NEAREST) {
        const bool in = ay.near >= 0 && az.near >= 0;
        const int64_t row = ((int64_t)az.near * W + ay.near) * D;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          out[j] = (in && sx[j].near >= 0) ? ld<DT>(cs, row + sx[j].near) : 0.0f;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) out[j] = perm_interp<DT>(cs, sx[j], ay, az, H, W, D);
      }
      st4v<DT>(cd, o, out);
    }
    return;
  }
  if (MODE == BA_NEAREST) {
    int64_t row;
    bool in;
    perm_row<MODE>(ay, az, H, W, D, row, in);
    float v[4], l, r;
    PermX p = px;
    p.need_l = p.need_r = false;
    perm_fetch<DT>(cs, row, in && act, p, D, v, l, r);
    perm_xlerp<false>(v, l, r, px, sx, out);
  } else {
    float v[4][4], l[4], r[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int dy = q & 1, dz = q >> 1;
      const bool need = (dy == 0 || ay.frac != 0.0f) && (dz == 0 || az.frac != 0.0f);
      const int yy = ay.lo + dy, zz = az.lo + dz;
      const bool in = act && need && (unsigned)yy < (unsigned)W && (unsigned)zz < (unsigned)H;
      perm_fetch<DT>(cs, ((int64_t)zz * W + yy) * D, in, px, D, v[q], l[q], r[q]);
    }
    float c[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) perm_xlerp<true>(v[q], l[q], r[q], px, sx, c[q]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float c0 = __fmaf_rn(ay.frac, __fsub_rn(c[1][j], c[0][j]), c[0][j]);
      const float c1 = __fmaf_rn(ay.frac, __fsub_rn(c[3][j], c[2][j]), c[2][j]);
      out[j] = __fmaf_rn(az.frac, __fsub_rn(c1, c0), c0);
    }
  }
  if (act) st4v<DT>(cd, o, out);
}

template <int S0, int S1, int R>
__device__ __forceinline__ void perm_rows_slow(const ResampleArgs& a, int64_t b, int H, int W,
                                               int D, int64_t orow0, int nr, int d, bool act,
                                               bool xok, const PermX& px, const PermAxis* sy,
                                               const PermAxis* sz, const PermAxis* sx) {
  constexpr int DT0 = spec_dt(S0);
  constexpr int S1K = S1 < 0 ? 0 : S1;
  constexpr int DT1 = spec_dt(S1K);
  const int64_t hwd = (int64_t)H * W * D;
  const KeyArgs& k0 = a.keys[0];
  const KeyArgs& k1 = a.keys[S1 >= 0 ? 1 : 0];
  const size_t e0 = DT0 == BA_BF16 ? 2 : 4, e1 = DT1 == BA_BF16 ? 2 : 4;
  for (int r = 0; r < nr; ++r) {
    const int64_t o = (orow0 + r) * D + d;
    for (int c = 0; c < k0.channels; ++c) {
      const size_t off = ((size_t)b * k0.channels + c) * hwd * e0;
      perm_row_slow<S0>((const char*)k0.src + off, (char*)k0.dst + off, H, W, D, o, act, xok, px,
                        sy[r], sz[r], sx);
    }
    if (S1 >= 0)
      for (int c = 0; c < k1.channels; ++c) {
        const size_t off = ((size_t)b * k1.channels + c) * hwd * e1;
        perm_row_slow<S1K>((const char*)k1.src + off, (char*)k1.dst + off, H, W, D, o, act, xok,
                           px, sy[r], sz[r], sx);
      }
  }
}

// R output rows per warp (4 for single-channel keys, so that each lane keeps
// four loads in flight; 1 otherwise, with four channels at a time).
template <int S0, int S1, int R>
__global__ void __launch_bounds__(PM_THREADS, 2) resample3d_perm_kernel(const __grid_constant__ ResampleArgs a) {
  constexpr int ROWS = PM_WARPS * R;
  __shared__ PermAxis s_x[PM_MAX_D];
  __shared__ PermAxis s_y[ROWS], s_z[ROWS];
  __shared__ float s_th[12];
  constexpr int PAD = spec_pad(S0);
  const bool ALIGN = a.align_corners != 0;
  const int H = a.H, W = a.W, D = a.D;
  const int hwd = H * W * D;
  const int64_t b = a.b0 + blockIdx.y;
  // the CTA walks groups of ROWS rows, gridDim.x apart
  const int n_groups = (H * W + ROWS - 1) / ROWS;
  const int t = threadIdx.x;
  if (!elem_active(a, b)) {
    // the reference's torch.where keeps a masked-out element: a group's rows
    // are one contiguous run per channel
    for (int g = blockIdx.x; g < n_groups; g += gridDim.x) {
      const int row0 = g * ROWS;
      const int rows = min(ROWS, H * W - row0);
      for (int ki = 0; ki < a.n_keys; ++ki) {
        const KeyArgs& kc = a.keys[ki];
        const int ke = kc.dtype == BA_BF16 ? 2 : 4;
        const int n4 = rows * D / 4;  // 4-voxel chunks
        for (int c = 0; c < kc.channels; ++c) {
          const int64_t i0 = (b * kc.channels + c) * (int64_t)hwd + (int64_t)row0 * D;
          for (int q = t; q < n4; q += PM_THREADS) {
            if (ke == 2)
              reinterpret_cast<uint2*>((uint16_t*)kc.dst + i0)[q] =
                  __ldg(reinterpret_cast<const uint2*>((const uint16_t*)kc.src + i0) + q);
            else
              reinterpret_cast<float4*>((float*)kc.dst + i0)[q] =
                  __ldg(reinterpret_cast<const float4*>((const float*)kc.src + i0) + q);
          }
        }
      }
    }
    return;
  }
  if (t < 12) {
    const int i = t / 4, j = t % 4;
    const float* x = elem_xform(a, b);
    if (a.xform_kind == BA_XFORM_AFFINE) {
      // monai_affine_to_theta: theta = P S_norm A S_inv P, P swapping 0 and 2.
      const int pi = 2 - i, pj = (j == 3) ? 3 : 2 - j;
      const float s_j = (pj == 3) ? 1.0f : a.si[pj];
      s_th[t] = (a.sn[pi] * x[pi * 4 + pj]) * s_j;
    } else {
      s_th[t] = x[i * 4 + j];
    }
  }
  __syncthreads();
  // the output axis (0: d, 1: w, 2: h) driving source axis r, and its sign
  int col[3];
  float sgn[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    col[r] = s_th[r * 4] != 0.0f ? 0 : (s_th[r * 4 + 1] != 0.0f ? 1 : 2);
    sgn[r] = s_th[r * 4 + col[r]];
  }
  for (int d = t; d < D; d += PM_THREADS)
    s_x[d] = perm_axis<PAD>(perm_coord(d, D, sgn[0], s_th[3], D, ALIGN), D);
  // the output index driving source y (r = 1, size W) and z (r = 2, size H)
  const int yc = col[1], zc = col[2];
  const float ys = sgn[1], zs = sgn[2], yt = s_th[7], zt = s_th[11];
  const int wr = (t / 32) * R, lane = t % 32;  // the warp's first row in a group
  for (int g = blockIdx.x; g < n_groups; g += gridDim.x) {
    const int row0 = g * ROWS;
    const int rows = min(ROWS, H * W - row0);
    __syncthreads();  // the previous group's row tables are read
    if (t < 2 * ROWS) {
      const int j = t % ROWS, r = 1 + t / ROWS;
      const int ri = min(row0 + j, H * W - 1);
      const int w = ri % W, h = ri / W;
      const int c = r == 1 ? yc : zc;
      const int i = c == 1 ? w : h;
      const int n = c == 1 ? W : H;
      const int size = r == 1 ? W : H;
      const PermAxis pa =
          perm_axis<PAD>(perm_coord(i, n, r == 1 ? ys : zs, r == 1 ? yt : zt, size, ALIGN), size);
      if (r == 1)
        s_y[j] = pa;
      else
        s_z[j] = pa;
    }
    __syncthreads();
    if (wr >= rows) continue;
    const int nr = min(R, rows - wr);
    // warp-uniform: every row of the warp on voxel centres along y and z
    bool centre = spec_mode(S0) == BA_NEAREST;
    if (!centre) {
      centre = true;
      for (int r = 0; r < nr; ++r)
        centre = centre && s_y[wr + r].frac == 0.0f && s_z[wr + r].frac == 0.0f;
    }
    for (int d0 = 0; d0 < D; d0 += 128) {
      const int d = d0 + 4 * lane;
      const bool act = d < D;
      const PermX px = perm_x(s_x + (act ? d : 0), D);
      const bool xok = __all_sync(0xFFFFFFFFu, !act || px.base >= 0);
      if (xok && centre)
        perm_rows_fast<S0, S1, R>(a, b, H, W, D, row0 + wr, nr, d, act, px, s_y + wr, s_z + wr,
                                  s_x + (act ? d : 0));
      else
        perm_rows_slow<S0, S1, R>(a, b, H, W, D, row0 + wr, nr, d, act, xok, px, s_y + wr,
                                  s_z + wr, s_x + (act ? d : 0));
    }
  }
}

// ===========================================================================
// TMA-staged signed-permutation resample: the default for signed-permutation
// launches whose H, W and D are at most PT_MAX_DIM (one tensor-map box spans
// a whole D row).  The output is cut into tiles of PT_TR x PT_TR (h, w) rows
// by the whole D extent.  A signed permutation maps a tile's rows onto a
// PT_TR x PT_TR block of source rows, which one cp.async.bulk.tensor load per
// (key, channel) copies into a shared-memory stage (zero-filled outside the
// volume).  A producer warp keeps PT_STAGES loads in flight on mbarriers; four
// consumer warps write the output rows from the stage as 16-byte (fp32) /
// 8-byte (bf16) vectors, reversed for a flip along D.  Voxels off a voxel
// centre take resample3d_perm_kernel's arithmetic: along x, a lerp with the
// neighbouring voxel of the staged row; rows off a centre along y or z (a
// plane or two per element) read their 2 or 4 source rows from global
// memory.  Masked-out elements are the identity copy.  All keys of the launch
// (any mix of modes and dtypes with one padding) go through one launch.
// Every mbarrier wait is bounded (PT_WAIT_NS): a wait that runs out records
// it in g_wait_timeouts (read by ba_wait_status) and the CTA stops, its
// producer first waiting, again bounded, for the loads it issued.
// ===========================================================================
constexpr int PT_TR = 4;                          // tile rows along h and w
constexpr int PT_ROWS = PT_TR * PT_TR;            // output rows per tile
constexpr int PT_CWARPS = 4;                      // consumer warps
constexpr int PT_THREADS = (PT_CWARPS + 1) * 32;  // + the producer warp
#ifndef BA_PT_STAGES
#define BA_PT_STAGES 4
#endif
constexpr int PT_STAGES = BA_PT_STAGES;
constexpr int PT_MAX_DIM = 256;  // tensor-map box extent limit; also the tables
constexpr unsigned long long PT_WAIT_NS = 2000000000ull;

// Bounded device waits that ran out (any kernel of this file); read and
// cleared by ba_wait_status.
__device__ unsigned int g_wait_timeouts;

struct PermTmaArgs {
  CUtensorMap maps[BA_MAX_KEYS];  // key k's (B * C, H, W, D) source, box (1, PT_TR, PT_TR, D)
  ResampleArgs r;
  int32_t stage_bytes;  // one stage: the largest key's box
};

__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return (unsigned)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// true once the barrier's phase of parity `parity` has completed; the
// thread may be suspended in the instruction until then, for at most
// PT_SUSPEND_NS (so waiting warps do not spin through issue slots)
constexpr unsigned PT_SUSPEND_NS = 1000000u;
__device__ __forceinline__ bool mbar_test(uint64_t* bar, unsigned parity) {
  unsigned done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(PT_SUSPEND_NS)
      : "memory");
  return done != 0;
}

// mbar_test until it succeeds or PT_WAIT_NS pass; false when the time ran out
#ifndef BA_PT_BACKOFF_NS
#define BA_PT_BACKOFF_NS 0
#endif
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_test(bar, parity)) {
    if (BA_PT_BACKOFF_NS > 0) __nanosleep(BA_PT_BACKOFF_NS);
    if (global_ns() - t0 > PT_WAIT_NS) return false;
  }
  return true;
}

// One box of a 4-D tensor map into shared memory, completing on `bar`.  The
// innermost coordinate is always 0 here (16-byte aligned), the others may lie
// outside the tensor (those elements read as zero).
__device__ __forceinline__ void tma_load4(void* dst, const CUtensorMap* map, int x, int y, int z,
                                          int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

template <int DT>
__device__ __forceinline__ void lds4(const unsigned char* row, int x, float* v) {
  if (DT == BA_BF16) {
    const uint2 u = *reinterpret_cast<const uint2*>(row + 2 * x);
    v[0] = __uint_as_float(u.x << 16);
    v[1] = __uint_as_float(u.x & 0xFFFF0000u);
    v[2] = __uint_as_float(u.y << 16);
    v[3] = __uint_as_float(u.y & 0xFFFF0000u);
  } else {
    const float4 f = *reinterpret_cast<const float4*>(row + 4 * x);
    v[0] = f.x;
    v[1] = f.y;
    v[2] = f.z;
    v[3] = f.w;
  }
}

template <int DT>
__device__ __forceinline__ float lds1(const unsigned char* row, int x) {
  if (DT == BA_BF16)
    return __uint_as_float((uint32_t)(*reinterpret_cast<const uint16_t*>(row + 2 * x)) << 16);
  return *reinterpret_cast<const float*>(row + 4 * x);
}

// Where a tile's source rows start along source axis y or z: the smaller of
// the nearest indices of the tile's first and last rows along the output axis
// driving it (the permutation is monotone along that axis).
__device__ __forceinline__ int permt_box_start(const PermAxis* tab, int o0, int n) {
  const int last = min(o0 + PT_TR - 1, n - 1);
  return min(tab[o0].near, tab[last].near);
}

// Rows a consumer warp writes for each tile: rows r = warp + PT_CWARPS * i
// of the tile, i < PT_RPW.
constexpr int PT_RPW = PT_ROWS / PT_CWARPS;

// A lane's 4 voxels d .. d+3 of one output row, copied from the staged
// source row: the chunk's bits as they are (a copy keeps NaN payloads),
// reversed for a flip along x.
template <int DT>
__device__ __forceinline__ void permt_chunk(const unsigned char* srow, char* cd, int o,
                                            const PermX& x) {
  if (DT == BA_BF16) {
    uint2 u = *reinterpret_cast<const uint2*>(srow + 2 * x.base);
    if (x.rev) u = make_uint2(__byte_perm(u.y, 0, 0x1032), __byte_perm(u.x, 0, 0x1032));
    *reinterpret_cast<uint2*>(cd + 2 * (int64_t)o) = u;
  } else {
    uint4 u = *reinterpret_cast<const uint4*>(srow + 4 * x.base);
    if (x.rev) u = make_uint4(u.w, u.z, u.y, u.x);
    *reinterpret_cast<uint4*>(cd + 4 * (int64_t)o) = u;
  }
}

// One consumer warp's rows of a tile, one key and channel, from the stage.
// The warp writes output column ow = w0 + warp of the tile, rows
// oh = h0 + i (i < PT_RPW), the i-th starting at orow0 + i * W * D.  srow[i]
// packs the stage row for a nearest key (low byte) and for a bilinear key
// (second byte): 0..PT_ROWS-1, PT_GLOBAL for the global-memory path, PT_NONE
// where the tile has no output row.  PT_GLOBAL rows are left to
// permt_fixups.
constexpr int PT_GLOBAL = 0xFF, PT_NONE = 0xFE;

template <int DT>
__device__ __forceinline__ float permt_tap(const unsigned char* srow, int x, int D) {
  return (unsigned)x < (unsigned)D ? lds1<DT>(srow, x) : 0.0f;
}

// A bilinear key's voxels of the chunk off a centre along x (one position
// per row): the fast kernel's lerp fma(f, hi - lo, lo) over the two source
// voxels of the staged row (zero outside the volume; trilerp2's lerps along y
// and z at fraction 0 return it unchanged), stored over the copied value.
template <int DT>
__device__ __forceinline__ void permt_xfix(const unsigned char* srow, char* cd, int o, int D,
                                           const PermAxis* sx) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const PermAxis ax = sx[j];
    if (ax.frac != 0.0f) {
      const float lo = permt_tap<DT>(srow, ax.lo, D), hi = permt_tap<DT>(srow, ax.lo + 1, D);
      st<DT>(cd, o + j, __fmaf_rn(ax.frac, __fsub_rn(hi, lo), lo));
    }
  }
}

template <int MODE, int DT, int NQ>
__device__ __forceinline__ void permt_rows(const KeyArgs& k, int64_t b, int c, int H, int W,
                                           int D, const unsigned char* stage, const int* srow,
                                           int orow0, const PermX& x0, const PermX& x1,
                                           const PermAxis* s_x, int lane) {
  constexpr int esz = DT == BA_BF16 ? 2 : 4;
  char* cd = (char*)k.dst + ((size_t)b * k.channels + c) * ((size_t)H * W * D) * esz;
  const int d0 = 4 * lane, d1 = d0 + 128, plane = W * D;
#pragma unroll
  for (int i = 0; i < PT_RPW; ++i) {
    const int sr = MODE == BA_NEAREST ? (srow[i] & 0xFF) : ((srow[i] >> 8) & 0xFF);
    if (sr < PT_ROWS) {
      const unsigned char* st = stage + sr * D * esz;
      const int o = orow0 + i * plane;
      if (d0 < D) {
        permt_chunk<DT>(st, cd, o + d0, x0);
        if (MODE != BA_NEAREST && x0.off) permt_xfix<DT>(st, cd, o + d0, D, s_x + d0);
      }
      if (NQ > 1 && d1 < D) {
        permt_chunk<DT>(st, cd, o + d1, x1);
        if (MODE != BA_NEAREST && x1.off) permt_xfix<DT>(st, cd, o + d1, D, s_x + d1);
      }
    }
  }
}

// After a tile's staged items: the warp's rows and chunks the stage did not
// serve, for every key and channel, by resample3d_perm_kernel's
// global-memory path: PT_GLOBAL rows (a bilinear key's rows off a voxel
// centre along y or z, a plane or two per element; rows outside the staged
// block).  Out of line, so the staged loop keeps its registers.
#ifndef BA_PT_FIXUPS_INLINE
#define BA_PT_FIXUPS_INLINE 1
#endif
#if BA_PT_FIXUPS_INLINE
#define BA_PT_FIXUPS_ATTR __forceinline__
#else
#define BA_PT_FIXUPS_ATTR __noinline__
#endif
template <int PAD, int NQ>
__device__ BA_PT_FIXUPS_ATTR void permt_fixups(const ResampleArgs& a, int64_t b, const int* srow,
                                          int orow0, int h0, int ow, int yc, int zc,
                                          const PermAxis* s_x, const PermAxis* s_y,
                                          const PermAxis* s_z, PermX x0, PermX x1, int lane) {
  static_assert(PT_RPW == 4, "four rows per warp");
  const int H = a.H, W = a.W, D = a.D, plane = W * D;
  const int d0 = 4 * lane, d1 = d0 + 128;
  for (int i = 0; i < PT_RPW; ++i) {
    // selects, not indexing, so the rows' codes stay in registers
    const int sv = (i & 2) ? ((i & 1) ? srow[3] : srow[2]) : ((i & 1) ? srow[1] : srow[0]);
    const int sn = sv & 0xFF, sb = (sv >> 8) & 0xFF;
    if (sn == PT_NONE) continue;
    const int oh = h0 + i, o = orow0 + i * plane;
    const PermAxis ay = s_y[yc == 1 ? ow : oh], az = s_z[zc == 1 ? ow : oh];
    for (int ki = 0; ki < a.n_keys; ++ki) {
      const KeyArgs& k = a.keys[ki];
      const bool nearest = k.mode == BA_NEAREST;
      if ((nearest ? sn : sb) != PT_GLOBAL) continue;
      const bool l0 = d0 < D, l1 = NQ > 1 && d1 < D;
      const int esz = k.dtype == BA_BF16 ? 2 : 4;
      for (int c = 0; c < k.channels; ++c) {
        const size_t coff = ((size_t)b * k.channels + c) * ((size_t)H * W * D) * esz;
        const char* cs = (const char*)k.src + coff;
        char* cd = (char*)k.dst + coff;
        switch (k.mode * 2 + k.dtype) {
#define BA_PT_FIX(M, T)                                                                       \
  case M * 2 + T:                                                                             \
    if (l0) perm_row_slow<spec_code(M, PAD, T)>(cs, cd, H, W, D, o + d0, true, x0.base >= 0, \
                                                x0, ay, az, s_x + d0);                        \
    if (l1) perm_row_slow<spec_code(M, PAD, T)>(cs, cd, H, W, D, o + d1, true, x1.base >= 0, \
                                                x1, ay, az, s_x + d1);                        \
    break;
          BA_PT_FIX(BA_BILINEAR, BA_F32)
          BA_PT_FIX(BA_BILINEAR, BA_BF16)
          BA_PT_FIX(BA_NEAREST, BA_F32)
          BA_PT_FIX(BA_NEAREST, BA_BF16)
#undef BA_PT_FIX
          default:
            break;
        }
      }
    }
  }
}

// CTAs per SM the permutation kernel's registers are bounded for.  Measured
// on B200: 5 (72 registers) and 6 (64) were no faster than 4 (96) on a
// four-channel vol + seg permutation and slower on a one-channel flip.
#ifndef BA_PT_MINBLOCKS
#define BA_PT_MINBLOCKS 4
#endif
// NQ: 16-byte chunks per lane and row (1 for D <= 128, 2 up to PT_MAX_DIM)
template <int PAD, int NQ>
__global__ void __launch_bounds__(PT_THREADS, BA_PT_MINBLOCKS)
    resample3d_permt_kernel(const __grid_constant__ PermTmaArgs p) {
  extern __shared__ __align__(128) unsigned char pt_stage[];
  __shared__ PermAxis s_x[PT_MAX_DIM], s_y[PT_MAX_DIM], s_z[PT_MAX_DIM];
  __shared__ __align__(8) uint64_t full[PT_STAGES], empty[PT_STAGES];
  __shared__ float s_th[12];
  const ResampleArgs& a = p.r;
  const bool ALIGN = a.align_corners != 0;
  const int H = a.H, W = a.W, D = a.D;
  const int64_t b = a.b0 + blockIdx.y;
  const bool act = elem_active(a, b);
  const int t = threadIdx.x, warp = t / 32, lane = t % 32;
  if (t < 12) {
    const int i = t / 4, j = t % 4;
    const float* x = elem_xform(a, b);
    if (a.xform_kind == BA_XFORM_AFFINE) {
      // monai_affine_to_theta: theta = P S_norm A S_inv P, P swapping 0 and 2.
      const int pi = 2 - i, pj = (j == 3) ? 3 : 2 - j;
      const float s_j = (pj == 3) ? 1.0f : a.si[pj];
      s_th[t] = (a.sn[pi] * x[pi * 4 + pj]) * s_j;
    } else {
      s_th[t] = x[i * 4 + j];
    }
  } else if (t == 32) {
    for (int i = 0; i < PT_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], PT_CWARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // the output axis (0: d, 1: w, 2: h) driving source axis r, and its sign;
  // a masked-out element is the identity copy
  int col[3];
  float sgn[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    col[r] = s_th[r * 4] != 0.0f ? 0 : (s_th[r * 4 + 1] != 0.0f ? 1 : 2);
    sgn[r] = s_th[r * 4 + col[r]];
  }
  const int yc = act ? col[1] : 1, zc = act ? col[2] : 2;
  const int ny = yc == 1 ? W : H, nz = zc == 1 ? W : H;
  for (int i = t; i < D; i += PT_THREADS)
    s_x[i] = act ? perm_axis<PAD>(perm_coord(i, D, sgn[0], s_th[3], D, ALIGN), D)
                 : PermAxis{i, 0.0f, i};
  for (int i = t; i < ny; i += PT_THREADS)
    s_y[i] = act ? perm_axis<PAD>(perm_coord(i, ny, sgn[1], s_th[7], W, ALIGN), W)
                 : PermAxis{i, 0.0f, i};
  for (int i = t; i < nz; i += PT_THREADS)
    s_z[i] = act ? perm_axis<PAD>(perm_coord(i, nz, sgn[2], s_th[11], H, ALIGN), H)
                 : PermAxis{i, 0.0f, i};
  __syncthreads();
  const int ntw = (W + PT_TR - 1) / PT_TR;
  const int ntiles = ((H + PT_TR - 1) / PT_TR) * ntw;
  if (warp == PT_CWARPS) {
    // producer: one lane issues every load of the CTA's items in order
    if (lane != 0) return;
    bool ok = true;
    int j = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      const int h0 = (tile / ntw) * PT_TR, w0 = (tile % ntw) * PT_TR;
      const int ys = permt_box_start(s_y, yc == 1 ? w0 : h0, ny);
      const int zs = permt_box_start(s_z, zc == 1 ? w0 : h0, nz);
      for (int ki = 0; ok && ki < a.n_keys; ++ki) {
        const KeyArgs& k = a.keys[ki];
        const unsigned bytes = (unsigned)(D * PT_ROWS * (k.dtype == BA_BF16 ? 2 : 4));
        for (int c = 0; c < k.channels; ++c, ++j) {
          const int s = j % PT_STAGES, round = j / PT_STAGES;
          if (!mbar_wait(&empty[s], (unsigned)(round & 1) ^ 1u)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], bytes);
          tma_load4(pt_stage + (size_t)s * p.stage_bytes, &p.maps[ki], 0, ys, zs,
                    (int)(b * k.channels + c), &full[s]);
        }
      }
    }
    if (!ok) atomicOr(&g_wait_timeouts, 1u);
    // every issued load (items 0 .. j-1) lands before the CTA may exit: the
    // last one of stage s is item s + PT_STAGES * ((j - 1 - s) / PT_STAGES)
    for (int s = 0; s < PT_STAGES && s < j; ++s) {
      const int round = (s + PT_STAGES * ((j - 1 - s) / PT_STAGES)) / PT_STAGES;
      if (!mbar_wait(&full[s], (unsigned)(round & 1))) atomicOr(&g_wait_timeouts, 1u);
    }
    return;
  }
  // consumers: the x side of the lane's chunks d = 4 lane and 4 lane + 128,
  // fixed for the element
  const int d0 = 4 * lane, d1 = d0 + 128;
  const PermX x0 = perm_x(s_x + (d0 < D ? d0 : 0), D);
  const PermX x1 = NQ > 1 ? perm_x(s_x + (d1 < D ? d1 : 0), D) : x0;
  const bool xok =
      __all_sync(0xFFFFFFFFu, (d0 >= D || x0.base >= 0) && (NQ == 1 || d1 >= D || x1.base >= 0));
  int j = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int h0 = (tile / ntw) * PT_TR, w0 = (tile % ntw) * PT_TR;
    const int ys = permt_box_start(s_y, yc == 1 ? w0 : h0, ny);
    const int zs = permt_box_start(s_z, zc == 1 ? w0 : h0, nz);
    // the warp's rows of this tile (column ow, rows h0 + i), for nearest and
    // for bilinear keys
    const int ow = w0 + warp;
    const int orow0 = (h0 * W + ow) * D;
    int srow[PT_RPW];
    bool fix = false;  // a row for permt_fixups (warp-uniform)
#pragma unroll
    for (int i = 0; i < PT_RPW; ++i) {
      const int oh = h0 + i;
      srow[i] = PT_NONE | (PT_NONE << 8);
      if (oh < H && ow < W) {
        const PermAxis ay = s_y[yc == 1 ? ow : oh], az = s_z[zc == 1 ? ow : oh];
        const int nyr = ay.near - ys, nzr = az.near - zs;
        const int lyr = ay.lo - ys, lzr = az.lo - zs;
        const int sn = xok && (unsigned)nyr < (unsigned)PT_TR && (unsigned)nzr < (unsigned)PT_TR
                           ? nzr * PT_TR + nyr
                           : PT_GLOBAL;
        const int sb = xok && ay.frac == 0.0f && az.frac == 0.0f &&
                               (unsigned)lyr < (unsigned)PT_TR && (unsigned)lzr < (unsigned)PT_TR
                           ? lzr * PT_TR + lyr
                           : PT_GLOBAL;
        srow[i] = sn | (sb << 8);
        fix = fix || sn == PT_GLOBAL || sb == PT_GLOBAL;
      }
    }
    for (int ki = 0; ki < a.n_keys; ++ki) {
      const KeyArgs& k = a.keys[ki];
      for (int c = 0; c < k.channels; ++c, ++j) {
        const int s = j % PT_STAGES, round = j / PT_STAGES;
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&full[s], (unsigned)(round & 1)));
        if (!ok) {
          if (lane == 0) atomicOr(&g_wait_timeouts, 1u);
          return;
        }
        const unsigned char* stage = pt_stage + (size_t)s * p.stage_bytes;
        switch (k.mode * 2 + k.dtype) {
          case BA_BILINEAR * 2 + BA_F32:
            permt_rows<BA_BILINEAR, BA_F32, NQ>(k, b, c, H, W, D, stage, srow, orow0, x0, x1, s_x,
                                            lane);
            break;
          case BA_BILINEAR * 2 + BA_BF16:
            permt_rows<BA_BILINEAR, BA_BF16, NQ>(k, b, c, H, W, D, stage, srow, orow0, x0, x1, s_x,
                                            lane);
            break;
          case BA_NEAREST * 2 + BA_F32:
            permt_rows<BA_NEAREST, BA_F32, NQ>(k, b, c, H, W, D, stage, srow, orow0, x0, x1, s_x,
                                            lane);
            break;
          case BA_NEAREST * 2 + BA_BF16:
            permt_rows<BA_NEAREST, BA_BF16, NQ>(k, b, c, H, W, D, stage, srow, orow0, x0, x1, s_x,
                                            lane);
            break;
          default:
            break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
    if (fix) permt_fixups<PAD, NQ>(a, b, srow, orow0, h0, ow, yc, zc, s_x, s_y, s_z, x0, x1, lane);
  }
}

// Opt the staged kernel in to its dynamic shared memory once per process
// (needed above 48 KB; idempotent, so concurrent first calls are harmless).
template <int S0, int S1, bool FAST>
void allow_staged_smem(int bytes) {
  static bool done = false;
  if (!done) {
    if (FAST) {
      cudaFuncSetAttribute(resample3d_fast_kernel<S0, S1, false>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      cudaFuncSetAttribute(resample3d_fast_kernel<S0, S1, true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    } else
      cudaFuncSetAttribute(resample3d_staged_kernel<S0, S1>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    done = true;
  }
}

bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
  const char* pa = (const char*)a;
  const char* pb = (const char*)b;
  return pa < pb + nb && pb < pa + na;
}

// ---------------------------------------------------------------------------
// Elastic field composed with a following affine (an extension: the
// reference resamples twice, elastic then affine).  For output voxel p the
// affine maps p into the elastic output's voxel space exactly as
// affine_grid + grid_sample(align_corners=False) would (u); the elastic grid
// F (grid_sample coordinates, align_corners=True, xyz order) is read there
// by trilinear interpolation at u clamped to the volume (uc), and the
// displacement is extended beyond the volume by clamping:
//   G(p) = F~(uc) + (u - uc) / half,   half = max((N-1)/2, 1e-6),
// so a voxel the affine moves out of view still lands outside and takes the
// key's padding when G is sampled.  Elements without the affine take
// G = F; elements without the elastic field take the identity grid for F.
// One thread per output voxel; grid (ceil(HWD / 256), B).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float lerp_rn(float a, float b, float g, float f) {
  return __fadd_rn(__fmul_rn(a, g), __fmul_rn(b, f));
}

// identity grid value of index q along an axis of n (elastic convention)
__device__ __forceinline__ float ident_coord(int q, int n) {
  const float half_lo = __fdiv_rn(__fsub_rn((float)n, 1.0f), 2.0f);
  const float step = __fdiv_rn(__fsub_rn(half_lo, -half_lo), __fsub_rn((float)n, 1.0f));
  const float c0 = linspace_at(-half_lo, half_lo, step, q, n);
  return __fdiv_rn(c0, half_lo < 1e-6f ? 1e-6f : half_lo);
}

__global__ void __launch_bounds__(256)
    compose_field_kernel(const float* __restrict__ field, const float* __restrict__ theta,
                         const uint8_t* __restrict__ mask_field,
                         const uint8_t* __restrict__ mask_affine, int H, int W, int D,
                         float* __restrict__ out) {
  const int64_t b = blockIdx.y;
  const int64_t hwd = (int64_t)H * W * D;
  const int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= hwd) return;
  const int h = (int)(s / ((int64_t)W * D)), w = (int)((s / D) % W), d = (int)(s % D);
  const bool has_field = mask_field == nullptr || mask_field[b] != 0;
  const bool has_affine = mask_affine == nullptr || mask_affine[b] != 0;
  const int n[3] = {D, W, H};  // x, y, z extents
  float* o = out + (b * hwd + s) * 3;
  auto F = [&](int z, int y, int x, int r) -> float {
    if (has_field) return __ldg(field + ((b * H + z) * (int64_t)W * D + (int64_t)y * D + x) * 3 + r);
    return ident_coord(r == 0 ? x : (r == 1 ? y : z), n[r]);
  };
  if (!has_affine) {
#pragma unroll
    for (int r = 0; r < 3; ++r) o[r] = F(h, w, d, r);
    return;
  }
  // affine_grid's coordinates (align_corners=False) and the bmm as the
  // resample kernel computes them: x*t0, fused y and z terms, translation
  const float bx = base_coord(d, D, 0), by = base_coord(w, W, 0), bz = base_coord(h, H, 0);
  const float* t = theta + b * 12;
  float u[3], uc[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const float g = __fadd_rn(
        __fmaf_rn(bz, __ldg(t + r * 4 + 2), __fmaf_rn(by, __ldg(t + r * 4 + 1), __fmul_rn(bx, __ldg(t + r * 4)))),
        __ldg(t + r * 4 + 3));
    // grid_sampler_unnormalize, align_corners=False
    u[r] = __fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(g, 1.0f), (float)n[r]), 1.0f), 0.5f);
    const float hi = (float)(n[r] - 1);
    uc[r] = u[r] != u[r] ? 0.0f : fminf(fmaxf(u[r], 0.0f), hi);  // NaN -> 0
  }
  int i0[3], i1[3];
  float f[3], g1[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    i0[r] = (int)floorf(uc[r]);
    i1[r] = i0[r] + 1 < n[r] ? i0[r] + 1 : i0[r];
    f[r] = __fsub_rn(uc[r], (float)i0[r]);
    g1[r] = __fsub_rn(1.0f, f[r]);
  }
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    // x, then y, then z
    const float c00 = lerp_rn(F(i0[2], i0[1], i0[0], r), F(i0[2], i0[1], i1[0], r), g1[0], f[0]);
    const float c01 = lerp_rn(F(i0[2], i1[1], i0[0], r), F(i0[2], i1[1], i1[0], r), g1[0], f[0]);
    const float c10 = lerp_rn(F(i1[2], i0[1], i0[0], r), F(i1[2], i0[1], i1[0], r), g1[0], f[0]);
    const float c11 = lerp_rn(F(i1[2], i1[1], i0[0], r), F(i1[2], i1[1], i1[0], r), g1[0], f[0]);
    const float c0 = lerp_rn(c00, c01, g1[1], f[1]);
    const float c1 = lerp_rn(c10, c11, g1[1], f[1]);
    const float fi = lerp_rn(c0, c1, g1[2], f[2]);
    const float half_lo = __fdiv_rn(__fsub_rn((float)n[r], 1.0f), 2.0f);
    const float half = half_lo < 1e-6f ? 1e-6f : half_lo;
    o[r] = __fadd_rn(fi, __fdiv_rn(__fsub_rn(u[r], uc[r]), half));
  }
}

// ===========================================================================
// Grid-driven resample (a grid_sample grid B x H x W x D x 3, the elastic
// path).  A warp takes 128 consecutive output voxels (flat index), each lane
// 4 of them 32 apart, so every gather instruction reads 32 consecutive
// voxels' taps (a few sectors for a near-identity map).  The lane's voxels
// are sampled as two packed pairs; every channel of each key is sampled at
// them with one tap base pointer per voxel (constant deltas inside the
// volume).  The arithmetic is resample3d_kernel's operation for operation,
// so results are identical.
// ===========================================================================
constexpr int G4_THREADS = 128;
constexpr int G4_VOX = 4;  // voxels per thread, 32 apart

template <int DT>
__device__ __forceinline__ float ldp(const char* p) {
  if (DT == BA_BF16) return bf16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t*>(p)));
  return __ldg(reinterpret_cast<const float*>(p));
}

// taps8 with one base pointer and constant deltas for an interior footprint
template <int DT>
__device__ __forceinline__ void taps8p(const char* cs, int x0, int y0, int z0, int H, int W, int D,
                                       bool interior, float* v) {
  constexpr int E = DT == BA_BF16 ? 2 : 4;
  if (interior) {
    const char* p = cs + (size_t)((z0 * W + y0) * D + x0) * E;
    const char* py = p + (size_t)D * E;
    const char* pz = p + (size_t)W * D * E;
    const char* pzy = pz + (size_t)D * E;
    v[0] = ldp<DT>(p);
    v[1] = ldp<DT>(p + E);
    v[2] = ldp<DT>(py);
    v[3] = ldp<DT>(py + E);
    v[4] = ldp<DT>(pz);
    v[5] = ldp<DT>(pz + E);
    v[6] = ldp<DT>(pzy);
    v[7] = ldp<DT>(pzy + E);
    return;
  }
  taps8<DT>(cs, x0, y0, z0, H, W, D, false, v);
}

// Trilinear set-up of a voxel pair, as sample_pair forms it.
struct Pair8 {
  Floor2 fx, fy, fz;
  float2 w[8];
  bool ia, ib;
};

template <int PAD, bool ALIGN>
__device__ __forceinline__ Pair8 pair_setup(float2 ix, float2 iy, float2 iz, int H, int W, int D) {
  const float2 px = pad2<PAD, ALIGN>(ix, D);
  const float2 py = pad2<PAD, ALIGN>(iy, W);
  const float2 pz = pad2<PAD, ALIGN>(iz, H);
  Pair8 q;
  q.fx = floor2(px);
  q.fy = floor2(py);
  q.fz = floor2(pz);
  const float2 one = f2(1.0f);
  const float2 wx1 = sub2(px, q.fx.f), wx0 = sub2(add2(q.fx.f, one), px);
  const float2 wy1 = sub2(py, q.fy.f), wy0 = sub2(add2(q.fy.f, one), py);
  const float2 wz1 = sub2(pz, q.fz.f), wz0 = sub2(add2(q.fz.f, one), pz);
  const float2 xy00 = mul2(wx0, wy0), xy10 = mul2(wx1, wy0);
  const float2 xy01 = mul2(wx0, wy1), xy11 = mul2(wx1, wy1);
  q.w[0] = mul2(xy00, wz0);
  q.w[1] = mul2(xy10, wz0);
  q.w[2] = mul2(xy01, wz0);
  q.w[3] = mul2(xy11, wz0);
  q.w[4] = mul2(xy00, wz1);
  q.w[5] = mul2(xy10, wz1);
  q.w[6] = mul2(xy01, wz1);
  q.w[7] = mul2(xy11, wz1);
  q.ia = (unsigned)q.fx.lo < (unsigned)(D - 1) && (unsigned)q.fy.lo < (unsigned)(W - 1) &&
         (unsigned)q.fz.lo < (unsigned)(H - 1);
  q.ib = (unsigned)q.fx.hi < (unsigned)(D - 1) && (unsigned)q.fy.hi < (unsigned)(W - 1) &&
         (unsigned)q.fz.hi < (unsigned)(H - 1);
  return q;
}

template <int DT>
__device__ __forceinline__ float2 pair_interp(const Pair8& q, const char* cs, int H, int W, int D) {
  float va[8], vb[8];
  taps8p<DT>(cs, q.fx.lo, q.fy.lo, q.fz.lo, H, W, D, q.ia, va);
  taps8p<DT>(cs, q.fx.hi, q.fy.hi, q.fz.hi, H, W, D, q.ib, vb);
  // products packed, sums scalar, in torch's tap order
  float2 acc = f2(0.0f);
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const float2 pr = mul2(f2(va[t], vb[t]), q.w[t]);
    acc.x = __fadd_rn(acc.x, pr.x);
    acc.y = __fadd_rn(acc.y, pr.y);
  }
  return acc;
}

// Every channel of key k at the lane's voxels fv[0..3]: pairs (0,1), (2,3),
// coordinates (ix, iy, iz)[p]; a voxel with ok[v] false is not stored.
template <int S, bool ALIGN>
__device__ __forceinline__ void sample_lane(const KeyArgs& k, int64_t b, int H, int W, int D,
                                            int hwd, const int* fv, const bool* ok,
                                            const float2* ix, const float2* iy,
                                            const float2* iz) {
  constexpr int MODE = spec_mode(S), PAD = spec_pad(S), DT = spec_dt(S);
  constexpr int E = DT == BA_BF16 ? 2 : 4;
  const size_t cstride = (size_t)hwd * E;
  const char* src_e = (const char*)k.src + (size_t)b * k.channels * cstride;
  char* dst_e = (char*)k.dst + (size_t)b * k.channels * cstride;
  if (MODE == BA_NEAREST) {
    int o[G4_VOX];
    bool in[G4_VOX];
#pragma unroll
    for (int v = 0; v < G4_VOX; ++v) {
      const int p = v / 2;
      const float2 px = pad2<PAD, ALIGN>(ix[p], D), py = pad2<PAD, ALIGN>(iy[p], W),
                   pz = pad2<PAD, ALIGN>(iz[p], H);
      // nearbyint (round half to even) in one conversion
      const int x = __float2int_rn(v & 1 ? px.y : px.x), y = __float2int_rn(v & 1 ? py.y : py.x),
                z = __float2int_rn(v & 1 ? pz.y : pz.x);
      in[v] = (unsigned)x < (unsigned)D && (unsigned)y < (unsigned)W && (unsigned)z < (unsigned)H;
      o[v] = in[v] ? ((z * W + y) * D + x) * E : 0;
    }
    for (int c = 0; c < k.channels; ++c) {
      const char* cs = src_e + c * cstride;
      char* cd = dst_e + c * cstride;
      float r[G4_VOX];
#pragma unroll
      for (int v = 0; v < G4_VOX; ++v) r[v] = in[v] ? ldp<DT>(cs + o[v]) : 0.0f;
#pragma unroll
      for (int v = 0; v < G4_VOX; ++v)
        if (ok[v]) st<DT>(cd, fv[v], r[v]);
    }
    return;
  }
  // one pair's set-up live at a time: the kernel runs 8 CTAs per SM (64
  // registers), the occupancy that hides the gathers' latency best
  static_assert(G4_VOX == 4, "two pairs per lane");
#pragma unroll 1
  for (int p = 0; p < 2; ++p) {
    // selects, not indexing, so the lane's values stay in registers
    const Pair8 q = pair_setup<PAD, ALIGN>(p ? ix[1] : ix[0], p ? iy[1] : iy[0],
                                           p ? iz[1] : iz[0], H, W, D);
    const int fa = p ? fv[2] : fv[0], fb = p ? fv[3] : fv[1];
    const bool oa = p ? ok[2] : ok[0], ob = p ? ok[3] : ok[1];
    for (int c = 0; c < k.channels; ++c) {
      const float2 r = pair_interp<DT>(q, src_e + c * cstride, H, W, D);
      char* cd = dst_e + c * cstride;
      if (oa) st<DT>(cd, fa, r.x);
      if (ob) st<DT>(cd, fb, r.y);
    }
  }
}

template <int S0, int S1>
__global__ void __launch_bounds__(G4_THREADS, 8) resample3d_grid4_kernel(const __grid_constant__ ResampleArgs a) {
  const int H = a.H, W = a.W, D = a.D;
  const int hwd = H * W * D;
  const int lane = threadIdx.x & 31;
  const int f0 = (int)blockIdx.x * (G4_THREADS * G4_VOX) + (int)(threadIdx.x >> 5) * 32 * G4_VOX + lane;
  if (f0 >= hwd) return;
  const int64_t b = a.b0 + blockIdx.y;
  int fv[G4_VOX];
  bool ok[G4_VOX];
#pragma unroll
  for (int v = 0; v < G4_VOX; ++v) {
    ok[v] = f0 + 32 * v < hwd;
    fv[v] = ok[v] ? f0 + 32 * v : f0;  // a voxel past the end recomputes f0, unstored
  }
  if (!elem_active(a, b)) {
    // the reference's torch.where keeps a masked-out element
    for (int ki = 0; ki < a.n_keys; ++ki) {
      const KeyArgs& k = a.keys[ki];
      for (int c = 0; c < k.channels; ++c) {
        const int64_t base = ((int64_t)b * k.channels + c) * hwd;
#pragma unroll
        for (int v = 0; v < G4_VOX; ++v)
          if (ok[v]) {
            if (k.dtype == BA_BF16)
              ((uint16_t*)k.dst)[base + fv[v]] = __ldg((const uint16_t*)k.src + base + fv[v]);
            else
              ((float*)k.dst)[base + fv[v]] = __ldg((const float*)k.src + base + fv[v]);
          }
      }
    }
    return;
  }
  float g[3][G4_VOX];
#pragma unroll
  for (int v = 0; v < G4_VOX; ++v) {
    const float* gp = a.xform + ((int64_t)b * hwd + fv[v]) * 3;
#pragma unroll
    for (int r = 0; r < 3; ++r) g[r][v] = __ldg(gp + r);
  }
  const float fD = (float)D, fW = (float)W, fH = (float)H;
  float2 ix[G4_VOX / 2], iy[G4_VOX / 2], iz[G4_VOX / 2];
  if (a.align_corners) {
#pragma unroll
    for (int p = 0; p < G4_VOX / 2; ++p) {
      ix[p] = unnormalize2<true>(f2(g[0][2 * p], g[0][2 * p + 1]), fD);
      iy[p] = unnormalize2<true>(f2(g[1][2 * p], g[1][2 * p + 1]), fW);
      iz[p] = unnormalize2<true>(f2(g[2][2 * p], g[2][2 * p + 1]), fH);
    }
    sample_lane<S0, true>(a.keys[0], b, H, W, D, hwd, fv, ok, ix, iy, iz);
    if (S1 >= 0) sample_lane<(S1 < 0 ? 0 : S1), true>(a.keys[1], b, H, W, D, hwd, fv, ok, ix, iy, iz);
  } else {
    const bool pD = (D & (D - 1)) == 0, pW = (W & (W - 1)) == 0, pH = (H & (H - 1)) == 0;
    auto un = [](float2 c, float size, bool pow2) {
      return pow2 ? unnormalize2_pow2(c, size) : unnormalize2<false>(c, size);
    };
#pragma unroll
    for (int p = 0; p < G4_VOX / 2; ++p) {
      ix[p] = un(f2(g[0][2 * p], g[0][2 * p + 1]), fD, pD);
      iy[p] = un(f2(g[1][2 * p], g[1][2 * p + 1]), fW, pW);
      iz[p] = un(f2(g[2][2 * p], g[2][2 * p + 1]), fH, pH);
    }
    sample_lane<S0, false>(a.keys[0], b, H, W, D, hwd, fv, ok, ix, iy, iz);
    if (S1 >= 0) sample_lane<(S1 < 0 ? 0 : S1), false>(a.keys[1], b, H, W, D, hwd, fv, ok, ix, iy, iz);
  }
}

}  // namespace
}  // namespace ba

namespace ba {
namespace {
int sm_count_rs() {
  static int cached = 0;
  if (cached == 0) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
      cached = n;
    else
      cached = 148;
  }
  return cached;
}

// True when every active element of a host-parameter launch maps by a
// signed permutation that resample3d_perm_kernel takes: theta's 3x3 part
// (derived from the affine with the kernel's own arithmetic) one +-1 per row
// and column, no translation, source x driven by output D, and a swapped
// (H, W) plane square.
bool perm_chunk(const ResampleArgs& a, int64_t nb) {
  if (!a.inline_params || a.xform_kind == BA_XFORM_GRID) return false;
  if (a.D % 4 != 0 || a.D > PM_MAX_D) return false;
  for (int64_t i = 0; i < nb; ++i) {
    if (!a.inl_mask[i]) continue;
    const float* x = a.inl_xform + i * a.xform_stride;
    float th[12];
    for (int t = 0; t < 12; ++t) {
      const int r = t / 4, j = t % 4;
      if (a.xform_kind == BA_XFORM_AFFINE) {
        const int pi = 2 - r, pj = (j == 3) ? 3 : 2 - j;
        const float s_j = (pj == 3) ? 1.0f : a.si[pj];
        th[t] = (a.sn[pi] * x[pi * 4 + pj]) * s_j;
      } else {
        th[t] = x[r * 4 + j];
      }
    }
    int used = 0;
    for (int r = 0; r < 3; ++r) {
      int nz = 0, c = -1;
      for (int j = 0; j < 3; ++j)
        if (th[r * 4 + j] != 0.0f) {
          ++nz;
          c = j;
        }
      if (nz != 1 || (th[r * 4 + c] != 1.0f && th[r * 4 + c] != -1.0f) || th[r * 4 + 3] != 0.0f)
        return false;
      if (used & (1 << c)) return false;
      used |= 1 << c;
      if (r == 0 && c != 0) return false;        // x from d
      if (r != 0 && c != r && a.H != a.W) return false;  // a swapped plane is square
    }
  }
  return true;
}

// cuTensorMapEncodeTiled from the driver the runtime loaded (no link-time
// dependency on libcuda); null when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    else
      cudaGetLastError();
  });
  return fn;
}

// Tensor maps of recent sources (a map depends only on the address, dtype
// and shape, so a cached one stays valid for any buffer at that address and
// shape): a Compose step resamples the same pipeline buffers every call, and
// encoding costs a driver call per key.  `make` encodes a missing one.
template <class F>
bool cached_tensor_map(const void* src, int dtype, const cuuint64_t* dims, F make,
                       CUtensorMap* out) {
  struct Entry {
    const void* src;
    int dtype;
    cuuint64_t dims[4];
    int dev;
    CUtensorMap map;
  };
  static std::mutex mu;
  static Entry cache[16];
  static int used = 0, next = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> g(mu);
    for (int i = 0; i < used; ++i) {
      const Entry& e = cache[i];
      if (e.src == src && e.dtype == dtype && e.dev == dev &&
          memcmp(e.dims, dims, sizeof(e.dims)) == 0) {
        *out = e.map;
        return true;
      }
    }
  }
  if (!make(out)) return false;
  std::lock_guard<std::mutex> g(mu);
  Entry& e = cache[next];
  e.src = src;
  e.dtype = dtype;
  memcpy(e.dims, dims, sizeof(e.dims));
  e.dev = dev;
  e.map = *out;
  next = (next + 1) % 16;
  used = std::max(used, next == 0 ? 16 : next);
  return true;
}

// The TMA-staged permutation kernel for a launch whose active elements are
// all signed permutations (perm_chunk), when every key qualifies: one
// padding (zeros or border) for all keys, bilinear keys only outside the
// exact mode, H, W, D <= PT_MAX_DIM, rows a multiple of 16 bytes, 16-byte
// aligned tensors.  Returns false (nothing launched) otherwise.
bool launch_perm_tma(const ba_resample_desc& d, const ResampleArgs& a, int64_t nb, bool exact,
                     cudaStream_t st) {
  if (!a.inline_params || a.xform_kind == BA_XFORM_GRID) return false;
  if (d.D > PT_MAX_DIM || d.H > PT_MAX_DIM || d.W > PT_MAX_DIM) return false;
  const int pad = a.keys[0].padding;
  if (pad == BA_PAD_REFLECTION) return false;
  int stage_bytes = 0;
  for (int i = 0; i < a.n_keys; ++i) {
    const KeyArgs& k = a.keys[i];
    const int esz = k.dtype == BA_BF16 ? 2 : 4;
    if (k.padding != pad || (exact && k.mode != BA_NEAREST)) return false;
    if ((d.D * esz) % 16 != 0 || ((uintptr_t)k.src % 16) != 0 || ((uintptr_t)k.dst % 16) != 0)
      return false;
    if (d.batch * k.channels > INT32_MAX) return false;
    stage_bytes = std::max(stage_bytes, (int)d.D * PT_ROWS * esz);
  }
  if (!perm_chunk(a, nb)) return false;
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  PermTmaArgs p;
  memset(&p, 0, sizeof(p));
  for (int i = 0; i < a.n_keys; ++i) {
    const KeyArgs& k = a.keys[i];
    if (k.channels == 0) continue;  // no items: the map is never read
    const cuuint64_t esz = k.dtype == BA_BF16 ? 2 : 4;
    const cuuint64_t dims[4] = {(cuuint64_t)d.D, (cuuint64_t)d.W, (cuuint64_t)d.H,
                                (cuuint64_t)(d.batch * k.channels)};
    const cuuint64_t strides[3] = {(cuuint64_t)d.D * esz, (cuuint64_t)(d.W * d.D) * esz,
                                   (cuuint64_t)(d.H * d.W * d.D) * esz};
    const cuuint32_t box[4] = {(cuuint32_t)d.D, PT_TR, PT_TR, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (!cached_tensor_map(k.src, k.dtype, dims, [&](CUtensorMap* m) {
          return encode(m,
                        k.dtype == BA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        4, const_cast<void*>(k.src), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        }, &p.maps[i]))
      return false;
  }
  p.r = a;
  p.stage_bytes = stage_bytes;
  const int smem = PT_STAGES * stage_bytes;
  const int64_t ntiles = ((d.H + PT_TR - 1) / PT_TR) * ((d.W + PT_TR - 1) / PT_TR);
  // one wave: as many CTAs as fit on the SMs at once (registers and this
  // stage size decide how many per SM), spread over the launch's elements,
  // each walking tiles
  // dynamic shared memory each instantiation allows (with the 9 KB of
  // static tables, even 48 KB of stages needs the opt-in)
  static int opted[4] = {0, 0, 0, 0};
  const int nq = d.D <= 128 ? 1 : 2;
  const int which = (pad == BA_PAD_BORDER ? 2 : 0) + (nq - 1);
  static int occ_smem[4] = {-1, -1, -1, -1}, occ[4] = {1, 1, 1, 1};  // last query per kernel
  auto grid_for = [&](const void* fn) {
    if (occ_smem[which] != smem) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, PT_THREADS, smem) !=
              cudaSuccess ||
          per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
      }
      occ[which] = per_sm;
      occ_smem[which] = smem;
    }
    const int per_sm = occ[which];
    const int64_t ctas = (int64_t)per_sm * sm_count_rs();
    const int64_t per_elem = std::max<int64_t>(1, ctas / nb);
    return dim3((unsigned)std::min<int64_t>(ntiles, per_elem), (unsigned)nb);
  };
  switch (which) {
#define BA_PT_LAUNCH(I, P, Q)                                                         \
  case I:                                                                             \
    if (smem > opted[I]) {                                                            \
      cudaFuncSetAttribute(resample3d_permt_kernel<P, Q>,                             \
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);        \
      opted[I] = smem;                                                                \
    }                                                                                 \
    resample3d_permt_kernel<P, Q><<<grid_for((const void*)resample3d_permt_kernel<P, Q>), \
                                    PT_THREADS, smem, st>>>(p);                       \
    break;
    BA_PT_LAUNCH(0, BA_PAD_ZEROS, 1)
    BA_PT_LAUNCH(1, BA_PAD_ZEROS, 2)
    BA_PT_LAUNCH(2, BA_PAD_BORDER, 1)
    BA_PT_LAUNCH(3, BA_PAD_BORDER, 2)
#undef BA_PT_LAUNCH
    default:
      return false;
  }
  return true;
}

// Launches of one resample over elements a.b0 .. a.b0 + nb - 1: the kernel
// each key group takes (TMA-staged row copies for signed permutations,
// staged / fast for affine maps with a bilinear key, grid kernel for grid
// maps, global-gather kernel otherwise).
// Keys whose min/max the staged affine kernel folded in one launch_resample
// call (by output pointer).
struct FoldLog {
  const void* dst[BA_MAX_KEYS];
  int n = 0;
  void add(const void* p) {
    if (n < BA_MAX_KEYS) dst[n++] = p;
  }
  bool has(const void* p) const {
    for (int i = 0; i < n; ++i)
      if (dst[i] == p) return true;
    return false;
  }
};

ba_status launch_resample(const ba_resample_desc& d, ResampleArgs& a, int64_t nb,
                          cudaStream_t st, FoldLog& folded) {
  const int64_t hwd = d.H * d.W * d.D;
  const int tiles_d = (int)((d.D + BD - 1) / BD);
  const int64_t gx = (int64_t)tiles_d * ((d.W + TY - 1) / TY);
  const int64_t gy = (d.H + TZ * NB - 1) / (TZ * NB);
  BA_REQUIRE(gx <= INT32_MAX && gy <= 65535, "ba_resample3d: spatial extent too large");
  const dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)nb);
  auto code = [](const KeyArgs& k) { return spec_code(k.mode, k.padding, k.dtype); };
  // The staged kernel serves a bilinear key (zeros or border padding) of an
  // affine map whose rows start on 16-byte (fp32) or 8-byte (bf16) boundaries.
  auto stageable = [&](const KeyArgs& k) {
    const uintptr_t align = k.dtype == BA_BF16 ? 8 : 16;
    return k.mode == BA_BILINEAR && k.padding != BA_PAD_REFLECTION &&
           a.xform_kind != BA_XFORM_GRID && (d.D % 4) == 0 && ((uintptr_t)k.src % align) == 0;
  };
  const int st_tiles = (int)(((d.D + ST_TD - 1) / ST_TD) * ((d.W + ST_TW - 1) / ST_TW));
  const dim3 st_grid((unsigned)st_tiles, (unsigned)((d.H + ST_TH - 1) / ST_TH), (unsigned)nb);
  const int st_smem = ST_MAX_FLOATS * (int)sizeof(float);
  const int fs_smem = FS_MAX_FLOATS * (int)sizeof(float);
  // returns false when (s0, s1) has no staged instantiation
  const bool exact = (d.flags & BA_RESAMPLE_EXACT) != 0;
  auto launch_staged = [&](const ResampleArgs& args, int s0, int s1) -> bool {
    if (!exact && args.keys[0].minmax != nullptr) folded.add(args.keys[0].dst);
    switch (s0 * 16 + (s1 + 1)) {
#define BA_ST(S0, S1)                                                                \
  case S0 * 16 + (S1 + 1):                                                           \
    if (exact) {                                                                     \
      allow_staged_smem<S0, S1, false>(st_smem);                                     \
      resample3d_staged_kernel<S0, S1><<<st_grid, ST_THREADS, st_smem, st>>>(args);  \
    } else {                                                                         \
      allow_staged_smem<S0, S1, true>(fs_smem);                                      \
      if (args.keys[0].minmax != nullptr)                                            \
        resample3d_fast_kernel<S0, S1, true><<<st_grid, ST_THREADS, fs_smem, st>>>(args); \
      else                                                                           \
        resample3d_fast_kernel<S0, S1, false><<<st_grid, ST_THREADS, fs_smem, st>>>(args); \
    }                                                                                \
    return true;
#define BA_ST_KEY(P, T0)                                                               \
  BA_ST(spec_code(BA_BILINEAR, P, T0), -1)                                             \
  BA_ST(spec_code(BA_BILINEAR, P, T0), spec_code(BA_NEAREST, P, BA_F32))               \
  BA_ST(spec_code(BA_BILINEAR, P, T0), spec_code(BA_NEAREST, P, BA_BF16))
      BA_ST_KEY(BA_PAD_ZEROS, BA_F32)
      BA_ST_KEY(BA_PAD_ZEROS, BA_BF16)
      BA_ST_KEY(BA_PAD_BORDER, BA_F32)
      BA_ST_KEY(BA_PAD_BORDER, BA_BF16)
#undef BA_ST_KEY
#undef BA_ST
      default:
        return false;
    }
  };
  // Signed permutations: the row-copy kernel, keys with zeros or border
  // padding whose rows are vector-aligned.
  auto perm_ok = [&](const KeyArgs& k) {
    const uintptr_t align = k.dtype == BA_BF16 ? 8 : 16;
    return k.padding != BA_PAD_REFLECTION && ((uintptr_t)k.src % align) == 0 &&
           ((uintptr_t)k.dst % align) == 0;
  };
  // about four CTAs per SM over the launch's elements, each walking row
  // groups; single-channel launches take 4 rows per warp
  auto launch_perm = [&](const ResampleArgs& args, int s0, int s1) -> bool {
    int nc = 0;
    for (int i = 0; i < args.n_keys; ++i) nc = std::max(nc, args.keys[i].channels);
    const int rpw = nc == 1 ? 4 : 1;
    const int64_t rows = (int64_t)PM_WARPS * rpw;
    const int64_t groups = (d.H * d.W + rows - 1) / rows;
    const int64_t per_elem = std::max<int64_t>(1, (4 * (int64_t)sm_count_rs() + nb - 1) / nb);
    const dim3 grid_pm((unsigned)std::min<int64_t>(groups, per_elem), (unsigned)nb);
    switch (s0 * 16 + (s1 + 1)) {
#define BA_PM(S0, S1)                                                                  \
  case S0 * 16 + (S1 + 1):                                                             \
    if (rpw == 4)                                                                      \
      resample3d_perm_kernel<S0, S1, 4><<<grid_pm, PM_THREADS, 0, st>>>(args);         \
    else                                                                               \
      resample3d_perm_kernel<S0, S1, 1><<<grid_pm, PM_THREADS, 0, st>>>(args);         \
    return true;
#define BA_PM_PAD(P)                                                                \
  BA_PM(spec_code(BA_BILINEAR, P, BA_F32), -1)                                      \
  BA_PM(spec_code(BA_BILINEAR, P, BA_BF16), -1)                                     \
  BA_PM(spec_code(BA_NEAREST, P, BA_F32), -1)                                       \
  BA_PM(spec_code(BA_NEAREST, P, BA_BF16), -1)                                      \
  BA_PM(spec_code(BA_BILINEAR, P, BA_F32), spec_code(BA_NEAREST, P, BA_F32))        \
  BA_PM(spec_code(BA_BILINEAR, P, BA_F32), spec_code(BA_NEAREST, P, BA_BF16))       \
  BA_PM(spec_code(BA_BILINEAR, P, BA_BF16), spec_code(BA_NEAREST, P, BA_F32))       \
  BA_PM(spec_code(BA_BILINEAR, P, BA_BF16), spec_code(BA_NEAREST, P, BA_BF16))
      BA_PM_PAD(BA_PAD_ZEROS)
      BA_PM_PAD(BA_PAD_BORDER)
#undef BA_PM_PAD
#undef BA_PM
      default:
        return false;
    }
  };
  // Signed permutations of every key in one TMA-staged launch.
  if (launch_perm_tma(d, a, nb, exact, st)) return check_launch("ba_resample3d");
  // Grid maps take the lane-per-voxel grid kernel.
  const bool grid4 = a.xform_kind == BA_XFORM_GRID;
  const dim3 g4_grid((unsigned)((hwd + G4_THREADS * G4_VOX - 1) / (G4_THREADS * G4_VOX)),
                     (unsigned)nb);
  // vol (bilinear) + seg (nearest) with one padding: one fused launch
#ifndef BA_RS_FUSE_PAIR
#define BA_RS_FUSE_PAIR 1
#endif
  if (BA_RS_FUSE_PAIR && a.n_keys == 2) {
    KeyArgs k0 = a.keys[0], k1 = a.keys[1];
    if (k0.mode == BA_NEAREST && k1.mode == BA_BILINEAR) {
      a.keys[0] = k1;
      a.keys[1] = k0;
      k0 = a.keys[0];
      k1 = a.keys[1];
    }
    if (!exact && perm_ok(a.keys[0]) && perm_ok(a.keys[1]) && k1.mode == BA_NEAREST &&
        k0.padding == k1.padding && perm_chunk(a, nb) && launch_perm(a, code(k0), code(k1)))
      return check_launch("ba_resample3d");
    if (k0.mode == BA_BILINEAR && k1.mode == BA_NEAREST && k0.padding == k1.padding &&
        stageable(k0) && launch_staged(a, code(k0), code(k1)))
      return check_launch("ba_resample3d");
    if (k0.mode == BA_BILINEAR && k1.mode == BA_NEAREST && k0.padding == k1.padding) {
      bool launched = true;
      switch (code(k0) * 16 + code(k1)) {
#define BA_PAIR(P, T0, T1)                                                                 \
  case spec_code(BA_BILINEAR, P, T0) * 16 + spec_code(BA_NEAREST, P, T1):                  \
    if (grid4)                                                                             \
      resample3d_grid4_kernel<spec_code(BA_BILINEAR, P, T0), spec_code(BA_NEAREST, P, T1)> \
          <<<g4_grid, G4_THREADS, 0, st>>>(a);                                             \
    else                                                                                   \
      resample3d_kernel<spec_code(BA_BILINEAR, P, T0), spec_code(BA_NEAREST, P, T1)>       \
          <<<grid, NTHREADS, 0, st>>>(a);                                                  \
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
  // a nearest key reads the same voxels in both modes, so its permutations
  // take the row-copy kernel in the exact mode too
  const bool perm = perm_chunk(a, nb);
  for (int i = 0; i < a.n_keys; ++i) {
    one.keys[0] = a.keys[i];
    if (perm && (!exact || one.keys[0].mode == BA_NEAREST) && perm_ok(one.keys[0]) &&
        launch_perm(one, code(one.keys[0]), -1)) {
      const ba_status s1 = check_launch("ba_resample3d");
      if (s1 != BA_OK) return s1;
      continue;
    }
    if (stageable(one.keys[0]) && launch_staged(one, code(one.keys[0]), -1)) {
      const ba_status s1 = check_launch("ba_resample3d");
      if (s1 != BA_OK) return s1;
      continue;
    }
    switch (code(one.keys[0])) {
#define BA_ONE(S)                                                      \
  case S:                                                              \
    if (grid4)                                                         \
      resample3d_grid4_kernel<S, -1><<<g4_grid, G4_THREADS, 0, st>>>(one); \
    else                                                               \
      resample3d_kernel<S, -1><<<grid, NTHREADS, 0, st>>>(one);        \
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
  BA_REQUIRE((d.flags & ~(BA_RESAMPLE_EXACT | BA_RESAMPLE_HOST_PARAMS)) == 0,
             "ba_resample3d: unknown flags 0x%x", d.flags);
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
    a.keys[i].minmax = k.minmax;
    if (k.minmax != nullptr)
      BA_REQUIRE(((uintptr_t)k.minmax % 4) == 0, "ba_resample3d: key %d minmax not 4-byte aligned",
                 i);
  }
  if (d.batch == 0) return BA_OK;
  const cudaStream_t st = (cudaStream_t)stream;
  // min/max outputs: reset, folded by the staged affine kernel as it writes,
  // reduced from the output by the other paths
  for (int i = 0; i < d.n_keys; ++i)
    if (a.keys[i].minmax != nullptr && a.keys[i].channels > 0) {
      const ba_status s = minmax_keys_init(a.keys[i].minmax, d.batch * a.keys[i].channels, st);
      if (s != BA_OK) return s;
    }
  int launches = 0, fold_count[BA_MAX_KEYS] = {0};
  auto run = [&](int64_t nb) -> ba_status {
    FoldLog folded;
    const ba_status s = launch_resample(d, a, nb, st, folded);
    ++launches;
    for (int i = 0; i < d.n_keys; ++i)
      if (folded.has(d.keys[i].dst)) ++fold_count[i];
    return s;
  };
  auto finish = [&]() -> ba_status {
    for (int i = 0; i < d.n_keys; ++i) {
      const ba_resample_key& k = d.keys[i];
      if (k.minmax == nullptr || k.channels == 0 || fold_count[i] == launches) continue;
      const ba_status s = minmax_keys_fold(k.dst, k.dtype, d.batch * k.channels, hwd, k.minmax, st);
      if (s != BA_OK) return s;
    }
    return BA_OK;
  };
  if (!(d.flags & BA_RESAMPLE_HOST_PARAMS)) {
    const ba_status s = run(d.batch);
    return s != BA_OK ? s : finish();
  }
  // host parameters: each launch of up to RS_INLINE_B elements carries their
  // transform and mask in its kernel parameters (read here, before return)
  BA_REQUIRE(d.xform_kind == BA_XFORM_GRID || d.xform_stride <= 16,
             "ba_resample3d: host xform_stride %lld > 16", (long long)d.xform_stride);
  a.inline_params = 1;
  for (int64_t b0 = 0; b0 < d.batch; b0 += RS_INLINE_B) {
    const int64_t nb = std::min<int64_t>(RS_INLINE_B, d.batch - b0);
    a.b0 = b0;
    for (int64_t i = 0; i < nb; ++i) {
      a.inl_mask[i] = d.mask == nullptr ? 1 : (d.mask[b0 + i] != 0);
      if (d.xform_kind != BA_XFORM_GRID)
        memcpy(a.inl_xform + i * d.xform_stride, d.xform + (b0 + i) * d.xform_stride,
               (size_t)d.xform_stride * sizeof(float));
    }
    const ba_status s = run(nb);
    if (s != BA_OK) return s;
  }
  return finish();
}

extern "C" ba_status ba_compose_field(const float* field, const float* theta,
                                      const uint8_t* mask_field, const uint8_t* mask_affine,
                                      int64_t batch, int64_t H, int64_t W, int64_t D, float* grid,
                                      ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(batch >= 0 && H > 0 && W > 0 && D > 0, "ba_compose_field: bad shape");
  BA_REQUIRE(batch <= 65535, "ba_compose_field: batch exceeds 65535");
  BA_REQUIRE(H * W * D < ((int64_t)1 << 31), "ba_compose_field: volume exceeds 2^31 voxels");
  if (batch == 0) return BA_OK;
  BA_REQUIRE(field && theta && grid, "ba_compose_field: NULL pointer");
  const int64_t hwd = H * W * D;
  dim3 g((unsigned)((hwd + 255) / 256), (unsigned)batch);
  compose_field_kernel<<<g, 256, 0, (cudaStream_t)stream>>>(field, theta, mask_field, mask_affine,
                                                          (int)H, (int)W, (int)D, grid);
  return check_launch("ba_compose_field");
}

extern "C" ba_status ba_wait_status(ba_stream_t stream) {
  using namespace ba;
  clear_error();
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) {
    set_error("ba_wait_status: %s", cudaGetErrorString(e));
    return BA_ECUDA;
  }
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v));
  if (e != cudaSuccess) {
    set_error("ba_wait_status: %s", cudaGetErrorString(e));
    return BA_ECUDA;
  }
  if (v == 0) return BA_OK;
  const unsigned int zero = 0;
  cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(zero));
  set_error("ba_wait_status: a bounded device wait ran out of time; the output of the kernel "
            "that recorded it is incomplete");
  return BA_ETIMEOUT;
}
