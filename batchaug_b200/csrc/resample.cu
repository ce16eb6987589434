// Fused 3-D resample: one kernel per Compose materialisation.
//
// Replaces batchaug/compose.py:71-110 (_materialize: monai_affine_to_theta,
// F.affine_grid, F.grid_sample on an fp32 copy, .to(dtype), torch.where) and
// the eager applies of RandAffine (affine.py:284-317), Rand3DElastic
// (elastic.py:101-125) and RandRotate90's non-square fallback
// (rotate90.py:100-112).
//
// Design (B200): no grid tensor and no fp32 copy of the input ever reach
// HBM.  Each thread owns VEC output voxels of one row along D (the
// contiguous axis), derives their source coordinates in registers from the
// element's theta (computed once per CTA in shared memory, straight from the
// MONAI affine when given one), and for every key of the group and every
// channel gathers the 8 trilinear taps (1 for nearest) through the read-only
// cache and blends them.  A CTA covers a compact 32(D) x 4(W) x 4(H) output
// brick so that its source footprint stays in L1; the input of an element
// fits in the 126 MB L2, so HBM sees each input byte about once.  Masked-out
// elements take a plain copy.
//
// Arithmetic reproduces torch's CPU affine_grid and grid_sample bit for bit:
// the base grid is torch.linspace's two-sided fused formula scaled by
// (N-1)/N, the bmm with theta is the fused chain MKL produces, and the
// unnormalise / clip / reflect / trilinear steps round exactly where torch's
// scalar code rounds (this file is compiled with -fmad=false).
#include <stdio.h>

#include "ba_common.cuh"

namespace ba {
namespace {

constexpr int TX = 8;  // threads along D (each VEC voxels)
constexpr int TY = 4;  // threads along W
constexpr int TZ = 4;  // threads along H
constexpr int NTHREADS = TX * TY * TZ;

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

// affine_grid's linspace_from_neg_one.
__device__ __forceinline__ float base_coord(int i, int n, int align_corners) {
  if (n <= 1) return 0.0f;
  float step = 2.0f / (float)(n - 1);
  float r = linspace_at(-1.0f, 1.0f, step, i, n);
  if (!align_corners) r = (r * (float)(n - 1)) / (float)n;
  return r;
}

__device__ __forceinline__ float unnormalize(float coord, int size, int align_corners) {
  if (align_corners) return ((coord + 1.0f) / 2.0f) * (float)(size - 1);
  return ((coord + 1.0f) * (float)size - 1.0f) / 2.0f;
}

// std::min(size-1, std::max(in, 0)) with std's argument order, so that a
// NaN coordinate clips to size-1 exactly as torch's sampler does.
__device__ __forceinline__ float clip_coord(float in, int size) {
  float lo = (in < 0.0f) ? 0.0f : in;
  float hi = (float)(size - 1);
  return (lo < hi) ? lo : hi;
}

__device__ __forceinline__ float reflect_coord(float in, int twice_low, int twice_high) {
  if (twice_low == twice_high) return 0.0f;
  float mn = (float)twice_low / 2.0f;
  float span = (float)(twice_high - twice_low) / 2.0f;
  in = fabsf(in - mn);
  float extra = fmodf(in, span);
  int flips = (int)floorf(in / span);
  if ((flips & 1) == 0) return extra + mn;
  return span - extra + mn;
}

// Padding transform of an unnormalised coordinate, then the guard torch's
// CUDA sampler applies before converting to an integer index (non-finite or
// huge coordinates become -100, i.e. out of bounds).
__device__ __forceinline__ float pad_coord(float coord, int size, int padding, int align_corners) {
  if (padding == BA_PAD_BORDER) {
    coord = clip_coord(coord, size);
  } else if (padding == BA_PAD_REFLECTION) {
    coord = align_corners ? reflect_coord(coord, 0, 2 * (size - 1))
                          : reflect_coord(coord, -1, 2 * size - 1);
    coord = clip_coord(coord, size);
  }
  if (!(fabsf(coord) < 1.0e9f)) coord = -100.0f;
  return coord;
}

// Precomputed sampling footprint of one output voxel for one key.
struct Tap8 {
  int32_t off[8];
  float w[8];
  uint32_t valid;  // bit k: tap k in bounds
};

__device__ __forceinline__ void trilinear_footprint(float ix, float iy, float iz, int H, int W,
                                                    int D, Tap8& t) {
  float x0f = floorf(ix), y0f = floorf(iy), z0f = floorf(iz);
  int x0 = (int)x0f, y0 = (int)y0f, z0 = (int)z0f;
  int x1 = x0 + 1, y1 = y0 + 1, z1 = z0 + 1;
  float wx0 = (float)x1 - ix, wx1 = ix - (float)x0;
  float wy0 = (float)y1 - iy, wy1 = iy - (float)y0;
  float wz0 = (float)z1 - iz, wz1 = iz - (float)z0;
  // torch's corner order tnw, tne, tsw, tse, bnw, bne, bsw, bse with each
  // weight a left-to-right product (x * y) * z.
  t.w[0] = wx0 * wy0 * wz0;
  t.w[1] = wx1 * wy0 * wz0;
  t.w[2] = wx0 * wy1 * wz0;
  t.w[3] = wx1 * wy1 * wz0;
  t.w[4] = wx0 * wy0 * wz1;
  t.w[5] = wx1 * wy0 * wz1;
  t.w[6] = wx0 * wy1 * wz1;
  t.w[7] = wx1 * wy1 * wz1;
  bool vx0 = (unsigned)x0 < (unsigned)D, vx1 = (unsigned)x1 < (unsigned)D;
  bool vy0 = (unsigned)y0 < (unsigned)W, vy1 = (unsigned)y1 < (unsigned)W;
  bool vz0 = (unsigned)z0 < (unsigned)H, vz1 = (unsigned)z1 < (unsigned)H;
  // Offsets of out-of-bounds taps are never dereferenced; unsigned
  // arithmetic keeps their computation well defined.
  const uint32_t uW = (uint32_t)W, uD = (uint32_t)D;
  uint32_t r00 = ((uint32_t)z0 * uW + (uint32_t)y0) * uD, r01 = ((uint32_t)z0 * uW + (uint32_t)y1) * uD;
  uint32_t r10 = ((uint32_t)z1 * uW + (uint32_t)y0) * uD, r11 = ((uint32_t)z1 * uW + (uint32_t)y1) * uD;
  t.off[0] = (int32_t)(r00 + (uint32_t)x0);
  t.off[1] = (int32_t)(r00 + (uint32_t)x1);
  t.off[2] = (int32_t)(r01 + (uint32_t)x0);
  t.off[3] = (int32_t)(r01 + (uint32_t)x1);
  t.off[4] = (int32_t)(r10 + (uint32_t)x0);
  t.off[5] = (int32_t)(r10 + (uint32_t)x1);
  t.off[6] = (int32_t)(r11 + (uint32_t)x0);
  t.off[7] = (int32_t)(r11 + (uint32_t)x1);
  t.valid = (uint32_t)(vz0 && vy0 && vx0) | ((uint32_t)(vz0 && vy0 && vx1) << 1) |
            ((uint32_t)(vz0 && vy1 && vx0) << 2) | ((uint32_t)(vz0 && vy1 && vx1) << 3) |
            ((uint32_t)(vz1 && vy0 && vx0) << 4) | ((uint32_t)(vz1 && vy0 && vx1) << 5) |
            ((uint32_t)(vz1 && vy1 && vx0) << 6) | ((uint32_t)(vz1 && vy1 && vx1) << 7);
}

template <int DT>
__device__ __forceinline__ float ld(const void* base, int64_t i) {
  if (DT == BA_BF16) return bf16_bits_to_f32(__ldg((const uint16_t*)base + i));
  return __ldg((const float*)base + i);
}

template <int DT>
__device__ __forceinline__ float gather8(const void* cbase, const Tap8& t) {
  float out = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float v = (t.valid >> k) & 1u ? ld<DT>(cbase, t.off[k]) : 0.0f;
    out = out + v * t.w[k];
  }
  return out;
}

template <int DT>
__device__ __forceinline__ void st(void* base, int64_t i, float v) {
  if (DT == BA_BF16)
    ((uint16_t*)base)[i] = f32_to_bf16_bits(v);
  else
    ((float*)base)[i] = v;
}

// All channels of one key at one output voxel (flat spatial index s).
template <int DT>
__device__ __forceinline__ void sample_voxel(const KeyArgs& k, const ResampleArgs& a,
                                             int64_t ebase, int64_t hwd, int64_t s, float ix,
                                             float iy, float iz) {
  const int H = a.H, W = a.W, D = a.D;
  const float px = pad_coord(ix, D, k.padding, a.align_corners);
  const float py = pad_coord(iy, W, k.padding, a.align_corners);
  const float pz = pad_coord(iz, H, k.padding, a.align_corners);
  if (k.mode == BA_NEAREST) {
    const int xn = (int)rintf(px), yn = (int)rintf(py), zn = (int)rintf(pz);
    const bool ok =
        (unsigned)xn < (unsigned)D && (unsigned)yn < (unsigned)W && (unsigned)zn < (unsigned)H;
    const int32_t off = ok ? (zn * W + yn) * D + xn : 0;
    for (int c = 0; c < k.channels; ++c) {
      const int64_t cb = ebase + (int64_t)c * hwd;
      st<DT>(k.dst, cb + s, ok ? ld<DT>(k.src, cb + off) : 0.0f);
    }
    return;
  }
  Tap8 t;
  trilinear_footprint(px, py, pz, H, W, D, t);
  for (int c = 0; c < k.channels; ++c) {
    const int64_t cb = ebase + (int64_t)c * hwd;
    const void* cbase = (DT == BA_BF16) ? (const void*)((const uint16_t*)k.src + cb)
                                        : (const void*)((const float*)k.src + cb);
    st<DT>(k.dst, cb + s, gather8<DT>(cbase, t));
  }
}

// A CTA covers a (TX*VEC)(D) x TY(W) x TZ(H) output brick.  Thread tx owns
// the voxels d = brick_d0 + v*TX + tx, v < VEC, so that for each v the lanes
// of a warp write TX consecutive voxels of TY rows (full 32-byte sectors for
// fp32) while only one tap footprint is live per thread.
template <int VEC>
__global__ void __launch_bounds__(NTHREADS, 8)
    resample3d_kernel(const __grid_constant__ ResampleArgs a) {
  const int H = a.H, W = a.W, D = a.D;
  const int tiles_d = (D + TX * VEC - 1) / (TX * VEC);
  const int tx = threadIdx.x % TX;
  const int ty = (threadIdx.x / TX) % TY;
  const int tz = threadIdx.x / (TX * TY);
  const int d_brick = (blockIdx.x % tiles_d) * (TX * VEC);
  const int w = (blockIdx.x / tiles_d) * TY + ty;
  const int h = blockIdx.y * TZ + tz;
  const int64_t b = blockIdx.z;
  const int64_t hwd = (int64_t)H * W * D;

  __shared__ float theta[12];
  const bool active = (a.mask == nullptr) || (a.mask[b] != 0);
  if (active && a.xform_kind != BA_XFORM_GRID && threadIdx.x < 12) {
    const int i = threadIdx.x / 4, j = threadIdx.x % 4;
    const float* x = a.xform + b * a.xform_stride;
    if (a.xform_kind == BA_XFORM_AFFINE) {
      // monai_affine_to_theta: theta = P S_norm A S_inv P, P swapping 0 and 2.
      const int pi = 2 - i, pj = (j == 3) ? 3 : 2 - j;
      const float s_i = a.sn[pi];
      const float s_j = (pj == 3) ? 1.0f : a.si[pj];
      theta[threadIdx.x] = (s_i * x[pi * 4 + pj]) * s_j;
    } else {
      theta[threadIdx.x] = x[i * 4 + j];
    }
  }
  __syncthreads();
  if (h >= H || w >= W) return;
  const int64_t row = ((int64_t)h * W + w) * D;

  if (!active) {
    for (int v = 0; v < VEC; ++v) {
      const int d = d_brick + v * TX + tx;
      if (d >= D) break;
      for (int ki = 0; ki < a.n_keys; ++ki) {
        const KeyArgs& k = a.keys[ki];
        for (int c = 0; c < k.channels; ++c) {
          const int64_t i = (b * k.channels + c) * hwd + row + d;
          if (k.dtype == BA_BF16)
            ((uint16_t*)k.dst)[i] = __ldg((const uint16_t*)k.src + i);
          else
            ((float*)k.dst)[i] = __ldg((const float*)k.src + i);
        }
      }
    }
    return;
  }

  // affine_grid's y and z base coordinates are shared by the thread's voxels.
  const float by = base_coord(w, W, a.align_corners);
  const float bz = base_coord(h, H, a.align_corners);
  for (int v = 0; v < VEC; ++v) {
    const int d = d_brick + v * TX + tx;
    if (d >= D) break;
    float gx, gy, gz;
    if (a.xform_kind == BA_XFORM_GRID) {
      const float* g = a.xform + (b * hwd + row + d) * 3;
      gx = __ldg(g);
      gy = __ldg(g + 1);
      gz = __ldg(g + 2);
    } else {
      // affine_grid's bmm as MKL accumulates it: x*t0, fused y and z terms,
      // then the translation.
      const float bx = base_coord(d, D, a.align_corners);
      gx = __fmaf_rn(bz, theta[2], __fmaf_rn(by, theta[1], bx * theta[0])) + theta[3];
      gy = __fmaf_rn(bz, theta[6], __fmaf_rn(by, theta[5], bx * theta[4])) + theta[7];
      gz = __fmaf_rn(bz, theta[10], __fmaf_rn(by, theta[9], bx * theta[8])) + theta[11];
    }
    const float ix = unnormalize(gx, D, a.align_corners);
    const float iy = unnormalize(gy, W, a.align_corners);
    const float iz = unnormalize(gz, H, a.align_corners);
    for (int ki = 0; ki < a.n_keys; ++ki) {
      const KeyArgs& k = a.keys[ki];
      const int64_t ebase = b * (int64_t)k.channels * hwd;
      if (k.dtype == BA_BF16)
        sample_voxel<BA_BF16>(k, a, ebase, hwd, row + d, ix, iy, iz);
      else
        sample_voxel<BA_F32>(k, a, ebase, hwd, row + d, ix, iy, iz);
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

  constexpr int VEC = 4;
  const int tiles_d = (int)((d.D + TX * VEC - 1) / (TX * VEC));
  const int64_t gx = (int64_t)tiles_d * ((d.W + TY - 1) / TY);
  const int64_t gy = (d.H + TZ - 1) / TZ;
  BA_REQUIRE(gx <= INT32_MAX && gy <= 65535, "ba_resample3d: spatial extent too large");
  dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)d.batch);
  resample3d_kernel<VEC><<<grid, NTHREADS, 0, (cudaStream_t)stream>>>(a);
  return check_launch("ba_resample3d");
}
