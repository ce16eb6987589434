// RandSimulateLowResolution (batchaug/pytorch/intensity/resolution.py:74-118):
// per element a target size t = max(1, rint(s * zoom)) per axis, then
// F.interpolate down to t and back up to the original size, each result
// cast to the tensor dtype.
//
// Per-axis index and weight arithmetic follows torch's CPU interpolate for
// 5-D inputs step by step (nearest: floor(o * n/m); nearest-exact:
// floor((o + 0.5) * n/m); trilinear: src = fma(n/m, o + 0.5, -0.5) clamped
// at 0, weights held in the dtype, each axis combined as
// fma(t0, w0, t1 * w1), H outer, D inner; area: box sum in the dtype, then
// divided by the box extent of each axis in turn), so results are
// bit-identical to the reference in fp32 and bf16.
//
// Two launch shapes:
//   - direct: a nearest or nearest-exact downsample only selects source
//     voxels, so it is folded into the upsample's per-axis maps; one pass
//     reads x and writes the output (the defaults take this path);
//   - two-pass: trilinear or area downsampling writes each element's small
//     volume to caller scratch (in the dtype, as torch rounds it), the
//     upsample reads it back.
#include <stdio.h>

#include <algorithm>

#include "ba_common.cuh"

namespace ba {
namespace {

enum { LR_NEAREST = 0, LR_NEAREST_EXACT = 1, LR_TRILINEAR = 2, LR_AREA = 3 };
enum { LR_PASS_DOWN = 0, LR_PASS_UP = 1, LR_PASS_DIRECT = 2 };

struct LowresArgs {
  const void* src;
  void* dst;
  const void* copy_src;  // masked-out elements copy this (up and direct passes)
  const float* zoom;
  const uint8_t* mask;
  int64_t C, H, W, D;
  int64_t ws_elem;  // workspace elements per batch element (C * largest target volume)
  int32_t dtype;
  int32_t mode;       // interpolation mode of this pass (the upsample mode when direct)
  int32_t align;      // align_corners of a trilinear pass
  int32_t pass;       // LR_PASS_*
  int32_t down_mode;  // direct pass: LR_NEAREST or LR_NEAREST_EXACT
  float max_zoom;     // zoom factors are clamped to this (the workspace bound)
};

__device__ __forceinline__ int32_t target_size(int64_t s, float zoom) {
  const int32_t v = (int32_t)rintf(__fmul_rn((float)s, zoom));
  return v < 1 ? 1 : v;
}

// Scale of a nearest / nearest-exact map (input n, output m): n / m.
// Scale of a trilinear map: (n-1)/(m-1) with align_corners, else n / m.
__device__ __forceinline__ float map_scale(int mode, bool align, int32_t n, int32_t m) {
  if (mode == LR_TRILINEAR && align) return m > 1 ? __fdiv_rn((float)(n - 1), (float)(m - 1)) : 0.0f;
  return __fdiv_rn((float)n, (float)m);
}

// nearest / nearest-exact source index of output o
__device__ __forceinline__ int32_t near_index(int mode, int32_t n, int32_t m, int32_t o, float s) {
  if (n == m) return o;
  const float p = mode == LR_NEAREST ? __fmul_rn((float)o, s) : __fmul_rn(__fadd_rn((float)o, 0.5f), s);
  const int32_t i = (int32_t)floorf(p);
  return i > n - 1 ? n - 1 : i;
}

struct Lin {
  int32_t i0, i1;
  float l0, l1;
};

template <int DT>
__device__ __forceinline__ Lin lin_map(int32_t n, int32_t m, int32_t o, bool align, float s) {
  Lin r;
  if (n == m) {
    r.i0 = r.i1 = o;
    r.l0 = 1.0f;
    r.l1 = 0.0f;
    return r;
  }
  float src;
  if (align) {
    src = __fmul_rn(s, (float)o);
  } else {
    src = __fmaf_rn(s, __fadd_rn((float)o, 0.5f), -0.5f);
    src = src < 0.0f ? 0.0f : src;
  }
  int32_t i0 = (int32_t)floorf(src);
  i0 = i0 > n - 1 ? n - 1 : i0;
  float l1 = __fsub_rn(src, (float)i0);
  l1 = l1 < 0.0f ? 0.0f : (l1 > 1.0f ? 1.0f : l1);
  l1 = round_dt<DT>(l1);
  r.i0 = i0;
  r.i1 = i0 + (i0 < n - 1 ? 1 : 0);
  r.l1 = l1;
  r.l0 = round_dt<DT>(__fsub_rn(1.0f, l1));
  return r;
}

template <int DT>
__device__ __forceinline__ float ld(const void* p, int64_t i) {
  return DT == BA_BF16 ? bf16_bits_to_f32(__ldg((const unsigned short*)p + i))
                       : __ldg((const float*)p + i);
}

// Per-(element, channel) constants of one pass, resolved once per CTA.
struct PassConst {
  int32_t n[3], m[3];   // input and output sizes of this pass
  int32_t t[3];         // the element's target size
  float s[3];           // this pass's map scale per axis
  float sd[3];          // direct pass: scale of the folded downsample (S -> t)
  int64_t in_base, out_base;
  int32_t off;          // masked-out element
};

// One output voxel.  Sources are gathered as src_at(a, b, e) with input
// indices; for the direct pass the indices are first mapped through the
// folded nearest downsample (fold(ax, i) -> source index along ax).
template <int DT, typename Src, typename Fold>
__device__ __forceinline__ float interp_voxel(int mode, bool align, const PassConst& k, int32_t h,
                                              int32_t w, int32_t d, Src src_at, Fold fold) {
  if (mode == LR_TRILINEAR) {
    const Lin A = lin_map<DT>(k.n[0], k.m[0], h, align, k.s[0]);
    const Lin Bw = lin_map<DT>(k.n[1], k.m[1], w, align, k.s[1]);
    const Lin Dd = lin_map<DT>(k.n[2], k.m[2], d, align, k.s[2]);
    const int32_t a0 = fold(0, A.i0), a1 = fold(0, A.i1), b0 = fold(1, Bw.i0), b1 = fold(1, Bw.i1);
    const int32_t e0 = fold(2, Dd.i0), e1 = fold(2, Dd.i1);
    float th[2];
#pragma unroll
    for (int ih = 0; ih < 2; ++ih) {
      const int32_t a = ih ? a1 : a0;
      float tw[2];
#pragma unroll
      for (int iw = 0; iw < 2; ++iw) {
        const int32_t b = iw ? b1 : b0;
        tw[iw] = __fmaf_rn(src_at(a, b, e0), Dd.l0, __fmul_rn(src_at(a, b, e1), Dd.l1));
      }
      th[ih] = __fmaf_rn(tw[0], Bw.l0, __fmul_rn(tw[1], Bw.l1));
    }
    return __fmaf_rn(th[0], A.l0, __fmul_rn(th[1], A.l1));
  }
  if (mode == LR_AREA) {
    const int32_t a0 = (int32_t)(((int64_t)h * k.n[0]) / k.m[0]);
    const int32_t a1 = (int32_t)(((int64_t)(h + 1) * k.n[0] + k.m[0] - 1) / k.m[0]);
    const int32_t b0 = (int32_t)(((int64_t)w * k.n[1]) / k.m[1]);
    const int32_t b1 = (int32_t)(((int64_t)(w + 1) * k.n[1] + k.m[1] - 1) / k.m[1]);
    const int32_t e0 = (int32_t)(((int64_t)d * k.n[2]) / k.m[2]);
    const int32_t e1 = (int32_t)(((int64_t)(d + 1) * k.n[2] + k.m[2] - 1) / k.m[2]);
    float acc = 0.0f;
    for (int32_t a = a0; a < a1; ++a)
      for (int32_t b = b0; b < b1; ++b)
        for (int32_t e = e0; e < e1; ++e)
          acc = round_dt<DT>(__fadd_rn(acc, src_at(fold(0, a), fold(1, b), fold(2, e))));
    acc = round_dt<DT>(__fdiv_rn(acc, (float)(a1 - a0)));
    acc = round_dt<DT>(__fdiv_rn(acc, (float)(b1 - b0)));
    return __fdiv_rn(acc, (float)(e1 - e0));
  }
  return src_at(fold(0, near_index(mode, k.n[0], k.m[0], h, k.s[0])),
                fold(1, near_index(mode, k.n[1], k.m[1], w, k.s[1])),
                fold(2, near_index(mode, k.n[2], k.m[2], d, k.s[2])));
}

// Grid (ceil(voxels / 256), B * C); voxels = the output volume of the pass
// (for the down pass the largest target volume; threads past an element's
// own target exit).  Zoom factors above max_zoom are clamped to it, so no
// element's target exceeds the workspace sized from max_zoom.
template <int DT>
__global__ void __launch_bounds__(256) lowres_kernel(const __grid_constant__ LowresArgs a) {
  __shared__ PassConst k;
  const int64_t bc = blockIdx.y;
  const int64_t b = bc / a.C, c = bc % a.C;
  const int32_t S[3] = {(int32_t)a.H, (int32_t)a.W, (int32_t)a.D};
  const int64_t HWD = a.H * a.W * a.D;
  const bool down = a.pass == LR_PASS_DOWN;
  if (threadIdx.x == 0) {
    const float z = fminf(a.zoom[b], a.max_zoom);
    for (int ax = 0; ax < 3; ++ax) {
      k.t[ax] = target_size(S[ax], z);
      k.n[ax] = down ? S[ax] : k.t[ax];
      k.m[ax] = down ? k.t[ax] : S[ax];
      k.s[ax] = map_scale(a.mode, a.align != 0, k.n[ax], k.m[ax]);
      k.sd[ax] = __fdiv_rn((float)S[ax], (float)k.t[ax]);
    }
    const int64_t tv = (int64_t)k.t[0] * k.t[1] * k.t[2];
    k.in_base = a.pass == LR_PASS_UP ? b * a.ws_elem + c * tv : bc * HWD;
    k.out_base = down ? b * a.ws_elem + c * tv : bc * HWD;
    k.off = a.mask != nullptr && a.mask[b] == 0;
  }
  __syncthreads();
  const int64_t mv = (int64_t)k.m[0] * k.m[1] * k.m[2];
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= mv) return;
  if (k.off) {
    if (!down) {
      const int64_t i = bc * HWD + o;
      if (DT == BA_BF16)
        ((uint16_t*)a.dst)[i] = ((const uint16_t*)a.copy_src)[i];
      else
        ((float*)a.dst)[i] = ((const float*)a.copy_src)[i];
    }
    return;
  }
  const int32_t m12 = k.m[1] * k.m[2];
  const int32_t oi = (int32_t)o;
  const int32_t h = oi / m12, w = (oi - h * m12) / k.m[2], d = oi - h * m12 - w * k.m[2];
  const int32_t n1 = k.n[1], n2 = k.n[2];
  const int64_t base = k.in_base;
  auto src_at = [&](int32_t i, int32_t j, int32_t e) {
    return ld<DT>(a.src, base + ((int64_t)i * n1 + j) * n2 + e);
  };
  float v;
  if (a.pass == LR_PASS_DIRECT) {
    // the nearest / nearest-exact downsample (S -> t) only picks source
    // voxels: gather from x through it; src_at then indexes x (sizes S)
    const int dm = a.down_mode;
    auto src_x = [&](int32_t i, int32_t j, int32_t e) {
      return ld<DT>(a.src, base + ((int64_t)i * S[1] + j) * S[2] + e);
    };
    v = interp_voxel<DT>(a.mode, a.align != 0, k, h, w, d, src_x, [&](int ax, int32_t i) {
      return near_index(dm, S[ax], k.t[ax], i, k.sd[ax]);
    });
  } else {
    v = interp_voxel<DT>(a.mode, a.align != 0, k, h, w, d, src_at,
                         [](int, int32_t i) { return i; });
  }
  const int64_t oo = k.out_base + o;
  if (DT == BA_BF16)
    ((uint16_t*)a.dst)[oo] = f32_to_bf16_bits(v);
  else
    ((float*)a.dst)[oo] = v;
}

// Trilinear direct and up passes by output rows: CTA (ceil(H * W /
// LR_ROW_ROWS), B * C) takes LR_ROW_ROWS consecutive (h, w) rows, one warp
// per row, lanes along D.  The D map (tap indices, through the folded
// nearest downsample of a direct pass, and weights) is tabulated once per
// CTA in shared memory; per row, the H and W maps and the four source rows
// they select are resolved once by its warp, and each lane gathers its D
// positions' 8 taps from those rows.  The arithmetic is interp_voxel's, so
// results are identical to lowres_kernel's.
constexpr int LR_ROW_THREADS = 128;
constexpr int LR_ROW_ROWS = 16;

// The D map of a row pass, the same for every row of an element: source
// indices of the two taps (through the folded nearest downsample of a
// direct pass) and their weights.
struct DTap {
  int32_t e0, e1;
  float l0, l1;
};

template <int DT, bool DIRECT>
__device__ __forceinline__ void lowres_row(const LowresArgs& a, const PassConst& k,
                                           const int32_t (&S)[3], int32_t row,
                                           const DTap* dmap) {
  const int32_t h = row / S[1], w = row - h * S[1];
  const int64_t orow = k.out_base + (int64_t)row * S[2];
  if (k.off) {
    for (int32_t d = (int32_t)(threadIdx.x & 31); d < S[2]; d += 32) {
      if (DT == BA_BF16)
        ((uint16_t*)a.dst)[orow + d] = ((const uint16_t*)a.copy_src)[orow + d];
      else
        ((float*)a.dst)[orow + d] = ((const float*)a.copy_src)[orow + d];
    }
    return;
  }
  const bool align = a.align != 0;
  const int dm = a.down_mode;
  auto fold = [&](int ax, int32_t i) {
    return DIRECT ? near_index(dm, S[ax], k.t[ax], i, k.sd[ax]) : i;
  };
  const Lin A = lin_map<DT>(k.n[0], k.m[0], h, align, k.s[0]);
  const Lin Bw = lin_map<DT>(k.n[1], k.m[1], w, align, k.s[1]);
  const int32_t a0 = fold(0, A.i0), a1 = fold(0, A.i1), b0 = fold(1, Bw.i0), b1 = fold(1, Bw.i1);
  // source rows (a, b): sizes S for a direct pass (x itself), the target for up
  const int64_t N1 = DIRECT ? S[1] : k.n[1], N2 = DIRECT ? S[2] : k.n[2];
  const int64_t r00 = k.in_base + ((int64_t)a0 * N1 + b0) * N2;
  const int64_t r01 = k.in_base + ((int64_t)a0 * N1 + b1) * N2;
  const int64_t r10 = k.in_base + ((int64_t)a1 * N1 + b0) * N2;
  const int64_t r11 = k.in_base + ((int64_t)a1 * N1 + b1) * N2;
  for (int32_t d = (int32_t)(threadIdx.x & 31); d < S[2]; d += 32) {
    const DTap t = dmap[d];
    auto tw = [&](int64_t r) {
      return __fmaf_rn(ld<DT>(a.src, r + t.e0), t.l0, __fmul_rn(ld<DT>(a.src, r + t.e1), t.l1));
    };
    const float th0 = __fmaf_rn(tw(r00), Bw.l0, __fmul_rn(tw(r01), Bw.l1));
    const float th1 = __fmaf_rn(tw(r10), Bw.l0, __fmul_rn(tw(r11), Bw.l1));
    const float v = __fmaf_rn(th0, A.l0, __fmul_rn(th1, A.l1));
    if (DT == BA_BF16)
      ((uint16_t*)a.dst)[orow + d] = f32_to_bf16_bits(v);
    else
      ((float*)a.dst)[orow + d] = v;
  }
}

template <int DT, bool DIRECT>
__global__ void __launch_bounds__(LR_ROW_THREADS) lowres_row_kernel(const __grid_constant__ LowresArgs a) {
  __shared__ PassConst k;
  extern __shared__ DTap dmap[];  // D entries
  const int64_t bc = blockIdx.y;
  const int64_t b = bc / a.C, c = bc % a.C;
  const int32_t S[3] = {(int32_t)a.H, (int32_t)a.W, (int32_t)a.D};
  const int64_t HWD = a.H * a.W * a.D;
  if (threadIdx.x < 3) {  // one axis per thread
    const int ax = threadIdx.x;
    const float z = fminf(a.zoom[b], a.max_zoom);
    k.t[ax] = target_size(S[ax], z);
    k.n[ax] = k.t[ax];
    k.m[ax] = S[ax];
    k.s[ax] = map_scale(a.mode, a.align != 0, k.n[ax], k.m[ax]);
    k.sd[ax] = __fdiv_rn((float)S[ax], (float)k.t[ax]);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int64_t tv = (int64_t)k.t[0] * k.t[1] * k.t[2];
    k.in_base = DIRECT ? bc * HWD : b * a.ws_elem + c * tv;
    k.out_base = bc * HWD;
    k.off = a.mask != nullptr && a.mask[b] == 0;
  }
  __syncthreads();
  if (!k.off) {
    const bool align = a.align != 0;
    for (int32_t d = threadIdx.x; d < S[2]; d += LR_ROW_THREADS) {
      const Lin Dd = lin_map<DT>(k.n[2], k.m[2], d, align, k.s[2]);
      DTap t;
      t.e0 = DIRECT ? near_index(a.down_mode, S[2], k.t[2], Dd.i0, k.sd[2]) : Dd.i0;
      t.e1 = DIRECT ? near_index(a.down_mode, S[2], k.t[2], Dd.i1, k.sd[2]) : Dd.i1;
      t.l0 = Dd.l0;
      t.l1 = Dd.l1;
      dmap[d] = t;
    }
    __syncthreads();
  }
  const int32_t rows = S[0] * S[1];
  const int32_t first = (int32_t)blockIdx.x * LR_ROW_ROWS;
  const int32_t last = min(rows, first + LR_ROW_ROWS);
  // one warp per row: a row's H/W maps and source rows are resolved once per
  // warp and amortised over its D / 32 voxels per lane
  for (int32_t row = first + (int32_t)(threadIdx.x >> 5); row < last; row += LR_ROW_THREADS / 32)
    lowres_row<DT, DIRECT>(a, k, S, row, dmap);
}

int64_t host_target(int64_t s, double zoom) {
  const int64_t v = (int64_t)std::nearbyint((double)((float)s * (float)zoom));
  return v < 1 ? 1 : v;
}

ba_status launch(const LowresArgs& a, int64_t voxels, int64_t planes, cudaStream_t st) {
  if (voxels <= 0) return BA_OK;
  const size_t dmap_bytes = (size_t)a.D * sizeof(DTap);
  if (a.mode == LR_TRILINEAR && a.pass != LR_PASS_DOWN && dmap_bytes <= 48 * 1024) {
    const dim3 g((unsigned)((a.H * a.W + LR_ROW_ROWS - 1) / LR_ROW_ROWS), (unsigned)planes);
    const bool bf = a.dtype == BA_BF16, direct = a.pass == LR_PASS_DIRECT;
    if (bf && direct)
      lowres_row_kernel<BA_BF16, true><<<g, LR_ROW_THREADS, dmap_bytes, st>>>(a);
    else if (bf)
      lowres_row_kernel<BA_BF16, false><<<g, LR_ROW_THREADS, dmap_bytes, st>>>(a);
    else if (direct)
      lowres_row_kernel<BA_F32, true><<<g, LR_ROW_THREADS, dmap_bytes, st>>>(a);
    else
      lowres_row_kernel<BA_F32, false><<<g, LR_ROW_THREADS, dmap_bytes, st>>>(a);
    return check_launch("ba_lowres3d");
  }
  dim3 g((unsigned)((voxels + 255) / 256), (unsigned)planes);
  if (a.dtype == BA_BF16)
    lowres_kernel<BA_BF16><<<g, 256, 0, st>>>(a);
  else
    lowres_kernel<BA_F32><<<g, 256, 0, st>>>(a);
  return check_launch("ba_lowres3d");
}

}  // namespace
}  // namespace ba

extern "C" size_t ba_lowres_workspace_bytes(const ba_lowres_desc* d) {
  using namespace ba;
  if (d == nullptr || d->batch < 0 || d->channels < 0 || d->H < 1 || d->W < 1 || d->D < 1)
    return 0;
  if (d->down_mode == LR_NEAREST || d->down_mode == LR_NEAREST_EXACT) return 0;
  const int64_t tv = host_target(d->H, d->max_zoom) * host_target(d->W, d->max_zoom) *
                     host_target(d->D, d->max_zoom);
  return (size_t)(d->batch * d->channels * tv) * (d->dtype == BA_BF16 ? 2 : 4);
}

extern "C" ba_status ba_lowres3d(const ba_lowres_desc* d, void* workspace, size_t workspace_bytes,
                                 ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(d != nullptr, "ba_lowres3d: desc is NULL");
  BA_REQUIRE(d->dtype == BA_F32 || d->dtype == BA_BF16, "ba_lowres3d: bad dtype %d", d->dtype);
  BA_REQUIRE(d->batch >= 0 && d->channels >= 0 && d->H > 0 && d->W > 0 && d->D > 0,
             "ba_lowres3d: bad shape");
  BA_REQUIRE(d->batch * d->channels <= 65535, "ba_lowres3d: batch*channels exceeds 65535");
  BA_REQUIRE(d->H * d->W * d->D < ((int64_t)1 << 31), "ba_lowres3d: volume exceeds 2^31 voxels");
  BA_REQUIRE(d->down_mode >= LR_NEAREST && d->down_mode <= LR_AREA && d->up_mode >= LR_NEAREST &&
                 d->up_mode <= LR_AREA,
             "ba_lowres3d: unknown interpolation mode");
  BA_REQUIRE(d->max_zoom > 0.0 && d->max_zoom <= 64.0, "ba_lowres3d: max_zoom %g not in (0, 64]",
             d->max_zoom);
  BA_REQUIRE(host_target(d->H, d->max_zoom) * host_target(d->W, d->max_zoom) *
                     host_target(d->D, d->max_zoom) <
                 ((int64_t)1 << 31),
             "ba_lowres3d: target volume at max_zoom exceeds 2^31 voxels");
  const int64_t HWD = d->H * d->W * d->D;
  if (d->batch * d->channels * HWD == 0) return BA_OK;
  BA_REQUIRE(d->src && d->dst && d->zoom, "ba_lowres3d: NULL pointer");
  const size_t esz = d->dtype == BA_BF16 ? 2 : 4;
  const int64_t n = d->batch * d->channels * HWD;
  BA_REQUIRE((const char*)d->src + n * esz <= (const char*)d->dst ||
                 (const char*)d->dst + n * esz <= (const char*)d->src,
             "ba_lowres3d: dst overlaps src");
  cudaStream_t st = (cudaStream_t)stream;
  LowresArgs a;
  memset(&a, 0, sizeof(a));
  a.zoom = d->zoom;
  a.mask = d->mask;
  a.C = d->channels;
  a.H = d->H;
  a.W = d->W;
  a.D = d->D;
  a.dtype = d->dtype;
  a.copy_src = d->src;
  a.max_zoom = (float)d->max_zoom;
  const int64_t planes = d->batch * d->channels;
  if (d->down_mode == LR_NEAREST || d->down_mode == LR_NEAREST_EXACT) {
    a.src = d->src;
    a.dst = d->dst;
    a.pass = LR_PASS_DIRECT;
    a.mode = d->up_mode;
    a.align = d->up_mode == LR_TRILINEAR ? (d->align_corners != 0) : 0;
    a.down_mode = d->down_mode;
    return launch(a, HWD, planes, st);
  }
  const size_t need = ba_lowres_workspace_bytes(d);
  BA_REQUIRE(workspace != nullptr && workspace_bytes >= need,
             "ba_lowres3d: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  const int64_t tv = host_target(d->H, d->max_zoom) * host_target(d->W, d->max_zoom) *
                     host_target(d->D, d->max_zoom);
  a.ws_elem = d->channels * tv;
  // down: x -> workspace (element b at b * ws_elem, channel c at c * its own
  // target volume)
  a.src = d->src;
  a.dst = workspace;
  a.pass = LR_PASS_DOWN;
  a.mode = d->down_mode;
  a.align = d->down_mode == LR_TRILINEAR ? (d->align_corners != 0) : 0;
  ba_status s = launch(a, tv, planes, st);
  if (s != BA_OK) return s;
  // up: workspace -> dst; masked-out elements copy src
  a.src = workspace;
  a.dst = d->dst;
  a.pass = LR_PASS_UP;
  a.mode = d->up_mode;
  a.align = d->up_mode == LR_TRILINEAR ? (d->align_corners != 0) : 0;
  return launch(a, HWD, planes, st);
}
