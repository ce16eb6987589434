// Separable Gaussian smoothing and the elastic displacement field.
//
// Reference semantics:
//   gaussian_1d_batch           batchaug/pytorch/intensity/smooth.py:9-34
//   separable_gaussian_conv3d   batchaug/pytorch/intensity/smooth.py:37-88
//   RandGaussianSmooth.apply    batchaug/pytorch/intensity/smooth.py:110-117
//   Rand3DElastic.sample_params batchaug/pytorch/geometric/elastic.py:37-99
//   RandGaussianSharpen.apply   batchaug/pytorch/intensity/sharpen.py:117-136
//
// Design: three axis passes (H, then W, then D, as the reference's three
// grouped conv3d calls) with per-element taps held in shared memory; the
// passes read and write fp32 intermediates in caller-provided scratch and the
// last pass writes the output dtype directly (and, for the elastic field,
// forms the grid_sample grid in place: centred MONAI grid + magnitude *
// displacement, divided by (N-1)/2, components reordered to x=D, y=W, z=H).
// The uniform draw of the elastic field is generated in-kernel by Philox
// unless the caller injects it.  Unsharp masking runs two smooths; the last
// pass of the second one combines its result with the first blur as it
// writes, so the double blur is never stored.
#include <stdio.h>

#include <algorithm>

#include "ba_common.cuh"
#include "philox.cuh"

namespace ba {
namespace {

constexpr int SM_THREADS = 256;
constexpr int MAX_TAPS = 255;

__device__ __forceinline__ float load_in(const void* p, int dtype, int64_t i) {
  return dtype == BA_BF16 ? bf16_bits_to_f32(((const uint16_t*)p)[i]) : ((const float*)p)[i];
}

// blurred + alpha * (blurred - double_blurred), one op at a time in the
// dtype with alpha cast to it first (sharpen.py:131); `db` is the second
// blur's fp32 sum before its cast.
__device__ __forceinline__ float sharpen_combine(float blurred, float db, float alpha, int dtype) {
  if (dtype == BA_BF16) {
    const float d = round_bf16(__fsub_rn(blurred, round_bf16(db)));
    const float t = round_bf16(__fmul_rn(round_bf16(alpha), d));
    return round_bf16(__fadd_rn(blurred, t));
  }
  return __fadd_rn(blurred, __fmul_rn(alpha, __fsub_rn(blurred, db)));
}

// One warp per element: the lanes evaluate the taps, lane 0 sums them in
// tap order (the order the normalisation has always used), every lane
// divides its taps by the sum.
constexpr int GT_THREADS = 128;

__global__ void gauss_taps_kernel(const float* sigmas, int64_t B, int64_t K, float* taps) {
  const int64_t b = blockIdx.x * (int64_t)(GT_THREADS / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (b >= B) return;
  const int64_t tail = K / 2;
  float s = sigmas[b];
  s = s < 1e-6f ? 1e-6f : s;
  const float t = 0.70710678f / s;
  float* o = taps + b * K;
  for (int64_t k = lane; k < K; k += 32) {
    const float x = (float)(k - tail);
    float v = 0.5f * (erff(t * (x + 0.5f)) - erff(t * (x - 0.5f)));
    o[k] = v < 0.0f ? 0.0f : v;
  }
  __syncwarp();  // the warp's tap stores are visible to lane 0
  float sum = 0.0f;
  if (lane == 0)
    for (int64_t k = 0; k < K; ++k) sum += o[k];
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int64_t k = lane; k < K; k += 32) o[k] = o[k] / sum;
}

// One zero-padded correlation along AXIS (0=H, 1=W, 2=D) of planes
// (B*P, H, W, D), P planes per element sharing that element's taps.  The
// output element is fp32 unless OUT_DT says otherwise; with `copy_src` set,
// masked-out elements copy copy_src instead (the last pass of a smooth).
struct AxisArgs {
  const void* in;
  int32_t in_dtype;
  void* out;
  int32_t out_dtype;
  const float* taps;
  int32_t K;
  int64_t P, H, W, D, HWD;
  int32_t padding;  // ba_smooth_pad
  const uint8_t* mask;
  const void* copy_src;
  // unsharp masking (last pass of the second blur): out = combine(sharp_blur, acc)
  const void* sharp_blur;
  const float* alpha;
};

// Source index of padded position q (may be outside [0, n)) along an axis of
// length n, or -1 for a zero tap.  "reflect" mirrors without repeating the
// edge sample, "replicate" repeats it (F.pad's modes).
__device__ __forceinline__ int64_t pad_index(int64_t q, int64_t n, int padding) {
  if (q >= 0 && q < n) return q;
  if (padding == BA_SMOOTH_REFLECT) {
    if (n == 1) return 0;
    const int64_t period = 2 * (n - 1);
    int64_t r = q % period;
    if (r < 0) r += period;
    return r < n ? r : period - r;
  }
  if (padding == BA_SMOOTH_REPLICATE) return q < 0 ? 0 : n - 1;
  return -1;
}

template <int AXIS>
__global__ void __launch_bounds__(SM_THREADS) axis_pass_kernel(const __grid_constant__ AxisArgs a) {
  __shared__ float w[MAX_TAPS];
  const int64_t plane = blockIdx.y;  // b * P + p
  const int64_t b = plane / a.P;
  for (int k = threadIdx.x; k < a.K; k += blockDim.x) w[k] = a.taps[b * a.K + k];
  __syncthreads();
  const int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= a.HWD) return;
  const int64_t idx = plane * a.HWD + s;
  if (a.copy_src != nullptr && a.mask != nullptr && a.mask[b] == 0) {
    if (a.out_dtype == BA_BF16)
      ((uint16_t*)a.out)[idx] = ((const uint16_t*)a.copy_src)[idx];
    else
      ((float*)a.out)[idx] = ((const float*)a.copy_src)[idx];
    return;
  }
  const int64_t n = AXIS == 0 ? a.H : (AXIS == 1 ? a.W : a.D);
  const int64_t stride = AXIS == 0 ? a.W * a.D : (AXIS == 1 ? a.D : 1);
  const int64_t pos = (s / stride) % n;
  const int pad = a.K / 2;
  const int64_t base = plane * a.HWD + s - pos * stride;
  float acc = 0.0f;
  for (int k = 0; k < a.K; ++k) {
    const int64_t q = pad_index(pos + k - pad, n, a.padding);
    if (q < 0) continue;
    acc = acc + load_in(a.in, a.in_dtype, base + q * stride) * w[k];
  }
  if (a.sharp_blur != nullptr)
    acc = sharpen_combine(load_in(a.sharp_blur, a.out_dtype, idx), acc, a.alpha[b], a.out_dtype);
  if (a.out_dtype == BA_BF16)
    ((uint16_t*)a.out)[idx] = f32_to_bf16_bits(acc);
  else
    ((float*)a.out)[idx] = acc;
}

// Uniform draw of the elastic field, mapped to [-1, 1): u * 2 - 1.
// One thread per Philox block: the four field values at positions 4q .. 4q+3
// of an element (p = comp * HWD + s), all four outputs of the block used.
__global__ void elastic_draw_kernel(const float* u, uint32_t seed_lo, uint32_t seed_hi,
                                    uint64_t elem_offset, int64_t HWD, int64_t batch,
                                    float* out) {
  const int64_t per = 3 * HWD;           // values per element
  const int64_t blocks = (per + 3) / 4;  // Philox blocks per element
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= batch * blocks) return;
  const int64_t b = i / blocks;
  const int64_t q = i - b * blocks;
  const int64_t p0 = 4 * q;
  const int n = per - p0 < 4 ? (int)(per - p0) : 4;
  float* o = out + b * per + p0;
  if (u != nullptr) {
    const float* x = u + b * per + p0;
    for (int l = 0; l < n; ++l) o[l] = x[l] * 2.0f - 1.0f;
    return;
  }
  const uint64_t eb = elem_offset + (uint64_t)b;
  const U4 ctr = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                  STREAM_ELASTIC | (uint32_t)((uint64_t)q >> 32)};
  const U4 r = philox4x32_10(ctr, seed_lo, seed_hi);
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int l = 0; l < 4; ++l)
    if (l < n) o[l] = u01(w[l]) * 2.0f - 1.0f;
}

// Last (D-axis) pass of the elastic field, forming the grid:
// grid[b,h,w,d,2-comp] = (centre_comp + smooth_comp * magnitude[b]) / half_comp.
__global__ void __launch_bounds__(SM_THREADS)
    elastic_grid_kernel(const float* in, const float* taps, int32_t K, const float* magnitude,
                        int64_t H, int64_t W, int64_t D, float* grid) {
  __shared__ float w[MAX_TAPS];
  const int64_t b = blockIdx.y;
  for (int k = threadIdx.x; k < K; k += blockDim.x) w[k] = taps[b * K + k];
  __syncthreads();
  const int64_t HWD = H * W * D;
  const int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= HWD) return;
  const int64_t z = s / (W * D), y = (s / D) % W, x = s % D;
  const int pad = K / 2;
  const float mag = magnitude[b];
  const int64_t sz[3] = {H, W, D};
  const int64_t idx[3] = {z, y, x};
  float* g = grid + (b * HWD + s) * 3;
  for (int comp = 0; comp < 3; ++comp) {
    const float* row = in + (b * 3 + comp) * HWD + s - x;
    float acc = 0.0f;
    for (int k = 0; k < K; ++k) {
      const int64_t q = x + k - pad;
      if (q < 0 || q >= D) continue;
      acc = acc + row[q] * w[k];
    }
    const float disp = acc * mag;
    const float n = (float)sz[comp];
    const float half_lo = (n - 1.0f) / 2.0f;
    const float c0 = linspace_at(-half_lo, half_lo, (half_lo - (-half_lo)) / (n - 1.0f),
                                 idx[comp], sz[comp]);
    float half = half_lo < 1e-6f ? 1e-6f : half_lo;
    g[2 - comp] = (c0 + disp) / half;
  }
}

// ===========================================================================
// Tiled separable smoothing (used when the taps fit TILE_KMAX).
//
// Pass A convolves each H-plane along D then W inside a shared-memory tile
// (halo loaded with the padding rule), writing an fp32 intermediate; pass B
// convolves along H over column strips of that intermediate and writes the
// result (the output dtype, or one component of the elastic grid).  Taps sit
// in shared memory zero-padded to a compile-time KMAX (one broadcast read per
// tap, reused for R outputs) and the input window rolls through registers,
// one shared-memory read per tap step.  Rows read with stride R per thread use the padded
// index q + q/8, which keeps those reads free of bank conflicts.  The three
// 1-D operators (each "pad, then correlate" along one axis) commute, so
// running D, W, H instead of the reference's H, W, D changes only rounding.
// ===========================================================================
constexpr int TS_THREADS = 256;
constexpr int TS_TD = 64;   // pass A tile extent along D
constexpr int TS_RD = 8;    // pass A D-outputs per thread unit
constexpr int TS_RW = 8;    // pass A W-outputs per thread unit
constexpr int TB_TD = 32;   // pass B tile extent along D
constexpr int TS_TH = 64;   // pass B tile extent along H
constexpr int TS_RH = 8;    // pass B H-outputs per thread (TS_TH / TS_RH = 8 groups)
constexpr int TILE_KMAX = 63;
constexpr int MAX_COLS = TS_TD + TILE_KMAX - 1;
constexpr int MAX_ROWS = TS_TH + TILE_KMAX - 1;  // pass B rows with halo
static_assert(TS_TH == (TS_THREADS / TB_TD) * TS_RH, "pass B: one run of TS_RH rows per thread group");

// Tile extent along W of pass A: wider tiles for wide kernels keep the
// D-pass halo rows (KMAX-1 of them) a small fraction of the work.
__host__ __device__ constexpr int plane_tw(int kmax) { return kmax > 23 ? 64 : 32; }

// Shared-memory row index with one pad word every 8: a thread reading R=8
// consecutive entries starting at 8*t hits distinct banks across a warp.
__host__ __device__ __forceinline__ int pidx(int q) { return q + (q >> 3); }

struct TiledArgs {
  const void* in;  // pass A: input volume (in_dtype), pass B: fp32 intermediate
  int32_t in_dtype;
  float* mid;      // fp32 intermediate (B*P, H, W, D)
  void* out;       // pass B output
  int32_t out_dtype;
  const float* taps_h;
  const float* taps_w;
  const float* taps_d;
  int32_t Kh, Kw, Kd;
  int32_t padding;
  int64_t P, H, W, D, HWD;
  const uint8_t* mask;    // masked-out elements copy `copy_src` in pass B
  const void* copy_src;
  // elastic grid output (pass B): grid != nullptr
  float* grid;
  const float* magnitude;
  // unsharp masking (pass B of the second blur): out = combine(sharp_blur, acc)
  const void* sharp_blur;
  const float* alpha;
};

// R outputs out[i] = sum_k w[k] * x[i + k] for k < KMAX from a register
// window x of R + KMAX - 1 values; taps come from shared memory (one
// broadcast read per tap, reused by all R outputs).
// R outputs acc[i] = sum_k w[k] * x[i + k], k < KMAX.  The window rolls:
// tap k loads x[k + R - 1] only, so R values of x are live at a time, not
// R + KMAX - 1 (which would not fit the registers for wide kernels).
template <int R, int KMAX, typename Load>
__device__ __forceinline__ void conv_rolling(Load x, const float* s_w, float* acc) {
  float xw[R + KMAX - 1];
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int j = 0; j < R - 1; ++j) xw[j] = x(j);
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    xw[k + R - 1] = x(k + R - 1);
    const float w = s_w[k];
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = __fmaf_rn(w, xw[i + k], acc[i]);
  }
}

template <int KMAX>
__device__ __forceinline__ void load_taps_smem(const float* taps, int64_t b, int K, float* s_w) {
  for (int k = threadIdx.x; k < KMAX; k += blockDim.x) s_w[k] = k < K ? taps[b * K + k] : 0.0f;
}

// Pass A: grid (tiles_w * tiles_d, H, B*P).
template <int KMAX>
__global__ void __launch_bounds__(TS_THREADS) smooth_plane_kernel(const __grid_constant__ TiledArgs a) {
  constexpr int TW = plane_tw(KMAX);
  extern __shared__ float sm[];
  __shared__ float s_wd[KMAX], s_ww[KMAX];
  __shared__ int s_di[MAX_COLS];
  const int64_t bp = blockIdx.z;
  const int64_t b = bp / a.P;
  if (a.mask != nullptr && a.mask[b] == 0) return;  // pass B copies the input
  const int W = (int)a.W, D = (int)a.D;
  const int h = blockIdx.y;
  const int tiles_d = (D + TS_TD - 1) / TS_TD;
  const int td0 = (blockIdx.x % tiles_d) * TS_TD;
  const int tw0 = (blockIdx.x / tiles_d) * TW;
  const int pd = a.Kd / 2, pw = a.Kw / 2;
  // tile with halo: KMAX-wide windows read up to KMAX-1 past each output
  constexpr int rowsA = TW + KMAX - 1, colsA = TS_TD + KMAX - 1;
  constexpr int PA = (colsA - 1) + ((colsA - 1) >> 3) + 1;
  float* A = sm;                   // rowsA x PA (padded index)
  float* Bm = sm + rowsA * PA;     // rowsA x TS_TD
  const int64_t plane = (bp * a.H + h) * (int64_t)W * D;
  for (int q = threadIdx.x; q < colsA; q += TS_THREADS)
    s_di[q] = q < TS_TD + 2 * pd ? (int)pad_index(td0 - pd + q, D, a.padding) : -1;
  load_taps_smem<KMAX>(a.taps_d, b, a.Kd, s_wd);
  load_taps_smem<KMAX>(a.taps_w, b, a.Kw, s_ww);
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int r = warp; r < rowsA; r += TS_THREADS / 32) {
    // rows and columns beyond the real halo meet zero taps; keep them finite
    const int64_t wi = r < TW + 2 * pw ? pad_index(tw0 - pw + r, W, a.padding) : -1;
    const int64_t row = plane + wi * D;
    for (int q = lane; q < colsA; q += 32) {
      const int di = s_di[q];
      A[r * PA + pidx(q)] = (wi >= 0 && di >= 0) ? load_in(a.in, a.in_dtype, row + di) : 0.0f;
    }
  }
  __syncthreads();
  // D pass: units of TS_RD consecutive outputs of one row
  constexpr int GROUPS_D = TS_TD / TS_RD;
  for (int u = threadIdx.x; u < rowsA * GROUPS_D; u += TS_THREADS) {
    const int r = u / GROUPS_D, q0 = (u % GROUPS_D) * TS_RD;
    float acc[TS_RD];
    const float* rowp = A + r * PA;
    conv_rolling<TS_RD, KMAX>([&](int j) { return rowp[pidx(q0 + j)]; }, s_wd, acc);
#pragma unroll
    for (int i = 0; i < TS_RD; ++i) Bm[r * TS_TD + q0 + i] = acc[i];
  }
  __syncthreads();
  // W pass: thread (q, group) produces rows group*TS_RW .. +TS_RW-1 of column q
  const int q = threadIdx.x % TS_TD;
  const int d = td0 + q;
  for (int wg = threadIdx.x / TS_TD; wg < TW / TS_RW; wg += TS_THREADS / TS_TD) {
    float acc[TS_RW];
    conv_rolling<TS_RW, KMAX>([&](int j) { return Bm[(wg * TS_RW + j) * TS_TD + q]; }, s_ww,
                              acc);
    if (d < D) {
#pragma unroll
      for (int i = 0; i < TS_RW; ++i) {
        const int w = tw0 + wg * TS_RW + i;
        if (w < W) a.mid[plane + (int64_t)w * D + d] = acc[i];
      }
    }
  }
}

// Pass B: grid (tiles_h * tiles_d, W, B*P); thread (q, group) of a
// TS_TH x TB_TD strip produces TS_RH consecutive h of column q.
template <int KMAX>
__global__ void __launch_bounds__(TS_THREADS) smooth_column_kernel(const __grid_constant__ TiledArgs a) {
  extern __shared__ float sm[];
  __shared__ float s_wh[KMAX];
  __shared__ int s_hi[MAX_ROWS];
  const int64_t bp = blockIdx.z;
  const int64_t b = bp / a.P;
  const int H = (int)a.H, W = (int)a.W, D = (int)a.D;
  const int w = blockIdx.y;
  const int tiles_d = (D + TB_TD - 1) / TB_TD;
  const int td0 = (blockIdx.x % tiles_d) * TB_TD;
  const int th0 = (blockIdx.x / tiles_d) * TS_TH;
  const int q = threadIdx.x % TB_TD, hg = threadIdx.x / TB_TD;
  const int d = td0 + q;
  const int64_t plane_stride = (int64_t)W * D;
  const int64_t col = bp * a.HWD + (int64_t)w * D + d;  // + h * plane_stride
  if (a.mask != nullptr && a.mask[b] == 0) {
    if (a.copy_src != nullptr && d < D) {
      for (int i = 0; i < TS_RH; ++i) {
        const int h = th0 + hg * TS_RH + i;
        if (h >= H) break;
        const int64_t o = col + h * plane_stride;
        if (a.out_dtype == BA_BF16)
          ((uint16_t*)a.out)[o] = ((const uint16_t*)a.copy_src)[o];
        else
          ((float*)a.out)[o] = ((const float*)a.copy_src)[o];
      }
    }
    return;
  }
  const int ph = a.Kh / 2;
  constexpr int rowsS = TS_TH + KMAX - 1;
  float* S = sm;  // rowsS x TB_TD
  for (int r = threadIdx.x; r < rowsS; r += TS_THREADS)
    s_hi[r] = r < TS_TH + 2 * ph ? (int)pad_index(th0 - ph + r, H, a.padding) : -1;
  load_taps_smem<KMAX>(a.taps_h, b, a.Kh, s_wh);
  __syncthreads();
  for (int r = hg; r < rowsS; r += TS_THREADS / TB_TD) {
    const int hi = s_hi[r];
    S[r * TB_TD + q] = (hi >= 0 && d < D) ? a.mid[bp * a.HWD + hi * plane_stride + (int64_t)w * D + d]
                                          : 0.0f;
  }
  __syncthreads();
  float acc[TS_RH];
  conv_rolling<TS_RH, KMAX>([&](int j) { return S[(hg * TS_RH + j) * TB_TD + q]; }, s_wh, acc);
  if (d >= D) return;
  if (a.grid != nullptr) {
    // elastic: the component (P index of bp) is the displacement axis
    const int comp = (int)(bp % a.P);
    const float mag = a.magnitude[b];
    const int64_t sz = comp == 0 ? a.H : (comp == 1 ? a.W : a.D);
    const float n = (float)sz;
    const float half_lo = (n - 1.0f) / 2.0f;
    const float step = (half_lo - (-half_lo)) / (n - 1.0f);
    const float half = half_lo < 1e-6f ? 1e-6f : half_lo;
#pragma unroll
    for (int i = 0; i < TS_RH; ++i) {
      const int h = th0 + hg * TS_RH + i;
      if (h < H) {
        const int64_t idx = comp == 0 ? h : (comp == 1 ? w : d);
        const float c0 = linspace_at(-half_lo, half_lo, step, idx, sz);
        const int64_t s = (int64_t)h * plane_stride + (int64_t)w * D + d;
        a.grid[(b * a.HWD + s) * 3 + (2 - comp)] = (c0 + acc[i] * mag) / half;
      }
    }
    return;
  }
  if (a.sharp_blur != nullptr) {
    const float al = a.alpha[b];
#pragma unroll
    for (int i = 0; i < TS_RH; ++i) {
      const int h = th0 + hg * TS_RH + i;
      if (h < H) {
        const int64_t o = col + h * plane_stride;
        acc[i] = sharpen_combine(load_in(a.sharp_blur, a.out_dtype, o), acc[i], al, a.out_dtype);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < TS_RH; ++i) {
    const int h = th0 + hg * TS_RH + i;
    if (h < H) {
      const int64_t o = col + h * plane_stride;
      if (a.out_dtype == BA_BF16)
        ((uint16_t*)a.out)[o] = f32_to_bf16_bits(acc[i]);
      else
        ((float*)a.out)[o] = acc[i];
    }
  }
}

int tiled_kmax(int K) {
  for (int k : {7, 15, 23, 31, 47, 63})
    if (K <= k) return k;
  return 0;
}

size_t plane_smem(int kmax) {
  const int rowsA = plane_tw(kmax) + kmax - 1, colsA = TS_TD + kmax - 1;
  const int PA = pidx(colsA - 1) + 1;
  return (size_t)(rowsA * PA + rowsA * TS_TD) * sizeof(float);
}

size_t column_smem(int kmax) { return (size_t)((TS_TH + kmax - 1) * TB_TD) * sizeof(float); }

template <int KMAX>
ba_status launch_tiled_kmax(const TiledArgs& a, int64_t planes, cudaStream_t st) {
  const size_t sa = plane_smem(KMAX), sb = column_smem(KMAX);
  // opt in to more than 48 KB of dynamic shared memory (B200: 227 KB per CTA)
  cudaFuncSetAttribute(smooth_plane_kernel<KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)sa);
  cudaFuncSetAttribute(smooth_column_kernel<KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)sb);
  constexpr int TW = plane_tw(KMAX);
  const int tiles_d = (int)((a.D + TS_TD - 1) / TS_TD);
  dim3 ga((unsigned)(tiles_d * ((a.W + TW - 1) / TW)), (unsigned)a.H, (unsigned)planes);
  smooth_plane_kernel<KMAX><<<ga, TS_THREADS, sa, st>>>(a);
  ba_status s = check_launch("smooth pass A");
  if (s != BA_OK) return s;
  const int tiles_db = (int)((a.D + TB_TD - 1) / TB_TD);
  dim3 gb((unsigned)(tiles_db * ((a.H + TS_TH - 1) / TS_TH)), (unsigned)a.W, (unsigned)planes);
  smooth_column_kernel<KMAX><<<gb, TS_THREADS, sb, st>>>(a);
  return check_launch("smooth pass B");
}

ba_status launch_tiled(const TiledArgs& a, int64_t planes, cudaStream_t st) {
  const int K = std::max(a.Kh, std::max(a.Kw, a.Kd));
  switch (tiled_kmax(K)) {
    case 7: return launch_tiled_kmax<7>(a, planes, st);
    case 15: return launch_tiled_kmax<15>(a, planes, st);
    case 23: return launch_tiled_kmax<23>(a, planes, st);
    case 31: return launch_tiled_kmax<31>(a, planes, st);
    case 47: return launch_tiled_kmax<47>(a, planes, st);
    default: return launch_tiled_kmax<63>(a, planes, st);
  }
}

// ===========================================================================
// Streaming separable smoothing (used for KMAX <= SS_KMAX_MAX).
//
// One CTA owns an SS_TW (W) x SS_TD (D) column block of one (element,
// channel) plane stack and walks its H range plane by plane:
//   1. the plane's tile with its W/D halo arrives one plane ahead: as whole
//      16-byte chunks copied by cp.async into a double-buffered raw stage
//      (rows 16-byte aligned), then converted once into the padded fp32 tile
//      with the D padding rule applied through a per-thread column map; or,
//      for unaligned rows, element by element through registers;
//   2. D correlation of every tile row (SS_RD outputs per thread unit);
//   3. W correlation (SS_RW outputs per thread), the result V of the plane
//      written to a per-thread ring of the last RING planes in shared memory;
//   4. every SS_RH planes, the H correlation of SS_RH output planes from the
//      ring, and the epilogue (cast, or the unsharp-mask combination).
// The ring holds one float4 (the thread's SS_RW columns) per plane and
// thread; a thread only reads back the entries it wrote, so the ring needs no
// barrier.  After each flush the slots of planes no later window reads are
// zeroed, so a window that runs past the fed planes (taps beyond the runtime
// K) meets exact zeros.  HBM sees one read of the input (plus the H halo of
// each chunk) and one write of the output; nothing intermediate leaves the
// SM.  Tile entries beyond the runtime halo are zero-filled likewise.
// ===========================================================================
constexpr int SS_THREADS = 128;
constexpr int SS_TD = 32;  // D extent of the block: one warp's lanes
constexpr int SS_TW = 16;  // W extent: 4 warps x SS_RW rows
constexpr int SS_RD = 8;   // D outputs per thread unit in step 2
constexpr int SS_RW = 4;   // W outputs per thread in step 3
constexpr int SS_RH = 4;   // H outputs per thread and column per flush
constexpr int SS_KMAX_MAX = 23;
static_assert(SS_TW == (SS_THREADS / SS_TD) * SS_RW, "step 3: one run of SS_RW rows per warp");

template <int KMAX>
struct SsGeom {
  static constexpr int ROWS = SS_TW + KMAX - 1;  // tile rows (W with halo)
  static constexpr int COLS = SS_TD + KMAX - 1;  // tile columns (D with halo)
  static constexpr int RS = COLS | 1;  // odd row stride: the step-2 reads hit 32 banks
  static constexpr int NLOAD = (ROWS * COLS + SS_THREADS - 1) / SS_THREADS;
  static constexpr int BS = SS_TD + 1;  // step-2 output row stride (conflict-free writes)
  static constexpr int DUNITS = ROWS * (SS_TD / SS_RD);
  static constexpr int RING = SS_RH + KMAX - 1;
  static constexpr int TILE_FLOATS = (ROWS * RS + 3) / 4 * 4;
  static constexpr int BM_FLOATS = (ROWS * BS + 3) / 4 * 4;
  static constexpr int RING_FLOATS = RING * SS_TW * SS_TD;
  static constexpr size_t SMEM = (size_t)(TILE_FLOATS + BM_FLOATS + RING_FLOATS) * sizeof(float);
};

// Raw staging of a plane's tile for the cp.async path: whole 16-byte chunks,
// the D window widened to chunk boundaries (XO elements each side).
template <int KMAX, int DT>
struct SsRaw {
  static constexpr int ESZ = DT == BA_BF16 ? 2 : 4;
  static constexpr int CH = 16 / ESZ;  // elements per chunk
  static constexpr int PMAX = (KMAX - 1) / 2;
  static constexpr int XO = (PMAX + CH - 1) / CH * CH;
  static constexpr int RP = SS_TD + 2 * XO;  // row pitch, elements (a whole number of chunks)
  static constexpr int CPR = RP / CH;
  static constexpr int ROWS = SS_TW + KMAX - 1;
  static constexpr int NCHUNK = ROWS * CPR;
  static constexpr int CPT = (NCHUNK + SS_THREADS - 1) / SS_THREADS;
  static constexpr int STAGE_BYTES = ROWS * RP * ESZ;
  static constexpr size_t SMEM = 2 * (size_t)STAGE_BYTES;
};

// R outputs acc[i] = sum_k w[k] * x(i + k), taps in registers.
template <int R, int KMAX, typename Load>
__device__ __forceinline__ void conv_regs(Load x, const float (&w)[KMAX], float* acc) {
  float xw[R + KMAX - 1];
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int j = 0; j < R - 1; ++j) xw[j] = x(j);
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    xw[k + R - 1] = x(k + R - 1);
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = __fmaf_rn(w[k], xw[i + k], acc[i]);
  }
}

// Taps of length K (odd, <= KMAX) centred in a KMAX array with zeros on both
// sides: correlating a window whose centre sits at PMAX = (KMAX-1)/2 then
// equals the K-tap correlation, the extra taps adding exact zeros.
template <int KMAX>
__device__ __forceinline__ void load_taps_centred(const float* taps, int64_t b, int K,
                                                  float (&w)[KMAX]) {
  const int off = (KMAX - K) / 2;
#pragma unroll
  for (int k = 0; k < KMAX; ++k)
    w[k] = (k >= off && k < off + K) ? __ldg(taps + b * K + (k - off)) : 0.0f;
}

template <int KMAX>
__device__ __forceinline__ void load_taps_regs(const float* taps, int64_t b, int K, float (&w)[KMAX]) {
#pragma unroll
  for (int k = 0; k < KMAX; ++k) w[k] = k < K ? __ldg(taps + b * K + k) : 0.0f;
}

template <int DT>
__device__ __forceinline__ float ld_dt(const void* p, int64_t i) {
  return DT == BA_BF16 ? bf16_bits_to_f32(__ldg((const unsigned short*)p + i))
                       : __ldg((const float*)p + i);
}

template <int DT>
__device__ __forceinline__ void st_dt(void* p, int64_t i, float v) {
  if (DT == BA_BF16)
    ((uint16_t*)p)[i] = f32_to_bf16_bits(v);
  else
    ((float*)p)[i] = v;
}

// Grid (tiles_d * tiles_w, n_chunks, B*P); chunk c covers output planes
// [c * h_chunk, min(H, (c+1) * h_chunk)).
template <int KMAX, int DT, bool ASYNC>
__global__ void __launch_bounds__(SS_THREADS, 4)
    smooth_stream_kernel(const __grid_constant__ TiledArgs a, int32_t h_chunk) {
  using G = SsGeom<KMAX>;
  using RW = SsRaw<KMAX, DT>;
  extern __shared__ float sm[];
  float* tile = sm;
  float* bm = sm + G::TILE_FLOATS;
  float4* ring4 = reinterpret_cast<float4*>(bm + G::BM_FLOATS);
  const int tid = threadIdx.x;
  const int64_t bp = blockIdx.z;
  const int64_t b = bp / a.P;
  const int H = (int)a.H, W = (int)a.W, D = (int)a.D;
  const int tiles_d = (D + SS_TD - 1) / SS_TD;
  const int d0 = (blockIdx.x % tiles_d) * SS_TD;
  const int w0 = (blockIdx.x / tiles_d) * SS_TW;
  const int hs = blockIdx.y * h_chunk;
  const int he = min(H, hs + h_chunk);
  const int lane_d = tid % SS_TD, wg = tid / SS_TD;
  const int64_t plane_sz = (int64_t)W * D;
  const int64_t stack = bp * (int64_t)H * plane_sz;  // offset of plane 0 of this stack

  if (a.mask != nullptr && a.mask[b] == 0) {
    // the reference's torch.where: masked-out elements keep the input
    if (a.copy_src == nullptr) return;
    const int d = d0 + lane_d;
    if (d >= D) return;
    for (int h = hs; h < he; ++h)
#pragma unroll
      for (int c = 0; c < SS_RW; ++c) {
        const int w = w0 + wg * SS_RW + c;
        if (w < W) {
          const int64_t o = stack + h * plane_sz + (int64_t)w * D + d;
          st_dt<DT>(a.out, o, ld_dt<DT>(a.copy_src, o));
        }
      }
    return;
  }

  const int ph = a.Kh / 2, pw = a.Kw / 2, pd = a.Kd / 2;
  float wd[KMAX], ww[KMAX], wh[KMAX];
  load_taps_regs<KMAX>(a.taps_d, b, a.Kd, wd);
  load_taps_regs<KMAX>(a.taps_w, b, a.Kw, ww);
  load_taps_regs<KMAX>(a.taps_h, b, a.Kh, wh);

  // Register path: in-plane source offset of each tile entry this thread
  // loads (-1: zero).  cp.async path: the in-plane source offset of each
  // raw chunk this thread copies (-1: none, the stage stays zero there) and
  // the raw column that feeds each of its two conversion columns.
  constexpr int NOFF = ASYNC ? RW::CPT : G::NLOAD;
  int32_t off[NOFF];
  int32_t rcol[2];
  unsigned char* raw = reinterpret_cast<unsigned char*>(ring4 + G::RING_FLOATS / 4);
  if constexpr (ASYNC) {
#pragma unroll
    for (int i = 0; i < RW::CPT; ++i) {
      const int c = tid + i * SS_THREADS;
      const int rr = c / RW::CPR, k = c % RW::CPR;
      const int r = rr - (RW::PMAX - pw);  // tile row fed by raw row rr
      int32_t o = -1;
      if (c < RW::NCHUNK && r >= 0 && r < SS_TW + 2 * pw) {
        const int64_t wi = pad_index(w0 - pw + r, W, a.padding);
        const int x = d0 - RW::XO + k * RW::CH;
        if (wi >= 0 && x >= 0 && x + RW::CH <= D) o = (int32_t)(wi * D + x);
      }
      off[i] = o;
    }
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int col = lane_d + SS_TD * cc;
      int32_t rc = -1;
      if (col < G::COLS && col < SS_TD + 2 * pd) {
        const int64_t dd = pad_index(d0 - pd + col, D, a.padding);
        if (dd >= 0) rc = (int32_t)(dd - (d0 - RW::XO));
      }
      rcol[cc] = rc;
    }
    // entries the conversion never writes stay zero; chunks never copied too
    for (int i = tid; i < G::TILE_FLOATS; i += SS_THREADS) tile[i] = 0.0f;
    for (int i = tid; i < (int)(RW::SMEM / 16); i += SS_THREADS)
      reinterpret_cast<float4*>(raw)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
#pragma unroll
    for (int i = 0; i < G::NLOAD; ++i) {
      const int e = tid + i * SS_THREADS;
      const int row = e / G::COLS, col = e % G::COLS;
      int32_t o = -1;
      if (e < G::ROWS * G::COLS && row < SS_TW + 2 * pw && col < SS_TD + 2 * pd) {
        const int64_t wi = pad_index(w0 - pw + row, W, a.padding);
        const int64_t di = pad_index(d0 - pd + col, D, a.padding);
        if (wi >= 0 && di >= 0) o = (int32_t)(wi * D + di);
      }
      off[i] = o;
    }
    rcol[0] = rcol[1] = -1;
  }
  // zero ring: taps beyond K and not-yet-fed planes meet zeros
  for (int i = tid; i < G::RING_FLOATS / 4; i += SS_THREADS)
    ring4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  int64_t obase[SS_RW];
  uint32_t col_ok = 0;
#pragma unroll
  for (int c = 0; c < SS_RW; ++c) {
    const int w = w0 + wg * SS_RW + c, d = d0 + lane_d;
    obase[c] = stack + (int64_t)w * D + d;
    if (w < W && d < D) col_ok |= 1u << c;
  }

  const int q_begin = hs - ph, q_end = he + ph;  // padded plane range fed through
  // source plane of padded index q (-1: a zero plane)
  auto src_plane = [&](int q) -> int { return (int)pad_index(q, H, a.padding); };
  float pre[ASYNC ? 1 : G::NLOAD];
  auto fetch = [&](int q) {
    const int sp = src_plane(q);
    if constexpr (ASYNC) {
      if (sp >= 0) {
        const char* pb = (const char*)a.in + (stack + sp * plane_sz) * RW::ESZ;
        unsigned char* st = raw + ((q - q_begin) & 1) * RW::STAGE_BYTES;
#pragma unroll
        for (int i = 0; i < RW::CPT; ++i) {
          const int c = tid + i * SS_THREADS;
          if (off[i] >= 0)
            cp_async16(st + (c / RW::CPR * RW::RP + c % RW::CPR * RW::CH) * RW::ESZ,
                       pb + (int64_t)off[i] * RW::ESZ);
        }
      }
      cp_async_commit();
    } else {
#pragma unroll
      for (int i = 0; i < G::NLOAD; ++i)
        pre[i] = (sp >= 0 && off[i] >= 0) ? ld_dt<DT>(a.in, stack + sp * plane_sz + off[i]) : 0.0f;
    }
  };
  if constexpr (ASYNC) __syncthreads();  // the zeroed stages before any copy lands
  fetch(q_begin);
  int next_out = hs;
  const float al = a.sharp_blur != nullptr ? a.alpha[b] : 0.0f;
  for (int q = q_begin; q < q_end; ++q) {
    const int slot = (q - q_begin) % G::RING;
    const bool zero_plane = src_plane(q) < 0;
    if constexpr (ASYNC) {
      // 1. copies of plane q+1 in flight; plane q's have landed (this
      //    thread's), the barrier makes every thread's visible
      if (q + 1 < q_end)
        fetch(q + 1);
      else
        cp_async_commit();
      cp_async_wait<1>();
      __syncthreads();
      if (!zero_plane) {
        const unsigned char* st = raw + ((q - q_begin) & 1) * RW::STAGE_BYTES;
        const int rofs = RW::PMAX - pw;
#pragma unroll
        for (int i = 0; i < (G::ROWS + 3) / 4; ++i) {
          const int r = wg + 4 * i;
          if (r < SS_TW + 2 * pw) {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              if (rcol[cc] >= 0) {
                const int ri = (r + rofs) * RW::RP + rcol[cc];
                tile[r * G::RS + lane_d + SS_TD * cc] =
                    DT == BA_BF16 ? bf16_bits_to_f32(((const uint16_t*)st)[ri])
                                  : ((const float*)st)[ri];
              }
            }
          }
        }
      }
      __syncthreads();
    } else {
      if (!zero_plane) {
        // 1. prefetched plane -> shared tile (the previous plane's step 2 is done)
#pragma unroll
        for (int i = 0; i < G::NLOAD; ++i) {
          const int e = tid + i * SS_THREADS;
          if (e < G::ROWS * G::COLS) tile[e + e / G::COLS * (G::RS - G::COLS)] = pre[i];
        }
      }
      __syncthreads();
      if (q + 1 < q_end) fetch(q + 1);
    }
    if (!zero_plane) {
      // 2. D correlation of every tile row
      for (int u = tid; u < G::DUNITS; u += SS_THREADS) {
        const int r = u / (SS_TD / SS_RD), q0 = (u % (SS_TD / SS_RD)) * SS_RD;
        const float* rowp = tile + r * G::RS + q0;
        float acc[SS_RD];
        conv_regs<SS_RD, KMAX>([&](int j) { return rowp[j]; }, wd, acc);
#pragma unroll
        for (int i = 0; i < SS_RD; ++i) bm[r * G::BS + q0 + i] = acc[i];
      }
    }
    __syncthreads();
    // 3. W correlation -> ring slot of plane q (own columns only)
    float v[SS_RW];
    if (!zero_plane) {
      conv_regs<SS_RW, KMAX>([&](int j) { return bm[(wg * SS_RW + j) * G::BS + lane_d]; }, ww,
                             v);
    } else {
#pragma unroll
      for (int c = 0; c < SS_RW; ++c) v[c] = 0.0f;
    }
    ring4[slot * SS_THREADS + tid] = make_float4(v[0], v[1], v[2], v[3]);
    // 4. flush SS_RH output planes once their last input plane is in
    const bool last = q + 1 == q_end;
    if (next_out + SS_RH - 1 + ph <= q || (last && next_out < he)) {
      const int base = (next_out - hs) % G::RING;
      const float4* p0 = ring4 + base * SS_THREADS + tid;
      float acc[SS_RW][SS_RH];
#pragma unroll
      for (int c = 0; c < SS_RW; ++c)
#pragma unroll
        for (int i = 0; i < SS_RH; ++i) acc[c][i] = 0.0f;
      auto xslot = [&](int j) {
        const float4* p = p0 + j * SS_THREADS;
        return *(j >= G::RING - base ? p - G::RING * SS_THREADS : p);
      };
      float4 xw[SS_RH + KMAX - 1];
#pragma unroll
      for (int j = 0; j < SS_RH - 1; ++j) xw[j] = xslot(j);
#pragma unroll
      for (int k = 0; k < KMAX; ++k) {
        xw[k + SS_RH - 1] = xslot(k + SS_RH - 1);
#pragma unroll
        for (int i = 0; i < SS_RH; ++i) {
          acc[0][i] = __fmaf_rn(wh[k], xw[i + k].x, acc[0][i]);
          acc[1][i] = __fmaf_rn(wh[k], xw[i + k].y, acc[1][i]);
          acc[2][i] = __fmaf_rn(wh[k], xw[i + k].z, acc[2][i]);
          acc[3][i] = __fmaf_rn(wh[k], xw[i + k].w, acc[3][i]);
        }
      }
      // planes before the next window are never read again: zero their slots
#pragma unroll
      for (int i = 0; i < SS_RH; ++i) {
        float4* p = const_cast<float4*>(p0) + i * SS_THREADS;
        *(i >= G::RING - base ? p - G::RING * SS_THREADS : p) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int c = 0; c < SS_RW; ++c) {
        if (!(col_ok & (1u << c))) continue;
#pragma unroll
        for (int i = 0; i < SS_RH; ++i) {
          const int h = next_out + i;
          if (h < he) {
            const int64_t o = obase[c] + h * plane_sz;
            float r = acc[c][i];
            if (a.sharp_blur != nullptr)
              r = sharpen_combine(ld_dt<DT>(a.sharp_blur, o), r, al, DT);
            st_dt<DT>(a.out, o, r);
          }
        }
      }
      next_out += SS_RH;
    }
  }
}

int sm_count_smooth() {
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

template <int KMAX, int DT, bool ASYNC>
ba_status launch_stream_kmax(const TiledArgs& a, int64_t planes, cudaStream_t st) {
  using G = SsGeom<KMAX>;
  const size_t smem = G::SMEM + (ASYNC ? SsRaw<KMAX, DT>::SMEM : 0);
  cudaFuncSetAttribute(smooth_stream_kernel<KMAX, DT, ASYNC>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int tiles_d = (int)((a.D + SS_TD - 1) / SS_TD);
  const int tiles_w = (int)((a.W + SS_TW - 1) / SS_TW);
  // chunk H until the grid covers the resident CTAs about twice
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, smooth_stream_kernel<KMAX, DT, ASYNC>,
                                                    SS_THREADS, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t slots = (int64_t)per_sm * sm_count_smooth();
  const int64_t blocks = (int64_t)tiles_d * tiles_w * planes;
  int64_t chunk = a.H;
  while (blocks * ((a.H + chunk - 1) / chunk) < 2 * slots && chunk / 2 >= 4 * KMAX) chunk /= 2;
  chunk = (chunk + SS_RH - 1) / SS_RH * SS_RH;
  dim3 g((unsigned)(tiles_d * tiles_w), (unsigned)((a.H + chunk - 1) / chunk), (unsigned)planes);
  smooth_stream_kernel<KMAX, DT, ASYNC><<<g, SS_THREADS, smem, st>>>(a, (int32_t)chunk);
  return check_launch("smooth stream");
}

// The cp.async path needs 16-byte aligned rows (D * element size a multiple
// of 16) and a 16-byte aligned source.
template <int DT, bool ASYNC>
ba_status launch_stream_a(const TiledArgs& a, int64_t planes, cudaStream_t st) {
  const int K = std::max(a.Kh, std::max(a.Kw, a.Kd));
  // an exact KMAX for the common sigma ranges (1.0 -> 9, 1.25 -> 11, 1.5 -> 13
  // taps at truncation 4): every zero tap is an FMA per voxel and axis
  if (K <= 7) return launch_stream_kmax<7, DT, ASYNC>(a, planes, st);
  if (K <= 9) return launch_stream_kmax<9, DT, ASYNC>(a, planes, st);
  if (K <= 11) return launch_stream_kmax<11, DT, ASYNC>(a, planes, st);
  if (K <= 13) return launch_stream_kmax<13, DT, ASYNC>(a, planes, st);
  if (K <= 15) return launch_stream_kmax<15, DT, ASYNC>(a, planes, st);
  return launch_stream_kmax<23, DT, ASYNC>(a, planes, st);
}

template <int DT>
ba_status launch_stream(const TiledArgs& a, int64_t planes, cudaStream_t st) {
  const int esz = DT == BA_BF16 ? 2 : 4;
  const bool aligned = (a.D * esz) % 16 == 0 && ((uintptr_t)a.in % 16) == 0;
  return aligned ? launch_stream_a<DT, true>(a, planes, st)
                 : launch_stream_a<DT, false>(a, planes, st);
}

// Uniform draw of the elastic field mapped to [-1,1), four values per thread
// from one Philox block (requires HWD % 4 == 0).
__global__ void elastic_draw4_kernel(uint32_t seed_lo, uint32_t seed_hi, uint64_t elem_offset,
                                     int64_t HWD, int64_t total4, float4* out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= total4) return;
  const int64_t per4 = 3 * HWD / 4;
  const int64_t b = i / per4;
  const uint64_t q = (uint64_t)(i - b * per4);  // (comp*HWD + s) >> 2
  const uint64_t eb = elem_offset + (uint64_t)b;
  const U4 ctr = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                  STREAM_ELASTIC | (uint32_t)(q >> 32)};
  const U4 r = philox4x32_10(ctr, seed_lo, seed_hi);
  out[i] = make_float4(u01(r.x) * 2.0f - 1.0f, u01(r.y) * 2.0f - 1.0f, u01(r.z) * 2.0f - 1.0f,
                       u01(r.w) * 2.0f - 1.0f);
}

ba_status launch_axis(int axis, const AxisArgs& a, int64_t planes, cudaStream_t st) {
  dim3 grid((unsigned)((a.HWD + SM_THREADS - 1) / SM_THREADS), (unsigned)planes);
  if (axis == 0)
    axis_pass_kernel<0><<<grid, SM_THREADS, 0, st>>>(a);
  else if (axis == 1)
    axis_pass_kernel<1><<<grid, SM_THREADS, 0, st>>>(a);
  else
    axis_pass_kernel<2><<<grid, SM_THREADS, 0, st>>>(a);
  return check_launch("axis pass");
}

// ===========================================================================
// Wide-tap separable smoothing (taps 24..63; the elastic field's K=43).
//
// Three coalesced passes, D then W then H, fp32 intermediates in scratch:
//   - D: a CTA stages RL_ROWS rows with their padded halo in shared memory
//     (for the elastic field the Philox draw is generated right there, so
//     the uniform field is never written) and correlates SS_RD outputs per
//     thread unit from a register window;
//   - W and H: a CTA stages the whole padded line of 32 D columns in
//     shared memory (roll_col_kernel) and each warp correlates chunks of
//     RC_R outputs from a register window, lanes along D.  Lines too long
//     to stage take a walk instead (roll_axis_kernel): each thread walks
//     one line, its outputs accumulating in a ring of KMAX registers (the
//     input at padded step q adds w[k] * x to output q - k, and output
//     q - (KMAX-1) is complete and stored), unrolled by KMAX so every ring
//     slot is a compile-time register.
// Every path accumulates the outputs in tap order, as the other smoothing
// paths do, so the two W/H forms give identical results.
// Taps are centred in KMAX-wide arrays (zeros outside the runtime K).  The
// H pass writes the output dtype (masked-out elements copy the input) or,
// for the elastic field, the grid_sample grid.
// ===========================================================================
constexpr int RL_THREADS = 128;
constexpr int RL_ROWS = 32;  // D pass: rows staged per CTA

// 4-byte cp.async (a thread stages its own inputs; no other thread reads them)
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(gmem) : "memory");
}

enum { RL_SRC_DT = 0, RL_SRC_PHILOX = 1, RL_SRC_UNIFORM = 2 };
enum { RL_OUT_F32 = 0, RL_OUT_DT = 1, RL_OUT_GRID = 2 };

struct RollArgs {
  const void* src;      // RL_SRC_DT: volume (in_dtype); RL_SRC_UNIFORM: u fp32
  int32_t in_dtype;
  void* dst;            // fp32 scratch, the output volume (out_dtype) or the grid
  int32_t out_dtype;
  const float* taps;    // (B, K) taps of this axis
  int32_t K;
  int32_t padding;
  int64_t batch, P, H, W, D;  // P planes per element
  const uint8_t* mask;  // RL_OUT_DT: masked-out elements copy copy_src (or are skipped)
  const void* copy_src;
  const void* sharp_blur;     // RL_OUT_DT: unsharp-mask combination with this blur
  const float* alpha;
  const float* magnitude;   // RL_OUT_GRID
  uint32_t seed_lo, seed_hi;  // RL_SRC_PHILOX
  uint64_t elem_offset;
  int32_t plane_major;  // W/H passes: planes along blockIdx.x
};

// D pass: grid (ceil(B*P*H*W / RL_ROWS)); each row is one line along D.
template <int KMAX, int SRC>
__global__ void __launch_bounds__(RL_THREADS) roll_d_kernel(const __grid_constant__ RollArgs a) {
  constexpr int PMAX = (KMAX - 1) / 2;
  extern __shared__ float srow[];
  const int D = (int)a.D;
  const int LS = D + KMAX - 1;  // staged row length
  // one pad word every 8 entries (the R=8 units of a row read distinct banks)
  // and SS_RD - 1 zero entries past the row, so a unit's window never needs
  // a bounds check
  const int LSP = pidx(LS + SS_RD - 2) + 1;
  const int64_t rows_per_elem = a.P * a.H * a.W;
  const int64_t total = a.batch * rows_per_elem;
  const int64_t row0 = (int64_t)blockIdx.x * RL_ROWS;
  const int nrows = (int)(total - row0 < RL_ROWS ? total - row0 : RL_ROWS);
  const int tid = threadIdx.x;
  // element and row-within-element of each staged row: one 64-bit division
  // per row for the whole CTA, none in the loops below
  __shared__ int32_t s_elem[RL_ROWS];
  __shared__ int64_t s_erow[RL_ROWS];
  if (tid < nrows) {
    const int64_t row = row0 + tid;
    const int64_t b = row / rows_per_elem;
    s_elem[tid] = (int32_t)b;
    s_erow[tid] = row - b * rows_per_elem;
  }
  if (SRC == RL_SRC_PHILOX) {
    // zero padding: PMAX entries before the row, PMAX + SS_RD - 1 after it
    const int npad = LS + SS_RD - 1 - D;
    {
      int r = tid / npad, j = tid % npad;
      const int step_r = RL_THREADS / npad, step_j = RL_THREADS % npad;
      while (r < nrows) {
        srow[r * LSP + pidx(j < PMAX ? j : D + j)] = 0.0f;
        j += step_j;
        r += step_r;
        if (j >= npad) j -= npad, ++r;
      }
    }
    __syncthreads();  // s_elem, s_erow
    // the elastic draw u*2-1 keyed as the standalone draw kernel keys it:
    // flat position p = comp*HWD + s of element b, four per Philox block
    // (D % 4 == 0, so a row starts a block); (row, block) pairs spread over
    // every thread of the CTA
    const int q4n = D / 4;
    int r = tid / q4n, q4 = tid % q4n;
    const int step_r = RL_THREADS / q4n, step_q = RL_THREADS % q4n;
    while (r < nrows) {
      const uint64_t q = (uint64_t)((s_erow[r] * D) >> 2) + (uint64_t)q4;
      const uint64_t eb = a.elem_offset + (uint64_t)s_elem[r];
      const U4 ctr = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                      STREAM_ELASTIC | (uint32_t)(q >> 32)};
      const U4 rr = philox4x32_10(ctr, a.seed_lo, a.seed_hi);
      float* sr = srow + r * LSP;
      const int j0 = PMAX + 4 * q4;
      sr[pidx(j0)] = u01(rr.x) * 2.0f - 1.0f;
      sr[pidx(j0 + 1)] = u01(rr.y) * 2.0f - 1.0f;
      sr[pidx(j0 + 2)] = u01(rr.z) * 2.0f - 1.0f;
      sr[pidx(j0 + 3)] = u01(rr.w) * 2.0f - 1.0f;
      q4 += step_q;
      r += step_r;
      if (q4 >= q4n) q4 -= q4n, ++r;
    }
  } else {
    for (int r = 0; r < nrows; ++r) {
      float* sr = srow + r * LSP;
      const int64_t base = (row0 + r) * D;
      for (int j = tid; j < LS + SS_RD - 1; j += RL_THREADS) {
        const int64_t di = j < LS ? pad_index(j - PMAX, D, a.padding) : -1;
        float v = 0.0f;
        if (di >= 0) {
          if (SRC == RL_SRC_UNIFORM)
            v = __ldg((const float*)a.src + base + di) * 2.0f - 1.0f;
          else
            v = load_in(a.src, a.in_dtype, base + di);
        }
        sr[pidx(j)] = v;
      }
    }
  }
  __syncthreads();
  float w[KMAX];
  const int nseg = (D + SS_RD - 1) / SS_RD;
  int cur_b = -1;
  int r = tid / nseg, seg = tid % nseg;
  const int step_r = RL_THREADS / nseg, step_s = RL_THREADS % nseg;
  while (r < nrows) {
    const int q0 = seg * SS_RD;
    const int64_t row = row0 + r;
    const int b = s_elem[r];
    if (b != cur_b) {
      load_taps_centred<KMAX>(a.taps, b, a.K, w);
      cur_b = b;
    }
    // q0 is a multiple of 8: pidx(q0 + j) = pidx(q0) + j + j / 8
    const float* x = srow + r * LSP + pidx(q0);
    float acc[SS_RD];
    conv_regs<SS_RD, KMAX>([&](int j) { return x[j + (j >> 3)]; }, w, acc);
    float* o = (float*)a.dst + row * D + q0;
    if ((D & 3) == 0 && q0 + SS_RD <= D) {
      reinterpret_cast<float4*>(o)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
#pragma unroll
      for (int i = 0; i < SS_RD; ++i)
        if (q0 + i < D) o[i] = acc[i];
    }
    seg += step_s;
    r += step_r;
    if (seg >= nseg) seg -= nseg, ++r;
  }
}

// Resident CTAs per SM the register budget is set for: the grid-writing H
// pass fits 4 at KMAX 43 without spills, the others 3.
constexpr int rl_axis_min_blocks(int kmax, int out) {
  return kmax > 47 ? 2 : (kmax > 43 ? 3 : (kmax > 31 && out != RL_OUT_GRID ? 3 : 4));
}

// W (AXIS 1) or H (AXIS 0) pass: a thread owns line (plane, o, d) with o
// the other in-plane axis and walks the axis of length N.  Grid
// (ceil(O*D / RL_THREADS), B*P), or (B*P, ceil(O*D / RL_THREADS)) with
// plane_major set, so that the CTAs writing the three interleaved
// components of one grid region run together.
//
// ZPAD (zero padding): the walk starts at the first real input (the PMAX
// padded steps before it would only add zeros to outputs below 0) and the
// steps past the last input skip their FMAs; skipping the addition of an
// exact zero product leaves every sum unchanged.
template <int KMAX, int AXIS, int OUT, bool ZPAD>
__global__ void __launch_bounds__(RL_THREADS, rl_axis_min_blocks(KMAX, OUT))
    roll_axis_kernel(const __grid_constant__ RollArgs a) {
  constexpr int PMAX = (KMAX - 1) / 2;
  constexpr int LEAD = ZPAD ? PMAX : 0;  // first walked step
  const int H = (int)a.H, W = (int)a.W, D = (int)a.D;
  const unsigned plane = a.plane_major ? blockIdx.x : blockIdx.y;  // b * P + p
  const unsigned lblk = a.plane_major ? blockIdx.y : blockIdx.x;
  const int b = (int)(plane / (unsigned)a.P);
  const int O = AXIS == 1 ? H : W;
  const int N = AXIS == 1 ? W : H;
  const unsigned idx = lblk * RL_THREADS + threadIdx.x;  // O * D < 2^31 (host check)
  if (idx >= (unsigned)O * (unsigned)D) return;
  const int o_ax = (int)(idx / (unsigned)D), d = (int)(idx - (unsigned)o_ax * (unsigned)D);
  const int64_t HWD = (int64_t)H * W * D;
  const int64_t stride = AXIS == 1 ? D : (int64_t)W * D;  // step along the walked axis
  const int64_t inplane = AXIS == 1 ? (int64_t)o_ax * W * D + d : (int64_t)o_ax * D + d;
  const int64_t base = (int64_t)plane * HWD + inplane;
  if (OUT == RL_OUT_DT && a.mask != nullptr && a.mask[b] == 0) {
    if (a.copy_src != nullptr)
      for (int n = 0; n < N; ++n) {
        const int64_t i = base + n * stride;
        if (a.out_dtype == BA_BF16)
          ((uint16_t*)a.dst)[i] = ((const uint16_t*)a.copy_src)[i];
        else
          ((float*)a.dst)[i] = ((const float*)a.copy_src)[i];
      }
    return;
  }
  float w[KMAX];
  load_taps_centred<KMAX>(a.taps, b, a.K, w);
  float acc[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) acc[k] = 0.0f;
  // grid epilogue constants (elastic): component = plane % 3
  const int comp = OUT == RL_OUT_GRID ? (int)(plane % 3u) : 0;
  float mag = 0.0f, half = 1.0f, rhalf = 0.0f, half_lo = 0.0f, step = 0.0f;
  int64_t csz = 1;
  if (OUT == RL_OUT_GRID) {
    mag = a.magnitude[b];
    csz = comp == 0 ? H : (comp == 1 ? W : D);
    const float n = (float)csz;
    half_lo = (n - 1.0f) / 2.0f;
    step = (half_lo - (-half_lo)) / (n - 1.0f);
    half = half_lo < 1e-6f ? 1e-6f : half_lo;
    rhalf = recip_for_div(half);
  }
  // grid coordinate of the components that do not vary along the walk
  float c_fixed = 0.0f;
  if (OUT == RL_OUT_GRID) {
    const int64_t cidx = comp == 2 ? d : o_ax;  // comp 1 (W) on the H walk, 0 (H) on a W walk
    c_fixed = linspace_at(-half_lo, half_lo, step, cidx, csz);
  }
  const bool walked = OUT == RL_OUT_GRID && comp == (AXIS == 0 ? 0 : 1);
  // grid element of output 0 of this line and the step between outputs
  const int64_t g0 = ((int64_t)b * HWD + inplane) * 3 + (2 - comp), gstep = 3 * stride;
  const float* src = (const float*)a.src;
  // Walk over padded steps t = LEAD .. N + KMAX - 2 in blocks of KMAX: step t
  // reads input t - PMAX and completes output t - (KMAX - 1).
  const int nblk = (N + KMAX - 1 - LEAD + KMAX - 1) / KMAX;
  extern __shared__ float xs[];  // 2 x KMAX x RL_THREADS: this thread's column
  auto stage_block = [&](int blk, int buf) {
    float* col = xs + buf * KMAX * RL_THREADS + threadIdx.x;
    const int p0 = LEAD + blk * KMAX - PMAX;  // input position of step 0
    if (p0 >= 0 && p0 + KMAX <= N) {
      const float* g = src + base + (int64_t)p0 * stride;
#pragma unroll
      for (int s = 0; s < KMAX; ++s) cp_async4(col + s * RL_THREADS, g + (int64_t)s * stride);
    } else {
      for (int s = 0; s < KMAX; ++s) {
        const int64_t pos = p0 + s < N + PMAX ? pad_index(p0 + s, N, a.padding) : -1;
        if (pos >= 0)
          cp_async4(col + s * RL_THREADS, src + base + pos * stride);
        else
          col[s * RL_THREADS] = 0.0f;
      }
    }
    cp_async_commit();
  };
  auto store = [&](int o, float v) {
    if (OUT == RL_OUT_F32) {
      ((float*)a.dst)[base + (int64_t)o * stride] = v;
    } else if (OUT == RL_OUT_DT) {
      const int64_t oi = base + (int64_t)o * stride;
      float r = v;
      if (a.sharp_blur != nullptr)
        r = sharpen_combine(load_in(a.sharp_blur, a.out_dtype, oi), v, a.alpha[b], a.out_dtype);
      if (a.out_dtype == BA_BF16)
        ((uint16_t*)a.dst)[oi] = f32_to_bf16_bits(r);
      else
        ((float*)a.dst)[oi] = r;
    } else {
      const float c0 = walked ? linspace_at(-half_lo, half_lo, step, o, csz) : c_fixed;
      ((float*)a.dst)[g0 + (int64_t)o * gstep] = div_rn(c0 + v * mag, half, rhalf);
    }
  };
  stage_block(0, 0);
  for (int blk = 0; blk < nblk; ++blk) {
    if (blk + 1 < nblk)
      stage_block(blk + 1, (blk + 1) & 1);
    else
      cp_async_commit();
    cp_async_wait<1>();
    const float* xb = xs + (blk & 1) * KMAX * RL_THREADS + threadIdx.x;
    const int o0 = LEAD + blk * KMAX - (KMAX - 1);  // output completed at step 0
    const int p0 = LEAD + blk * KMAX - PMAX;        // input read at step 0
    const bool all_out = o0 >= 0 && o0 + KMAX <= N;
    const int s_end = N - o0;                 // steps s < s_end complete an output
    const int s_in = ZPAD ? N - p0 : KMAX;    // steps s < s_in read a real input
#pragma unroll
    for (int s = 0; s < KMAX; ++s) {
      const int o = o0 + s;
      if (s >= s_end) break;  // past the last output
      if (!ZPAD || s < s_in) {
        const float x = xb[s * RL_THREADS];
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
          const int slot = (LEAD + s - k + KMAX) % KMAX;
          acc[slot] = __fmaf_rn(w[k], x, acc[slot]);
        }
      }
      const int slot_done = (LEAD + s + 1) % KMAX;
      if (all_out || o >= 0) store(o, acc[slot_done]);
      acc[slot_done] = 0.0f;
    }
  }
}

// W (AXIS 1) or H (AXIS 0) pass as a column tile: a CTA stages the whole
// padded line (N + KMAX - 1 positions) of RC_LANES consecutive D columns of
// one (plane, o) in shared memory, and each warp correlates chunks of RC_R
// consecutive outputs from a register window, lanes along D.  No input is
// staged twice and the loop body is one chunk, so the code stays small.
// Grid (B*P, O * ceil(D / RC_LANES)): planes fastest, so the CTAs writing
// the three interleaved components of one grid region run together.
constexpr int RC_LANES = 32;
constexpr int RC_WARPS = 4;
constexpr int RC_R = 8;

__host__ __device__ constexpr int rc_rows(int N, int kmax) { return N + kmax - 1 + RC_R - 1; }

template <int KMAX, int AXIS, int OUT>
__global__ void __launch_bounds__(RC_WARPS * 32) roll_col_kernel(const __grid_constant__ RollArgs a) {
  constexpr int PMAX = (KMAX - 1) / 2;
  extern __shared__ __align__(16) float col[];  // [rc_rows][RC_LANES]
  const int H = (int)a.H, W = (int)a.W, D = (int)a.D;
  const int N = AXIS == 1 ? W : H;
  const int dblocks = (D + RC_LANES - 1) / RC_LANES;
  const unsigned plane = blockIdx.x;  // b * P + p
  const int o_ax = (int)(blockIdx.y / (unsigned)dblocks);
  const int d0 = (int)(blockIdx.y - (unsigned)o_ax * (unsigned)dblocks) * RC_LANES;
  const int nd = min(RC_LANES, D - d0);
  const int b = (int)(plane / (unsigned)a.P);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t HWD = (int64_t)H * W * D;
  const int64_t stride = AXIS == 1 ? D : (int64_t)W * D;  // step along the walked axis
  const int64_t inplane = (AXIS == 1 ? (int64_t)o_ax * W * D : (int64_t)o_ax * D) + d0;
  const int64_t base = (int64_t)plane * HWD + inplane;  // position 0 of column d0
  if (OUT == RL_OUT_DT && a.mask != nullptr && a.mask[b] == 0) {
    if (a.copy_src != nullptr && lane < nd)
      for (int n = warp; n < N; n += RC_WARPS) {
        const int64_t i = base + n * stride + lane;
        if (a.out_dtype == BA_BF16)
          ((uint16_t*)a.dst)[i] = ((const uint16_t*)a.copy_src)[i];
        else
          ((float*)a.dst)[i] = ((const float*)a.copy_src)[i];
      }
    return;
  }
  // stage rows r = padded position (input r - PMAX); rows past the padded
  // line and lanes past D are zero
  const float* src = (const float*)a.src;
  const int rows = rc_rows(N, KMAX);
  if ((D & 3) == 0) {
    // 16-byte copies: 8 per row, 16 rows per pass of the CTA
    const int q = threadIdx.x & 7;
    for (int r = threadIdx.x >> 3; r < rows; r += RC_WARPS * 4) {
      const int64_t pos = r < N + KMAX - 1 ? pad_index(r - PMAX, N, a.padding) : -1;
      float* dstp = col + r * RC_LANES + 4 * q;
      if (pos >= 0 && 4 * q < nd)
        cp_async16(dstp, src + base + pos * stride + 4 * q);
      else
        *reinterpret_cast<float4*>(dstp) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  } else {
    for (int r = warp; r < rows; r += RC_WARPS) {
      const int64_t pos = r < N + KMAX - 1 ? pad_index(r - PMAX, N, a.padding) : -1;
      if (pos >= 0 && lane < nd)
        cp_async4(col + r * RC_LANES + lane, src + base + pos * stride + lane);
      else
        col[r * RC_LANES + lane] = 0.0f;
    }
  }
  cp_async_commit();
  float w[KMAX];
  load_taps_centred<KMAX>(a.taps, b, a.K, w);
  // grid epilogue constants (elastic): component = plane % 3
  const int comp = OUT == RL_OUT_GRID ? (int)(plane % 3u) : 0;
  float mag = 0.0f, half = 1.0f, rhalf = 0.0f, half_lo = 0.0f, step = 0.0f, c_fixed = 0.0f;
  int64_t csz = 1;
  if (OUT == RL_OUT_GRID) {
    mag = a.magnitude[b];
    csz = comp == 0 ? H : (comp == 1 ? W : D);
    const float n = (float)csz;
    half_lo = (n - 1.0f) / 2.0f;
    step = (half_lo - (-half_lo)) / (n - 1.0f);
    half = half_lo < 1e-6f ? 1e-6f : half_lo;
    rhalf = recip_for_div(half);
    // the coordinate of a component that does not vary along the walk
    const int64_t cidx = comp == 2 ? d0 + lane : o_ax;
    c_fixed = linspace_at(-half_lo, half_lo, step, cidx, csz);
  }
  const bool walked = OUT == RL_OUT_GRID && comp == (AXIS == 0 ? 0 : 1);
  const int64_t g0 = ((int64_t)b * HWD + inplane + lane) * 3 + (2 - comp), gstep = 3 * stride;
  cp_async_wait<0>();
  __syncthreads();
  const int nchunk = (N + RC_R - 1) / RC_R;
  for (int c = warp; c < nchunk; c += RC_WARPS) {
    const int q0 = c * RC_R;
    const float* x = col + q0 * RC_LANES + lane;
    float acc[RC_R];
    conv_regs<RC_R, KMAX>([&](int j) { return x[j * RC_LANES]; }, w, acc);
    if (lane < nd && q0 + RC_R <= N && OUT != RL_OUT_DT) {
      // a whole chunk: stores by pointer steps, no per-output bounds
      if (OUT == RL_OUT_F32) {
        float* op = (float*)a.dst + base + (int64_t)q0 * stride + lane;
#pragma unroll
        for (int i = 0; i < RC_R; ++i, op += stride) *op = acc[i];
      } else {
        // the grid: c0 + field * mag divided by half; every quotient takes
        // div_rn's fast path (RN(a*y) corrected by one fma) unless one of
        // the chunk's needs its slow path, then all go through div_rn
        float av[RC_R], r[RC_R];
        bool fast = rhalf != 0.0f;
#pragma unroll
        for (int i = 0; i < RC_R; ++i) {
          const float cw = walked ? linspace_at32(-half_lo, half_lo, step, q0 + i, (int)csz)
                                  : c_fixed;
          av[i] = cw + acc[i] * mag;
          const float q = __fmul_rn(av[i], rhalf);
          const float aq = fabsf(q);
          fast = fast && av[i] != 0.0f && aq >= 0x1p-100f && aq <= 0x1p100f;
          r[i] = __fmaf_rn(__fmaf_rn(-q, half, av[i]), rhalf, q);
        }
        if (!fast)
#pragma unroll
          for (int i = 0; i < RC_R; ++i) r[i] = div_rn(av[i], half, rhalf);
        float* gp = (float*)a.dst + g0 + (int64_t)q0 * gstep;
#pragma unroll
        for (int i = 0; i < RC_R; ++i, gp += gstep) *gp = r[i];
      }
    } else if (lane < nd) {
#pragma unroll
      for (int i = 0; i < RC_R; ++i) {
        const int o = q0 + i;
        if (o < N) {
          const float v = acc[i];
          const int64_t oi = base + (int64_t)o * stride + lane;
          if (OUT == RL_OUT_F32) {
            ((float*)a.dst)[oi] = v;
          } else if (OUT == RL_OUT_DT) {
            float r = v;
            if (a.sharp_blur != nullptr)
              r = sharpen_combine(load_in(a.sharp_blur, a.out_dtype, oi), v, a.alpha[b],
                                  a.out_dtype);
            if (a.out_dtype == BA_BF16)
              ((uint16_t*)a.dst)[oi] = f32_to_bf16_bits(r);
            else
              ((float*)a.dst)[oi] = r;
          } else {
            const float c0 = walked ? linspace_at(-half_lo, half_lo, step, o, csz) : c_fixed;
            ((float*)a.dst)[g0 + (int64_t)o * gstep] = div_rn(c0 + v * mag, half, rhalf);
          }
        }
      }
    }
  }
}

int roll_kmax(int K) {
  // 43 is the elastic field's K (sigma 7, truncated 3): no zero taps
  for (int k : {23, 31, 43, 47, 63})
    if (K <= k) return k;
  return 0;
}

// The column-tile pass when its staged line fits in shared memory and the
// (O, D-block) count fits grid.y; the ring walk otherwise.
template <int KMAX, int AXIS, int OUT>
bool launch_axis_col(const RollArgs& a, int64_t planes, cudaStream_t st) {
  const int64_t N = AXIS == 1 ? a.W : a.H, O = AXIS == 1 ? a.H : a.W;
  const int64_t yblocks = O * ((a.D + RC_LANES - 1) / RC_LANES);
  const size_t smem = (size_t)rc_rows((int)N, KMAX) * RC_LANES * sizeof(float);
  if (smem > 96 * 1024 || yblocks > 65535 || planes > 65535) return false;
  cudaFuncSetAttribute(roll_col_kernel<KMAX, AXIS, OUT>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  roll_col_kernel<KMAX, AXIS, OUT>
      <<<dim3((unsigned)planes, (unsigned)yblocks), RC_WARPS * 32, smem, st>>>(a);
  return true;
}

template <int KMAX, int AXIS, int OUT, bool ZPAD>
ba_status launch_axis_roll(const RollArgs& a, int64_t planes, cudaStream_t st, const char* what) {
  if (launch_axis_col<KMAX, AXIS, OUT>(a, planes, st)) return check_launch(what);
  const size_t xs = (size_t)2 * KMAX * RL_THREADS * sizeof(float);
  cudaFuncSetAttribute(roll_axis_kernel<KMAX, AXIS, OUT, ZPAD>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)xs);
  const int64_t lines = (AXIS == 1 ? a.H : a.W) * a.D;
  const unsigned lb = (unsigned)((lines + RL_THREADS - 1) / RL_THREADS);
  const dim3 g = a.plane_major ? dim3((unsigned)planes, lb) : dim3(lb, (unsigned)planes);
  roll_axis_kernel<KMAX, AXIS, OUT, ZPAD><<<g, RL_THREADS, xs, st>>>(a);
  return check_launch(what);
}

template <int KMAX>
ba_status launch_roll_kmax(int src_kind, int out_kind, const RollArgs& ad, const RollArgs& aw,
                           const RollArgs& ah, int64_t batch, cudaStream_t st) {
  const int64_t rows = batch * ad.P * ad.H * ad.W;
  const size_t smem =
      (size_t)RL_ROWS * (pidx((int)ad.D + KMAX - 1 + SS_RD - 2) + 1) * sizeof(float);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(roll_d_kernel<KMAX, RL_SRC_DT>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
        cudaFuncSetAttribute(roll_d_kernel<KMAX, RL_SRC_PHILOX>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
        cudaFuncSetAttribute(roll_d_kernel<KMAX, RL_SRC_UNIFORM>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 gd((unsigned)((rows + RL_ROWS - 1) / RL_ROWS));
  if (src_kind == RL_SRC_PHILOX)
    roll_d_kernel<KMAX, RL_SRC_PHILOX><<<gd, RL_THREADS, smem, st>>>(ad);
  else if (src_kind == RL_SRC_UNIFORM)
    roll_d_kernel<KMAX, RL_SRC_UNIFORM><<<gd, RL_THREADS, smem, st>>>(ad);
  else
    roll_d_kernel<KMAX, RL_SRC_DT><<<gd, RL_THREADS, smem, st>>>(ad);
  ba_status s = check_launch("wide smooth D pass");
  if (s != BA_OK) return s;
  const int64_t planes = batch * aw.P;
  const bool zp = aw.padding == BA_SMOOTH_ZEROS;
  s = zp ? launch_axis_roll<KMAX, 1, RL_OUT_F32, true>(aw, planes, st, "wide smooth W pass")
         : launch_axis_roll<KMAX, 1, RL_OUT_F32, false>(aw, planes, st, "wide smooth W pass");
  if (s != BA_OK) return s;
  if (out_kind == RL_OUT_GRID)  // the elastic field is zero-padded
    return launch_axis_roll<KMAX, 0, RL_OUT_GRID, true>(ah, planes, st, "wide smooth H pass");
  return zp ? launch_axis_roll<KMAX, 0, RL_OUT_DT, true>(ah, planes, st, "wide smooth H pass")
            : launch_axis_roll<KMAX, 0, RL_OUT_DT, false>(ah, planes, st, "wide smooth H pass");
}

ba_status launch_roll(int kmax, int src_kind, int out_kind, const RollArgs& ad, const RollArgs& aw,
                      const RollArgs& ah, int64_t batch, cudaStream_t st) {
  switch (kmax) {
    case 23: return launch_roll_kmax<23>(src_kind, out_kind, ad, aw, ah, batch, st);
    case 31: return launch_roll_kmax<31>(src_kind, out_kind, ad, aw, ah, batch, st);
    case 43: return launch_roll_kmax<43>(src_kind, out_kind, ad, aw, ah, batch, st);
    case 47: return launch_roll_kmax<47>(src_kind, out_kind, ad, aw, ah, batch, st);
    default: return launch_roll_kmax<63>(src_kind, out_kind, ad, aw, ah, batch, st);
  }
}

}  // namespace
}  // namespace ba

extern "C" int64_t ba_gauss_taps_len(double max_sigma, double truncated) {
  double s = max_sigma < 1e-6 ? 1e-6 : max_sigma;
  // sigma is clamped in fp32 by the reference; max_sigma arrives as the
  // float32 value widened to double (Tensor.item()).
  s = (double)(float)s;
  const double t = s * truncated;
  const int64_t tail = (int64_t)((t > 0.5 ? t : 0.5) + 0.5);
  return 2 * tail + 1;
}

extern "C" ba_status ba_gauss_taps(const float* sigmas, int64_t batch, int64_t K, float* taps,
                                   ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(batch >= 0, "ba_gauss_taps: negative batch");
  BA_REQUIRE(K >= 1 && K <= MAX_TAPS && (K % 2) == 1, "ba_gauss_taps: K=%lld must be odd, 1..%d",
             (long long)K, MAX_TAPS);
  if (batch == 0) return BA_OK;
  BA_REQUIRE(sigmas && taps, "ba_gauss_taps: NULL pointer");
  gauss_taps_kernel<<<(unsigned)((batch + GT_THREADS / 32 - 1) / (GT_THREADS / 32)), GT_THREADS, 0,
                      (cudaStream_t)stream>>>(sigmas, batch, K, taps);
  return check_launch("ba_gauss_taps");
}

extern "C" size_t ba_smooth_workspace_bytes(int64_t batch, int64_t channels, int64_t H, int64_t W,
                                            int64_t D) {
  if (batch < 0 || channels < 0 || H < 0 || W < 0 || D < 0) return 0;
  return (size_t)(2 * batch * channels * H * W * D) * sizeof(float);
}

namespace ba {
namespace {

// One separable smooth of (planes = B*P, H, W, D) from `src` (in_dtype) to
// `dst` (out_dtype), scratch t0/t1 (fp32, planes*HWD each; the tiled path
// uses t0 only).  Masked-out elements copy copy_src (or are skipped when it
// is NULL); with sharp_blur set, the last pass writes the unsharp-mask
// combination instead of the blur.
struct SmoothJob {
  const void* src;
  int32_t in_dtype;
  void* dst;
  int32_t out_dtype;
  int64_t P, planes, H, W, D;
  const float* taps[3];  // H, W, D
  int64_t K[3];
  int32_t padding;
  const uint8_t* mask;
  const void* copy_src;
  const void* sharp_blur;
  const float* alpha;
  float* t0;
  float* t1;
};

ba_status run_smooth(const SmoothJob& j, cudaStream_t st) {
  const int64_t HWD = j.H * j.W * j.D;
  const int64_t kmax = std::max(j.K[0], std::max(j.K[1], j.K[2]));
  const bool streamable = kmax <= SS_KMAX_MAX && j.in_dtype == j.out_dtype &&
                          j.W * j.D < ((int64_t)1 << 31) &&
                          ((j.D + SS_TD - 1) / SS_TD) * ((j.W + SS_TW - 1) / SS_TW) <= 0x7FFFFFFF;
  const bool rollable = !streamable && roll_kmax((int)kmax) != 0 &&
                        j.H * j.D <= ((int64_t)1 << 31) && j.W * j.D <= ((int64_t)1 << 31);
  if (rollable) {
    RollArgs r;
    memset(&r, 0, sizeof(r));
    r.batch = j.planes / j.P;
    r.P = j.P;
    r.H = j.H;
    r.W = j.W;
    r.D = j.D;
    r.padding = j.padding;
    RollArgs rd = r, rw = r, rh = r;
    rd.src = j.src;
    rd.in_dtype = j.in_dtype;
    rd.dst = j.t0;
    rd.taps = j.taps[2];
    rd.K = (int32_t)j.K[2];
    rw.src = j.t0;
    rw.dst = j.t1;
    rw.taps = j.taps[1];
    rw.K = (int32_t)j.K[1];
    rh.src = j.t1;
    rh.dst = j.dst;
    rh.out_dtype = j.out_dtype;
    rh.taps = j.taps[0];
    rh.K = (int32_t)j.K[0];
    rh.mask = j.mask;
    rh.copy_src = j.copy_src;
    rh.sharp_blur = j.sharp_blur;
    rh.alpha = j.alpha;
    return launch_roll(roll_kmax((int)kmax), RL_SRC_DT, RL_OUT_DT, rd, rw, rh, r.batch, st);
  }
  if (streamable || (tiled_kmax((int)kmax) != 0 && j.H <= 65535 && j.W <= 65535)) {
    TiledArgs t;
    memset(&t, 0, sizeof(t));
    t.in = j.src;
    t.in_dtype = j.in_dtype;
    t.mid = j.t0;
    t.out = j.dst;
    t.out_dtype = j.out_dtype;
    t.taps_h = j.taps[0];
    t.taps_w = j.taps[1];
    t.taps_d = j.taps[2];
    t.Kh = (int32_t)j.K[0];
    t.Kw = (int32_t)j.K[1];
    t.Kd = (int32_t)j.K[2];
    t.padding = j.padding;
    t.P = j.P;
    t.H = j.H;
    t.W = j.W;
    t.D = j.D;
    t.HWD = HWD;
    t.mask = j.mask;
    t.copy_src = j.copy_src;
    t.sharp_blur = j.sharp_blur;
    t.alpha = j.alpha;
    if (streamable)
      return j.out_dtype == BA_BF16 ? launch_stream<BA_BF16>(t, j.planes, st)
                                    : launch_stream<BA_F32>(t, j.planes, st);
    return launch_tiled(t, j.planes, st);
  }
  AxisArgs a;
  memset(&a, 0, sizeof(a));
  a.P = j.P;
  a.H = j.H;
  a.W = j.W;
  a.D = j.D;
  a.HWD = HWD;
  a.padding = j.padding;
  // H pass: src -> t0
  a.in = j.src;
  a.in_dtype = j.in_dtype;
  a.out = j.t0;
  a.out_dtype = BA_F32;
  a.taps = j.taps[0];
  a.K = (int32_t)j.K[0];
  ba_status s = launch_axis(0, a, j.planes, st);
  if (s != BA_OK) return s;
  // W pass: t0 -> t1
  a.in = j.t0;
  a.in_dtype = BA_F32;
  a.out = j.t1;
  a.taps = j.taps[1];
  a.K = (int32_t)j.K[1];
  s = launch_axis(1, a, j.planes, st);
  if (s != BA_OK) return s;
  // D pass: t1 -> dst; masked-out elements copy copy_src
  a.in = j.t1;
  a.out = j.dst;
  a.out_dtype = j.out_dtype;
  a.taps = j.taps[2];
  a.K = (int32_t)j.K[2];
  a.mask = j.mask;
  a.copy_src = j.mask ? j.copy_src : nullptr;
  a.sharp_blur = j.sharp_blur;
  a.alpha = j.alpha;
  return launch_axis(2, a, j.planes, st);
}

ba_status check_taps(const char* who, const int64_t* K, int64_t H, int64_t W, int64_t D,
                     int32_t padding) {
  for (int i = 0; i < 3; ++i)
    BA_REQUIRE(K[i] >= 1 && K[i] <= MAX_TAPS && (K[i] % 2) == 1, "%s: K=%lld must be odd, 1..%d",
               who, (long long)K[i], MAX_TAPS);
  if (padding == BA_SMOOTH_REFLECT) {
    // F.pad(mode="reflect") needs the pad to be smaller than the axis
    BA_REQUIRE(K[0] / 2 < H && K[1] / 2 < W && K[2] / 2 < D,
               "%s: reflect padding needs K/2 < size along every axis", who);
  }
  return BA_OK;
}

size_t align16(size_t n) { return (n + 15) & ~(size_t)15; }

}  // namespace
}  // namespace ba

extern "C" ba_status ba_smooth3d(const void* src, void* dst, int32_t dtype, int64_t batch,
                                 int64_t channels, int64_t H, int64_t W, int64_t D,
                                 const float* taps_h, int64_t Kh, const float* taps_w, int64_t Kw,
                                 const float* taps_d, int64_t Kd, int32_t padding,
                                 const uint8_t* mask, void* workspace, size_t workspace_bytes,
                                 ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(dtype == BA_F32 || dtype == BA_BF16, "ba_smooth3d: bad dtype %d", dtype);
  BA_REQUIRE(batch >= 0 && channels >= 0 && H > 0 && W > 0 && D > 0, "ba_smooth3d: bad shape");
  BA_REQUIRE(batch * channels <= 65535, "ba_smooth3d: batch*channels exceeds 65535");
  BA_REQUIRE(padding >= BA_SMOOTH_ZEROS && padding <= BA_SMOOTH_REPLICATE,
             "ba_smooth3d: unknown padding %d", padding);
  const int64_t K[3] = {Kh, Kw, Kd};
  ba_status s = check_taps("ba_smooth3d", K, H, W, D, padding);
  if (s != BA_OK) return s;
  const int64_t n = batch * channels * H * W * D;
  if (n == 0) return BA_OK;
  BA_REQUIRE(src && dst && taps_h && taps_w && taps_d, "ba_smooth3d: NULL pointer");
  const size_t need = ba_smooth_workspace_bytes(batch, channels, H, W, D);
  BA_REQUIRE(workspace && workspace_bytes >= need,
             "ba_smooth3d: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  const size_t esz = dtype == BA_BF16 ? 2 : 4;
  BA_REQUIRE((const char*)src + n * esz <= (const char*)dst ||
                 (const char*)dst + n * esz <= (const char*)src,
             "ba_smooth3d: dst overlaps src");
  SmoothJob j;
  memset(&j, 0, sizeof(j));
  j.src = src;
  j.in_dtype = dtype;
  j.dst = dst;
  j.out_dtype = dtype;
  j.P = channels;
  j.planes = batch * channels;
  j.H = H;
  j.W = W;
  j.D = D;
  j.taps[0] = taps_h;
  j.taps[1] = taps_w;
  j.taps[2] = taps_d;
  for (int i = 0; i < 3; ++i) j.K[i] = K[i];
  j.padding = padding;
  j.mask = mask;
  j.copy_src = src;
  j.t0 = (float*)workspace;
  j.t1 = j.t0 + n;
  return run_smooth(j, (cudaStream_t)stream);
}

extern "C" size_t ba_sharpen_workspace_bytes(const ba_sharpen_desc* d) {
  using namespace ba;
  if (d == nullptr || d->batch < 0 || d->channels < 0 || d->H < 0 || d->W < 0 || d->D < 0)
    return 0;
  const size_t n = (size_t)(d->batch * d->channels * d->H * d->W * d->D);
  const size_t esz = d->dtype == BA_BF16 ? 2 : 4;
  return align16(2 * n * sizeof(float)) + n * esz;
}

extern "C" ba_status ba_sharpen3d(const ba_sharpen_desc* d, void* workspace,
                                  size_t workspace_bytes, ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(d != nullptr, "ba_sharpen3d: desc is NULL");
  BA_REQUIRE(d->dtype == BA_F32 || d->dtype == BA_BF16, "ba_sharpen3d: bad dtype %d", d->dtype);
  BA_REQUIRE(d->batch >= 0 && d->channels >= 0 && d->H > 0 && d->W > 0 && d->D > 0,
             "ba_sharpen3d: bad shape");
  BA_REQUIRE(d->batch * d->channels <= 65535, "ba_sharpen3d: batch*channels exceeds 65535");
  BA_REQUIRE(d->padding >= BA_SMOOTH_ZEROS && d->padding <= BA_SMOOTH_REPLICATE,
             "ba_sharpen3d: unknown padding %d", d->padding);
  ba_status s = check_taps("ba_sharpen3d", d->K1, d->H, d->W, d->D, d->padding);
  if (s != BA_OK) return s;
  s = check_taps("ba_sharpen3d", d->K2, d->H, d->W, d->D, d->padding);
  if (s != BA_OK) return s;
  const int64_t n = d->batch * d->channels * d->H * d->W * d->D;
  if (n == 0) return BA_OK;
  BA_REQUIRE(d->src && d->dst && d->alpha, "ba_sharpen3d: NULL pointer");
  for (int i = 0; i < 3; ++i)
    BA_REQUIRE(d->taps1[i] && d->taps2[i], "ba_sharpen3d: NULL taps");
  const size_t need = ba_sharpen_workspace_bytes(d);
  BA_REQUIRE(workspace && workspace_bytes >= need,
             "ba_sharpen3d: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  BA_REQUIRE((uintptr_t)workspace % 16 == 0, "ba_sharpen3d: workspace not 16-byte aligned");
  const size_t esz = d->dtype == BA_BF16 ? 2 : 4;
  BA_REQUIRE((const char*)d->src + n * esz <= (const char*)d->dst ||
                 (const char*)d->dst + n * esz <= (const char*)d->src,
             "ba_sharpen3d: dst overlaps src");
  cudaStream_t st = (cudaStream_t)stream;
  float* t0 = (float*)workspace;
  float* t1 = t0 + n;
  void* blurred = (char*)workspace + align16(2 * (size_t)n * sizeof(float));
  SmoothJob j;
  memset(&j, 0, sizeof(j));
  j.in_dtype = d->dtype;
  j.out_dtype = d->dtype;
  j.P = d->channels;
  j.planes = d->batch * d->channels;
  j.H = d->H;
  j.W = d->W;
  j.D = d->D;
  j.padding = d->padding;
  j.t0 = t0;
  j.t1 = t1;
  // blurred = smooth(src, taps1), cast to dtype; masked-out elements are not
  // needed (the second blur copies src for them)
  j.src = d->src;
  j.dst = blurred;
  for (int i = 0; i < 3; ++i) {
    j.taps[i] = d->taps1[i];
    j.K[i] = d->K1[i];
  }
  j.mask = d->mask;
  j.copy_src = nullptr;
  s = run_smooth(j, st);
  if (s != BA_OK) return s;
  // dst = combine(blurred, smooth(blurred, taps2)); masked-out elements copy src
  j.src = blurred;
  j.dst = d->dst;
  for (int i = 0; i < 3; ++i) {
    j.taps[i] = d->taps2[i];
    j.K[i] = d->K2[i];
  }
  j.copy_src = d->src;
  j.sharp_blur = blurred;
  j.alpha = d->alpha;
  return run_smooth(j, st);
}

extern "C" size_t ba_elastic_workspace_bytes(int64_t batch, int64_t H, int64_t W, int64_t D) {
  if (batch < 0 || H < 0 || W < 0 || D < 0) return 0;
  return (size_t)(2 * batch * 3 * H * W * D) * sizeof(float);
}

extern "C" ba_status ba_elastic_grid(const float* u, uint64_t seed, uint64_t elem_offset,
                                     int64_t batch, int64_t H, int64_t W, int64_t D,
                                     const float* taps, int64_t K, const float* magnitude,
                                     float* grid, void* workspace, size_t workspace_bytes,
                                     ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(batch >= 0 && H > 0 && W > 0 && D > 0, "ba_elastic_grid: bad shape");
  BA_REQUIRE(batch * 3 <= 65535, "ba_elastic_grid: batch exceeds 21845");
  BA_REQUIRE(K >= 1 && K <= MAX_TAPS && (K % 2) == 1, "ba_elastic_grid: K=%lld must be odd, 1..%d",
             (long long)K, MAX_TAPS);
  const int64_t HWD = H * W * D;
  if (batch * HWD == 0) return BA_OK;
  BA_REQUIRE(taps && magnitude && grid, "ba_elastic_grid: NULL pointer");
  const size_t need = ba_elastic_workspace_bytes(batch, H, W, D);
  BA_REQUIRE(workspace && workspace_bytes >= need,
             "ba_elastic_grid: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  cudaStream_t st = (cudaStream_t)stream;
  float* t0 = (float*)workspace;
  float* t1 = t0 + batch * 3 * HWD;
  const int64_t total = batch * 3 * HWD;
  // elastic_draw_kernel threads: one per Philox block of four field values
  const int64_t draw_threads = batch * ((3 * HWD + 3) / 4);
  ba_status s;
  if (roll_kmax((int)K) != 0 && H * D <= ((int64_t)1 << 31) && W * D <= ((int64_t)1 << 31)) {
    // D pass straight from the Philox draw (or the injected u); W; H into
    // the grid.  An unaligned D takes the draw through scratch first.
    RollArgs r;
    memset(&r, 0, sizeof(r));
    r.batch = batch;
    r.P = 3;
    r.H = H;
    r.W = W;
    r.D = D;
    r.padding = BA_SMOOTH_ZEROS;
    r.taps = taps;
    r.K = (int32_t)K;
    RollArgs rd = r, rw = r, rh = r;
    int src_kind;
    if (u != nullptr) {
      src_kind = RL_SRC_UNIFORM;
      rd.src = u;
    } else if ((D % 4) == 0) {
      src_kind = RL_SRC_PHILOX;
      rd.seed_lo = (uint32_t)seed;
      rd.seed_hi = (uint32_t)(seed >> 32);
      rd.elem_offset = elem_offset;
    } else {
      elastic_draw_kernel<<<(unsigned)((draw_threads + 255) / 256), 256, 0, st>>>(
          nullptr, (uint32_t)seed, (uint32_t)(seed >> 32), elem_offset, HWD, batch, t1);
      s = check_launch("ba_elastic_grid");
      if (s != BA_OK) return s;
      src_kind = RL_SRC_DT;
      rd.src = t1;
      rd.in_dtype = BA_F32;
    }
    rd.dst = t0;
    rw.src = t0;
    rw.dst = t1;
    rh.src = t1;
    rh.dst = grid;
    rh.magnitude = magnitude;
    rh.plane_major = (W * D + RL_THREADS - 1) / RL_THREADS <= 65535;
    return launch_roll(roll_kmax((int)K), src_kind, RL_OUT_GRID, rd, rw, rh, batch, st);
  }
  if (u == nullptr && (HWD % 4) == 0) {
    const int64_t total4 = total / 4;
    elastic_draw4_kernel<<<(unsigned)((total4 + 255) / 256), 256, 0, st>>>(
        (uint32_t)seed, (uint32_t)(seed >> 32), elem_offset, HWD, total4, (float4*)t0);
  } else {
    elastic_draw_kernel<<<(unsigned)((draw_threads + 255) / 256), 256, 0, st>>>(
        u, (uint32_t)seed, (uint32_t)(seed >> 32), elem_offset, HWD, batch, t0);
  }
  s = check_launch("ba_elastic_grid");
  if (s != BA_OK) return s;
  if (tiled_kmax((int)K) != 0 && H <= 65535 && W <= 65535) {
    TiledArgs t;
    memset(&t, 0, sizeof(t));
    t.in = t0;
    t.in_dtype = BA_F32;
    t.mid = t1;
    t.taps_h = t.taps_w = t.taps_d = taps;
    t.Kh = t.Kw = t.Kd = (int32_t)K;
    t.padding = BA_SMOOTH_ZEROS;
    t.P = 3;
    t.H = H;
    t.W = W;
    t.D = D;
    t.HWD = HWD;
    t.grid = grid;
    t.magnitude = magnitude;
    return launch_tiled(t, batch * 3, st);
  }
  AxisArgs a;
  memset(&a, 0, sizeof(a));
  a.P = 3;
  a.H = H;
  a.W = W;
  a.D = D;
  a.HWD = HWD;
  a.taps = taps;
  a.K = (int32_t)K;
  a.in = t0;
  a.in_dtype = BA_F32;
  a.out = t1;
  a.out_dtype = BA_F32;
  s = launch_axis(0, a, batch * 3, st);
  if (s != BA_OK) return s;
  a.in = t1;
  a.out = t0;
  s = launch_axis(1, a, batch * 3, st);
  if (s != BA_OK) return s;
  dim3 g((unsigned)((HWD + SM_THREADS - 1) / SM_THREADS), (unsigned)batch);
  elastic_grid_kernel<<<g, SM_THREADS, 0, st>>>(t0, taps, (int32_t)K, magnitude, H, W, D, grid);
  return check_launch("ba_elastic_grid");
}
