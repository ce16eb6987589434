// Separable Gaussian smoothing and the elastic displacement field.
//
// Reference semantics:
//   gaussian_1d_batch           batchaug/pytorch/intensity/smooth.py:9-34
//   separable_gaussian_conv3d   batchaug/pytorch/intensity/smooth.py:37-88
//   RandGaussianSmooth.apply    batchaug/pytorch/intensity/smooth.py:110-117
//   Rand3DElastic.sample_params batchaug/pytorch/geometric/elastic.py:37-99
//
// Design: three axis passes (H, then W, then D, as the reference's three
// grouped conv3d calls) with per-element taps held in shared memory; the
// passes read and write fp32 intermediates in caller-provided scratch and the
// last pass writes the output dtype directly (and, for the elastic field,
// forms the grid_sample grid in place: centred MONAI grid + magnitude *
// displacement, divided by (N-1)/2, components reordered to x=D, y=W, z=H).
// The uniform draw of the elastic field is generated in-kernel by Philox
// unless the caller injects it.
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

__global__ void gauss_taps_kernel(const float* sigmas, int64_t B, int64_t K, float* taps) {
  const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t tail = K / 2;
  float s = sigmas[b];
  s = s < 1e-6f ? 1e-6f : s;
  const float t = 0.70710678f / s;
  float* o = taps + b * K;
  float sum = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    const float x = (float)(k - tail);
    float v = 0.5f * (erff(t * (x + 0.5f)) - erff(t * (x - 0.5f)));
    v = v < 0.0f ? 0.0f : v;
    o[k] = v;
    sum += v;
  }
  for (int64_t k = 0; k < K; ++k) o[k] = o[k] / sum;
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
  if (a.out_dtype == BA_BF16)
    ((uint16_t*)a.out)[idx] = f32_to_bf16_bits(acc);
  else
    ((float*)a.out)[idx] = acc;
}

// Uniform draw of the elastic field, mapped to [-1, 1): u * 2 - 1.
__global__ void elastic_draw_kernel(const float* u, uint32_t seed_lo, uint32_t seed_hi,
                                    uint64_t elem_offset, int64_t HWD, int64_t total,
                                    float* out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= total) return;
  float x;
  if (u != nullptr) {
    x = u[i];
  } else {
    const int64_t per = 3 * HWD;
    const int64_t b = i / per;
    const int64_t p = i - b * per;  // comp * HWD + s
    const uint64_t eb = elem_offset + (uint64_t)b;
    const uint64_t q = (uint64_t)p >> 2;
    const U4 ctr = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                    STREAM_ELASTIC | (uint32_t)(q >> 32)};
    const U4 r = philox4x32_10(ctr, seed_lo, seed_hi);
    const int l = (int)(p & 3);
    x = u01(l == 0 ? r.x : (l == 1 ? r.y : (l == 2 ? r.z : r.w)));
  }
  out[i] = x * 2.0f - 1.0f;
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
  gauss_taps_kernel<<<(unsigned)((batch + 127) / 128), 128, 0, (cudaStream_t)stream>>>(
      sigmas, batch, K, taps);
  return check_launch("ba_gauss_taps");
}

extern "C" size_t ba_smooth_workspace_bytes(int64_t batch, int64_t channels, int64_t H, int64_t W,
                                            int64_t D) {
  if (batch < 0 || channels < 0 || H < 0 || W < 0 || D < 0) return 0;
  return (size_t)(2 * batch * channels * H * W * D) * sizeof(float);
}

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
  for (int64_t K : {Kh, Kw, Kd})
    BA_REQUIRE(K >= 1 && K <= MAX_TAPS && (K % 2) == 1, "ba_smooth3d: K=%lld must be odd, 1..%d",
               (long long)K, MAX_TAPS);
  BA_REQUIRE(padding >= BA_SMOOTH_ZEROS && padding <= BA_SMOOTH_REPLICATE,
             "ba_smooth3d: unknown padding %d", padding);
  if (padding == BA_SMOOTH_REFLECT) {
    // F.pad(mode="reflect") needs the pad to be smaller than the axis
    BA_REQUIRE(Kh / 2 < H && Kw / 2 < W && Kd / 2 < D,
               "ba_smooth3d: reflect padding needs K/2 < size along every axis");
  }
  const int64_t HWD = H * W * D;
  const int64_t n = batch * channels * HWD;
  if (n == 0) return BA_OK;
  BA_REQUIRE(src && dst && taps_h && taps_w && taps_d, "ba_smooth3d: NULL pointer");
  const size_t need = ba_smooth_workspace_bytes(batch, channels, H, W, D);
  BA_REQUIRE(workspace && workspace_bytes >= need,
             "ba_smooth3d: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  const size_t esz = dtype == BA_BF16 ? 2 : 4;
  BA_REQUIRE((const char*)src + n * esz <= (const char*)dst ||
                 (const char*)dst + n * esz <= (const char*)src,
             "ba_smooth3d: dst overlaps src");
  float* t0 = (float*)workspace;
  float* t1 = t0 + n;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t planes = batch * channels;
  AxisArgs a;
  memset(&a, 0, sizeof(a));
  a.P = channels;
  a.H = H;
  a.W = W;
  a.D = D;
  a.HWD = HWD;
  a.padding = padding;
  // H pass: src (dtype) -> t0
  a.in = src;
  a.in_dtype = dtype;
  a.out = t0;
  a.out_dtype = BA_F32;
  a.taps = taps_h;
  a.K = (int32_t)Kh;
  ba_status s = launch_axis(0, a, planes, st);
  if (s != BA_OK) return s;
  // W pass: t0 -> t1
  a.in = t0;
  a.in_dtype = BA_F32;
  a.out = t1;
  a.taps = taps_w;
  a.K = (int32_t)Kw;
  s = launch_axis(1, a, planes, st);
  if (s != BA_OK) return s;
  // D pass: t1 -> dst (dtype); masked-out elements copy src
  a.in = t1;
  a.out = dst;
  a.out_dtype = dtype;
  a.taps = taps_d;
  a.K = (int32_t)Kd;
  a.mask = mask;
  a.copy_src = mask ? src : nullptr;
  return launch_axis(2, a, planes, st);
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
  elastic_draw_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
      u, (uint32_t)seed, (uint32_t)(seed >> 32), elem_offset, HWD, total, t0);
  ba_status s = check_launch("ba_elastic_grid");
  if (s != BA_OK) return s;
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
