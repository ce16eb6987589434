// Shared device helpers for the batchaug_b200 kernels (sm_100a).
//
// Every file of this library is compiled with -fmad=false: each float
// multiply and add rounds on its own, as in torch's scalar CPU kernels that
// the reference results come from.  Fused multiply-adds appear only where
// written explicitly (__fmaf_rn), at the places where torch's own CPU path
// fuses (MKL's bmm inside affine_grid, linspace, the einsum of the bias field).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/batchaug_b200.h"

namespace ba {

// ---------------------------------------------------------------------------
// Host-side error reporting (thread-local message + status).
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();
ba_status check_launch(const char* what);

// Checks of an intensity-chain descriptor (shape, dtype, ops, pointers);
// defined in intensity.cu.
ba_status validate_chain(const ba_chain_desc* d);

// Per-group min/max keys (the chain's statistics format) for
// ba_resample3d's minmax output: reset, and fold a tensor's groups of
// group_size consecutive values into them; defined in intensity.cu.
ba_status minmax_keys_init(int32_t* keys, int64_t groups, cudaStream_t st);
ba_status minmax_keys_fold(const void* x, int dtype, int64_t groups, int64_t group_size,
                           int32_t* keys, cudaStream_t st);

#define BA_REQUIRE(cond, ...)        \
  do {                               \
    if (!(cond)) {                   \
      ::ba::set_error(__VA_ARGS__);  \
      return BA_EINVAL;              \
    }                                \
  } while (0)

// ---------------------------------------------------------------------------
// Element access.  bf16 is stored as the upper half of an fp32 and rounded
// to nearest even on store, which is what c10::BFloat16 does.  (NaN payload
// bits may differ from c10's canonical 0x7FC0; NaN stays NaN.)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float(((uint32_t)h) << 16);
}

// Round-to-nearest-even through the hardware conversion (cvt.rn.bf16.f32),
// the same result c10::BFloat16 gives for every non-NaN value.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Two values rounded and packed (lo = a, hi = b) in one conversion.
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Round an fp32 value to the nearest bf16 and back (one torch bf16 op's
// rounding of its fp32 result).
__device__ __forceinline__ float round_bf16(float f) {
  return __bfloat162float(__float2bfloat16_rn(f));
}

template <int DT>
__device__ __forceinline__ float round_dt(float f) {
  return DT == BA_BF16 ? round_bf16(f) : f;
}

__device__ __forceinline__ float load_f(const void* p, int dtype, int64_t i) {
  if (dtype == BA_BF16) return bf16_bits_to_f32(__ldg((const uint16_t*)p + i));
  return __ldg((const float*)p + i);
}

__device__ __forceinline__ void store_f(void* p, int dtype, int64_t i, float v) {
  if (dtype == BA_BF16)
    ((uint16_t*)p)[i] = f32_to_bf16_bits(v);
  else
    ((float*)p)[i] = v;
}

// ---------------------------------------------------------------------------
// torch.linspace(start, end, n)[i]: step = fl((end - start) / (n - 1)),
// first half fma(step, i, start), second half fma(-step, n-1-i, end).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float linspace_at(float start, float end, float step, int64_t i,
                                             int64_t n) {
  if (n == 1) return start;
  if (i < n / 2) return __fmaf_rn(step, (float)i, start);
  return __fmaf_rn(-step, (float)(n - 1 - i), end);
}
// linspace_at for 32-bit indices (the same values: the conversions are exact
// below 2^24)
__device__ __forceinline__ float linspace_at32(float start, float end, float step, int i, int n) {
  if (n == 1) return start;
  if (i < n / 2) return __fmaf_rn(step, (float)i, start);
  return __fmaf_rn(-step, (float)(n - 1 - i), end);
}

// ---------------------------------------------------------------------------
// Order-preserving int32 keys for float min/max with atomics.  NaN maps to
// the extreme key in each direction so that a NaN anywhere wins both the
// min and the max, as torch.min / torch.max propagate NaN.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int32_t fkey(float f) {
  int32_t k = __float_as_int(f);
  return k >= 0 ? k : (k ^ 0x7FFFFFFF);
}
__device__ __forceinline__ float fkey_inv(int32_t k) {
  return __int_as_float(k >= 0 ? k : (k ^ 0x7FFFFFFF));
}
// ---------------------------------------------------------------------------
// Asynchronous 16-byte global->shared copies (cp.async, sm_80+).  A thread
// waits for its own groups with cp.async.wait_group, a hardware wait.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

constexpr int32_t KEY_MIN_NAN = (int32_t)0x80000000;  // below key(-inf)
constexpr int32_t KEY_MAX_NAN = (int32_t)0x7FFFFFFF;  // above key(+inf)
constexpr int32_t KEY_POS_INF = (int32_t)0x7F800000;
constexpr int32_t KEY_NEG_INF = (int32_t)(0xFF800000u ^ 0x7FFFFFFFu);

// RN(1/b) when a/b can take the reciprocal path of div_rn, else 0.
__device__ __forceinline__ float recip_for_div(float b) {
  const float m = fabsf(b);
  return (m >= 0x1p-120f && m <= 0x1p120f) ? __frcp_rn(b) : 0.0f;
}

// a / b rounded to nearest, from y = RN(1/b) (recip_for_div): q = RN(a*y),
// the remainder r = a - b*q is exact in one fma, and RN(q + r*y) is the
// correctly rounded quotient (P. Markstein, "IA-64 and Elementary Functions",
// 2000, the correction step for a correctly rounded reciprocal) whenever a, b
// and the quotient are normal.  Zero, tiny, huge and non-finite quotients take
// the plain division.
__device__ __forceinline__ float div_rn(float a, float b, float y) {
  if (y != 0.0f) {
    const float q = __fmul_rn(a, y);
    const float aq = fabsf(q);
    if (a == 0.0f) return q;
    if (aq >= 0x1p-100f && aq <= 0x1p100f) return __fmaf_rn(__fmaf_rn(-q, b, a), y, q);
  }
  return __fdiv_rn(a, b);
}

__device__ __forceinline__ float decode_min_key(int32_t k) {
  return k == KEY_MIN_NAN ? __int_as_float(0x7FC00000) : fkey_inv(k);
}
__device__ __forceinline__ float decode_max_key(int32_t k) {
  return k == KEY_MAX_NAN ? __int_as_float(0x7FC00000) : fkey_inv(k);
}

}  // namespace ba
