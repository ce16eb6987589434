// Counter-based random numbers: Philox4x32-10 (Salmon, Moraes, Dror, Shaw,
// "Parallel Random Numbers: As Easy as 1, 2, 3", SC'11) and the Box-Muller
// transform (Box & Muller, 1958).  Written from the published descriptions:
// ten rounds of two 32x32->64 multiplies with the paper's multipliers and
// Weyl key increments.
//
// Streams are keyed so that every value depends only on
// (seed, global element index, stream id, position): identical across keys of
// a dict transform, across ranks of a sharded run and across launch shapes.
#pragma once

#include <stdint.h>

namespace ba {

struct U4 {
  uint32_t x, y, z, w;
};

__host__ __device__ __forceinline__ void mulhilo32(uint32_t a, uint32_t b, uint32_t& hi,
                                                    uint32_t& lo) {
#ifdef __CUDA_ARCH__
  lo = a * b;
  hi = __umulhi(a, b);
#else
  uint64_t p = (uint64_t)a * (uint64_t)b;
  lo = (uint32_t)p;
  hi = (uint32_t)(p >> 32);
#endif
}

// Philox4x32 with 10 rounds: counter ctr, key (k0, k1).
__host__ __device__ __forceinline__ U4 philox4x32_10(U4 ctr, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(M0, ctr.x, hi0, lo0);
    mulhilo32(M1, ctr.z, hi1, lo1);
    U4 n;
    n.x = hi1 ^ ctr.y ^ k0;
    n.y = lo1;
    n.z = hi0 ^ ctr.w ^ k1;
    n.w = lo0;
    ctr = n;
    k0 += W0;
    k1 += W1;
  }
  return ctr;
}

// Uniform in (0, 1]: 24 random bits, never 0 (safe for log).
__host__ __device__ __forceinline__ float u01_open0(uint32_t r) {
  return ((float)(r >> 8) + 1.0f) * (1.0f / 16777216.0f);
}

// Uniform in [0, 1): 24 random bits, as torch.rand's float32 resolution.
__host__ __device__ __forceinline__ float u01(uint32_t r) {
  return (float)(r >> 8) * (1.0f / 16777216.0f);
}

#ifdef __CUDACC__
// Uniform in (0, 1] from the top 23 bits, built in the float's bit pattern
// (2 - [1, 2)), so the integer-to-float conversion unit is not needed.
__device__ __forceinline__ float u01_open0_bits(uint32_t r) {
  return 2.0f - __uint_as_float(0x3F800000u | (r >> 9));
}
// Uniform in [-pi, pi) from the top 23 bits: pi * ([1, 2) * 2 - 3).
__device__ __forceinline__ float angle_bits(uint32_t r) {
  constexpr float PI = 3.141592653589793f;
  return (__uint_as_float(0x3F800000u | (r >> 9)) * 2.0f - 3.0f) * PI;
}
__device__ __forceinline__ float sqrt_approx(float x) {
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Four standard normals from one Philox block (two Box-Muller pairs).  The
// angle is drawn in [-pi, pi), where the hardware sine/cosine are accurate to
// about 2^-21; only the distribution matters for augmentation noise.
__device__ __forceinline__ void normal4(U4 r, float* z) {
  const float r0 = sqrt_approx(-2.0f * __logf(u01_open0_bits(r.x)));
  const float r1 = sqrt_approx(-2.0f * __logf(u01_open0_bits(r.z)));
  float s0, c0, s1, c1;
  __sincosf(angle_bits(r.y), &s0, &c0);
  __sincosf(angle_bits(r.w), &s1, &c1);
  z[0] = r0 * c0;
  z[1] = r0 * s0;
  z[2] = r1 * c1;
  z[3] = r1 * s1;
}
#endif

// Stream ids (the counter's high word) of the library's random streams.
constexpr uint32_t STREAM_NOISE = 0x4E4F0000u;    // Gaussian noise volume
constexpr uint32_t STREAM_ELASTIC = 0x454C0000u;  // elastic uniform field
constexpr uint32_t STREAM_PARAMS = 0x50410000u;   // per-element scalar params
constexpr uint32_t STREAM_RICIAN1 = 0x52310000u;  // Rician noise, first component
constexpr uint32_t STREAM_RICIAN2 = 0x52320000u;  // Rician noise, second component

}  // namespace ba
