// Fused intensity chain and min/max reduction.
//
// Reference semantics (batchaug PyTorch backend, op by op in the tensor
// dtype):
//   RandGaussianNoise.apply     batchaug/pytorch/intensity/noise.py:62-66
//   RandAdjustContrast.apply    batchaug/pytorch/intensity/contrast.py:116-131
//   RandScaleIntensity.apply    batchaug/pytorch/intensity/scale_shift.py:51-56
//   RandShiftIntensity.apply    batchaug/pytorch/intensity/scale_shift.py:106-113
//   RandBiasField.apply         batchaug/pytorch/intensity/bias_field.py:99-112
//   ScaleIntensity.apply        batchaug/pytorch/intensity/contrast.py:35-68
// replacing the Triton kernels batchaug/triton/kernels/{reduce,elementwise,
// scale_shift,bias_field}.py.
//
// Design (B200): a chain of these transforms is one kernel per "segment".
// CONTRAST and RESCALE need the min/max of their own input, so the chain is
// cut in front of each of them; a segment streams 16-byte vectors, applies its
// ops in registers (rounding to the tensor dtype after every op, as torch
// does), writes the result and folds its min/max into per-group int32 keys
// with one atomic per CTA and group.  The next segment re-reads that result.
// Data streams through a per-thread cp.async ring in shared memory (deep
// memory-level parallelism without register cost).  Gaussian noise is
// generated in registers (Philox4x32-10 + Box-Muller) instead of being
// materialised.
#include <stdio.h>

#include <algorithm>
#include <vector>

#include "ba_common.cuh"
#include "philox.cuh"

namespace ba {
namespace {

constexpr int CHAIN_THREADS = 256;
// Chunks in flight per thread in the cp.async ring (8 x 16 B x 256 threads =
// 32 KB of shared memory per CTA) and the resident CTAs per SM it is sized
// for: ~128 KB in flight per SM, enough to stream HBM at full rate.
constexpr int CHAIN_PIPE = 8;
constexpr int CHAIN_MINBLOCKS = 4;
// bf16 segments hold more live values per thread (packed words plus the
// unpacked fallback): one CTA fewer per SM keeps them out of local memory.
template <int DT>
constexpr int chain_minblocks() { return DT == BA_BF16 ? 3 : CHAIN_MINBLOCKS; }
constexpr int CHAIN_MIN_CHUNKS = 16;

struct OpArgs {
  int32_t kind;
  int32_t flags;
  const uint8_t* mask;
  const float* param;
  const float* param2;
  const float* noise;
  const int32_t* stats_in;     // keys (groups, 2) the op reads (CONTRAST, RESCALE)
  const double* moments_in;    // (groups, 3): sum, sum of squares, nonzero count
                               // (STD_SHIFT, FIXED_MEAN, relative RICIAN)
  int64_t moments_n;           // values per moments group
  int32_t stats_per_channel;
  int32_t degree;
  uint32_t seed_lo, seed_hi;
  uint64_t elem_offset;
  float minv, span, factor1p;  // RESCALE constants as the reference rounds them
  float mean;                  // RICIAN noise mean
};

struct ChainArgs {
  const void* src;
  void* dst;
  int64_t C, H, W, D, HWD;
  int32_t b0;       // first element of this launch
  int32_t n_ops;
  int32_t stats_mode;  // 0: none, 1: per element, 2: per (element, channel)
  int32_t stats_moments;  // 0: min/max keys, 1: moments
  int64_t tile;        // spatial positions per CTA (multiple of VEC)
  int32_t* stats_out;  // keys (groups, 2)
  double* moments_out;  // moments (groups, 3)
  OpArgs ops[BA_MAX_OPS];
};

// ---------------------------------------------------------------------------
// Bias field: Legendre values along one axis with the reference recurrence
// p_n = ((2n-1) * c * p_{n-1} - (n-1) * p_{n-2}) / n  (bias_field.py:38-43).
// ---------------------------------------------------------------------------
template <int DEG>
__device__ __forceinline__ void legendre(float c, float* p) {
  p[0] = 1.0f;
  if (DEG >= 1) p[1] = c;
#pragma unroll
  for (int n = 2; n <= DEG; ++n) {
    float a = ((float)(2 * n - 1) * c) * p[n - 1];
    float s = (float)(n - 1) * p[n - 2];
    p[n] = (a - s) / (float)n;
  }
}

__device__ __forceinline__ float axis_coord(int64_t i, int64_t n) {
  if (n == 1) return -1.0f;
  return linspace_at(-1.0f, 1.0f, 2.0f / (float)(n - 1), i, n);
}

// exp(sum_t c_t * L_i(x) L_j(y) L_k(z)) over (i,j,k), i+j+k <= DEG, in the
// reference's triplet order (bias_field.py:24-28); the sum is the fused chain
// torch's CPU einsum produces and each basis value is (Li*Lj)*Lk.
template <int DEG>
__device__ __forceinline__ float bias_multiplier(const float* coeffs, const float* lx,
                                                 const float* ly, const float* lz) {
  float acc = 0.0f;
  int t = 0;
#pragma unroll
  for (int i = 0; i <= DEG; ++i)
#pragma unroll
    for (int j = 0; j <= DEG - i; ++j) {
      const float pij = lx[i] * ly[j];
#pragma unroll
      for (int k = 0; k <= DEG - i - j; ++k) {
        const float basis = pij * lz[k];
        const float c = __ldg(coeffs + t);
        acc = (t == 0) ? c * basis : __fmaf_rn(c, basis, acc);
        ++t;
      }
    }
  return expf(acc);
}

template <int DEG, int VEC>
__device__ __forceinline__ void bias_run(const OpArgs& op, int64_t b, int64_t s0, int n,
                                         const ChainArgs& a, float* v) {
  constexpr int NC = (DEG + 1) * (DEG + 2) * (DEG + 3) / 6;
  const float* coeffs = op.param + b * NC;
  int64_t h = s0 / (a.W * a.D);
  int64_t rem = s0 - h * a.W * a.D;
  int64_t w = rem / a.D;
  int64_t z = rem - w * a.D;
  float lx[DEG + 1], ly[DEG + 1], lz[DEG + 1];
  legendre<DEG>(axis_coord(h, a.H), lx);
  legendre<DEG>(axis_coord(w, a.W), ly);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    if (i < n) {
      legendre<DEG>(axis_coord(z, a.D), lz);
      v[i] = v[i] * bias_multiplier<DEG>(coeffs, lx, ly, lz);
      if (++z == a.D) {
        z = 0;
        if (++w == a.W) {
          w = 0;
          ++h;
          legendre<DEG>(axis_coord(h, a.H), lx);
        }
        legendre<DEG>(axis_coord(w, a.W), ly);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Per-(element, channel) constants of each op, resolved once per channel into
// shared memory so the per-vector loop reads no parameters from global memory.
// ---------------------------------------------------------------------------
struct OpConst {
  float k0, k1, k2, k3, k4, k5;
  int on;
  // bf16 kernels: operands as bf16x2 splats, and whether the op can run on
  // packed bf16 arithmetic (every scalar it uses is a bf16 value)
  uint32_t h0, h1, h2;
  int packed;
};

__device__ __forceinline__ bool is_bf16_value(float f) { return round_bf16(f) == f; }
__device__ __forceinline__ uint32_t splat_bf16(float f) { return pack_bf16x2(f, f); }

// a / b rounded to fp32 and then to bf16, for bf16 values a and b: the
// bf16 rounding of RN(a * RN(1/b)) already equals it.  Reason: a/b of two
// 8-bit significands is never a bf16 midpoint and, when not exact, is at
// least ~2^-17 (relative) away from one, while a * RN(1/b) is within 2^-23 of
// a/b; fp32-then-bf16 rounding of a quotient equals its bf16 rounding because
// fp32 carries more than 2*8+2 bits (Figueroa, "When is double rounding
// innocuous?", 1995).  Checked exhaustively over all significand pairs.
__device__ __forceinline__ float div_for_bf16(float a, float b, float y) {
  if (y != 0.0f) {
    const float q = __fmul_rn(a, y);
    const float aq = fabsf(q);
    if (a == 0.0f || (aq >= 0x1p-100f && aq <= 0x1p100f)) return q;
  }
  return __fdiv_rn(a, b);
}

// torch.std (unbiased) of a group from its moments (sum, sum of squares,
// nonzero count) in double; with nonzero, of the nonzero values when there
// are at least two of them (scale_shift.py:174-189).  Fewer than two values:
// NaN, as torch gives.
__device__ __forceinline__ float moment_std(const double* m, int64_t g, int64_t n, bool nonzero) {
  const double s = m[3 * g], ss = m[3 * g + 1], nnz = m[3 * g + 2];
  const double cnt = (nonzero && nnz > 1.0) ? nnz : (double)n;
  if (cnt < 2.0) return __int_as_float(0x7FC00000);
  double v = (ss - s * (s / cnt)) / (cnt - 1.0);
  v = v < 0.0 ? 0.0 : v;
  return (float)sqrt(v);
}

template <int DT>
__device__ __forceinline__ void resolve_op(const ChainArgs& a, int oi, int64_t b, int64_t c,
                                           OpConst& o) {
  const OpArgs& op = a.ops[oi];
  o.on = (op.mask == nullptr || op.mask[b] != 0) ? 1 : 0;
  o.k0 = o.k1 = o.k2 = o.k3 = o.k4 = o.k5 = 0.0f;
  o.h0 = o.h1 = o.h2 = 0u;
  o.packed = 0;
  switch (op.kind) {
    case BA_OP_NOISE:
      if (op.flags & BA_NOISE_PHILOX) {
        o.k0 = op.param[b];   // std
        o.k1 = op.param2[b];  // mean
      }
      o.h0 = splat_bf16(o.on ? 1.0f : 0.0f);
      break;
    case BA_OP_CONTRAST: {
      const float mn = decode_min_key(op.stats_in[2 * b]);
      const float mx = decode_max_key(op.stats_in[2 * b + 1]);
      const float rng = mx - mn;
      o.k0 = mn;
      o.k1 = rng;
      o.k2 = rng + 1e-7f;
      o.k3 = op.param[b];  // gamma
      o.k4 = 1.0f / o.k2;
      o.k5 = powf(0.0f, o.k3);  // 0^gamma, taken apart from the fast power below
      break;
    }
    case BA_OP_SCALE:
      o.k0 = round_dt<DT>(1.0f + round_dt<DT>(op.param[b]));
      o.h0 = splat_bf16(o.k0);
      break;
    case BA_OP_SHIFT:
      o.k0 = round_dt<DT>(op.param[b]);
      o.h0 = splat_bf16(o.k0);
      break;
    case BA_OP_RESCALE:
      if (!(op.flags & BA_RESCALE_FACTOR) && (op.flags & (BA_RESCALE_MINV | BA_RESCALE_MAXV))) {
        const int64_t g = op.stats_per_channel ? b * a.C + c : b;
        const float mn = decode_min_key(op.stats_in[2 * g]);
        const float mx = decode_max_key(op.stats_in[2 * g + 1]);
        float den = round_dt<DT>(mx - mn);
        const bool is_const = den == 0.0f;
        o.k0 = mn;
        o.k1 = is_const ? 1.0f : den;
        o.k2 = is_const ? 1.0f : 0.0f;
        o.k3 = recip_for_div(o.k1);
        o.h0 = splat_bf16(mn);
        o.h1 = splat_bf16(op.span);
        o.h2 = splat_bf16(op.minv);
        o.packed = !is_const && is_bf16_value(op.span) && is_bf16_value(op.minv);
      } else if (op.flags & BA_RESCALE_FACTOR) {
        o.h0 = splat_bf16(op.factor1p);
        o.packed = is_bf16_value(op.factor1p);
      }
      break;
    case BA_OP_RICIAN: {
      float sd = op.param[b];
      if (op.flags & BA_RICIAN_RELATIVE) sd = sd * moment_std(op.moments_in, b, op.moments_n, false);
      o.k0 = sd;
      o.k1 = op.mean;
      break;
    }
    case BA_OP_STD_SHIFT: {
      const int64_t g = op.stats_per_channel ? b * a.C + c : b;
      o.k0 = op.param[b] * moment_std(op.moments_in, g, op.moments_n, op.flags & BA_STD_NONZERO);
      break;
    }
    case BA_OP_FIXED_MEAN: {
      const int64_t g = op.stats_per_channel ? b * a.C + c : b;
      o.k0 = (float)(op.moments_in[3 * g] / (double)op.moments_n);
      o.k1 = 1.0f + op.param[b];
      break;
    }
    default:
      break;
  }
}

// Apply op oi to n consecutive values of one channel (positions
// s0..s0+n-1), rounding its result to the tensor dtype as torch does.
// KIND >= 0: the op is known to be of that kind (an op of a sequence given
// at compile time), so the dispatch folds away.
template <int DT, int VEC, int KIND = -1>
__device__ __forceinline__ void apply_one(const ChainArgs& a, int oi, const OpConst& k, int64_t b,
                                          int64_t c, int64_t s0, int n, float* v) {
  {
    const OpArgs& op = a.ops[oi];
    const bool on = k.on != 0;
    switch (KIND >= 0 ? KIND : op.kind) {
      case BA_OP_NOISE: {
        // x + dt(noise) * dt(mask).  A masked-out element with generated noise
        // adds a zero; injected noise keeps the product (its sign of zero).
        if (!on && (op.flags & BA_NOISE_PHILOX)) {
#pragma unroll
          for (int i = 0; i < VEC; ++i) v[i] = v[i] + 0.0f;
          break;
        }
        const float m = on ? 1.0f : 0.0f;
        float nz[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) nz[i] = 0.0f;
        if (op.flags & BA_NOISE_PHILOX) {
          // Noise of flat position p = c*HWD + s of element b is normal
          // (p & 3) of Philox block (seed; p >> 2, element, NOISE stream),
          // times std plus mean in fp32 as torch.randn(...) * std + mean.
          if (on) {
            const uint64_t eb = op.elem_offset + (uint64_t)b;
            const int64_t first = c * a.HWD + s0;
            if (VEC >= 4) {
              // vector path: first is a multiple of 4 (HWD % VEC == 0)
#pragma unroll
              for (int base = 0; base < VEC; base += 4) {
                const uint64_t q = (uint64_t)(first + base) >> 2;
                const U4 ctr = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                                STREAM_NOISE | (uint32_t)(q >> 32)};
                float z4[4];
                normal4(philox4x32_10(ctr, op.seed_lo, op.seed_hi), z4);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  if (base + i < VEC) nz[base + i] = z4[i] * k.k0 + k.k1;
              }
            } else {
              const uint64_t q = (uint64_t)first >> 2;
              const U4 ctr = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                              STREAM_NOISE | (uint32_t)(q >> 32)};
              float z4[4];
              normal4(philox4x32_10(ctr, op.seed_lo, op.seed_hi), z4);
              const int l = (int)(first & 3);
              const float z = l == 0 ? z4[0] : (l == 1 ? z4[1] : (l == 2 ? z4[2] : z4[3]));
              nz[0] = z * k.k0 + k.k1;
            }
          }
        } else {
          const float* np = op.noise + (b * a.C + c) * a.HWD + s0;
#pragma unroll
          for (int i = 0; i < VEC; ++i) nz[i] = (i < n) ? __ldg(np + i) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const float nm = round_dt<DT>(round_dt<DT>(nz[i]) * m);
          v[i] = round_dt<DT>(v[i] + nm);
        }
        break;
      }
      case BA_OP_CONTRAST: {
        if (!on) break;
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          // the power below is approximate (a few fp32 ulp), so the
          // normalisation takes the reciprocal instead of a rounded division
          float nrm = (v[i] - k.k0) * k.k4;
          nrm = (nrm < 0.0f) ? 0.0f : nrm;
          // nrm in [0, 1]: the hardware exp2(gamma * log2(nrm)) power is
          // within a few fp32 ulp there (far inside the op's tolerance)
          const float pw = nrm == 0.0f ? k.k5 : __powf(nrm, k.k3);
          v[i] = round_dt<DT>(pw * k.k1 + k.k0);
        }
        break;
      }
      case BA_OP_SCALE: {
        if (!on) break;
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[i] = round_dt<DT>(v[i] * k.k0);
        break;
      }
      case BA_OP_SHIFT: {
        if (!on) break;
        const bool safe = op.flags & BA_SHIFT_SAFE;
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          float r = round_dt<DT>(v[i] + k.k0);
          if (safe) r = (r < 0.0f) ? 0.0f : ((r > 1.0f) ? 1.0f : r);
          v[i] = r;
        }
        break;
      }
      case BA_OP_BIAS_FIELD: {
        if (!on) break;
        float t[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) t[i] = v[i];
        switch (op.degree) {
          case 1: bias_run<1, VEC>(op, b, s0, n, a, t); break;
          case 2: bias_run<2, VEC>(op, b, s0, n, a, t); break;
          case 3: bias_run<3, VEC>(op, b, s0, n, a, t); break;
          case 4: bias_run<4, VEC>(op, b, s0, n, a, t); break;
          case 5: bias_run<5, VEC>(op, b, s0, n, a, t); break;
          default: bias_run<6, VEC>(op, b, s0, n, a, t); break;
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[i] = round_dt<DT>(t[i]);
        break;
      }
      case BA_OP_RICIAN: {
        // sqrt((x + n1)^2 + n2^2), n = mean + std * u in fp32 (noise.py:146-164)
        if (!on) break;
        float u1[VEC], u2[VEC];
        if (op.flags & BA_RICIAN_PHILOX) {
          // u of flat position p = c*HWD + s of element b is normal (p & 3)
          // of Philox block (seed; p >> 2, element, RICIAN1 / RICIAN2 stream)
          const uint64_t eb = op.elem_offset + (uint64_t)b;
          const int64_t first = c * a.HWD + s0;
#pragma unroll
          for (int base = 0; base < (VEC >= 4 ? VEC : 4); base += 4) {
            const uint64_t q = (uint64_t)(first + (VEC >= 4 ? base : 0)) >> 2;
            const U4 c1 = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                           STREAM_RICIAN1 | (uint32_t)(q >> 32)};
            const U4 c2 = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                           STREAM_RICIAN2 | (uint32_t)(q >> 32)};
            float z1[4], z2[4];
            normal4(philox4x32_10(c1, op.seed_lo, op.seed_hi), z1);
            normal4(philox4x32_10(c2, op.seed_lo, op.seed_hi), z2);
            if (VEC >= 4) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (base + i < VEC) {
                  u1[base + i] = z1[i];
                  u2[base + i] = z2[i];
                }
            } else {
              const int l = (int)(first & 3);
              u1[0] = l == 0 ? z1[0] : (l == 1 ? z1[1] : (l == 2 ? z1[2] : z1[3]));
              u2[0] = l == 0 ? z2[0] : (l == 1 ? z2[1] : (l == 2 ? z2[2] : z2[3]));
            }
          }
        } else {
          const int64_t off = (b * a.C + c) * a.HWD + s0;
#pragma unroll
          for (int i = 0; i < VEC; ++i) {
            u1[i] = (i < n) ? __ldg(op.noise + off + i) : 0.0f;
            u2[i] = (i < n) ? __ldg(op.param2 + off + i) : 0.0f;
          }
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const float n1 = __fadd_rn(__fmul_rn(k.k0, u1[i]), k.k1);
          const float n2 = __fadd_rn(__fmul_rn(k.k0, u2[i]), k.k1);
          const float x1 = __fadd_rn(v[i], n1);
          v[i] = round_dt<DT>(__fsqrt_rn(__fadd_rn(__fmul_rn(x1, x1), __fmul_rn(n2, n2))));
        }
        break;
      }
      case BA_OP_STD_SHIFT: {
        // x + factor * std, fp32, one cast (scale_shift.py:168-198)
        if (!on) break;
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[i] = round_dt<DT>(__fadd_rn(v[i], k.k0));
        break;
      }
      case BA_OP_FIXED_MEAN: {
        // mean + (x - mean) * (1 + factor), fp32, one cast (scale_shift.py:252-274)
        if (!on) break;
#pragma unroll
        for (int i = 0; i < VEC; ++i)
          v[i] = round_dt<DT>(__fadd_rn(k.k0, __fmul_rn(__fsub_rn(v[i], k.k0), k.k1)));
        break;
      }
      case BA_OP_RESCALE: {
        if (op.flags & BA_RESCALE_FACTOR) {
#pragma unroll
          for (int i = 0; i < VEC; ++i) v[i] = round_dt<DT>(v[i] * op.factor1p);
          break;
        }
        const bool has_min = op.flags & BA_RESCALE_MINV, has_max = op.flags & BA_RESCALE_MAXV;
        if (!has_min && !has_max) break;
        const bool is_const = k.k2 != 0.0f;
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const float nrm = round_dt<DT>(div_rn(round_dt<DT>(v[i] - k.k0), k.k1, k.k3));
          float r = nrm;
          if (has_min && has_max) r = round_dt<DT>(round_dt<DT>(nrm * op.span) + op.minv);
          if (has_min && is_const) r = round_dt<DT>(v[i] * op.minv);
          v[i] = r;
        }
        break;
      }
      default:
        break;
    }
  }
}

// The segment's ops, in order, on n consecutive values of one channel.
// SEQ >= 0: the ops' kinds in compile-time form, four bits each, the first
// op in the lowest bits (0 ends the sequence); -1: any ops.
template <int DT, int VEC, int SEQ>
__device__ __forceinline__ void apply_seq(const ChainArgs& a, const OpConst* oc, int oi,
                                          int64_t b, int64_t c, int64_t s0, int n, float* v) {
  if constexpr (SEQ != 0) {
    apply_one<DT, VEC, (SEQ & 15)>(a, oi, oc[oi], b, c, s0, n, v);
    apply_seq<DT, VEC, (SEQ >> 4)>(a, oc, oi + 1, b, c, s0, n, v);
  }
}

template <int DT, int VEC, int SEQ = -1>
__device__ __forceinline__ void apply_ops(const ChainArgs& a, const OpConst* oc, int64_t b,
                                          int64_t c, int64_t s0, int n, float* v) {
  if constexpr (SEQ >= 0)
    apply_seq<DT, VEC, SEQ>(a, oc, 0, b, c, s0, n, v);
  else
    for (int oi = 0; oi < a.n_ops; ++oi) apply_one<DT, VEC>(a, oi, oc[oi], b, c, s0, n, v);
}

// ---------------------------------------------------------------------------
// bf16 tensors: 8 values (one 16-byte chunk) as four bf16x2 words.  For two
// bf16 operands, torch's "compute in fp32, round to bf16" equals one
// correctly rounded bf16 operation (fp32 has more than 2*8+2 significand
// bits, so the double rounding is innocuous for +, -, *, /), which is what
// the packed bf16x2 instructions compute.  Ops whose scalars are all bf16
// values run packed; the others (contrast, bias field, fp32 scalars, clamped
// shift) take the fp32 path of apply_one on the unpacked values.
// ---------------------------------------------------------------------------
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t w) {
  return *reinterpret_cast<const __nv_bfloat162*>(&w);
}
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 h) {
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ void unpack_words(const uint32_t* w, float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = __uint_as_float(w[j] << 16);
    v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}
// values already rounded to bf16: the packing is a byte permutation
__device__ __forceinline__ void pack_words(const float* v, uint32_t* w) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = __byte_perm(__float_as_uint(v[2 * j]), __float_as_uint(v[2 * j + 1]), 0x7632);
}

// Op oi of the segment on one chunk of 8 bf16 values (four bf16x2 words);
// KIND >= 0: the op's kind, known at compile time.
template <int KIND>
__device__ __forceinline__ void apply_one_bf16x8(const ChainArgs& a, int oi, const OpConst& k,
                                                 int64_t b, int64_t c, int64_t s0, uint32_t* w) {
  {
    const OpArgs& op = a.ops[oi];
    const bool on = k.on != 0;
    bool done = true;
    switch (KIND >= 0 ? KIND : op.kind) {
      case BA_OP_NOISE:
        if (op.flags & BA_NOISE_PHILOX) {
          if (!on) {
#pragma unroll
            for (int j = 0; j < 4; ++j) w[j] = as_u32(__hadd2_rn(as_bf2(w[j]), as_bf2(0u)));
            break;
          }
          const uint64_t eb = op.elem_offset + (uint64_t)b;
          const int64_t first = c * a.HWD + s0;  // a multiple of 8
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint64_t q = (uint64_t)(first + 4 * half) >> 2;
            const U4 ctr = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                            STREAM_NOISE | (uint32_t)(q >> 32)};
            float z[4];
            normal4(philox4x32_10(ctr, op.seed_lo, op.seed_hi), z);
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              // torch.randn(...) * std + mean in fp32, then .to(bf16)
              const float n0 = __fadd_rn(__fmul_rn(z[2 * t], k.k0), k.k1);
              const float n1 = __fadd_rn(__fmul_rn(z[2 * t + 1], k.k0), k.k1);
              const int j = 2 * half + t;
              w[j] = as_u32(__hadd2_rn(as_bf2(w[j]), __floats2bfloat162_rn(n0, n1)));
            }
          }
        } else {
          const float* np = op.noise + (b * a.C + c) * a.HWD + s0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 n2 = __floats2bfloat162_rn(__ldg(np + 2 * j), __ldg(np + 2 * j + 1));
            w[j] = as_u32(__hadd2_rn(as_bf2(w[j]), __hmul2_rn(n2, as_bf2(k.h0))));
          }
        }
        break;
      case BA_OP_SCALE:
        if (!on) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = as_u32(__hmul2_rn(as_bf2(w[j]), as_bf2(k.h0)));
        break;
      case BA_OP_SHIFT:
        if (!on) break;
        if (op.flags & BA_SHIFT_SAFE) {
          done = false;
          break;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = as_u32(__hadd2_rn(as_bf2(w[j]), as_bf2(k.h0)));
        break;
      case BA_OP_RESCALE:
        if (op.flags & BA_RESCALE_FACTOR) {
          if (!k.packed) {
            done = false;
            break;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) w[j] = as_u32(__hmul2_rn(as_bf2(w[j]), as_bf2(k.h0)));
          break;
        }
        if (!(op.flags & (BA_RESCALE_MINV | BA_RESCALE_MAXV))) break;
        if (!k.packed) {
          done = false;
          break;
        }
        {
          const bool both = (op.flags & BA_RESCALE_MINV) && (op.flags & BA_RESCALE_MAXV);
          // (x - mn) / den in bf16, then * (maxv - minv) + minv in bf16; the
          // 8 quotients take div_for_bf16's reciprocal path unless one of
          // them needs its division, then all go through div_for_bf16
          float nv[8], q[8];
          bool fast = k.k3 != 0.0f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t num = as_u32(__hsub2_rn(as_bf2(w[j]), as_bf2(k.h0)));
            nv[2 * j] = __uint_as_float(num << 16);
            nv[2 * j + 1] = __uint_as_float(num & 0xFFFF0000u);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            q[i] = __fmul_rn(nv[i], k.k3);
            const float aq = fabsf(q[i]);
            fast = fast && (nv[i] == 0.0f || (aq >= 0x1p-100f && aq <= 0x1p100f));
          }
          if (!fast)
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = div_for_bf16(nv[i], k.k1, k.k3);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            __nv_bfloat162 r = __floats2bfloat162_rn(q[2 * j], q[2 * j + 1]);
            if (both) r = __hadd2_rn(__hmul2_rn(r, as_bf2(k.h1)), as_bf2(k.h2));
            w[j] = as_u32(r);
          }
        }
        break;
      default:
        done = false;  // contrast, bias field: fp32 arithmetic, one rounding
        break;
    }
    if (!done) {
      float v[8];
      unpack_words(w, v);
      apply_one<BA_BF16, 8, KIND>(a, oi, k, b, c, s0, 8, v);
      pack_words(v, w);
    }
  }
}

// A segment's ops given at compile time: SEQ holds their kinds, four bits
// each, the first op in the lowest bits (0 ends the sequence).
template <int SEQ>
__device__ __forceinline__ void apply_seq_bf16x8(const ChainArgs& a, const OpConst* oc, int oi,
                                                 int64_t b, int64_t c, int64_t s0, uint32_t* w) {
  if constexpr (SEQ != 0) {
    apply_one_bf16x8<(SEQ & 15)>(a, oi, oc[oi], b, c, s0, w);
    apply_seq_bf16x8<(SEQ >> 4)>(a, oc, oi + 1, b, c, s0, w);
  }
}

// The segment's ops on one chunk of 8 bf16 values.  SEQ >= 0: the ops'
// kinds in compile-time form (apply_seq_bf16x8), -1: any ops.
template <int SEQ = -1>
__device__ __forceinline__ void apply_ops_bf16x8(const ChainArgs& a, const OpConst* oc,
                                                 int64_t b, int64_t c, int64_t s0, uint32_t* w) {
  if constexpr (SEQ >= 0)
    apply_seq_bf16x8<SEQ>(a, oc, 0, b, c, s0, w);
  else
    for (int oi = 0; oi < a.n_ops; ++oi) apply_one_bf16x8<-1>(a, oi, oc[oi], b, c, s0, w);
}

__device__ __forceinline__ void fold_minmax_bf16x8(const uint32_t* w, __nv_bfloat162& mn,
                                                   __nv_bfloat162& mx) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    mn = __hmin2_nan(mn, as_bf2(w[j]));
    mx = __hmax2_nan(mx, as_bf2(w[j]));
  }
}

// Block-wide min/max of (mn, mx) followed by one atomic pair.
__device__ __forceinline__ void block_minmax_commit(float mn, float mx, int32_t* keys) {
  __shared__ int32_t s_min[CHAIN_THREADS / 32], s_max[CHAIN_THREADS / 32];
  const bool nan = (mn != mn) || (mx != mx);
  int32_t kmin = nan ? KEY_MIN_NAN : fkey(mn);
  int32_t kmax = nan ? KEY_MAX_NAN : fkey(mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xFFFFFFFFu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xFFFFFFFFu, kmax, o));
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();  // s_min/s_max may still be read by a previous commit
  if (lane == 0) {
    s_min[warp] = kmin;
    s_max[warp] = kmax;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < CHAIN_THREADS / 32; ++i) {
      kmin = min(kmin, s_min[i]);
      kmax = max(kmax, s_max[i]);
    }
    if (kmin != fkey(INFINITY)) atomicMin(keys, kmin);
    if (kmax != fkey(-INFINITY)) atomicMax(keys + 1, kmax);
  }
}

// NaN-propagating min/max (PTX min.NaN / max.NaN, sm_80+): a NaN anywhere
// makes the running value NaN, as torch.min / torch.max propagate it.
__device__ __forceinline__ float min_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

template <int VEC>
__device__ __forceinline__ void fold_minmax(const float* v, int n, float& mn, float& mx) {
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    if (i < n) {
      mn = min_nan(mn, v[i]);
      mx = max_nan(mx, v[i]);
    }
  }
}

// Per-thread moments of a segment's results (STD_SHIFT, FIXED_MEAN and
// relative RICIAN read the mean / std of their input): each chunk is summed
// in fp32, the chunk sums are accumulated in double.
struct Moments {
  double s, ss, nz;
};

template <int VEC>
__device__ __forceinline__ void fold_moments(const float* v, int n, Moments& mo) {
  float cs = 0.0f, css = 0.0f, cnz = 0.0f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    if (i < n) {
      cs = __fadd_rn(cs, v[i]);
      css = __fmaf_rn(v[i], v[i], css);
      cnz = __fadd_rn(cnz, v[i] != 0.0f ? 1.0f : 0.0f);
    }
  }
  mo.s += (double)cs;
  mo.ss += (double)css;
  mo.nz += (double)cnz;
}

// Block-wide sum of the moments followed by one atomic per quantity.
__device__ __forceinline__ void block_moments_commit(Moments mo, double* out) {
  __shared__ double s_m[3][CHAIN_THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mo.s += __shfl_xor_sync(0xFFFFFFFFu, mo.s, o);
    mo.ss += __shfl_xor_sync(0xFFFFFFFFu, mo.ss, o);
    mo.nz += __shfl_xor_sync(0xFFFFFFFFu, mo.nz, o);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) {
    s_m[0][warp] = mo.s;
    s_m[1][warp] = mo.ss;
    s_m[2][warp] = mo.nz;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < CHAIN_THREADS / 32; ++i) {
      mo.s += s_m[0][i];
      mo.ss += s_m[1][i];
      mo.nz += s_m[2][i];
    }
    atomicAdd(out, mo.s);
    atomicAdd(out + 1, mo.ss);
    atomicAdd(out + 2, mo.nz);
  }
}

// 16 bytes <-> VEC floats of the dtype.
template <int DT, int VEC>
__device__ __forceinline__ void unpack16(const uint4& t, float* v) {
  const uint32_t w[4] = {t.x, t.y, t.z, t.w};
  if (DT == BA_BF16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(w[i]);
  }
}

template <int DT, int VEC>
__device__ __forceinline__ uint4 pack16(const float* v) {
  uint4 t;
  if (DT == BA_BF16) {
    t.x = pack_bf16x2(v[0], v[1]);
    t.y = pack_bf16x2(v[2], v[3]);
    t.z = pack_bf16x2(v[4], v[5]);
    t.w = pack_bf16x2(v[6], v[7]);
  } else {
    t = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                   __float_as_uint(v[3]));
  }
  return t;
}

// Vector path over positions [s_begin, s_end) of one channel: 16-byte chunks
// handed to threads round-robin, each thread streaming its own chunks through
// a private ring of PIPE slots in shared memory with cp.async, so PIPE chunks
// per thread are in flight without holding registers.  A thread only reads
// the slots it filled itself, so cp.async.wait_group alone orders the data.
template <int DT, int VEC, bool WRITE, int SEQ>
__device__ __forceinline__ void run_range_vec(const ChainArgs& a, const OpConst* oc, int64_t b,
                                              int64_t c, int64_t s_begin, int64_t s_end,
                                              bool stats, float& mn, float& mx, Moments& mo,
                                              uint4* ring) {
  const int tid = threadIdx.x;
  const int64_t n_chunks = (s_end - s_begin) / VEC;
  const int64_t base = (b * a.C + c) * a.HWD + s_begin;
  __nv_bfloat162 mn2 = __floats2bfloat162_rn(INFINITY, INFINITY);
  __nv_bfloat162 mx2 = __floats2bfloat162_rn(-INFINITY, -INFINITY);
  const uint4* src = reinterpret_cast<const uint4*>(
      (const char*)a.src + base * (DT == BA_BF16 ? 2 : 4));
  uint4* dst = reinterpret_cast<uint4*>((char*)a.dst + base * (DT == BA_BF16 ? 2 : 4));
#pragma unroll
  for (int k = 0; k < CHAIN_PIPE - 1; ++k) {
    const int64_t j = tid + (int64_t)k * CHAIN_THREADS;
    if (j < n_chunks) cp_async16(&ring[k * CHAIN_THREADS + tid], src + j);
    cp_async_commit();
  }
  int slot = 0;
  for (int64_t j = tid; j < n_chunks; j += CHAIN_THREADS) {
    const int64_t jp = j + (int64_t)(CHAIN_PIPE - 1) * CHAIN_THREADS;
    const int pslot = slot == 0 ? CHAIN_PIPE - 1 : slot - 1;
    if (jp < n_chunks) cp_async16(&ring[pslot * CHAIN_THREADS + tid], src + jp);
    cp_async_commit();
    cp_async_wait<CHAIN_PIPE - 1>();
    if constexpr (DT == BA_BF16) {
      const uint4 t = ring[slot * CHAIN_THREADS + tid];
      uint32_t w[4] = {t.x, t.y, t.z, t.w};
      apply_ops_bf16x8<SEQ>(a, oc, b, c, s_begin + j * VEC, w);
      if (WRITE) dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
      if (stats) {
        if (a.stats_moments) {
          float v[8];
          unpack_words(w, v);
          fold_moments<8>(v, 8, mo);
        } else {
          fold_minmax_bf16x8(w, mn2, mx2);
        }
      }
    } else {
      float v[VEC];
      unpack16<DT, VEC>(ring[slot * CHAIN_THREADS + tid], v);
      apply_ops<DT, VEC, SEQ>(a, oc, b, c, s_begin + j * VEC, VEC, v);
      if (WRITE) dst[j] = pack16<DT, VEC>(v);
      if (stats) {
        if (a.stats_moments)
          fold_moments<VEC>(v, VEC, mo);
        else
          fold_minmax<VEC>(v, VEC, mn, mx);
      }
    }
    slot = slot + 1 == CHAIN_PIPE ? 0 : slot + 1;
  }
  cp_async_wait<0>();
  if constexpr (DT == BA_BF16) {
    mn = min_nan(mn, min_nan(__low2float(mn2), __high2float(mn2)));
    mx = max_nan(mx, max_nan(__low2float(mx2), __high2float(mx2)));
  }
}

// Scalar path (spatial size not a multiple of the vector width, or
// unaligned pointers): one element at a time.
template <int DT, bool WRITE>
__device__ __forceinline__ void run_range_scalar(const ChainArgs& a, const OpConst* oc,
                                                 int64_t b, int64_t c, int64_t s_begin,
                                                 int64_t s_end, bool stats, float& mn, float& mx,
                                                 Moments& mo) {
  const int64_t base = (b * a.C + c) * a.HWD;
  for (int64_t s = s_begin + threadIdx.x; s < s_end; s += CHAIN_THREADS) {
    float v[1];
    v[0] = load_f(a.src, DT, base + s);
    apply_ops<DT, 1>(a, oc, b, c, s, 1, v);
    if (WRITE) store_f(a.dst, DT, base + s, v[0]);
    if (stats) {
      if (a.stats_moments)
        fold_moments<1>(v, 1, mo);
      else
        fold_minmax<1>(v, 1, mn, mx);
    }
  }
}

// One segment of the chain.  CTA (x, y) handles spatial positions
// [x * tile, +tile) of channel y % C of element b0 + y / C, so the cp.async
// ring runs uninterrupted over the whole range and the op constants are
// resolved once per CTA.  SEQ >= 0: the segment's op kinds, four bits each
// (first op lowest), so their dispatch is resolved at compile time; -1: any
// ops.
template <int DT, int VEC, bool WRITE, int SEQ = -1>
__global__ void __launch_bounds__(CHAIN_THREADS, chain_minblocks<DT>())
    chain_kernel(const __grid_constant__ ChainArgs a) {
  __shared__ OpConst s_oc[BA_MAX_OPS];
  __shared__ uint4 s_ring[VEC > 1 ? CHAIN_PIPE * CHAIN_THREADS : 1];
  const int64_t b = a.b0 + blockIdx.y / a.C;
  const int64_t c = blockIdx.y % a.C;
  const int64_t s_begin = (int64_t)blockIdx.x * a.tile;
  const int64_t s_end = min(s_begin + a.tile, a.HWD);
  if (threadIdx.x < a.n_ops) resolve_op<DT>(a, threadIdx.x, b, c, s_oc[threadIdx.x]);
  __syncthreads();
  float mn = INFINITY, mx = -INFINITY;
  Moments mo = {0.0, 0.0, 0.0};
  if (VEC > 1)
    run_range_vec<DT, VEC, WRITE, SEQ>(a, s_oc, b, c, s_begin, s_end, a.stats_mode != 0, mn, mx,
                                       mo, s_ring);
  else
    run_range_scalar<DT, WRITE>(a, s_oc, b, c, s_begin, s_end, a.stats_mode != 0, mn, mx, mo);
  if (a.stats_mode != 0) {
    const int64_t g = a.stats_mode == 2 ? b * a.C + c : b;
    if (a.stats_moments)
      block_moments_commit(mo, a.moments_out + 3 * g);
    else
      block_minmax_commit(mn, mx, a.stats_out + 2 * g);
  }
}

__global__ void init_keys_kernel(int32_t* keys, int64_t n_groups) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n_groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    keys[2 * g] = fkey(INFINITY);
    keys[2 * g + 1] = fkey(-INFINITY);
  }
}

__global__ void decode_keys_kernel(float* stats, int64_t n_groups) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n_groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int32_t* k = (const int32_t*)stats;
    const float mn = decode_min_key(k[2 * g]);
    const float mx = decode_max_key(k[2 * g + 1]);
    stats[2 * g] = mn;
    stats[2 * g + 1] = mx;
  }
}

// Plain per-group min/max over a (n_groups, group_size) view, streamed
// through the same per-thread cp.async ring as the chain.
template <int DT, int VEC>
__global__ void __launch_bounds__(CHAIN_THREADS, CHAIN_MINBLOCKS)
    minmax_kernel(const void* x, int64_t group_size, int64_t tile, int32_t* keys) {
  __shared__ uint4 s_ring[VEC > 1 ? CHAIN_PIPE * CHAIN_THREADS : 1];
  const int64_t g = blockIdx.y;
  const int64_t s_begin = (int64_t)blockIdx.x * tile;
  const int64_t s_end = min(s_begin + tile, group_size);
  float mn = INFINITY, mx = -INFINITY;
  if (VEC > 1) {
    const int tid = threadIdx.x;
    const int64_t n_chunks = (s_end - s_begin) / VEC;
    const uint4* src = reinterpret_cast<const uint4*>(
        (const char*)x + (g * group_size + s_begin) * (DT == BA_BF16 ? 2 : 4));
    __nv_bfloat162 mn2 = __floats2bfloat162_rn(INFINITY, INFINITY);
    __nv_bfloat162 mx2 = __floats2bfloat162_rn(-INFINITY, -INFINITY);
#pragma unroll
    for (int k = 0; k < CHAIN_PIPE - 1; ++k) {
      const int64_t j = tid + (int64_t)k * CHAIN_THREADS;
      if (j < n_chunks) cp_async16(&s_ring[k * CHAIN_THREADS + tid], src + j);
      cp_async_commit();
    }
    int slot = 0;
    for (int64_t j = tid; j < n_chunks; j += CHAIN_THREADS) {
      const int64_t jp = j + (int64_t)(CHAIN_PIPE - 1) * CHAIN_THREADS;
      const int pslot = slot == 0 ? CHAIN_PIPE - 1 : slot - 1;
      if (jp < n_chunks) cp_async16(&s_ring[pslot * CHAIN_THREADS + tid], src + jp);
      cp_async_commit();
      cp_async_wait<CHAIN_PIPE - 1>();
      if constexpr (DT == BA_BF16) {
        const uint4 t = s_ring[slot * CHAIN_THREADS + tid];
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
        fold_minmax_bf16x8(w, mn2, mx2);
      } else {
        float v[VEC];
        unpack16<DT, VEC>(s_ring[slot * CHAIN_THREADS + tid], v);
        fold_minmax<VEC>(v, VEC, mn, mx);
      }
      slot = slot + 1 == CHAIN_PIPE ? 0 : slot + 1;
    }
    cp_async_wait<0>();
    if constexpr (DT == BA_BF16) {
      mn = min_nan(mn, min_nan(__low2float(mn2), __high2float(mn2)));
      mx = max_nan(mx, max_nan(__low2float(mx2), __high2float(mx2)));
    }
  } else {
    for (int64_t s = s_begin + threadIdx.x; s < s_end; s += CHAIN_THREADS) {
      float v[1] = {load_f(x, DT, g * group_size + s)};
      fold_minmax<1>(v, 1, mn, mx);
    }
  }
  block_minmax_commit(mn, mx, keys + 2 * g);
}

int sm_count() {
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

// Spatial positions per CTA: enough CTAs for about two waves, but at least
// CHAIN_MIN_CHUNKS 16-byte chunks per thread so the cp.async ring is full
// for most of a CTA's life.
int64_t pick_tile(int64_t positions, int64_t n_blocks_y, int vec) {
  const int64_t target_blocks = (int64_t)sm_count() * CHAIN_MINBLOCKS * 2;
  const int64_t per_y = std::max<int64_t>(1, target_blocks / std::max<int64_t>(1, n_blocks_y));
  const int64_t quantum = (int64_t)CHAIN_THREADS * vec;
  int64_t tile = (positions + per_y - 1) / per_y;
  tile = std::max<int64_t>(tile, quantum * (vec > 1 ? CHAIN_MIN_CHUNKS : 1));
  tile = (tile + quantum - 1) / quantum * quantum;
  return tile;
}

// Ops that read statistics of their own input: min/max (CONTRAST, min/max
// RESCALE) or moments (STD_SHIFT, FIXED_MEAN, relative RICIAN).
bool needs_moments(const ba_op& op) {
  return op.kind == BA_OP_STD_SHIFT || op.kind == BA_OP_FIXED_MEAN ||
         (op.kind == BA_OP_RICIAN && (op.flags & BA_RICIAN_RELATIVE));
}

// RESCALE with its min/max given (BA_RESCALE_GIVEN, ba_op.stats)
bool stats_given(const ba_op& op) {
  return op.kind == BA_OP_RESCALE && (op.flags & BA_RESCALE_GIVEN) &&
         !(op.flags & BA_RESCALE_FACTOR) && (op.flags & (BA_RESCALE_MINV | BA_RESCALE_MAXV));
}

bool needs_stats(const ba_op& op) {
  if (op.kind == BA_OP_CONTRAST || needs_moments(op)) return true;
  if (op.kind == BA_OP_RESCALE)
    return !(op.flags & BA_RESCALE_FACTOR) && (op.flags & (BA_RESCALE_MINV | BA_RESCALE_MAXV)) &&
           !(op.flags & BA_RESCALE_GIVEN);
  return false;
}

bool stats_per_channel(const ba_op& op) {
  if (op.kind == BA_OP_RESCALE) return op.flags & BA_RESCALE_CHANNEL;
  if (op.kind == BA_OP_STD_SHIFT || op.kind == BA_OP_FIXED_MEAN) return op.flags & BA_STAT_CHANNEL;
  return false;
}

int64_t stats_groups(const ba_op& op, int64_t B, int64_t C) {
  return stats_per_channel(op) ? B * C : B;
}

// int32 words of workspace per statistics group: two order-preserving keys
// (min/max) or three doubles (moments).
int64_t stats_words(const ba_op& op) { return needs_moments(op) ? 6 : 2; }

struct Segment {
  int first, last;      // ops [first, last)
  int stats_for;        // op index whose stats this segment produces, -1 none
  int64_t stats_offset;  // int32 offset of those stats in the workspace (8-byte aligned)
};

void plan_segments(const ba_chain_desc* d, std::vector<Segment>& segs, int64_t& ws_ints) {
  segs.clear();
  ws_ints = 0;
  int first = 0;
  for (int i = 0; i <= d->n_ops; ++i) {
    const bool cut = (i == d->n_ops) || needs_stats(d->ops[i]);
    if (!cut) continue;
    Segment s;
    s.first = first;
    s.last = i;
    s.stats_for = (i < d->n_ops) ? i : -1;
    s.stats_offset = 0;
    if (s.stats_for >= 0) {
      ws_ints = (ws_ints + 1) & ~(int64_t)1;  // doubles stay 8-byte aligned
      s.stats_offset = ws_ints;
      ws_ints += stats_words(d->ops[i]) * stats_groups(d->ops[i], d->batch, d->channels);
    }
    segs.push_back(s);
    first = i;
  }
}

template <int DT, int VEC>
ba_status launch_segment(ChainArgs& a, int64_t nb, bool write, cudaStream_t st) {
  const int64_t tile = pick_tile(a.HWD, nb * a.C, VEC);
  a.tile = tile;
  dim3 grid((unsigned)((a.HWD + tile - 1) / tile), (unsigned)(nb * a.C));
  // segments of common op sequences run without the op loop and kind
  // dispatch: any lone op (a rescale on given statistics is the usual last
  // segment; ops that read their input's statistics cut the chain into
  // one-op segments), and contrast -> scale -> shift
  if constexpr (VEC > 1) {
    int seq = 0;
    for (int i = a.n_ops - 1; i >= 0 && a.n_ops <= 3; --i) seq = (seq << 4) | a.ops[i].kind;
    if (write) {
      switch (a.n_ops <= 3 ? seq : -1) {
#define BA_SEQ(S)                                                        \
  case S:                                                                \
    chain_kernel<DT, VEC, true, (S)><<<grid, CHAIN_THREADS, 0, st>>>(a); \
    return check_launch("ba_intensity_chain");
        BA_SEQ(BA_OP_NOISE)
        BA_SEQ(BA_OP_CONTRAST)
        BA_SEQ(BA_OP_SCALE)
        BA_SEQ(BA_OP_SHIFT)
        BA_SEQ(BA_OP_BIAS_FIELD)
        BA_SEQ(BA_OP_RESCALE)
        BA_SEQ(BA_OP_RICIAN)
        BA_SEQ(BA_OP_STD_SHIFT)
        BA_SEQ(BA_OP_FIXED_MEAN)
        BA_SEQ(BA_OP_CONTRAST | BA_OP_SCALE << 4 | BA_OP_SHIFT << 8)
#undef BA_SEQ
        default:
          break;
      }
    } else if (a.n_ops == 0) {
      // a statistics pass over the input alone (no ops, no write)
      chain_kernel<DT, VEC, false, 0><<<grid, CHAIN_THREADS, 0, st>>>(a);
      return check_launch("ba_intensity_chain");
    }
  }
  if (write)
    chain_kernel<DT, VEC, true><<<grid, CHAIN_THREADS, 0, st>>>(a);
  else
    chain_kernel<DT, VEC, false><<<grid, CHAIN_THREADS, 0, st>>>(a);
  return check_launch("ba_intensity_chain");
}

}  // namespace

// Per-group min/max keys for ba_resample3d's minmax output: set them to the
// empty fold, and fold a tensor's groups into them (a group: group_size
// consecutive values; the same keys and kernel as a chain's statistics).
ba_status minmax_keys_init(int32_t* keys, int64_t groups, cudaStream_t st) {
  if (groups <= 0) return BA_OK;
  init_keys_kernel<<<(unsigned)std::min<int64_t>((groups + 255) / 256, 1024), 256, 0, st>>>(
      keys, groups);
  return check_launch("ba_resample3d minmax");
}

ba_status minmax_keys_fold(const void* x, int dtype, int64_t groups, int64_t group_size,
                           int32_t* keys, cudaStream_t st) {
  if (groups <= 0 || group_size <= 0) return BA_OK;
  const int vec = dtype == BA_BF16 ? 8 : 4;
  const bool vec_ok = (group_size % vec) == 0 && ((uintptr_t)x % 16) == 0;
  const int64_t tile = pick_tile(group_size, groups, vec_ok ? vec : 1);
  dim3 grid((unsigned)((group_size + tile - 1) / tile), (unsigned)groups);
  if (dtype == BA_BF16) {
    if (vec_ok)
      minmax_kernel<BA_BF16, 8><<<grid, CHAIN_THREADS, 0, st>>>(x, group_size, tile, keys);
    else
      minmax_kernel<BA_BF16, 1><<<grid, CHAIN_THREADS, 0, st>>>(x, group_size, tile, keys);
  } else {
    if (vec_ok)
      minmax_kernel<BA_F32, 4><<<grid, CHAIN_THREADS, 0, st>>>(x, group_size, tile, keys);
    else
      minmax_kernel<BA_F32, 1><<<grid, CHAIN_THREADS, 0, st>>>(x, group_size, tile, keys);
  }
  return check_launch("ba_resample3d minmax");
}

// Shape, dtype, op and pointer checks of a chain descriptor, shared with
// ba_intensity_chain_noalloc (noalloc.cu).
ba_status validate_chain(const ba_chain_desc* d) {
  BA_REQUIRE(d != nullptr, "ba_intensity_chain: desc is NULL");
  BA_REQUIRE(d->batch >= 0 && d->channels >= 0 && d->H > 0 && d->W > 0 && d->D > 0,
             "ba_intensity_chain: bad shape");
  BA_REQUIRE(d->batch * d->channels <= 65535,
             "ba_intensity_chain: batch * channels exceeds 65535");
  BA_REQUIRE(d->dtype == BA_F32 || d->dtype == BA_BF16, "ba_intensity_chain: bad dtype %d",
             d->dtype);
  BA_REQUIRE(d->n_ops >= 1 && d->n_ops <= BA_MAX_OPS, "ba_intensity_chain: n_ops=%d not in 1..%d",
             d->n_ops, BA_MAX_OPS);
  for (int i = 0; i < d->n_ops; ++i) {
    const ba_op& op = d->ops[i];
    BA_REQUIRE(op.kind >= BA_OP_NOISE && op.kind <= BA_OP_FIXED_MEAN,
               "ba_intensity_chain: op %d unknown kind %d", i, op.kind);
    switch (op.kind) {
      case BA_OP_NOISE:
        if (op.flags & BA_NOISE_PHILOX)
          BA_REQUIRE(op.param && op.param2, "ba_intensity_chain: op %d NOISE needs std and mean",
                     i);
        else
          BA_REQUIRE(op.noise, "ba_intensity_chain: op %d NOISE needs an injected noise tensor",
                     i);
        break;
      case BA_OP_CONTRAST:
      case BA_OP_SCALE:
      case BA_OP_SHIFT:
        BA_REQUIRE(op.param, "ba_intensity_chain: op %d needs its per-element parameter", i);
        break;
      case BA_OP_RICIAN:
        BA_REQUIRE(op.param, "ba_intensity_chain: op %d RICIAN needs noise_std", i);
        if (!(op.flags & BA_RICIAN_PHILOX))
          BA_REQUIRE(op.noise && op.param2,
                     "ba_intensity_chain: op %d RICIAN needs injected u1 and u2", i);
        break;
      case BA_OP_STD_SHIFT:
      case BA_OP_FIXED_MEAN:
        BA_REQUIRE(op.param, "ba_intensity_chain: op %d needs its per-element factor", i);
        break;
      case BA_OP_RESCALE:
        if (op.flags & BA_RESCALE_GIVEN)
          BA_REQUIRE(op.stats && (op.flags & BA_RESCALE_CHANNEL) &&
                         !(op.flags & BA_RESCALE_FACTOR),
                     "ba_intensity_chain: op %d RESCALE with BA_RESCALE_GIVEN needs stats and "
                     "BA_RESCALE_CHANNEL",
                     i);
        break;
      case BA_OP_BIAS_FIELD:
        BA_REQUIRE(op.param, "ba_intensity_chain: op %d BIAS_FIELD needs coefficients", i);
        if (op.degree < 1 || op.degree > 6) {
          set_error("ba_intensity_chain: op %d BIAS_FIELD degree %d not in 1..6", i, op.degree);
          return BA_EUNSUPPORTED;
        }
        break;
      default:
        break;
    }
  }
  const int64_t n = d->batch * d->channels * d->H * d->W * d->D;
  if (n > 0) {
    BA_REQUIRE(d->src && d->dst, "ba_intensity_chain: NULL src or dst");
    const size_t esz = d->dtype == BA_BF16 ? 2 : 4;
    const char* s = (const char*)d->src;
    const char* t = (const char*)d->dst;
    BA_REQUIRE(s == t || s + n * esz <= t || t + n * esz <= s,
               "ba_intensity_chain: dst partially overlaps src");
    BA_REQUIRE((uintptr_t)s % esz == 0 && (uintptr_t)t % esz == 0,
               "ba_intensity_chain: pointers not aligned to the element size");
  }
  return BA_OK;
}

}  // namespace ba

extern "C" size_t ba_intensity_workspace_bytes(const ba_chain_desc* desc) {
  using namespace ba;
  if (desc == nullptr || desc->n_ops < 1 || desc->n_ops > BA_MAX_OPS) return 0;
  // a malformed shape has no workspace size (ba_intensity_chain rejects it)
  if (desc->batch < 0 || desc->channels < 0 || desc->batch * desc->channels > 65535) return 0;
  std::vector<Segment> segs;
  int64_t ints = 0;
  plan_segments(desc, segs, ints);
  return (size_t)ints * sizeof(int32_t);
}

extern "C" ba_status ba_intensity_chain(const ba_chain_desc* desc, void* workspace,
                                        size_t workspace_bytes, ba_stream_t stream) {
  using namespace ba;
  clear_error();
  ba_status st = validate_chain(desc);
  if (st != BA_OK) return st;
  const ba_chain_desc& d = *desc;
  std::vector<Segment> segs;
  int64_t ws_ints = 0;
  plan_segments(&d, segs, ws_ints);
  BA_REQUIRE(workspace_bytes >= (size_t)ws_ints * sizeof(int32_t),
             "ba_intensity_chain: workspace of %zu bytes, %lld needed", workspace_bytes,
             (long long)(ws_ints * sizeof(int32_t)));
  BA_REQUIRE(ws_ints == 0 || workspace != nullptr, "ba_intensity_chain: workspace is NULL");
  BA_REQUIRE(ws_ints == 0 || (uintptr_t)workspace % 16 == 0,
             "ba_intensity_chain: workspace not 16-byte aligned");
  const int64_t HWD = d.H * d.W * d.D;
  if (d.batch * d.channels * HWD == 0) return BA_OK;
  cudaStream_t cs = (cudaStream_t)stream;
  int32_t* keys = (int32_t*)workspace;
  for (const Segment& sg : segs) {
    if (sg.stats_for < 0) continue;
    const ba_op& op = d.ops[sg.stats_for];
    const int64_t groups = stats_groups(op, d.batch, d.channels);
    if (needs_moments(op)) {
      if (cudaMemsetAsync(keys + sg.stats_offset, 0, (size_t)groups * 3 * sizeof(double), cs) !=
          cudaSuccess) {
        set_error("ba_intensity_chain: clearing the statistics failed");
        return BA_ECUDA;
      }
    } else {
      init_keys_kernel<<<(unsigned)std::min<int64_t>((groups + 255) / 256, 1024), 256, 0, cs>>>(
          keys + sg.stats_offset, groups);
      st = check_launch("ba_intensity_chain");
      if (st != BA_OK) return st;
    }
  }

  const int vec = d.dtype == BA_BF16 ? 8 : 4;
  const bool vec_ok = (HWD % vec) == 0 && ((uintptr_t)d.src % 16) == 0 &&
                      ((uintptr_t)d.dst % 16) == 0 &&
                      [&] {
                        for (int i = 0; i < d.n_ops; ++i) {
                          const ba_op& op = d.ops[i];
                          if (op.kind == BA_OP_NOISE && !(op.flags & BA_NOISE_PHILOX) &&
                              ((uintptr_t)op.noise % 16) != 0)
                            return false;
                          if (op.kind == BA_OP_RICIAN && !(op.flags & BA_RICIAN_PHILOX) &&
                              (((uintptr_t)op.noise % 16) != 0 || ((uintptr_t)op.param2 % 16) != 0))
                            return false;
                        }
                        return true;
                      }();

  const int64_t slice = d.batch;  // measured: slicing the batch for L2 reuse did not pay

  ChainArgs a;
  memset(&a, 0, sizeof(a));
  a.C = d.channels;
  a.H = d.H;
  a.W = d.W;
  a.D = d.D;
  a.HWD = HWD;
  for (int64_t b0 = 0; b0 < d.batch; b0 += slice) {
    const int64_t nb = std::min(slice, d.batch - b0);
    bool written = false;
    for (size_t si = 0; si < segs.size(); ++si) {
      const Segment& sg = segs[si];
      const bool has_ops = sg.last > sg.first;
      const bool is_last = si + 1 == segs.size();
      // A segment without ops only reduces (a chain starting with a stats
      // consumer); the last segment always writes dst.
      const bool write = has_ops || (is_last && !written);
      a.src = written ? d.dst : d.src;
      a.dst = d.dst;
      a.b0 = (int32_t)b0;
      a.n_ops = sg.last - sg.first;
      for (int i = sg.first; i < sg.last; ++i) {
        const ba_op& op = d.ops[i];
        OpArgs& o = a.ops[i - sg.first];
        memset(&o, 0, sizeof(o));
        o.kind = op.kind;
        o.flags = op.flags;
        o.mask = op.mask;
        o.param = op.param;
        o.param2 = op.param2;
        o.noise = op.noise;
        o.degree = op.degree;
        o.seed_lo = (uint32_t)op.seed;
        o.seed_hi = (uint32_t)(op.seed >> 32);
        o.elem_offset = op.elem_offset;
        o.minv = (float)op.c0;
        o.span = (float)(op.c1 - op.c0);
        o.factor1p = (float)(1.0 + op.c0);
        o.mean = (float)op.c0;
        if (stats_given(op)) {
          // min/max per (element, channel) from the resample that wrote src
          o.stats_per_channel = 1;
          o.stats_in = op.stats;
        } else if (needs_stats(op)) {
          // Stats come from the previous segment.
          const Segment& prev = segs[si - 1];
          o.stats_per_channel = stats_per_channel(op) ? 1 : 0;
          if (needs_moments(op)) {
            o.moments_in = (const double*)(keys + prev.stats_offset);
            o.moments_n = o.stats_per_channel ? HWD : d.channels * HWD;
          } else {
            o.stats_in = keys + prev.stats_offset;
          }
        }
      }
      a.stats_out = nullptr;
      a.moments_out = nullptr;
      a.stats_mode = 0;
      a.stats_moments = 0;
      if (sg.stats_for >= 0) {
        const ba_op& nx = d.ops[sg.stats_for];
        a.stats_mode = stats_per_channel(nx) ? 2 : 1;
        a.stats_moments = needs_moments(nx) ? 1 : 0;
        if (a.stats_moments)
          a.moments_out = (double*)(keys + sg.stats_offset);
        else
          a.stats_out = keys + sg.stats_offset;
      }
      if (!write && a.stats_mode == 0) continue;
      if (d.dtype == BA_BF16)
        st = vec_ok ? launch_segment<BA_BF16, 8>(a, nb, write, cs)
                    : launch_segment<BA_BF16, 1>(a, nb, write, cs);
      else
        st = vec_ok ? launch_segment<BA_F32, 4>(a, nb, write, cs)
                    : launch_segment<BA_F32, 1>(a, nb, write, cs);
      if (st != BA_OK) return st;
      if (write) written = true;
    }
  }
  return BA_OK;
}

extern "C" ba_status ba_minmax(const void* x, int32_t dtype, int64_t n_groups, int64_t group_size,
                               float* stats, ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(dtype == BA_F32 || dtype == BA_BF16, "ba_minmax: bad dtype %d", dtype);
  BA_REQUIRE(n_groups >= 0 && group_size >= 0, "ba_minmax: negative size");
  BA_REQUIRE(n_groups <= 65535, "ba_minmax: n_groups %lld exceeds 65535", (long long)n_groups);
  if (n_groups == 0) return BA_OK;
  BA_REQUIRE(stats != nullptr, "ba_minmax: stats is NULL");
  BA_REQUIRE((uintptr_t)stats % 8 == 0, "ba_minmax: stats not 8-byte aligned");
  BA_REQUIRE(group_size == 0 || x != nullptr, "ba_minmax: x is NULL");
  cudaStream_t cs = (cudaStream_t)stream;
  int32_t* keys = (int32_t*)stats;
  init_keys_kernel<<<(unsigned)std::min<int64_t>((n_groups + 255) / 256, 1024), 256, 0, cs>>>(
      keys, n_groups);
  ba_status st = check_launch("ba_minmax");
  if (st != BA_OK) return st;
  if (group_size > 0) {
    const int vec = dtype == BA_BF16 ? 8 : 4;
    const bool vec_ok = (group_size % vec) == 0 && ((uintptr_t)x % 16) == 0;
    const int v = vec_ok ? vec : 1;
    const int64_t tile = pick_tile(group_size, n_groups, v);
    dim3 grid((unsigned)((group_size + tile - 1) / tile), (unsigned)n_groups);
    if (dtype == BA_BF16) {
      if (vec_ok)
        minmax_kernel<BA_BF16, 8><<<grid, CHAIN_THREADS, 0, cs>>>(x, group_size, tile, keys);
      else
        minmax_kernel<BA_BF16, 1><<<grid, CHAIN_THREADS, 0, cs>>>(x, group_size, tile, keys);
    } else {
      if (vec_ok)
        minmax_kernel<BA_F32, 4><<<grid, CHAIN_THREADS, 0, cs>>>(x, group_size, tile, keys);
      else
        minmax_kernel<BA_F32, 1><<<grid, CHAIN_THREADS, 0, cs>>>(x, group_size, tile, keys);
    }
    st = check_launch("ba_minmax");
    if (st != BA_OK) return st;
  }
  decode_keys_kernel<<<(unsigned)std::min<int64_t>((n_groups + 255) / 256, 1024), 256, 0, cs>>>(
      stats, n_groups);
  return check_launch("ba_minmax");
}
