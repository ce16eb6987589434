// Library-wide C ABI pieces: thread-local error reporting, the version, the
// launch counter and the host-side Philox draw of per-element parameters.
#include <math.h>
#include <string.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "ba_common.cuh"
#include "philox.cuh"

namespace ba {
namespace {
thread_local char g_last_error[512] = {0};
std::atomic<uint64_t> g_launches{0};
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

ba_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
    return BA_ECUDA;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return BA_OK;
}

}  // namespace ba

extern "C" const char* ba_last_error(void) { return ba::g_last_error; }

extern "C" void ba_host_uniform(uint64_t seed, uint32_t stream, uint64_t elem_offset,
                                int64_t n_elems, int64_t per_elem, float* out) {
  if (out == nullptr || n_elems <= 0 || per_elem <= 0) return;
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  for (int64_t e = 0; e < n_elems; ++e) {
    const uint64_t eb = elem_offset + (uint64_t)e;
    for (int64_t q = 0; q * 4 < per_elem; ++q) {
      const ba::U4 ctr = {(uint32_t)q, (uint32_t)eb, (uint32_t)(eb >> 32),
                          ba::STREAM_PARAMS | (stream & 0xFFFFu)};
      const ba::U4 r = ba::philox4x32_10(ctr, k0, k1);
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
      for (int l = 0; l < 4 && q * 4 + l < per_elem; ++l)
        out[e * per_elem + q * 4 + l] = ba::u01(w[l]);
    }
  }
}

namespace {

// c = a @ b for 4x4 row-major fp32, each sum accumulated k = 0..3 with every
// product and addition rounded on its own.
void matmul4(const float* a, const float* b, float* c) {
  float t[16];
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j) {
      float acc = a[i * 4] * b[j];
      for (int k = 1; k < 4; ++k) acc = acc + a[i * 4 + k] * b[k * 4 + j];
      t[i * 4 + j] = acc;
    }
  memcpy(c, t, sizeof(t));
}

void eye4(float* m) {
  memset(m, 0, 16 * sizeof(float));
  m[0] = m[5] = m[10] = m[15] = 1.0f;
}

}  // namespace

extern "C" void ba_host_rand_affine(const float* u, int64_t batch, int64_t u_stride, float prob,
                                    const float* range_a, const float* range_b,
                                    const float* range_c, uint32_t present, uint32_t groups,
                                    int64_t H, int64_t W, int64_t D, uint8_t* mask,
                                    float* affine, float* theta) {
  if (u == nullptr || batch <= 0) return;
  const float sn[3] = {(float)(2.0 / (double)H), (float)(2.0 / (double)W),
                       (float)(2.0 / (double)D)};
  const float si[3] = {(float)((double)H / 2.0), (float)((double)W / 2.0),
                       (float)((double)D / 2.0)};
  for (int64_t e = 0; e < batch; ++e) {
    const float* ue = u + e * u_stride;
    float v[15];
    for (int k = 0; k < 15; ++k)
      v[k] = ((present >> k) & 1u) ? (ue[1 + k] * range_a[k] + range_b[k]) + range_c[k]
                                   : range_c[k];
    float A[16], M[16];
    eye4(A);
    if (groups & 1u) {  // Rx(a0) @ Ry(a1) @ Rz(a2)
      float rx[16], ry[16], rz[16];
      eye4(rx);
      eye4(ry);
      eye4(rz);
      const float c0 = cosf(v[0]), s0 = sinf(v[0]), c1 = cosf(v[1]), s1 = sinf(v[1]);
      const float c2 = cosf(v[2]), s2 = sinf(v[2]);
      rx[5] = c0, rx[6] = -s0, rx[9] = s0, rx[10] = c0;
      ry[0] = c1, ry[2] = s1, ry[8] = -s1, ry[10] = c1;
      rz[0] = c2, rz[1] = -s2, rz[4] = s2, rz[5] = c2;
      matmul4(rx, ry, M);
      matmul4(M, rz, M);
      matmul4(A, M, A);
    }
    if (groups & 2u) {  // shear: (0,1) (0,2) (1,0) (1,2) (2,0) (2,1)
      eye4(M);
      M[1] = v[3], M[2] = v[4], M[4] = v[5], M[6] = v[6], M[8] = v[7], M[9] = v[8];
      matmul4(A, M, A);
    }
    if (groups & 4u) {  // translation
      eye4(M);
      M[3] = v[9], M[7] = v[10], M[11] = v[11];
      matmul4(A, M, A);
    }
    if (groups & 8u) {  // scale
      eye4(M);
      M[0] = v[12], M[5] = v[13], M[10] = v[14];
      matmul4(A, M, A);
    }
    if (mask) mask[e] = ue[0] < prob ? 1 : 0;
    if (affine) memcpy(affine + e * 16, A, sizeof(A));
    if (theta) {
      // monai_affine_to_theta: theta[i][j] = (sn[p(i)] * A[p(i)][p(j)]) * si[p(j)],
      // p swapping axes 0 and 2, sn[3] = si[3] = 1
      for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) {
          const int pi = i == 3 ? 3 : 2 - i, pj = j == 3 ? 3 : 2 - j;
          const float s_i = pi == 3 ? 1.0f : sn[pi];
          const float s_j = pj == 3 ? 1.0f : si[pj];
          theta[e * 16 + i * 4 + j] = (s_i * A[pi * 4 + pj]) * s_j;
        }
    }
  }
}

extern "C" int32_t ba_version(void) { return (1 << 16) | 0; }

extern "C" uint64_t ba_kernel_launches(void) {
  return ba::g_launches.load(std::memory_order_relaxed);
}
