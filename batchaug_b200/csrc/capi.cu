// Library-wide C ABI pieces: thread-local error reporting, the version, the
// launch counter and the host-side Philox draw of per-element parameters.
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

extern "C" int32_t ba_version(void) { return (1 << 16) | 0; }

extern "C" uint64_t ba_kernel_launches(void) {
  return ba::g_launches.load(std::memory_order_relaxed);
}
