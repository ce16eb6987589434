// ba_intensity_chain_noalloc: the intensity chain for callers that cannot
// allocate device memory.
//
// Some hosts of this library own every byte of device memory through their
// own fixed pool (plugin hosts, embedded pipelines) or run the chain in a
// loop where a cudaMalloc/cudaFree — which may synchronise the device — is
// not acceptable, and so cannot provide the chain's scratch buffer.  This
// entry point takes the scratch from a statically sized array in device
// memory instead: a file-scope __device__ array of BA_NOALLOC_CHAIN_SCRATCH
// bytes, which every GPU that loads the library holds until the process
// exits.  It allocates nothing: no cudaMalloc, no cudaFree, no allocating
// library routine.
//
// In host code the array's name is only a host-side stand-in, not a device
// address, so the address is looked up once per device with
// cudaGetSymbolAddress while that device is current (on the first call on
// that device), cached, and passed to the unchanged ba_intensity_chain.
#include <mutex>

#include "ba_common.cuh"

namespace ba {
namespace {

constexpr int kMaxDevices = 64;

// Min/max statistics keys of the chain's segments (int32 pairs per group).
static __device__ __align__(256) unsigned char g_chain_scratch[BA_NOALLOC_CHAIN_SCRATCH];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

ba_status scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("ba_intensity_chain_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return BA_ECUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("ba_intensity_chain_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
    return BA_EUNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_chain_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("ba_intensity_chain_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return BA_ECUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return BA_OK;
}

}  // namespace
}  // namespace ba

extern "C" ba_status ba_intensity_chain_noalloc(const ba_chain_desc* desc, ba_stream_t stream) {
  using namespace ba;
  clear_error();
  BA_REQUIRE(desc != nullptr, "ba_intensity_chain_noalloc: desc is NULL");
  // the descriptor first, so a malformed shape reports itself and not a
  // scratch size derived from it
  const ba_status v = validate_chain(desc);
  if (v != BA_OK) return v;
  const size_t need = ba_intensity_workspace_bytes(desc);
  BA_REQUIRE(need <= (size_t)BA_NOALLOC_CHAIN_SCRATCH,
             "ba_intensity_chain_noalloc: this chain needs %zu bytes of scratch, more than the "
             "%d-byte static array; use ba_intensity_chain with a caller-provided workspace",
             need, BA_NOALLOC_CHAIN_SCRATCH);
  void* scratch = nullptr;
  if (need > 0) {
    const ba_status s = scratch_for_current_device(&scratch);
    if (s != BA_OK) return s;
  }
  // The chain re-initialises every statistics key it uses at the start of
  // the call, so nothing left in the array by an earlier call is read.
  return ba_intensity_chain(desc, scratch, need, stream);
}

extern "C" size_t ba_noalloc_chain_scratch_bytes(void) { return (size_t)BA_NOALLOC_CHAIN_SCRATCH; }
