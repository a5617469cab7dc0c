// gdn_fwd_sm100_noalloc: the chunked GDN forward for callers that must not
// allocate device memory when they call it.
//
// Who needs this.  The regular entry point takes its scratch (the per-chunk
// operand packets of the two-kernel path) from the caller, and the Python
// layer gets it from the framework's allocator.  Some callers cannot do that:
// runtimes that plan every byte of device memory when they start and forbid
// allocation afterwards, plug-ins whose host framework owns the device memory
// pool and gives them none, and latency-critical code that cannot afford the
// device-wide synchronisation cudaMalloc may perform.  This entry point runs
// the same two kernels with their scratch in a fixed array that is part of
// this library, so a call allocates nothing.
//
// The array (kScratchBytes = 32 MiB) lives in this file's device module.  With
// the CUDA driver's default lazy module loading it is reserved on a device
// when this library's device code is first used there (any of its entry
// points); with CUDA_MODULE_LOADING=EAGER it is reserved when the context is
// created, whether or not this entry point is ever called.  Either way it
// stays reserved on that device until the process exits.  Its device address
// is looked up once per device, by the first call made with that device
// current, and cached for the life of the process: a cudaDeviceReset (or any
// other reset of the primary context) invalidates the cached address, so this
// entry point must not be used after one.
//
// Every call uses the same array and leaves the last call's data in it.  The
// kernels never read a scratch byte that the same call has not written first
// (the work counter in the array's first bytes is zeroed by the call itself,
// before each prep launch), so nothing has to start at zero.  Calls that can run at the same time on the
// GPU (different streams, or different host threads on one device) race on
// the array: serialise them.
#include "../../include/gdn_b200.h"
#include "gdn_wy_scan.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

namespace gdn {
namespace {

constexpr uint64_t kScratchBytes = GDN_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the array for the current device (looked up once).
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDN_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // leave no sticky error behind for the caller
      return GDN_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return GDN_OK;
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_fwd_sm100_noalloc(const gdn_fwd_args* args, void* stream) {
  // An invalid or unsupported request is reported as such, before the size
  // check: a caller must not be told to shrink B*H when the shape is the problem.
  const int vrc = gdn::validate_fwd_args(args);
  if (vrc != GDN_OK) return vrc;
  // One chunk per (batch, head) must fit, next to one fp32 state per (b, h):
  // the sequence is then processed in as many segments as the array needs.
  const uint64_t pairs = uint64_t(args->B) * uint64_t(args->H);
  const uint64_t per_pair = gdn::kPacketBytesPerChunk + uint64_t(args->K) * uint64_t(args->V) * 4ull;
  if (pairs > (gdn::kScratchBytes - gdn::kWorkspaceHeaderBytes) / per_pair) return GDN_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rc = gdn::scratch_for_current_device(&scratch);
  if (rc != GDN_OK) return rc;
  gdn_fwd_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = gdn::kScratchBytes;
  return gdn_fwd_sm100(&a, stream);
}
