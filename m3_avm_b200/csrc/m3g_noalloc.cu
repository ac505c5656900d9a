// m3g_noalloc.cu -- greedy vocab head that allocates no device memory.
//
// m3g_matvec_greedy_noalloc runs the head GEMV with the argmax epilogue (the
// last GEMV of a decode step) and writes only the greedy token id.  Its
// logits and its 64-bit reduction key live in one file-scope static device
// array instead of buffers from cudaMalloc.  It is for callers that may not
// allocate device memory at all: a host runtime that owns the whole device
// through its own allocator or runs under a fixed memory budget, where a
// hidden cudaMalloc would both escape that budget and synchronise the device
// in the middle of its token loop.
//
// Setup: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress and reads the SM count
// and shared-memory limits; later calls reuse them.  Make that first call
// before any stream capture begins.  The address belongs to the device's
// current context: a call that finds another context current (after
// cudaDeviceReset, say) repeats the set-up instead of using a stale address.
//
// Limits and sharing: at most kMaxRows output rows (the logits fit the
// array); one call at a time per device -- calls on different streams that
// overlap use the same array and race.  Calls on one stream are ordered.
#include <mutex>

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/m3gemv.h"
#include "m3g_device.cuh"
#include "m3g_internal.h"

namespace m3g {
int host_fail(int code, const char* fmt, ...);
}  // namespace m3g

namespace {

constexpr uint64_t kMaxRows = 262144;  // 1 MiB of logits: vocabularies up to 256 Ki entries
constexpr size_t kKeyOff = 0;          // u64 greedy key: must be zero when the GEMV starts
constexpr size_t kStatusOff = 8;       // u32 status word of the GEMV's bounded waits
constexpr size_t kLogitsOff = 256;     // f32 logits[kMaxRows]
constexpr size_t kScratchBytes = kLogitsOff + 4 * kMaxRows;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DevSetup {
  unsigned char* scratch = nullptr;
  CUcontext ctx = nullptr;  // context the address was looked up in
  int sms = 0, smem_per_sm = 0, smem_optin = 0;
};
constexpr int kMaxDev = 64;
std::mutex g_mu;
DevSetup g_setup[kMaxDev];

// cuCtxGetCurrent through the runtime's driver entry point (no libcuda link).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(p);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  return fn;
}

CUcontext current_context() {
  CUcontext c = nullptr;
  CtxGetCurrentFn fn = ctx_get_current();
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

int setup_current_device(DevSetup* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDev) return m3g::host_fail(M3G_EINVAL, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DevSetup& s = g_setup[dev];
  // A context other than the one the address came from (the device was
  // reset, or no context is current on this thread yet) repeats the look-up.
  const bool by_ctx = ctx_get_current() != nullptr;
  if (!s.scratch || (by_ctx && current_context() != s.ctx)) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    DevSetup t;
    t.scratch = static_cast<unsigned char*>(p);
    t.ctx = by_ctx ? current_context() : nullptr;
    if ((e = cudaDeviceGetAttribute(&t.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&t.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) !=
            cudaSuccess ||
        (e = cudaDeviceGetAttribute(&t.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return m3g::host_fail(M3G_ECUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    s = t;
  }
  *out = s;
  return M3G_OK;
}

// token = the pick encoded in the key (0xFFFFFFFF when a bounded wait of
// the GEMV gave up); the key and status are cleared for the next call.
__global__ void k_greedy_finish(unsigned long long* key, uint32_t* status, uint32_t* token) {
  m3g::grid_dep_wait();
  const unsigned long long k = *key;
  const uint32_t pick = k ? 0xFFFFFFFFu - static_cast<uint32_t>(k) : 0u;
  *token = (*status & m3g::kStatusCopyTimeout) ? 0xFFFFFFFFu : pick;
  *key = 0ull;
  *status = 0u;
}

}  // namespace

extern "C" {

M3G_API int m3g_matvec_greedy_noalloc(const float* x, const uint8_t* raw, uint64_t raw_len, uint32_t dtype,
                                      uint64_t in_dim, uint64_t out_dim, uint32_t* token, void* stream) {
  if (!x || !raw || !token) return m3g::host_fail(M3G_EINVAL, "null argument");
  if (out_dim > kMaxRows)
    return m3g::host_fail(M3G_EINVAL, "out_dim %llu exceeds the no-alloc scratch (at most %llu rows)",
                          static_cast<unsigned long long>(out_dim), static_cast<unsigned long long>(kMaxRows));
  if (out_dim == 0 || in_dim == 0) return m3g::host_fail(M3G_ENONE, "zero dimension");
  DevSetup s;
  if (int rc = setup_current_device(&s)) return rc;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
  auto* key = reinterpret_cast<unsigned long long*>(s.scratch + kKeyOff);
  auto* status = reinterpret_cast<uint32_t*>(s.scratch + kStatusOff);
  auto* logits = reinterpret_cast<float*>(s.scratch + kLogitsOff);
  // The key is the only word that must start at zero; the logits are fully
  // overwritten.  Clearing it here also covers a call that failed midway.
  cudaError_t e = cudaMemsetAsync(key, 0, sizeof *key, st);
  if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  if (int rc = m3g::gemv_greedy_on(dtype, raw, raw_len, x, logits, static_cast<long long>(in_dim),
                                   static_cast<long long>(out_dim), st, s.sms, s.smem_per_sm, s.smem_optin, status,
                                   key))
    return rc;
  k_greedy_finish<<<1, 1, 0, st>>>(key, status, token);
  e = cudaGetLastError();
  if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "k_greedy_finish launch: %s", cudaGetErrorString(e));
  return M3G_OK;
}

}  // extern "C"
