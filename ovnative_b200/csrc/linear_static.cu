// linear_static.cu -- ovb_linear_static: fp32 activations in, quantised and
// multiplied like ovb_linear, but with no device memory from the caller.
//
// Why it exists.  ovb_linear needs a device workspace for the quantised
// activations (aq/asc) and leaves it to the caller to provide one.  Some
// callers cannot allocate device memory at the point where they run the
// layer:
//   - hosts that hand all device memory to their own pool or arena (engines
//     and plugins embedding the engine through its C ABI) and do not let a
//     library call cudaMalloc behind their back;
//   - latency-critical callers, such as a streaming TTS step, that must not
//     pay for cudaMalloc/cudaFree, which can synchronise the whole device;
//   - thin FFI bindings that can pass host or device pointers in but have no
//     way to own and later free a device buffer.
// For them the scratch lives in a fixed device array inside this library.
//
// Rules of use.
//   - Limit: M x K must fit kStaticScratchBytes (8 MiB) as laid out by
//     ovb_linear_workspace_bytes(M, K); e.g. M = 2048 rows at K = 3072, or
//     M = 6144 at K = 1024.  Larger calls are rejected with
//     OVB_ERR_INVALID_ARG -- use ovb_linear with a workspace instead.
//   - Every GPU that loads the library holds the 8 MiB array until the
//     process exits.
//   - One array per device, shared by every call on that device: calls whose
//     executions overlap on the GPU (different streams, or different host
//     threads, without ordering between them) race on it and give wrong
//     results.  Order them on one stream or with events.
//   - The array keeps the last call's contents.  Nothing needs clearing: the
//     quantiser writes every aq byte (tail padding included) and every scale
//     before the GEMM reads them.
//   - Arguments are checked before anything is enqueued: a rejected call
//     leaves the array (and any ordered call still reading it) untouched.
//   - The first call in a CUDA context looks up the array's device address
//     (cudaGetSymbolAddress, with that context current) and caches it under
//     the context's unique id.  A symbol's address belongs to a context, so a
//     host that binds its own driver-API context, or a process that calls
//     cudaDeviceReset and continues in a new context, gets a fresh lookup
//     rather than a stale address.  Make the first call in each context
//     before any CUDA stream capture in it.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/ovb200.h"
#include "ovb_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t{8} << 20;
constexpr int kCacheEntries = 64;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_linear_scratch[kStaticScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <class Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

// Unique id of the calling thread's current CUDA context (0 with none).
bool current_context_id(unsigned long long* id) {
  static const CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  *id = 0;
  if (!get_current || !get_id) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return false;
  if (!ctx) return true;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

struct CacheEntry {
  unsigned long long ctx_id;
  void* addr;
};
std::mutex g_scratch_mu;
CacheEntry g_cache[kCacheEntries] = {};
int g_cache_next = 0;

// Device address of g_linear_scratch in the current context (looked up once
// per context).  Returns OVB_OK or a status with ovb_last_error() set.
int scratch_address(void** out) {
  unsigned long long id = 0;
  if (!current_context_id(&id)) {
    ovb::set_error("ovb_linear_static: cannot identify the current CUDA context");
    return OVB_ERR_INTERNAL;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (id != 0)
    for (const CacheEntry& e : g_cache)
      if (e.ctx_id == id && e.addr) {
        *out = e.addr;
        return OVB_OK;
      }
  // With no context current yet, this lookup creates the device's primary
  // context; its id is read afterwards.
  void* p = nullptr;
  if (ovb::cuda_failed(cudaGetSymbolAddress(&p, g_linear_scratch),
                       "cudaGetSymbolAddress(static scratch)"))
    return OVB_ERR_INTERNAL;
  if (id == 0 && (!current_context_id(&id) || id == 0)) {
    ovb::set_error("ovb_linear_static: no CUDA context after the symbol lookup");
    return OVB_ERR_INTERNAL;
  }
  g_cache[g_cache_next] = {id, p};
  g_cache_next = (g_cache_next + 1) % kCacheEntries;
  *out = p;
  return OVB_OK;
}

int invalid(const char* msg) {
  ovb::set_error(msg);
  return OVB_ERR_INVALID_ARG;
}

}  // namespace

extern "C" int ovb_linear_static(int64_t M, const ovb_weight* w, const float* A, int64_t lda,
                                 float* C, int64_t ldc, int accumulate, void* stream) {
  if (M <= 0) return OVB_OK;
  // Every check comes before the first enqueue (see the rules above).
  if (!w) return invalid("weight handle is null");
  if (!A || !C) return invalid("A/C must be non-null");
  if (w->K <= 0 || w->N <= 0) return invalid("weight has no elements");
  if (lda < w->K) return invalid("lda < K");
  if (ldc < w->N) return invalid("ldc < N");
  // Bound M before any size arithmetic, so that a huge M cannot wrap the
  // byte count below the limit: a row needs 32 * Kb quantised bytes and
  // Kb fp32 scales.
  const int64_t kb = (w->K + 31) / 32;
  const int64_t max_rows = static_cast<int64_t>(kStaticScratchBytes / (36 * static_cast<size_t>(kb)));
  const size_t need = M <= max_rows ? ovb_linear_workspace_bytes(M, w->K) : 0;
  if (M > max_rows || need > kStaticScratchBytes) {
    char buf[240];
    std::snprintf(buf, sizeof buf,
                  "ovb_linear_static: M=%lld x K=%lld needs more than the %zu-byte static "
                  "scratch; use ovb_linear with a workspace",
                  static_cast<long long>(M), static_cast<long long>(w->K), kStaticScratchBytes);
    return invalid(buf);
  }
  void* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st != OVB_OK) return st;
  // Same layout as ovb_linear's workspace: aq, padded to 256 bytes, then asc.
  const size_t qb = static_cast<size_t>(ovb_quant_bytes(M, w->K));
  auto* aq = static_cast<int8_t*>(scratch);
  auto* asc = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + ((qb + 255) / 256) * 256);
  st = ovb_quantize(M, w->K, A, lda, aq, asc, 0, stream);
  if (st != OVB_OK) return st;
  return ovb_linear_q(M, w, aq, asc, C, ldc, accumulate, stream);
}
