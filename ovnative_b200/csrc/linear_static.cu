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
//   - The first call on a device looks up the array's device address (with
//     that device current) and caches it.  Make that first call before any
//     CUDA stream capture on the device.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/ovb200.h"
#include "ovb_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t{8} << 20;
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_linear_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_linear_scratch on the current device (looked up once
// per device).  Returns OVB_OK or a status with ovb_last_error() set.
int scratch_address(void** out) {
  int dev = 0;
  if (ovb::cuda_failed(cudaGetDevice(&dev), "cudaGetDevice")) return OVB_ERR_INTERNAL;
  if (dev < 0 || dev >= kMaxDevices) {
    ovb::set_error("ovb_linear_static: device index beyond the supported 64");
    return OVB_ERR_INTERNAL;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (ovb::cuda_failed(cudaGetSymbolAddress(&p, g_linear_scratch),
                         "cudaGetSymbolAddress(static scratch)"))
      return OVB_ERR_INTERNAL;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return OVB_OK;
}

}  // namespace

extern "C" int ovb_linear_static(int64_t M, const ovb_weight* w, const float* A, int64_t lda,
                                 float* C, int64_t ldc, int accumulate, void* stream) {
  if (M <= 0) return OVB_OK;
  if (!w) {
    ovb::set_error("weight handle is null");
    return OVB_ERR_INVALID_ARG;
  }
  const size_t need = ovb_linear_workspace_bytes(M, w->K);
  if (need > kStaticScratchBytes) {
    char buf[200];
    std::snprintf(buf, sizeof buf,
                  "ovb_linear_static: M=%lld x K=%lld needs %zu bytes of scratch, above the "
                  "%zu-byte static limit; use ovb_linear with a workspace",
                  static_cast<long long>(M), static_cast<long long>(w->K), need,
                  kStaticScratchBytes);
    ovb::set_error(buf);
    return OVB_ERR_INVALID_ARG;
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
