// weights.cu -- load-time packers from the two OVW1 int8 layouts into the
// device layout the GEMM reads: [N, Kp] int8, K-major (one output channel per
// row, Kp = 32*ceil(K/32), zero tail bytes).  With this layout one 32-k
// quantisation block of 128 output channels is a (32 B x 128 rows) TMA box,
// i.e. exactly the B operand of one tcgen05 kind::i8 MMA (K = 32).
//
// Replaces s8_nk_pack (gemm.cpp:584-621, VNNI 4x8 tiles + wsum) and the CUDA
// runner's dequantise-at-load (cuda_lm.cu:228-238, :840-873).  No wsum is
// needed: the GEMM multiplies signed q by signed w directly, so there is no
// +128 zero point to remove.
#include <cuda_fp16.h>

#include "ovb_internal.h"

namespace ovb {
namespace {

// [N, K] -> [N, Kp]: one thread per 16 output bytes.
__global__ void pack_nk_kernel(const int8_t* __restrict__ src, int64_t N, int64_t K,
                               int8_t* __restrict__ dst, int64_t Kp) {
  const int64_t chunks = Kp / 16;
  const int64_t total = N * chunks;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = t / chunks, k0 = (t - n * chunks) * 16;
    uint32_t word[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int64_t k = k0 + i;
      const uint32_t b = (k < K) ? static_cast<uint8_t>(src[n * K + k]) : 0u;
      word[i >> 2] |= b << (8 * (i & 3));
    }
    *reinterpret_cast<uint4*>(dst + n * Kp + k0) = make_uint4(word[0], word[1], word[2], word[3]);
  }
}

// [K, N] -> [N, Kp]: 32x32 transpose through shared memory.
__global__ void pack_kn_kernel(const int8_t* __restrict__ src, int64_t N, int64_t K,
                               int8_t* __restrict__ dst, int64_t Kp) {
  __shared__ int8_t tile[32][33];
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int64_t k = k0 + i, n = n0 + tx;
    tile[i][tx] = (k < K && n < N) ? src[k * N + n] : static_cast<int8_t>(0);
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int64_t n = n0 + i, k = k0 + tx;
    if (n < N && k < Kp) dst[n * Kp + k] = tile[tx][i];
  }
}

// int8 -> fp16 bit patterns, 16 values per thread (n is a multiple of 16:
// rows of Kp = 32 * Kb bytes).  Integers |v| <= 2048 are exact in fp16.
__global__ void widen_f16_kernel(const int8_t* __restrict__ src, int64_t n16,
                                 uint16_t* __restrict__ dst) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int4 v = reinterpret_cast<const int4*>(src)[i];
    const int8_t* b = reinterpret_cast<const int8_t*>(&v);
    uint16_t h[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) h[j] = __half_as_ushort(__short2half_rn(b[j]));
    reinterpret_cast<int4*>(dst)[2 * i] = *reinterpret_cast<const int4*>(&h[0]);
    reinterpret_cast<int4*>(dst)[2 * i + 1] = *reinterpret_cast<const int4*>(&h[8]);
  }
}

}  // namespace

cudaError_t launch_widen_f16(const int8_t* src, int64_t n, uint16_t* dst, cudaStream_t s) {
  if (n % 16 != 0) return cudaErrorInvalidValue;
  const int64_t n16 = n / 16;
  const int grid = static_cast<int>(std::min<int64_t>((n16 + 255) / 256, 4096));
  widen_f16_kernel<<<grid, 256, 0, s>>>(src, n16, dst);
  return cudaGetLastError();
}

cudaError_t launch_pack_nk(const int8_t* src, int64_t N, int64_t K, int8_t* dst, int64_t Kp,
                           cudaStream_t s) {
  const int64_t total = N * (Kp / 16);
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, 65535));
  pack_nk_kernel<<<grid, 256, 0, s>>>(src, N, K, dst, Kp);
  return cudaGetLastError();
}

cudaError_t launch_pack_kn(const int8_t* src, int64_t N, int64_t K, int8_t* dst, int64_t Kp,
                           cudaStream_t s) {
  // Kp/32 k-tiles cover the zero tail as well.
  const dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>(Kp / 32));
  pack_kn_kernel<<<grid, dim3(32, 8), 0, s>>>(src, N, K, dst, Kp);
  return cudaGetLastError();
}

}  // namespace ovb
