// quant.cu -- per-row, per-32-k activation quantisers for the int8 GEMM.
//
// Three producers, each writing asc (fp32 block scales) and aq in one of three
// forms (`mode`): int8 q (0), the reference's u8 q+128 (1, OVB_AQ_U8), or the
// dequantised activation fp16(q * asc) for the fp16 tensor-core mainloop (2,
// OVB_AQ_F16; aq is then [M, Kp] fp16).  A fourth form (3, OVB_AQ_F16_RAW)
// skips the quantisation: fp16 of the fp32 value itself, no asc, the input
// of fp32 linear weights (ovb_weight_create_f32).  q and asc are bit-identical to the
// reference CPU path:
//   quantize_kernel          quantize_a_u8          gemm.cpp:379-430
//   rmsnorm_quantize_kernel  rmsnorm_quantize_avx2  gemm.cpp:638-707
//   silu_mul_quantize_kernel silu_mul_quant_avx2    ops_cpu.cpp:144-198
//
// All three are HBM-bound (about 4-8 bytes read and ~1 byte written per
// element).  Every fp32 operation is an explicit round-to-nearest intrinsic so
// that nvcc can neither contract nor reorder anything; denormals are kept
// (no -ftz / fast-math on this file).
#include <cuda_fp16.h>

#include <climits>

#include "ovb_internal.h"
#include "ovb_ptx.cuh"
#include "ovb_quant.cuh"

namespace ovb {

// Status of the fp16 output form: bit 16 = a dequantised activation left the
// fp16 range (it would be stored as +-inf).  Reported by ovb_device_status.
__device__ int g_status_q;

namespace {

constexpr int kModeU8 = 1;
constexpr int kModeF16 = 2;
constexpr int kModeF16Raw = 3;  // fp16(a) itself, not quantised (asc not written)
constexpr int kErrF16Range = 16;
constexpr int kErrSelftest = 64;  // the wait self-test's deliberate timeout

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }

// fp16(q * scale) of 8 consecutive values (padding -> 0), packed in 16 bytes.
__device__ __forceinline__ uint4 dequant8_f16(const float (&v)[8], int nv, float inv,
                                              float scale) {
  uint32_t w[4];
  bool range_ok = true;
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    float d[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (i + j < nv) {
        int z = cvt_rne_x86(__fmul_rn(v[i + j], inv));
        z = z < -127 ? -127 : (z > 127 ? 127 : z);
        d[j] = __fmul_rn(static_cast<float>(z), scale);
        range_ok = range_ok && fabsf(d[j]) <= 65504.f;
      } else {
        d[j] = 0.f;
      }
    }
    const __half2 h = __floats2half2_rn(d[0], d[1]);
    w[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
  }
  if (!range_ok) atomicOr(&g_status_q, kErrF16Range);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// The same for 4 consecutive values (4 bytes of q, or 8 bytes of fp16).
template <int kMode>
__device__ __forceinline__ void store4(uint8_t* aq, int64_t idx, const float (&v)[4], int nv,
                                       float inv, float scale) {
  if constexpr (kMode == kModeF16Raw) {
    const __half2 h0 = __floats2half2_rn(nv > 0 ? v[0] : 0.f, nv > 1 ? v[1] : 0.f);
    const __half2 h1 = __floats2half2_rn(nv > 2 ? v[2] : 0.f, nv > 3 ? v[3] : 0.f);
    bool range_ok = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) range_ok = range_ok && !(i < nv && !(fabsf(v[i]) <= 65504.f));
    if (!range_ok) atomicOr(&g_status_q, kErrF16Range);
    *reinterpret_cast<uint2*>(aq + 2 * idx) = make_uint2(*reinterpret_cast<const uint32_t*>(&h0),
                                                         *reinterpret_cast<const uint32_t*>(&h1));
  } else if constexpr (kMode == kModeF16) {
    uint32_t w[2];
    bool range_ok = true;
#pragma unroll
    for (int i = 0; i < 4; i += 2) {
      float d[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (i + j < nv) {
          int z = cvt_rne_x86(__fmul_rn(v[i + j], inv));
          z = z < -127 ? -127 : (z > 127 ? 127 : z);
          d[j] = __fmul_rn(static_cast<float>(z), scale);
          range_ok = range_ok && fabsf(d[j]) <= 65504.f;
        } else {
          d[j] = 0.f;
        }
      }
      const __half2 h = __floats2half2_rn(d[0], d[1]);
      w[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
    }
    if (!range_ok) atomicOr(&g_status_q, kErrF16Range);
    *reinterpret_cast<uint2*>(aq + 2 * idx) = make_uint2(w[0], w[1]);
  } else {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      word |= ((i < nv) ? quant_byte(v[i], inv, kMode == kModeU8) : 0u) << (8 * i);
    *reinterpret_cast<uint32_t*>(aq + idx) = word;
  }
}

// Write the 8 quantised values of element k of a row in the chosen form.
template <int kMode>
__device__ __forceinline__ void store8(uint8_t* aq, int64_t idx, const float (&v)[8], int nv,
                                       float inv, float scale) {
  if constexpr (kMode == kModeF16Raw) {
    const float lo[4] = {v[0], v[1], v[2], v[3]};
    const float hi[4] = {v[4], v[5], v[6], v[7]};
    store4<kModeF16Raw>(aq, idx, lo, nv < 4 ? nv : 4, inv, scale);
    store4<kModeF16Raw>(aq, idx + 4, hi, nv > 4 ? nv - 4 : 0, inv, scale);
  } else if constexpr (kMode == kModeF16)
    *reinterpret_cast<uint4*>(aq + 2 * idx) = dequant8_f16(v, nv, inv, scale);
  else
    *reinterpret_cast<uint2*>(aq + idx) = quant8(v, nv, inv, kMode == kModeU8);
}

// Load 8 floats starting at p, the first nv of them valid (others 0).
__device__ __forceinline__ void load8(const float* p, int nv, bool vec_ok, float (&v)[8]) {
  if (nv == 8 && vec_ok) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (i < nv) ? __ldg(p + i) : 0.f;
  }
}

// ------------------------------------------------------------ quantize
// Four threads per 32-k block (8 values each); the block absmax is reduced
// over the four with shuffles (max is order-independent, so this equals the
// reference's 8-lane max followed by a scalar tail).
template <int kMode>
__global__ void __launch_bounds__(256) quantize_kernel(int64_t M, int64_t K, const float* A,
                                                       int64_t lda, uint8_t* aq, float* asc) {
  pdl_wait();  // the producer of this kernel's input is complete
  pdl_launch_dependents();
  const int64_t Kb = (K + 31) / 32, Kp = Kb * 32;
  const int64_t total = M * Kb * 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int lane = threadIdx.x & 31;
  const bool vec_ok = ((lda & 3) == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t - lane < total;
       t += stride) {
    const bool valid = t < total;
    const int64_t task = valid ? t >> 2 : 0;
    const int sub = static_cast<int>(t & 3);
    const int64_t row = task / Kb, b = task - row * Kb;
    const int64_t k = b * 32 + sub * 8;
    const int nv = valid ? static_cast<int>(imax64(0, imin64(8, K - k))) : 0;
    float v[8];
    load8(A + row * lda + k, nv, vec_ok, v);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    float scale, inv;
    block_scales(amax, &scale, &inv);
    if (valid) {
      store8<kMode>(aq, row * Kp + k, v, nv, inv, scale);
      if (kMode != kModeF16Raw && sub == 0) asc[row * Kb + b] = scale;
    }
  }
}

// Copy n floats from global src to shared dst with `threads` threads (this
// one is `tid`): 16-byte loads when aligned, eight loads in flight per thread
// before their stores.
__device__ __forceinline__ void stage_row(const float* __restrict__ src, int64_t n, float* dst,
                                          int tid, int threads) {
  const bool vec = ((n & 3) == 0) && ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
  if (vec) {
    const int64_t n4 = n / 4;
    for (int64_t i0 = tid; i0 < n4; i0 += 8 * static_cast<int64_t>(threads)) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t i = i0 + u * static_cast<int64_t>(threads);
        v[u] = i < n4 ? __ldg(reinterpret_cast<const float4*>(src) + i) : make_float4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t i = i0 + u * static_cast<int64_t>(threads);
        if (i < n4) reinterpret_cast<float4*>(dst)[i] = v[u];
      }
    }
  } else {
    for (int64_t i0 = tid; i0 < n; i0 += 8 * static_cast<int64_t>(threads)) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t i = i0 + u * static_cast<int64_t>(threads);
        v[u] = i < n ? __ldg(src + i) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t i = i0 + u * static_cast<int64_t>(threads);
        if (i < n) dst[i] = v[u];
      }
    }
  }
}

// ---------------------------------------------------- rmsnorm + quantize
// One warp per row.  The row is staged in shared memory with coalesced
// float4 loads; lanes 0..7 then run the reference's eight sequential FMA
// chains (lane l: elements l, l+8, ...; gemm.cpp:655-658), every lane sums
// the eight partials left to right plus the cols%8 tail (:661-663) and forms
// scale = 1/sqrt(sum/cols + eps) (:664).  The warp then quantises
// (x*scale)*w (:672-704) four 32-k blocks at a time: eight lanes per block,
// four consecutive elements per lane (one 16-byte shared-memory and gain
// load each), the block absmax reduced over the eight lanes with shuffles
// (max is order-independent, so this equals the reference's).
template <int kMode>
__global__ void __launch_bounds__(256) rmsnorm_quantize_kernel(int64_t rows, int64_t cols,
                                                               const float* x, const float* w,
                                                               float eps, uint8_t* aq,
                                                               float* asc) {
  pdl_wait();  // the producer of this kernel's input is complete
  pdl_launch_dependents();
  extern __shared__ float srow_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  float* srow = srow_all + static_cast<int64_t>(warp) * cols;
  // The gain vector, staged once per block (after the rows' slots).  Loads
  // are issued in batches of 8 before their stores so their latencies overlap.
  float* sw = srow_all + static_cast<int64_t>(warps) * cols;
  stage_row(w, cols, sw, threadIdx.x, blockDim.x);
  __syncthreads();
  const int64_t Kb = (cols + 31) / 32, Kp = Kb * 32;
  const bool vec_ok = ((cols & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * warps + warp; r < rows;
       r += static_cast<int64_t>(gridDim.x) * warps) {
    stage_row(x + r * cols, cols, srow, lane, 32);
    __syncwarp();
    const int64_t nvec = cols / 8;
    float acc = 0.f;
    if (lane < 8)
#pragma unroll 8
      for (int64_t j = 0; j < nvec; ++j) {
        const float v = srow[j * 8 + lane];
        acc = __fmaf_rn(v, v, acc);
      }
    float sum = __shfl_sync(0xffffffffu, acc, 0);
#pragma unroll
    for (int l = 1; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, acc, l));
    for (int64_t i = nvec * 8; i < cols; ++i) sum = __fadd_rn(sum, __fmul_rn(srow[i], srow[i]));
    const float scale =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(cols)), eps)));
    const int sub = lane & 7;  // this lane's quarter-of-a-quarter of the block
#pragma unroll 2
    for (int64_t b0 = 0; b0 < Kb; b0 += 4) {
      const int64_t b = b0 + (lane >> 3);
      const int64_t k = b * 32 + sub * 4;
      const int nv = b < Kb ? static_cast<int>(imax64(0, imin64(4, cols - k))) : 0;
      float xv[4], wv[4];
      if (nv == 4 && vec_ok) {
        const float4 a = *reinterpret_cast<const float4*>(srow + k);
        const float4 c = *reinterpret_cast<const float4*>(sw + k);
        xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
        wv[0] = c.x; wv[1] = c.y; wv[2] = c.z; wv[3] = c.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xv[i] = i < nv ? srow[k + i] : 0.f;
          wv[i] = i < nv ? sw[k + i] : 0.f;
        }
      }
      float v[4];
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[i] = (i < nv) ? __fmul_rn(__fmul_rn(xv[i], scale), wv[i]) : 0.f;
        amax = fmaxf(amax, fabsf(v[i]));
      }
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      float bs, inv;
      block_scales(amax, &bs, &inv);
      if (b < Kb) {
        if (kMode != kModeF16Raw && sub == 0) asc[r * Kb + b] = bs;
        store4<kMode>(aq, r * Kp + k, v, nv, inv, bs);
      }
    }
    __syncwarp();
  }
}

// The same for rows of at most 1024 elements (cols % 4 == 0, 16-byte aligned
// x and w) -- the LM's hidden size -- with one 128-thread block (4 warps) per
// row, so that the quantisation, serial within a warp, is spread over four:
// all threads stage the row in shared memory; lanes 0..7 of warp 0 run the
// reference-ordered sum of squares and publish the scale; then warp q
// quantises the groups i = 2q, 2q+1 (128 elements each: eight lanes per
// 32-k block, four elements per lane, as in the general kernel).
constexpr int kSmallCols = 1024;
constexpr int kSmallThreads = 128;

template <int kMode>
__global__ void __launch_bounds__(kSmallThreads) rmsnorm_quantize_small_kernel(
    int64_t rows, int64_t cols, const float* x, const float* w, float eps, uint8_t* aq,
    float* asc) {
  pdl_wait();  // the producer of this kernel's input is complete
  pdl_launch_dependents();
  __shared__ __align__(16) float srow[kSmallCols];
  __shared__ float s_scale;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t Kb = (cols + 31) / 32, Kp = Kb * 32;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = x + r * cols;
    // Each thread's two float4 of the row (positions 128*i + 4*lane of its
    // warp's groups), kept in registers for the quantisation.
    float4 xr[2], wr[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t k = 128 * (2 * warp + u) + 4 * lane;
      xr[u] = k < cols ? __ldg(reinterpret_cast<const float4*>(row + k)) : make_float4(0, 0, 0, 0);
      wr[u] = k < cols ? __ldg(reinterpret_cast<const float4*>(w + k)) : make_float4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t k = 128 * (2 * warp + u) + 4 * lane;
      if (k < cols) *reinterpret_cast<float4*>(srow + k) = xr[u];
    }
    __syncthreads();
    if (warp == 0) {
      const int64_t nvec = cols / 8;
      float acc = 0.f;
      if (lane < 8) {
        for (int64_t j0 = 0; j0 < nvec; j0 += 16) {
          float t[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) t[u] = j0 + u < nvec ? srow[(j0 + u) * 8 + lane] : 0.f;
#pragma unroll
          for (int u = 0; u < 16; ++u)
            if (j0 + u < nvec) acc = __fmaf_rn(t[u], t[u], acc);
        }
      }
      float sum = __shfl_sync(0xffffffffu, acc, 0);
#pragma unroll
      for (int l = 1; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, acc, l));
      for (int64_t i = nvec * 8; i < cols; ++i) sum = __fadd_rn(sum, __fmul_rn(srow[i], srow[i]));
      if (lane == 0)
        s_scale =
            __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(cols)), eps)));
    }
    __syncthreads();
    const float scale = s_scale;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = 2 * warp + u;
      const int64_t b = 4 * i + (lane >> 3);
      const int64_t k = 128 * i + 4 * lane;
      const int nv = k < cols ? 4 : 0;  // cols % 4 == 0
      const float xv[4] = {xr[u].x, xr[u].y, xr[u].z, xr[u].w};
      const float wv[4] = {wr[u].x, wr[u].y, wr[u].z, wr[u].w};
      float v[4];
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = (j < nv) ? __fmul_rn(__fmul_rn(xv[j], scale), wv[j]) : 0.f;
        amax = fmaxf(amax, fabsf(v[j]));
      }
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      float bs, inv;
      block_scales(amax, &bs, &inv);
      if (b < Kb) {
        if (kMode != kModeF16Raw && (lane & 7) == 0) asc[r * Kb + b] = bs;
        store4<kMode>(aq, r * Kp + k, v, nv, inv, bs);
      }
    }
    __syncthreads();  // srow and s_scale are reused by the next row
  }
}

// ------------------------------------ rmsnorm + quantize, rows in batches
// For many rows of at most 1024 columns (cols % 32 == 0, 16-byte aligned x
// and w): each warp takes four rows at a time.  The rows are staged in shared
// memory (16-byte chunks XOR-swizzled by their 8-chunk group, and each row
// slot padded by one chunk, so that both access patterns below are free of
// bank conflicts); lanes 8g .. 8g + 7 run row g's eight reference-ordered
// FMA chains (gemm.cpp:655-663) and every lane of the group forms the row's
// scale; then, row by row, lane b quantises 32-k block b on its own: the
// block scale's two IEEE divisions run once per block instead of once per
// eight lanes, and the rounding uses the exact identity
//   rne(y) = fl(y + 1.5 * 2^23) - 1.5 * 2^23   for |y| < 2^22
// (|v * inv| <= 127 (1 + 2^-23) inside a finite block), so the bytes equal
// quantize_a_u8's; a block holding a NaN or an infinity takes the
// x86-conversion path of the other kernels.
constexpr int kRows4 = 4;      // rows per warp
constexpr int kRows4Warps = 4;  // warps per block

__device__ __forceinline__ int swz4(int c) { return c ^ ((c >> 3) & 7); }

// 16-byte asynchronous copy global -> shared (through L2 only), and the wait
// for all of this thread's copies.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// max(m, |a|, |b|) in one instruction, NaN if any input is NaN.
__device__ __forceinline__ float fmax3_nan_abs(float m, float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return r;
}

// Packed f32x2 multiply (each lane an IEEE round-to-nearest product):
// (r0, r1) = (a0 * b0, a1 * b1).
__device__ __forceinline__ void mul2(float a0, float a1, float b0, float b1, float& r0, float& r1) {
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "mul.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

template <int kMode>
__global__ void __launch_bounds__(kRows4Warps * 32) rmsnorm_quantize_rows4_kernel(
    int64_t rows, int cols, const float* x, const float* w, float eps, uint8_t* aq, float* asc) {
  pdl_wait();  // the producer of this kernel's input is complete
  pdl_launch_dependents();
  extern __shared__ float4 sm4[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = cols / 4, rstride = nch + 1, Kb = cols / 32;
  float4* sw = sm4;
  float4* srows = sm4 + nch + warp * kRows4 * rstride;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int c = threadIdx.x; c < nch; c += blockDim.x) sw[swz4(c)] = __ldg(w4 + c);
  __syncthreads();
  const int64_t step = static_cast<int64_t>(gridDim.x) * kRows4Warps * kRows4;
  for (int64_t r0 = (static_cast<int64_t>(blockIdx.x) * kRows4Warps + warp) * kRows4; r0 < rows;
       r0 += step) {
    const int nr = static_cast<int>(imin64(kRows4, rows - r0));
    // ---- stage the rows: asynchronous 16-byte copies global -> shared
    // (coalesced, all four rows' in flight at once, no registers)
#pragma unroll
    for (int g = 0; g < kRows4; ++g) {
      if (g < nr) {
        const float4* xr = reinterpret_cast<const float4*>(x + (r0 + g) * cols);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int c = lane + 32 * k;
          if (c < nch) cp_async16(srows + g * rstride + swz4(c), xr + c);
        }
      }
    }
    cp_async_wait_all();
    __syncwarp();
    // ---- sum of squares in the reference's order: lane 8g + q, chain q of row g
    const int g = lane >> 3, q = lane & 7;
    float acc = 0.f;
    if (g < nr) {
      const float* rowf = reinterpret_cast<const float*>(srows + g * rstride);
#pragma unroll 8
      for (int i = 0; i < cols / 8; ++i) {
        const int f = 8 * i + q;
        const float v = rowf[swz4(f >> 2) * 4 + (f & 3)];
        acc = __fmaf_rn(v, v, acc);
      }
    }
    float sum = __shfl_sync(0xffffffffu, acc, 8 * g);
#pragma unroll
    for (int l = 1; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, acc, 8 * g + l));
    const float rscale =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(cols)), eps)));
    // ---- quantise: lane b takes 32-k block b of each row in turn
    for (int gg = 0; gg < nr; ++gg) {
      const float s = __shfl_sync(0xffffffffu, rscale, 8 * gg);
      if (lane < Kb) {
        const int64_t row = r0 + gg;
        float v[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // chunk j of block `lane`: the swizzle puts lanes 0-7 (one
          // quarter-warp phase) in distinct bank groups
          const int c = lane * 8 + j;
          const float4 a = srows[gg * rstride + swz4(c)];
          const float4 b = sw[swz4(c)];
          const int o = j * 4;
          // (x * s) * w, two elements per packed multiply
          float t0, t1, t2, t3;
          mul2(a.x, a.y, s, s, t0, t1);
          mul2(a.z, a.w, s, s, t2, t3);
          mul2(t0, t1, b.x, b.y, v[o], v[o + 1]);
          mul2(t2, t3, b.z, b.w, v[o + 2], v[o + 3]);
        }
        uint8_t* out = aq + (row * Kb + lane) * 32 * (kMode >= kModeF16 ? 2 : 1);
        if constexpr (kMode == kModeF16Raw) {
          bool range_ok = true;
          uint32_t hw[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            range_ok = range_ok && fabsf(v[2 * i]) <= 65504.f && fabsf(v[2 * i + 1]) <= 65504.f;
            const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            hw[i] = *reinterpret_cast<const uint32_t*>(&h);
          }
          if (!range_ok) atomicOr(&g_status_q, kErrF16Range);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<uint4*>(out)[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2],
                                                          hw[4 * i + 3]);
        } else {
          // the block maximum, NaN if the block holds one (two chains of
          // 3-input maxima); for a finite block it is the reference's amax
          float an0 = 0.f, an1 = 0.f;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            an0 = fmax3_nan_abs(an0, v[i], v[i + 1]);
            an1 = fmax3_nan_abs(an1, v[i + 2], v[i + 3]);
          }
          const float anan = fmax_nan(an0, an1);
          if (!(anan <= 3.402823466e38f)) {  // a NaN or an infinity: the x86 conversion path
            bool bad = false;
            asc[row * Kb + lane] = quant_block32(v, out, kMode, &bad);
            if (bad) atomicOr(&g_status_q, kErrF16Range);
            continue;
          }
          const float amax = anan;
          float bs, inv;
          block_scales(amax, &bs, &inv);
          asc[row * Kb + lane] = bs;
          if constexpr (kMode == kModeF16) {
            constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
            uint32_t hw[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              // rne(v * inv) * bs; the rounding steps stay scalar (a packed
              // multiply followed by a packed add can be contracted into one
              // fused multiply-add, which changes the rounding), the final
              // products are packed
              const float z0 =
                  __fsub_rn(__fadd_rn(__fmul_rn(v[2 * i], inv), kMagic), kMagic);
              const float z1 =
                  __fsub_rn(__fadd_rn(__fmul_rn(v[2 * i + 1], inv), kMagic), kMagic);
              float d0, d1;
              mul2(z0, z1, bs, bs, d0, d1);
              const __half2 h = __floats2half2_rn(d0, d1);
              hw[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
            // the largest |q * asc| is 127 * asc (the block's maximum maps to 127)
            if (amax > 0.f && __fmul_rn(127.f, bs) > 65504.f) atomicOr(&g_status_q, kErrF16Range);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<uint4*>(out)[i] = make_uint4(hw[4 * i], hw[4 * i + 1],
                                                            hw[4 * i + 2], hw[4 * i + 3]);
          } else {
            constexpr float kMagic = 12582912.0f;
            uint32_t wq[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              uint32_t word = 0;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int z = __float_as_int(__fadd_rn(__fmul_rn(v[4 * i + e], inv), kMagic)) -
                              0x4B400000;
                const uint32_t byte =
                    kMode == kModeU8 ? static_cast<uint32_t>(z + 128) : static_cast<uint32_t>(z & 0xFF);
                word |= byte << (8 * e);
              }
              wq[i] = word;
            }
            reinterpret_cast<uint4*>(out)[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
            reinterpret_cast<uint4*>(out)[1] = make_uint4(wq[4], wq[5], wq[6], wq[7]);
          }
        }
      }
    }
    __syncwarp();  // the row slots are reused by the next rows
  }
}

// ------------------------------------------------- silu(gate)*up + quantize
template <int kMode>
__global__ void __launch_bounds__(256) silu_mul_quantize_kernel(int64_t M, int64_t K,
                                                                const float* gate, int64_t ldg,
                                                                const float* up, int64_t ldu,
                                                                uint8_t* aq, float* asc) {
  pdl_wait();  // the producer of this kernel's input is complete
  pdl_launch_dependents();
  const int64_t Kb = (K + 31) / 32, Kp = Kb * 32;
  const int64_t total = M * Kb * 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int lane = threadIdx.x & 31;
  const bool vg = ((ldg & 3) == 0) && ((reinterpret_cast<uintptr_t>(gate) & 15) == 0);
  const bool vu = ((ldu & 3) == 0) && ((reinterpret_cast<uintptr_t>(up) & 15) == 0);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t - lane < total;
       t += stride) {
    const bool valid = t < total;
    const int64_t task = valid ? t >> 2 : 0;
    const int sub = static_cast<int>(t & 3);
    const int64_t row = task / Kb, b = task - row * Kb;
    const int64_t k = b * 32 + sub * 8;
    const int nv = valid ? static_cast<int>(imax64(0, imin64(8, K - k))) : 0;
    const int kn = static_cast<int>(imin64(32, K - b * 32));
    // This thread's 8 values are in the block's vector body when they form a
    // whole group of 8 inside the block (ops_cpu.cpp:163-165).
    const bool body = (sub * 8 + 8) <= kn;
    float g[8], u[8], v[8];
    load8(gate + row * ldg + k, nv, vg, g);
    load8(up + row * ldu + k, nv, vu, u);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[i] = (i < nv) ? (body ? silu_up_vec(g[i], u[i]) : silu_up_tail(g[i], u[i])) : 0.f;
      amax = fmaxf(amax, fabsf(v[i]));
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    float scale, inv;
    block_scales(amax, &scale, &inv);
    if (valid) {
      store8<kMode>(aq, row * Kp + k, v, nv, inv, scale);
      if (kMode != kModeF16Raw && sub == 0) asc[row * Kb + b] = scale;
    }
  }
}

int grid_for(int64_t threads_needed) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t blocks = (threads_needed + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms(dev)) * 8;
  return static_cast<int>(imax64(1, imin64(blocks, cap)));
}

}  // namespace

cudaError_t launch_quantize(int64_t M, int64_t K, const float* A, int64_t lda, void* aq,
                            float* asc, int mode, cudaStream_t s) {
  const int64_t Kb = (K + 31) / 32;
  const dim3 grid(grid_for(M * Kb * 4));
  auto* q8 = static_cast<uint8_t*>(aq);
  switch (mode) {
    case 0: return launch_plain(quantize_kernel<0>, grid, dim3(256), 0, s, M, K, A, lda, q8, asc);
    case 1: return launch_plain(quantize_kernel<1>, grid, dim3(256), 0, s, M, K, A, lda, q8, asc);
    case 3: return launch_plain(quantize_kernel<3>, grid, dim3(256), 0, s, M, K, A, lda, q8, asc);
    default: return launch_plain(quantize_kernel<2>, grid, dim3(256), 0, s, M, K, A, lda, q8, asc);
  }
}

cudaError_t launch_rmsnorm_quantize(int64_t rows, int64_t cols, const float* x, const float* w,
                                    float eps, void* aq, float* asc, int mode, cudaStream_t s) {
  // One warp per row; shared memory holds one row per warp.  Fewer warps per
  // block when there are few rows, so that the rows spread over all SMs.
  const int64_t row_bytes = cols * 4;
  int dev0 = 0;
  cudaGetDevice(&dev0);
  const int64_t per_block = imax64(1, rows / (2 * static_cast<int64_t>(num_sms(dev0))));
  int warps = static_cast<int>(imin64(imin64(8, per_block), imax64(1, (96 * 1024) / row_bytes)));
  const size_t smem = static_cast<size_t>(warps + 1) * row_bytes;  // rows + the gain vector
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    for (auto* k : {rmsnorm_quantize_kernel<0>, rmsnorm_quantize_kernel<1>,
                    rmsnorm_quantize_kernel<2>, rmsnorm_quantize_kernel<3>}) {
      cudaError_t e =
          cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (e != cudaSuccess) return e;
    }
    configured_dev = dev;
  }
  const int64_t blocks = (rows + warps - 1) / warps;
  const int grid = static_cast<int>(imin64(blocks, static_cast<int64_t>(num_sms(dev)) * 16));
  // The block-per-row kernel spreads one row over four warps, which suits a
  // few hundred rows; with many rows the warp-per-row kernel keeps four times
  // as many rows (and their loads) in flight per SM.  Both follow the
  // reference's order and write the same bytes.
  const bool small = cols <= kSmallCols && (cols & 3) == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                     rows <= static_cast<int64_t>(num_sms(dev)) * 8;
  const bool batched = cols <= kSmallCols && (cols & 31) == 0 &&
                       (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                       rows > static_cast<int64_t>(num_sms(dev)) * 8;
  if (batched) {
    static thread_local int configured_dev4 = -1;
    const size_t smem4 = static_cast<size_t>(cols / 4 + kRows4Warps * kRows4 * (cols / 4 + 1)) * 16;
    if (configured_dev4 != dev) {
      for (auto* k : {rmsnorm_quantize_rows4_kernel<0>, rmsnorm_quantize_rows4_kernel<1>,
                      rmsnorm_quantize_rows4_kernel<2>, rmsnorm_quantize_rows4_kernel<3>}) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem4));
        if (e != cudaSuccess) return e;
      }
      configured_dev4 = dev;
    }
    const int64_t per_block = kRows4Warps * kRows4;
    const int g4 = static_cast<int>(imin64((rows + per_block - 1) / per_block,
                                           static_cast<int64_t>(num_sms(dev)) * 3));
    auto* q8b = static_cast<uint8_t*>(aq);
    const int c = static_cast<int>(cols);
    switch (mode) {
      case 0: return launch_plain(rmsnorm_quantize_rows4_kernel<0>, dim3(g4), dim3(kRows4Warps * 32),
                                smem4, s, rows, c, x, w, eps, q8b, asc);
      case 1: return launch_plain(rmsnorm_quantize_rows4_kernel<1>, dim3(g4), dim3(kRows4Warps * 32),
                                smem4, s, rows, c, x, w, eps, q8b, asc);
      case 3: return launch_plain(rmsnorm_quantize_rows4_kernel<3>, dim3(g4), dim3(kRows4Warps * 32),
                                smem4, s, rows, c, x, w, eps, q8b, asc);
      default: return launch_plain(rmsnorm_quantize_rows4_kernel<2>, dim3(g4),
                                 dim3(kRows4Warps * 32), smem4, s, rows, c, x, w, eps, q8b, asc);
    }
  }
  if (small) {
    const int sgrid = static_cast<int>(imin64(rows, static_cast<int64_t>(num_sms(dev)) * 16));
    auto* q8s = static_cast<uint8_t*>(aq);
    switch (mode) {
      case 0: return launch_plain(rmsnorm_quantize_small_kernel<0>, dim3(sgrid), dim3(kSmallThreads),
                                0, s, rows, cols, x, w, eps, q8s, asc);
      case 1: return launch_plain(rmsnorm_quantize_small_kernel<1>, dim3(sgrid), dim3(kSmallThreads),
                                0, s, rows, cols, x, w, eps, q8s, asc);
      case 3: return launch_plain(rmsnorm_quantize_small_kernel<3>, dim3(sgrid), dim3(kSmallThreads),
                                0, s, rows, cols, x, w, eps, q8s, asc);
      default: return launch_plain(rmsnorm_quantize_small_kernel<2>, dim3(sgrid),
                                 dim3(kSmallThreads), 0, s, rows, cols, x, w, eps, q8s, asc);
    }
  }
  auto* q8 = static_cast<uint8_t*>(aq);
  switch (mode) {
    case 0: return launch_plain(rmsnorm_quantize_kernel<0>, dim3(grid), dim3(warps * 32), smem, s,
                              rows, cols, x, w, eps, q8, asc);
    case 1: return launch_plain(rmsnorm_quantize_kernel<1>, dim3(grid), dim3(warps * 32), smem, s,
                              rows, cols, x, w, eps, q8, asc);
    case 3: return launch_plain(rmsnorm_quantize_kernel<3>, dim3(grid), dim3(warps * 32), smem, s,
                              rows, cols, x, w, eps, q8, asc);
    default: return launch_plain(rmsnorm_quantize_kernel<2>, dim3(grid), dim3(warps * 32), smem, s,
                               rows, cols, x, w, eps, q8, asc);
  }
}

cudaError_t launch_silu_mul_quantize(int64_t M, int64_t K, const float* gate, int64_t ldg,
                                     const float* up, int64_t ldu, void* aq, float* asc, int mode,
                                     cudaStream_t s) {
  const int64_t Kb = (K + 31) / 32;
  const dim3 grid(grid_for(M * Kb * 4));
  auto* q8 = static_cast<uint8_t*>(aq);
  switch (mode) {
    case 0: return launch_plain(silu_mul_quantize_kernel<0>, grid, dim3(256), 0, s, M, K, gate, ldg,
                              up, ldu, q8, asc);
    case 1: return launch_plain(silu_mul_quantize_kernel<1>, grid, dim3(256), 0, s, M, K, gate, ldg,
                              up, ldu, q8, asc);
    case 3: return launch_plain(silu_mul_quantize_kernel<3>, grid, dim3(256), 0, s, M, K, gate, ldg,
                              up, ldu, q8, asc);
    default: return launch_plain(silu_mul_quantize_kernel<2>, grid, dim3(256), 0, s, M, K, gate, ldg,
                               up, ldu, q8, asc);
  }
}

namespace {
// One mbarrier that nothing ever arrives on, waited on with the kernels'
// bounded wait (ovb_wait): the wait gives up at its limit (~1 s at the SM
// clock), thread 0 records kErrSelftest, and the kernel ends normally.
__global__ void wait_selftest_kernel() {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  volatile int never = 0;
  const bool got = ovb_wait(smem_u32(&bar), 0u, &never);
  if (!got && threadIdx.x == 0) atomicOr(&g_status_q, kErrSelftest);
}
}  // namespace

cudaError_t launch_wait_selftest(cudaStream_t s) {
  return launch_plain(wait_selftest_kernel, dim3(1), dim3(32), 0, s);
}

cudaError_t read_and_clear_status_q(int* out, cudaStream_t s) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_status_q, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_status_q, &zero, sizeof(int));
}

}  // namespace ovb
