// ovb_quant.cuh -- the reference's activation-quantiser and SiLU arithmetic
// as device functions, shared by the quantiser kernels (quant.cu) and the
// GEMM epilogues that quantise their own output (gate|up + SiLU*up).  Every
// fp32 operation is an explicit round-to-nearest intrinsic so nvcc can
// neither contract nor reorder anything.
#pragma once

#include <cuda_fp16.h>

#include <climits>
#include <cstdint>

namespace ovb {

// _mm256_cvtps_epi32 under the default MXCSR: round to nearest even, and
// 0x80000000 ("integer indefinite") for NaN or values outside int32.
__device__ __forceinline__ int cvt_rne_x86(float v) {
  if (!(v == v) || v >= 2147483648.0f || v < -2147483648.0f) return INT_MIN;
  return __float2int_rn(v);
}

__device__ __forceinline__ uint32_t quant_byte(float v, float inv, bool u8) {
  int z = cvt_rne_x86(__fmul_rn(v, inv));
  z = z < -127 ? -127 : (z > 127 ? 127 : z);
  return u8 ? static_cast<uint32_t>(z + 128) : static_cast<uint32_t>(z & 0xFF);
}

// Block scale and its reciprocal exactly as gemm.cpp:407-408.
__device__ __forceinline__ void block_scales(float amax, float* scale, float* inv) {
  *scale = __fdiv_rn(amax, 127.0f);
  *inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
}

// Quantise 8 consecutive values (the first `nv` valid, the rest padding -> 0).
__device__ __forceinline__ uint2 quant8(const float (&v)[8], int nv, float inv, bool u8) {
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t b = (i < nv) ? quant_byte(v[i], inv, u8) : 0u;
    if (i < 4)
      lo |= b << (8 * i);
    else
      hi |= b << (8 * (i - 4));
  }
  return make_uint2(lo, hi);
}

// exp256_ps (ops_cpu.cpp:75-92) for one lane, operation for operation:
// clamp to [-87, 88], n = rne(x*log2e), r = x - n*ln2 (product, then
// difference), degree-6 Horner with fused multiply-adds, times 2^n built in
// the exponent field.
__device__ __forceinline__ float exp_ref(float x) {
  x = (x < 88.0f) ? x : 88.0f;
  x = (x > -87.0f) ? x : -87.0f;
  const float n = rintf(__fmul_rn(x, 1.4426950408889634f));
  const float r = __fsub_rn(x, __fmul_rn(n, 0.6931471805599453f));
  float p = 1.0f / 720;
  p = __fmaf_rn(p, r, 1.0f / 120);
  p = __fmaf_rn(p, r, 1.0f / 24);
  p = __fmaf_rn(p, r, 1.0f / 6);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = __float2int_rn(n);
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

// silu_up8 (ops_cpu.cpp:138-142): (g / (1 + exp(0 - g))) * u.
__device__ __forceinline__ float silu_up_vec(float g, float u) {
  const float d = __fadd_rn(1.0f, exp_ref(__fsub_rn(0.0f, g)));
  return __fmul_rn(__fdiv_rn(g, d), u);
}

// The scalar tail of a block (kn % 8 trailing elements, ops_cpu.cpp:166)
// uses silu() with the C library's expf.  A correctly rounded exp is formed
// here from the double-precision exp, which agrees with the host expf except
// in the rare cases where the host's result is not correctly rounded.
__device__ __forceinline__ float silu_up_tail(float g, float u) {
  const float e = static_cast<float>(exp(static_cast<double>(-g)));
  const float d = __fadd_rn(1.0f, e);
  return __fmul_rn(__fdiv_rn(g, d), u);
}

// Quantise the 32 values of one block (all valid) with the block's absmax
// rule and store them at `out` in form `mode` (0 int8 q, 1 u8 q+128, 2 fp16
// q*scale); returns the block scale.  Sets *range_bad when an fp16 value
// would overflow.
__device__ __forceinline__ float quant_block32(const float (&v)[32], uint8_t* out, int mode,
                                               bool* range_bad) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  float scale, inv;
  block_scales(amax, &scale, &inv);
  if (mode == 2) {
    uint4 w[4];
    uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float d[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        int z = cvt_rne_x86(__fmul_rn(v[i + j], inv));
        z = z < -127 ? -127 : (z > 127 ? 127 : z);
        d[j] = __fmul_rn(static_cast<float>(z), scale);
        if (fabsf(d[j]) > 65504.f) *range_bad = true;
      }
      const __half2 h = __floats2half2_rn(d[0], d[1]);
      wp[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(out)[i] = w[i];
  } else {
    uint32_t wq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) word |= quant_byte(v[4 * i + j], inv, mode == 1) << (8 * j);
      wq[i] = word;
    }
    reinterpret_cast<uint4*>(out)[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
    reinterpret_cast<uint4*>(out)[1] = make_uint4(wq[4], wq[5], wq[6], wq[7]);
  }
  return scale;
}

// quant_block32 with the same outputs, faster for blocks whose values are all
// finite: y = v * inv satisfies |y| <= 127 (1 + 2^-23) there, so
// fl(y + 1.5 * 2^23) holds rne(y) in its low mantissa bits and
// fl(fl(y + 1.5 * 2^23) - 1.5 * 2^23) = rne(y) exactly -- no conversion to
// an integer and no clamp (|rne(y)| <= 127).  An fp16 value can overflow only
// if 127 * scale does (the block's largest value maps to +-127).  Blocks with
// an infinity or a NaN take quant_block32.
__device__ __forceinline__ float quant_block32_fast(const float (&v)[32], uint8_t* out, int mode,
                                                    bool* range_bad) {
  float anan = 0.f;  // max |v|, NaN if any value is NaN
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(anan), "f"(fabsf(v[i])));
    anan = r;
  }
  if (!(anan <= 3.402823466e38f)) return quant_block32(v, out, mode, range_bad);
  float scale, inv;
  block_scales(anan, &scale, &inv);
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  if (mode == 2) {
    if (anan > 0.f && __fmul_rn(127.f, scale) > 65504.f) *range_bad = true;
    uint4 w[4];
    uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const float z0 = __fsub_rn(__fadd_rn(__fmul_rn(v[i], inv), kMagic), kMagic);
      const float z1 = __fsub_rn(__fadd_rn(__fmul_rn(v[i + 1], inv), kMagic), kMagic);
      const __half2 h = __floats2half2_rn(__fmul_rn(z0, scale), __fmul_rn(z1, scale));
      wp[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(out)[i] = w[i];
  } else {
    const int bias = mode == 1 ? 128 : 0;
    uint32_t wq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float t = __fadd_rn(__fmul_rn(v[4 * i + j], inv), kMagic);
        const int q = __float_as_int(t) - 0x4B400000 + bias;  // rne(v * inv) (+ 128)
        word |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);
      }
      wq[i] = word;
    }
    reinterpret_cast<uint4*>(out)[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
    reinterpret_cast<uint4*>(out)[1] = make_uint4(wq[4], wq[5], wq[6], wq[7]);
  }
  return scale;
}

}  // namespace ovb
