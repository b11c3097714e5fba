/*
 * ovb_oracle.c -- scalar CPU restatement of OVNative's int8 LM GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * ovnative_b200/csrc; only tests/, __graft_entry__.smoke() and the cpu
 * baseline leg of bench.py load it.  The product path never calls it.
 *
 * Parity is pinned: tests/test_oracle.py checks every function here byte for
 * byte against the reference's own code (gemm.cpp / ops_cpu.cpp compiled from
 * source into oracle/_ref/libovref.so by oracle/Makefile) and against the
 * committed golden vectors in tests/golden/.
 *
 * Exception: ovo_guided_sample (the sampler, cpp/src/model/tts.cpp:91-101,
 * :291-326) is a restatement only -- parity unpinned.  The reference's loop
 * lives inside a Pipeline method and its log_softmax in an anonymous
 * namespace, so neither can be called on its own, and no reference test or
 * golden vector covers it.
 *
 * Reference files cited below are paths inside the OVNative project
 * (cpp/src/backend/cpu/gemm.cpp, cpp/src/backend/cpu/ops_cpu.cpp,
 * cpp/src/model/tts.cpp).
 *
 * Numerics follow the reference operation for operation:
 *   - every product, sum and quotient is a separately rounded IEEE fp32 op
 *     (this file is built with -ffp-contract=off), fused multiply-adds appear
 *     only where the reference uses _mm256_fmadd_ps, and are written fmaf();
 *   - float->int conversion is round-to-nearest-even (cvtps_epi32 /
 *     nearbyint under the default MXCSR), out-of-range / NaN give INT32_MIN
 *     like cvtps_epi32's "integer indefinite" before the clamp.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define OVO_API __attribute__((visibility("default")))

static int64_t kblocks(int64_t K) { return (K + 31) / 32; }

/* cvtps_epi32 with the default rounding mode: RNE, and 0x80000000 for NaN or
 * anything outside int32. */
static int32_t cvt_rne_x86(float v) {
  if (!(v == v)) return INT32_MIN;
  if (v >= 2147483648.0f || v < -2147483648.0f) return INT32_MIN;
  return (int32_t)nearbyintf(v);
}

/* One 32-k block of quantize_a_u8: gemm.cpp:392-428.  `v` holds the kn
 * (<= 32) activations of the block; writes 32 bytes of q (u8 = q+128, tail
 * bytes 0) and returns the block scale. */
static float quant_block_u8(const float* v, int64_t kn, uint8_t* q) {
  /* amax exactly as the reference forms it (gemm.cpp:396-406), NaN included:
   * eight lanes, each folding the block's whole 8-vectors with MAXPS
   * (_mm256_max_ps(m, x) = (m > x) ? m : x -- a NaN on either side yields x),
   * then the lanes and the tail folded with std::max(amax, x) = (amax < x) ?
   * x : amax, which never lets a NaN through.  For finite values this is the
   * plain maximum of |v|. */
  float lane[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int64_t k = 0;
  for (; k + 8 <= kn; k += 8)
    for (int j = 0; j < 8; ++j) {
      const float a = fabsf(v[k + j]);
      lane[j] = (lane[j] > a) ? lane[j] : a;
    }
  float amax = 0.f;
  for (int j = 0; j < 8; ++j) amax = (amax < lane[j]) ? lane[j] : amax;
  for (; k < kn; ++k) {
    const float a = fabsf(v[k]);
    amax = (amax < a) ? a : amax;
  }
  const float scale = amax / 127.0f;                 /* gemm.cpp:407 */
  const float inv = amax > 0.f ? 127.0f / amax : 0.f; /* gemm.cpp:408 */
  for (int64_t k = 0; k < kn; ++k) {
    const float prod = v[k] * inv;
    int32_t z = cvt_rne_x86(prod);
    z = z < -127 ? -127 : (z > 127 ? 127 : z);
    q[k] = (uint8_t)(z + 128);
  }
  for (int64_t k = kn; k < 32; ++k) q[k] = 0; /* gemm.cpp:427 */
  return scale;
}

/* s8_nk_quantize / quantize_a_u8: gemm.cpp:379-430, :709-720.
 * aq: u8 [M, Kb*32]; asc: fp32 [M, Kb]. */
OVO_API void ovo_quantize_u8(int64_t M, int64_t K, const float* A, uint8_t* aq, float* asc) {
  if (M <= 0 || K <= 0) return;
  const int64_t Kb = kblocks(K), Kp = Kb * 32;
  for (int64_t i = 0; i < M; ++i)
    for (int64_t b = 0; b < Kb; ++b) {
      const int64_t k0 = b * 32, kn = (K - k0 < 32) ? (K - k0) : 32;
      asc[i * Kb + b] = quant_block_u8(A + i * K + k0, kn, aq + i * Kp + k0);
    }
}

/* rmsnorm_quantize_avx2: gemm.cpp:638-707 (and rmsnorm_avx2, ops_cpu.cpp:38-62).
 * Sum of squares: eight running fp32 lanes, lane l accumulating elements
 * i = l, l+8, ... with FMA in order (gemm.cpp:655-658), then the lanes summed
 * left to right (:661-662), then the cols%8 tail added one product at a time
 * (:663), then scale = 1/sqrt(sum/cols + eps) (:664).  The normalised value is
 * (x*scale)*w with two roundings (:675, :677). */
OVO_API void ovo_rmsnorm_quantize_u8(int64_t rows, int64_t cols, const float* x, const float* w,
                                     float eps, uint8_t* aq, float* asc) {
  if (rows <= 0 || cols <= 0) return;
  const int64_t Kb = kblocks(cols), Kp = Kb * 32;
  for (int64_t r = 0; r < rows; ++r) {
    const float* row = x + r * cols;
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t i = 0;
    for (; i + 8 <= cols; i += 8)
      for (int l = 0; l < 8; ++l) lane[l] = fmaf(row[i + l], row[i + l], lane[l]);
    float sum = lane[0] + lane[1];
    sum = sum + lane[2];
    sum = sum + lane[3];
    sum = sum + lane[4];
    sum = sum + lane[5];
    sum = sum + lane[6];
    sum = sum + lane[7];
    for (; i < cols; ++i) {
      const float p = row[i] * row[i];
      sum = sum + p;
    }
    const float scale = 1.f / sqrtf(sum / (float)cols + eps);
    for (int64_t b = 0; b < Kb; ++b) {
      const int64_t k0 = b * 32, kn = (cols - k0 < 32) ? (cols - k0) : 32;
      float v[32];
      for (int64_t k = 0; k < kn; ++k) {
        const float t = row[k0 + k] * scale;
        v[k] = t * w[k0 + k];
      }
      asc[r * Kb + b] = quant_block_u8(v, kn, aq + r * Kp + k0);
    }
  }
}

/* exp256_ps: ops_cpu.cpp:75-92, one lane.  Clamp to [-87, 88]; n = x*log2(e)
 * rounded to nearest even; r = x - n*ln2 (a product then a difference, not
 * fused); degree-6 Horner with FMA; scale by 2^n built from the exponent
 * bits. */
static float exp_ref(float x) {
  x = (x < 88.0f) ? x : 88.0f;   /* _mm256_min_ps(x, 88) returns 88 for NaN x */
  x = (x > -87.0f) ? x : -87.0f; /* _mm256_max_ps(x, -87) */
  const float n = nearbyintf(x * 1.4426950408889634f);
  const float nl = n * 0.6931471805599453f;
  const float r = x - nl;
  float p = 1.0f / 720;
  p = fmaf(p, r, 1.0f / 120);
  p = fmaf(p, r, 1.0f / 24);
  p = fmaf(p, r, 1.0f / 6);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int32_t ni = cvt_rne_x86(n);
  const uint32_t bits = (uint32_t)(ni + 127) << 23;
  float sc;
  memcpy(&sc, &bits, 4);
  return p * sc;
}

/* silu_up8 for one lane: ops_cpu.cpp:138-142: (g / (1 + exp(0 - g))) * u. */
static float silu_up_ref(float g, float u) {
  const float e = exp_ref(0.0f - g);
  const float d = 1.0f + e;
  const float s = g / d;
  return s * u;
}

/* silu_mul_quant_avx2: ops_cpu.cpp:144-198.  The vector body covers the
 * first (kn/8)*8 elements of each block with exp256_ps; the last kn%8 use
 * the scalar silu() with std::exp (:166).  std::exp is libm's, so those tail
 * elements are computed with expf here as well (both sides use the host
 * libm). */
OVO_API void ovo_silu_mul_quantize_u8(int64_t M, int64_t K, const float* gate, const float* up,
                                      uint8_t* aq, float* asc) {
  if (M <= 0 || K <= 0) return;
  const int64_t Kb = kblocks(K), Kp = Kb * 32;
  for (int64_t r = 0; r < M; ++r)
    for (int64_t b = 0; b < Kb; ++b) {
      const int64_t k0 = b * 32, kn = (K - k0 < 32) ? (K - k0) : 32;
      const float* g = gate + r * K + k0;
      const float* u = up + r * K + k0;
      float v[32];
      int64_t i = 0;
      for (; i + 8 <= kn; i += 8)
        for (int l = 0; l < 8; ++l) v[i + l] = silu_up_ref(g[i + l], u[i + l]);
      for (; i < kn; ++i) {
        const float d = 1.f + expf(-g[i]);
        v[i] = (g[i] / d) * u[i];
      }
      asc[r * Kb + b] = quant_block_u8(v, kn, aq + r * Kp + k0);
    }
}

/* Per-32-k block integer products P[m][n][b] = sum_{k in b} q[m,k] * W[n,k],
 * q = aq - 128.  This is what the 8 vpdpbusd + zero-point correction of
 * gemm.cpp:455-474 compute exactly (|P| <= 32*127*127 fits int32).
 * W is [N, K] (OVW1 layout=0). P: int32 [M, N, Kb]. */
OVO_API void ovo_block_products(int64_t M, int64_t N, int64_t K, const uint8_t* aq,
                                const int8_t* W, int32_t* P) {
  const int64_t Kb = kblocks(K), Kp = Kb * 32;
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n)
      for (int64_t b = 0; b < Kb; ++b) {
        const int64_t k0 = b * 32, kn = (K - k0 < 32) ? (K - k0) : 32;
        int32_t s = 0;
        for (int64_t k = 0; k < kn; ++k)
          s += ((int32_t)aq[m * Kp + k0 + k] - 128) * (int32_t)W[n * K + k0 + k];
        P[(m * N + n) * Kb + b] = s;
      }
}

/* linear_s8_nk_vnni_tile_at epilogue: gemm.cpp:455-501.
 * f = 0; for b in order: f = fma((float)P_b, asc[m,b], f);  o = f * wscale[n];
 * accumulate: o = o + C[m,n] (kept as a separate add, :487).
 * W is [N, K]; C row stride ldc. */
OVO_API void ovo_linear_q(int64_t M, int64_t N, int64_t K, const uint8_t* aq, const float* asc,
                          const int8_t* W, const float* wscale, float* C, int64_t ldc,
                          int accumulate) {
  if (M <= 0 || N <= 0 || K <= 0) return;
  const int64_t Kb = kblocks(K), Kp = Kb * 32;
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float f = 0.f;
      for (int64_t b = 0; b < Kb; ++b) {
        const int64_t k0 = b * 32, kn = (K - k0 < 32) ? (K - k0) : 32;
        int32_t s = 0;
        for (int64_t k = 0; k < kn; ++k)
          s += ((int32_t)aq[m * Kp + k0 + k] - 128) * (int32_t)W[n * K + k0 + k];
        f = fmaf((float)s, asc[m * Kb + b], f);
      }
      float o = f * wscale[n];
      if (accumulate) o = o + C[m * ldc + n];
      C[m * ldc + n] = o;
    }
}

/* Unfused producers, used to pin the fused-equals-composed identities of
 * test_gemm.cpp:182-201 and :331-351 on the oracle itself. */

/* rmsnorm_avx2: ops_cpu.cpp:38-62. */
OVO_API void ovo_rmsnorm_into(float* dst, const float* src, const float* w, int64_t rows,
                              int64_t cols, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* row = src + r * cols;
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t i = 0;
    for (; i + 8 <= cols; i += 8)
      for (int l = 0; l < 8; ++l) lane[l] = fmaf(row[i + l], row[i + l], lane[l]);
    float sum = lane[0] + lane[1];
    for (int l = 2; l < 8; ++l) sum = sum + lane[l];
    for (; i < cols; ++i) {
      const float p = row[i] * row[i];
      sum = sum + p;
    }
    const float scale = 1.f / sqrtf(sum / (float)cols + eps);
    for (i = 0; i < cols; ++i) {
      const float t = row[i] * scale;
      dst[r * cols + i] = t * w[i];
    }
  }
}

/* silu_mul_avx2: ops_cpu.cpp:126-136 (vector body on the first n/8*8
 * elements of the flat array, libm tail). */
OVO_API void ovo_silu_mul(float* out, const float* gate, const float* up, int64_t n) {
  int64_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int l = 0; l < 8; ++l) out[i + l] = silu_up_ref(gate[i + l], up[i + l]);
  for (; i < n; ++i) {
    const float d = 1.f + expf(-gate[i]);
    out[i] = (gate[i] / d) * up[i];
  }
}

/* ------------------------------------------------ guided argmax (sampler)
 * log_softmax: cpp/src/model/tts.cpp:91-101, operation for operation (max
 * as std::max(m, x) = m < x ? x : m; exp values summed left to right; then
 * x - lse).  `out` may be `x`, as in the reference's call at tts.cpp:313 --
 * its third loop then reads the exp values the second loop stored. */
static void log_softmax_ref(const float* x, int n, float* out) {
  float m = -INFINITY;
  for (int i = 0; i < n; ++i) m = (m < x[i]) ? x[i] : m;
  float sum = 0.f;
  for (int i = 0; i < n; ++i) {
    out[i] = expf(x[i] - m);
    sum += out[i];
  }
  const float lse = logf(sum) + m;
  for (int i = 0; i < n; ++i) out[i] = x[i] - lse;
}

/* The per-step guidance + argmax loop, cpp/src/model/tts.cpp:291-326 (the
 * non-B2 plane layout: cond row at token cond_seq - T + t, uncond row at
 * token t of its own plane, both [seq, C * V]).  in_place != 0 reproduces
 * the reference's in-place log_softmax of the mix (tts.cpp:313, scores
 * exp(mix - max) - lse); in_place == 0 gives the log-probabilities that
 * call intends, which the reference's CUDA kernel computes
 * (cpp/src/backend/cuda/cuda_lm.cu:717-740).  pred is the same either way.
 * mask_id outside [0, V) masks nothing.  scratch: 4 * V floats. */
OVO_API void ovo_guided_sample(const float* cond, int cond_seq, const float* uncond, int C,
                               int V, int T, float guidance, float penalty, int mask_id,
                               int in_place, int32_t* pred, float* scores, float* scratch) {
  float* lp_c = scratch;
  float* lp_u = scratch + V;
  float* mix = scratch + 2 * (int64_t)V;
  float* mix2 = scratch + 3 * (int64_t)V;
  const int64_t CV = (int64_t)C * V;
  for (int64_t idx = 0; idx < (int64_t)C * T; ++idx) {
    const int c = (int)(idx / T);
    const int t = (int)(idx - (int64_t)c * T);
    const float* lc = cond + ((int64_t)cond_seq - T + t) * CV + (int64_t)c * V;
    const float* lu = uncond + (int64_t)t * CV + (int64_t)c * V;
    log_softmax_ref(lc, V, lp_c);
    log_softmax_ref(lu, V, lp_u);
    float* lp_mix = mix;
    if (guidance != 0.f) {
      for (int v = 0; v < V; ++v) mix[v] = lp_c[v] + guidance * (lp_c[v] - lp_u[v]);
      if (in_place) {
        log_softmax_ref(mix, V, mix);
      } else {
        log_softmax_ref(mix, V, mix2);
        lp_mix = mix2;
      }
    } else {
      memcpy(mix, lp_c, sizeof(float) * (size_t)V);
    }
    if (mask_id >= 0 && mask_id < V) lp_mix[mask_id] = -INFINITY;
    int best = 0;
    float best_val = -INFINITY;
    for (int v = 0; v < V; ++v) {
      if (lp_mix[v] > best_val) {
        best_val = lp_mix[v];
        best = v;
      }
    }
    pred[idx] = best;
    scores[idx] = best_val - (float)c * penalty;
  }
}
