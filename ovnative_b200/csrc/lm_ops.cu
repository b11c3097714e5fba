// lm_ops.cu -- the steps of the LM forward that are not GEMMs, quantisers or
// attention: the embedding gather, the RoPE table, the per-head RMSNorm + RoPE
// of q and k (the int8 path; the fp16 path fuses it into the q|k|v GEMM), and
// the logits permute of the batched forward.
// They are what LM::forward / LM::forward_cfg (cpp/src/model/lm.cpp:343-454)
// run between the hot-path kernels, so that a whole forward stays on the
// device (ovb_lm_*, lm.cpp in this directory).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "ovb_internal.h"

namespace ovb {

__device__ int g_status_lm;

namespace {

constexpr int kErrLmIndex = 128;  // a token / codebook id outside its table (row left zero)
constexpr int kErrLmF16Range = 16;  // a q / k / v value beyond the fp16 range

// One row of an embedding table as Emb::gather reads it (mat.cpp:52-66):
// int8 entries times the row's scale, or fp32 entries.
__device__ __forceinline__ float emb_at(const EmbTable& t, int64_t row, int c) {
  if (t.i8) return __fmul_rn(static_cast<float>(t.i8[row * t.cols + c]), t.scale[row]);
  return t.f32[row * t.cols + c];
}

}  // namespace

// LM::embed / embed_cfg (lm.cpp:178-215): row r of the packed batch (batch
// row b = r / seq, position s = r % seq) takes the token embedding of
// ids[b][0][s] when mask[r] is 0, else the sum over codebooks c of the audio
// embeddings of ids[b][c][s] + offsets[c], accumulated in codebook order from
// 0.  ids are [B][C][seq] (forward_cfg: B = 1, seq = rows).  One block per
// row; an id outside its table leaves the row zero and sets status bit 128.
// Four consecutive elements of row `row` (c % 4 == 0, cols % 4 == 0): the
// same values as emb_at, with one 4- or 16-byte load.
__device__ __forceinline__ float4 emb_at4(const EmbTable& t, int64_t row, int c) {
  if (t.i8) {
    const char4 q = *reinterpret_cast<const char4*>(t.i8 + row * t.cols + c);
    const float sc = t.scale[row];
    return make_float4(__fmul_rn(static_cast<float>(q.x), sc), __fmul_rn(static_cast<float>(q.y), sc),
                       __fmul_rn(static_cast<float>(q.z), sc), __fmul_rn(static_cast<float>(q.w), sc));
  }
  return *reinterpret_cast<const float4*>(t.f32 + row * t.cols + c);
}

constexpr int kEmbMaxC = 32;  // codebooks the vector path stages

__global__ void embed_kernel(const int64_t* ids, const uint8_t* mask, const int64_t* offsets,
                             int C, int seq, EmbTable tok, EmbTable aud, float* out, int H) {
  const int64_t r = blockIdx.x;
  const int64_t b = r / seq, s = r % seq;
  const int64_t* base = ids + b * C * seq;
  float* o = out + r * H;
  // Vector path: the row's ids read once into shared memory, then four
  // consecutive columns per thread and load (the row's arithmetic unchanged:
  // the same products, summed in codebook order).
  const bool vec = C <= kEmbMaxC && (H & 3) == 0 && (tok.cols & 3) == 0 && (aud.cols & 3) == 0;
  if (vec) {
    __shared__ int64_t sid[kEmbMaxC];
    __shared__ int s_bad;
    const bool text = !mask[r];
    if (threadIdx.x == 0) s_bad = 0;
    __syncthreads();
    if (threadIdx.x < (text ? 1 : C)) {
      const int cb = threadIdx.x;
      const int64_t id = text ? base[s] : base[static_cast<int64_t>(cb) * seq + s] + offsets[cb];
      sid[cb] = id;
      if (!(id >= 0 && id < (text ? tok.rows : aud.rows))) atomicOr(&s_bad, 1);
    }
    __syncthreads();
    const bool ok = s_bad == 0;
    for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ok && text) {
        acc = emb_at4(tok, sid[0], c);
      } else if (ok) {
        for (int cb = 0; cb < C; ++cb) {
          const float4 e = emb_at4(aud, sid[cb], c);
          acc = make_float4(__fadd_rn(acc.x, e.x), __fadd_rn(acc.y, e.y), __fadd_rn(acc.z, e.z),
                            __fadd_rn(acc.w, e.w));
        }
      }
      *reinterpret_cast<float4*>(o + c) = acc;
    }
    if (!ok && threadIdx.x == 0) atomicOr(&g_status_lm, kErrLmIndex);
    return;
  }
  if (!mask[r]) {
    const int64_t id = base[s];
    const bool ok = id >= 0 && id < tok.rows;
    for (int c = threadIdx.x; c < H; c += blockDim.x) o[c] = ok ? emb_at(tok, id, c) : 0.f;
    if (!ok && threadIdx.x == 0) atomicOr(&g_status_lm, kErrLmIndex);
    return;
  }
  bool ok = true;
  for (int cb = 0; cb < C; ++cb) {
    const int64_t id = base[static_cast<int64_t>(cb) * seq + s] + offsets[cb];
    ok = ok && id >= 0 && id < aud.rows;
  }
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float acc = 0.f;
    if (ok)
      for (int cb = 0; cb < C; ++cb)
        acc = __fadd_rn(acc, emb_at(aud, base[static_cast<int64_t>(cb) * seq + s] + offsets[cb], c));
    o[c] = acc;
  }
  if (!ok && threadIdx.x == 0) atomicOr(&g_status_lm, kErrLmIndex);
}

// The RoPE table of a forward: cos and sin of angle_i = fl(fl(pos[r]) *
// inv_freq[i]) for i < 64, inv_freq[i] = (float) theta^(-2i/D) computed on
// the host as the reference does.  A row is 128 floats in 32 groups of four,
// group j = (cos angle_2j, cos angle_2j+1, sin angle_2j, sin angle_2j+1), so
// that a consumer rotating two adjacent elements reads both cosines and both
// sines as register pairs (rope_cos_sin).  The reference tabulates the same
// per row and keeps the table across layers while the positions do not
// change (qk_norm_rope_f32, ops_cpu.cpp:945-986); here it is built once per
// forward.  cos / sin are CUDA's (not glibc's): they agree to a few ulps.
// One thread per (row, i).
__global__ void rope_table_kernel(const int64_t* pos, RopeFreq f, int64_t rows, float* tab) {
  const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (t >= rows * 64) return;
  const int64_t r = t >> 6;
  const int i = static_cast<int>(t & 63);
  const float angle = __fmul_rn(static_cast<float>(pos[r]), f.inv_freq[i]);
  float* g = tab + r * 128 + 4 * (i >> 1) + (i & 1);
  g[0] = cosf(angle);
  g[2] = sinf(angle);
}

// (cos, sin) of angle i of a table row (rope_table_kernel's grouping).
__device__ __forceinline__ float2 rope_cos_sin(const float* row, int i) {
  const float* g = row + 4 * (i >> 1) + (i & 1);
  return make_float2(g[0], g[2]);
}

// qk_norm_rope_f32 (ops_cpu.cpp:945-1013) for head_dim 128, written as fp16
// into q16 / k16 (the attention's operands), and v converted to fp16 into
// v16, in one pass over the row; q, k, v (fp32, from the q|k|v GEMM) are only
// read.  Each head vector x of q (n_heads per row) and k (n_kv per row) is
// RMS-normalised with its weight, then rotated by the row's angles:
//   scale = 1 / sqrt(sum(x^2) / D + eps);  a = (x[i] scale) w[i],
//   b = (x[i+64] scale) w[i+64];  x[i] = a cos - b sin;  x[i+64] = b cos + a sin.
// One block per row, one warp per head vector; lane l holds elements l,
// l+32, l+64, l+96 and the sum of squares runs in a warp tree (the fused q|k|v
// GEMM epilogue, gemm_f16.cu, reproduces this order).  An output that
// rounds to an fp16 infinity (|x| >= 65520) or is NaN sets status bit 16.
__global__ void qk_norm_rope_f16_kernel(const float* q, const float* k, const float* v,
                                        __half* q16, __half* k16, __half* v16, const float* qw,
                                        const float* kw, const float* tab, int64_t rows,
                                        int n_heads, int n_kv, float eps) {
  constexpr int D = 128, half = 64;
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = static_cast<int>(blockDim.x >> 5);
  const float2 cs0 = rope_cos_sin(tab + r * D, lane), cs1 = rope_cos_sin(tab + r * D, lane + 32);
  bool range_ok = true;
  // Each warp's head vectors (q, then k, then v heads), loaded in groups of
  // four before any of them is reduced, so that their loads are in flight
  // together.
  const int nvec = n_heads + 2 * n_kv;
  for (int h0 = warp; h0 < nvec; h0 += 4 * nw) {
    float xs[4][4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int h = h0 + g * nw;
      const float* src = h < n_heads ? q + (r * n_heads + h) * D
                         : h < n_heads + n_kv ? k + (r * n_kv + (h - n_heads)) * D
                                              : v + (r * n_kv + (h - n_heads - n_kv)) * D;
#pragma unroll
      for (int j = 0; j < 4; ++j) xs[g][j] = h < nvec ? src[lane + 32 * j] : 0.f;
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) {
    const int h = h0 + g * nw;
    if (h >= nvec) break;
    if (h >= n_heads + n_kv) {  // v: convert only
      const int64_t base = (r * n_kv + (h - n_heads - n_kv)) * D;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x = xs[g][j];
        range_ok = range_ok && fabsf(x) < 65520.f;
        v16[base + lane + 32 * j] = __float2half_rn(x);
      }
      continue;
    }
    const bool is_q = h < n_heads;
    const int64_t base = is_q ? (r * n_heads + h) * D : (r * n_kv + (h - n_heads)) * D;
    __half* dst = is_q ? q16 + base : k16 + base;
    const float* w = is_q ? qw : kw;
    float x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = xs[g][j];
    float sum = __fadd_rn(__fadd_rn(__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1])),
                          __fadd_rn(__fmul_rn(x[2], x[2]), __fmul_rn(x[3], x[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float scale =
        __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(D)), eps)));
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = lane + 32 * j;  // 0 .. 63
      const float cs = j ? cs1.x : cs0.x, sn = j ? cs1.y : cs0.y;
      const float a = __fmul_rn(__fmul_rn(x[j], scale), w[i]);
      const float b = __fmul_rn(__fmul_rn(x[j + 2], scale), w[i + half]);
      const float lo = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
      const float hi = __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
      range_ok = range_ok && fabsf(lo) < 65520.f && fabsf(hi) < 65520.f;
      dst[i] = __float2half_rn(lo);
      dst[i + half] = __float2half_rn(hi);
    }
    }
  }
  if (!range_ok) atomicOr(&g_status_lm, kErrLmF16Range);
}

// [B*S, C*V] -> [B, C, S, V] (lm.cpp:387-398).  One block per (b, s) row.
__global__ void permute_logits_kernel(const float* src, float* dst, int S, int C, int V) {
  const int64_t r = blockIdx.x;
  const int64_t b = r / S, s = r % S;
  const float* in = src + r * C * static_cast<int64_t>(V);
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(C) * V; i += blockDim.x) {
    const int64_t c = i / V, t = i % V;
    dst[((b * C + c) * S + s) * V + t] = in[i];
  }
}

cudaError_t launch_embed(const int64_t* ids, const uint8_t* mask, const int64_t* offsets, int C,
                         int64_t rows, int seq, const EmbTable& tok, const EmbTable& aud,
                         float* out, int H, cudaStream_t s) {
  return launch_plain(embed_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, s, ids,
                      mask, offsets, C, seq, tok, aud, out, H);
}

cudaError_t launch_rope_table(const int64_t* pos, const RopeFreq& f, int64_t rows, float* tab,
                              cudaStream_t s) {
  const int64_t n = rows * 64;
  return launch_plain(rope_table_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256),
                      0, s, pos, f, rows, tab);
}

cudaError_t launch_qk_norm_rope_f16(const float* q, const float* k, const float* v, void* q16,
                                    void* k16, void* v16, const float* qw, const float* kw,
                                    const float* tab, int64_t rows, int n_heads, int n_kv,
                                    float eps, cudaStream_t s) {
  return launch_plain(qk_norm_rope_f16_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, s,
                      q, k, v, static_cast<__half*>(q16), static_cast<__half*>(k16),
                      static_cast<__half*>(v16), qw, kw, tab,
                      rows, n_heads, n_kv, eps);
}

cudaError_t launch_permute_logits(const float* src, float* dst, int B, int S, int C, int V,
                                  cudaStream_t s) {
  return launch_plain(permute_logits_kernel, dim3(static_cast<unsigned>(B * S)), dim3(256), 0, s,
                      src, dst, S, C, V);
}

cudaError_t read_and_clear_status_lm(int* out, cudaStream_t s) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_status_lm, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_status_lm, &zero, sizeof(int));
}

}  // namespace ovb
