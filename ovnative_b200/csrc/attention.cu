// attention.cu -- the attention of one OVNative LM layer on the tensor cores:
// for every attention segment (one half of a CFG pair, or one batch row: its
// q/k/v rows and an additive bias [rows, rows] or none) and query head h (kv
// head h / group),
//
//   out = softmax(q k^T * scale + bias) v,  rows whose scores are all below
//   -1e29 (fully masked) -> 0,
//
// as ov::attention_head_f32 computes it (cpp/src/backend/cpu/ops_cpu.cpp:
// 907-943, called per (segment, head) by LM::run_layer, cpp/src/model/
// lm.cpp:256-274; the reference's CUDA runner dispatches between a SIMT fp32
// kernel and TF32 strided-batched cuBLAS, cpp/src/backend/cuda/cuda_lm.cu:
// 393-421, :423-606, :1132-1145).  head_dim is 128.
//
// One CTA of 256 threads (OVB_ATT_THREADS) per (segment, head, block of 128
// query rows).  Warp w reads TMEM lanes 32 (w % 4) .. + 31 (the rows) and
// column group w / 4: half of the tile's keys and of O's columns; the two
// threads of a row combine their maxima and sums through shared memory.  Per
// tile of 128 keys:
//   - TMA brings the fp32 K and V tiles (128 x 128, 64 KB each) into staging
//     shared memory one tile ahead of their use;
//   - the threads convert them to fp16: K into the 128-byte-swizzled K-major
//     layout the MMA reads, V transposed (keys along K), keys past the
//     segment zeroed;
//   - S = Q K^T (tcgen05.mma kind::f16, fp32 in TMEM);
//   - the tile's bias, loaded by whole rows (coalesced) while the operands
//     are converted, is staged in the K staging buffer (the next K tile's
//     TMA waits until the scores are read);
//   - each thread turns its row of S into scaled, biased scores, moves its
//     softmax reference point m when the tile's maximum exceeds it by more
//     than 8 (then rescaling its running sum and its row of O in TMEM), and
//     writes P = exp(score - m) as fp16 into TMEM;
//   - O += P V with P as the A operand from TMEM.
// Finally O / sum goes to the output.  Keeping m up to 8 below the running
// maximum bounds P by e^8 (well inside fp16) and skips most rescales; the
// result is the same softmax.  The fp16 operands make the output agree with
// the fp32 reference to ~1e-3 relative (2^-11 rounding per element).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <functional>
#include <queue>
#include <utility>
#include <vector>

#include "ovb_internal.h"
#include "ovb_ptx.cuh"
#include "ovb_quant.cuh"

namespace ovb {

__device__ int g_status_att;

namespace {

constexpr int kErrAttRange = 16;  // an input beyond the fp16 range
constexpr int kErrAttWait = 32;   // a TMA or MMA-completion wait gave up
constexpr int kAttD = 128;
constexpr int kAttRows = 128;     // query rows per CTA = TMEM lanes
constexpr int kAttKeys = 128;     // keys per tile
#ifndef OVB_ATT_THREADS
#define OVB_ATT_THREADS 256
#endif
constexpr int kAttThreads = OVB_ATT_THREADS;
constexpr int kCG = kAttThreads / 128;   // column groups (threads per row)
constexpr int kGCols = kAttKeys / kCG;   // S / O columns per thread
static_assert(kGCols % 32 == 0, "whole 32-column TMEM chunks per thread");
constexpr float kRescale = 8.f;   // move m once a tile's max exceeds it by this
constexpr uint32_t kF16Tile = 128 * 128 * 2;  // one fp16 operand tile
constexpr uint32_t kF32Tile = 128 * 128 * 4;  // one fp32 staging tile (TMA box)
constexpr uint32_t kOffQ = 0, kOffK = kF16Tile, kOffV = 2 * kF16Tile;
constexpr uint32_t kOffStK = 3 * kF16Tile, kOffStV = kOffStK + kF32Tile;
constexpr uint32_t kOffCtl = kOffStV + kF32Tile;
constexpr uint32_t kColS = 0, kColP = 128, kColO = 256, kTmemCols = 512;

struct AttnCtl {
  uint64_t ld_k;   // TMA: K tile (phase i = tile i)
  uint64_t ld_v;   // TMA: Q (phase 0), then V tile i (phase i + 1)
  uint64_t mma_s;  // S = Q K^T of tile i complete (phase i)
  uint64_t mma_o;  // O += P V of tile i complete (phase i)
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kAttSmem = 1024 + kOffCtl + sizeof(AttnCtl);
static_assert(kAttSmem <= 227 * 1024, "attention shared memory");

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Byte offset of fp16 element (r, c) of a 128 x 128 operand stored as two K
// chunks of [128 rows][64 fp16] with the 128-byte swizzle (16-byte chunk j of
// row r at position j ^ (r % 8)).
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return static_cast<uint32_t>((c >> 6) * (kF16Tile / 2) + r * 128 +
                               ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}

// Rows of a row-major fp32 staging tile [128][128] into an fp16 operand
// tile, rows >= valid as zeros.  Warp w converts rows w, w + kAttThreads/32,
// ...; lane l columns 4l .. 4l + 3 (one 512-byte row per warp instruction, no
// bank conflicts).  Returns the largest |value| converted (NaN ignored).
__device__ __forceinline__ float convert_rows(uint8_t* dst, const float* st, int valid) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c4 = lane * 4;
  float amax = 0.f;
#pragma unroll
  for (int r = warp; r < kAttKeys; r += kAttThreads / 32) {
    float4 a = *reinterpret_cast<const float4*>(st + r * kAttD + c4);
    if (r >= valid) a = make_float4(0.f, 0.f, 0.f, 0.f);
    amax = fmaxf(fmaxf(amax, fabsf(a.x)), fmaxf(fabsf(a.y), fmaxf(fabsf(a.z), fabsf(a.w))));
    *reinterpret_cast<uint2*>(dst + sw_off(r, c4)) = make_uint2(pack2(a.x, a.y), pack2(a.z, a.w));
  }
  return amax;
}

// V^T of a row-major fp32 staging tile [128 keys][128 dims]: thread (g, p)
// writes rows 2p and 2p + 1 of the operand (keys along K) for the groups of
// 8 keys g, g + kCG', ... (kCG' = kAttThreads / 64), keys >= valid as zeros.
// Each 8-byte load instruction of a warp reads 256 consecutive bytes of one
// key row.  Returns the largest |value| converted.
__device__ __forceinline__ float convert_vt(uint8_t* dst, const float* st, int valid) {
  constexpr int kGroups = kAttThreads / 64;
  const int p = threadIdx.x & 63, g = threadIdx.x >> 6;
  float amax = 0.f;
#pragma unroll
  for (int kg = g; kg < kAttKeys / 8; kg += kGroups) {
    float2 x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = kg * 8 + j;
      x[j] = t < valid ? *reinterpret_cast<const float2*>(st + t * kAttD + 2 * p)
                       : make_float2(0.f, 0.f);
      amax = fmaxf(amax, fmaxf(fabsf(x[j].x), fabsf(x[j].y)));
    }
    *reinterpret_cast<uint4*>(dst + sw_off(2 * p, kg * 8)) =
        make_uint4(pack2(x[0].x, x[1].x), pack2(x[2].x, x[3].x), pack2(x[4].x, x[5].x),
                   pack2(x[6].x, x[7].x));
    *reinterpret_cast<uint4*>(dst + sw_off(2 * p + 1, kg * 8)) =
        make_uint4(pack2(x[0].y, x[1].y), pack2(x[2].y, x[3].y), pack2(x[4].y, x[5].y),
                   pack2(x[6].y, x[7].y));
  }
  return amax;
}

// 32 consecutive fp32 TMEM columns of this warp's 32 lanes <- r.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  uint32_t a[16], b[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    a[j] = r[j];
    b[j] = r[16 + j];
  }
  tmem_st16(taddr, a);
  tmem_st16(taddr + 16, b);
}

}  // namespace

__global__ void __launch_bounds__(kAttThreads, 1)
    attention_kernel(const __grid_constant__ AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  AttnCtl* ctl = reinterpret_cast<AttnCtl*>(smem + kOffCtl);
  const float* stk = reinterpret_cast<const float*>(smem + kOffStK);
  const float* stv = reinterpret_cast<const float*>(smem + kOffStV);
  // float [kCG][128] for combining the four threads of a row: the fp16 K
  // tile, free from the completion of S = Q K^T until the next tile's
  // conversion (and after the last tile).
  float* red = reinterpret_cast<float*>(smem + kOffK);
  const uint32_t sbase = smem_u32(smem);
  volatile int* abort = &ctl->abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rloc = (warp & 3) * 32 + lane;  // this thread's row (TMEM lane)
  const int cg = warp >> 2;                 // its column group

  // (segment, query block, head) of this CTA
  const int head = static_cast<int>(blockIdx.x % static_cast<unsigned>(args.n_heads));
  const int qb = static_cast<int>(blockIdx.x / static_cast<unsigned>(args.n_heads));
  int si = 0;
  for (int i = 1; i < args.n_segs; ++i)
    if (qb >= args.segs[i].qblock0) si = i;
  const AttnSeg& sg = args.segs[si];
  const int row0 = (qb - sg.qblock0) * kAttRows;
  const int S = sg.rows;
  const int kv = head / args.group;
  const int ntiles = (S + kAttKeys - 1) / kAttKeys;
  const int kx = sg.kv_x + kv * kAttD;

  if (tid == 0) {
    mbar_init(smem_u32(&ctl->ld_k), 1);
    mbar_init(smem_u32(&ctl->ld_v), 1);
    mbar_init(smem_u32(&ctl->mma_s), 1);
    mbar_init(smem_u32(&ctl->mma_o), 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const uint32_t s_col = tmem + lane_off + kColS + static_cast<uint32_t>(cg * kGCols);
  const uint32_t p_col = tmem + lane_off + kColP + static_cast<uint32_t>(cg * kGCols / 2);
  const uint32_t o_col = tmem + lane_off + kColO + static_cast<uint32_t>(cg * kGCols);
  uint32_t ph_k = 0, ph_v = 0, ph_s = 0, ph_o = 0;
  bool ok = true;
  float amax = 0.f;  // largest |q|, |k|, |v| converted (fp16 range check)
  auto wait = [&](uint64_t* bar, uint32_t& phase) {
    if (!ovb_wait(smem_u32(bar), phase, abort)) {
      ok = false;
      *abort = 1;
    }
    phase ^= 1u;
  };

  if (tid == 0) {
    mbar_arrive_expect_tx(smem_u32(&ctl->ld_v), kF32Tile);
    tma_load_2d(sbase + kOffStV, &args.tm_q, sg.q_x + head * kAttD, sg.q_y + row0,
                smem_u32(&ctl->ld_v));
    mbar_arrive_expect_tx(smem_u32(&ctl->ld_k), kF32Tile);
    tma_load_2d(sbase + kOffStK, &args.tm_k, kx, sg.kv_y, smem_u32(&ctl->ld_k));
  }
  wait(&ctl->ld_v, ph_v);
  amax = fmaxf(amax, convert_rows(smem + kOffQ, stv, S - row0));
  __syncthreads();  // staging of V free again
  if (tid == 0) {
    mbar_arrive_expect_tx(smem_u32(&ctl->ld_v), kF32Tile);
    tma_load_2d(sbase + kOffStV, &args.tm_v, kx, sg.kv_y, smem_u32(&ctl->ld_v));
  }

  const int row = row0 + rloc;
  const bool row_ok = row < S;
  const bool has_bias = sg.bias != nullptr;
  // (S % 4 == 0 with a 16-byte aligned base: every bias row and every 4-key
  // group of a tile is 16-byte aligned and lies wholly inside or past the row)
  const bool bias_vec = (S & 3) == 0 && (reinterpret_cast<uintptr_t>(sg.bias) & 15) == 0;
  // The bias tile [128 rows][128 keys] staged in the K staging buffer as
  // 16-byte chunks, chunk c of row r at position c ^ (r % 8): the eight rows
  // that a quarter-warp reads at one key group fall in distinct banks.
  float4* bst = reinterpret_cast<float4*>(smem + kOffStK);
  constexpr int kWarps = kAttThreads / 32;
  constexpr int kBRows = kAttRows / kWarps;  // bias rows each warp loads per tile
  float m = -INFINITY;   // softmax reference point (running max - 8 <= m <= running max)
  float mt = -INFINITY;  // running maximum of this thread's scores (fully-masked test)
  float l = 0.f;         // this thread's part of the sum of exp(score - m)

  for (int t = 0; t < ntiles; ++t) {
    const int valid = S - t * kAttKeys;
    // The tile's bias, loaded by whole rows (warp w rows w, w + kWarps, ...;
    // lane l keys 4l .. 4l + 3: one 512-byte row per warp instruction) while
    // the conversions and the MMA run.
    float4 bv[kBRows];
    if (has_bias) {
      const int kb = t * kAttKeys + lane * 4;
#pragma unroll
      for (int i = 0; i < kBRows; ++i) {
        const int r = row0 + warp + i * kWarps;
        const bool in = r < S;
        const float* p = sg.bias + static_cast<int64_t>(in ? r : 0) * S + kb;
        if (bias_vec) {
          bv[i] = ld_f4_if(p, in && kb < S);
        } else {
          bv[i].x = in && kb < S ? p[0] : 0.f;
          bv[i].y = in && kb + 1 < S ? p[1] : 0.f;
          bv[i].z = in && kb + 2 < S ? p[2] : 0.f;
          bv[i].w = in && kb + 3 < S ? p[3] : 0.f;
        }
      }
    }
    wait(&ctl->ld_k, ph_k);
    amax = fmaxf(amax, convert_rows(smem + kOffK, stk, valid));
    if (t > 0) wait(&ctl->mma_o, ph_o);  // P V of the previous tile done: V^T and P free
    wait(&ctl->ld_v, ph_v);
    amax = fmaxf(amax, convert_vt(smem + kOffV, stv, valid));
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();  // operands staged, staging buffers free
    if (tid == 0) {
      if (t + 1 < ntiles) {
        const int ky = sg.kv_y + (t + 1) * kAttKeys;
        if (!has_bias) {  // with a bias, K's staging holds it until the scores are read
          mbar_arrive_expect_tx(smem_u32(&ctl->ld_k), kF32Tile);
          tma_load_2d(sbase + kOffStK, &args.tm_k, kx, ky, smem_u32(&ctl->ld_k));
        }
        mbar_arrive_expect_tx(smem_u32(&ctl->ld_v), kF32Tile);
        tma_load_2d(sbase + kOffStV, &args.tm_v, kx, ky, smem_u32(&ctl->ld_v));
      }
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kAttD / 16; ++kk) {
        const uint32_t off = static_cast<uint32_t>((kk >> 2) * (kF16Tile / 2) + (kk & 3) * 32);
        mma_f16_ss(tmem + kColS, sw128_kmajor_desc(sbase + kOffQ, off),
                   sw128_kmajor_desc(sbase + kOffK, off), idesc_f16(kAttRows, kAttKeys),
                   kk > 0 ? 1u : 0u);
      }
      tc_commit(smem_u32(&ctl->mma_s));
    }
    if (has_bias) {
#pragma unroll
      for (int i = 0; i < kBRows; ++i) {
        const int r = warp + i * kWarps;
        bst[r * (kAttKeys / 4) + (lane ^ (r & 7))] = bv[i];
      }
      __syncthreads();  // the bias tile is staged
    }
    wait(&ctl->mma_s, ph_s);
    tc_fence_after();

    // scores (scaled, biased, -inf past the segment) back into S; tile max
    const int key0 = t * kAttKeys + cg * kGCols;
    float tmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < kGCols / 32; ++c) {
      uint32_t u[32];
      tmem_ld32(s_col + static_cast<uint32_t>(c * 32), u);
      tc_wait_ld32(u);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const int kc = (cg * kGCols + c * 32 + j) >> 2;  // key group within the tile
        const float4 b = has_bias ? bst[rloc * (kAttKeys / 4) + (kc ^ (rloc & 7))]
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        const float bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + c * 32 + j + e;
          float x = __fmul_rn(__uint_as_float(u[j + e]), args.scale);
          if (has_bias) x = __fadd_rn(x, bb[e]);
          x = key < S ? x : -INFINITY;
          tmax = fmaxf(tmax, x);
          u[j + e] = __float_as_uint(x);
        }
      }
      tmem_st32(s_col + static_cast<uint32_t>(c * 32), u);
    }
    mt = fmaxf(mt, tmax);
    red[cg * kAttRows + rloc] = tmax;
    __syncthreads();  // also: every thread has read its bias
    if (has_bias && tid == 0 && t + 1 < ntiles) {
      fence_proxy_async();
      mbar_arrive_expect_tx(smem_u32(&ctl->ld_k), kF32Tile);
      tma_load_2d(sbase + kOffStK, &args.tm_k, kx, sg.kv_y + (t + 1) * kAttKeys,
                  smem_u32(&ctl->ld_k));
    }
#pragma unroll
    for (int g = 0; g < kCG; ++g) tmax = fmaxf(tmax, red[g * kAttRows + rloc]);
    float factor = 1.f;
    if (tmax > m + kRescale) {  // also the first finite tile max (m = -inf)
      factor = m == -INFINITY ? 0.f : __expf(__fsub_rn(m, tmax));
      l = __fmul_rn(l, factor);
      m = tmax;
    }
    tc_wait_st();
    if (t > 0 && __any_sync(0xffffffffu, factor != 1.f)) {
#pragma unroll
      for (int c = 0; c < kGCols / 32; ++c) {
        uint32_t u[32];
        tmem_ld32(o_col + static_cast<uint32_t>(c * 32), u);
        tc_wait_ld32(u);
#pragma unroll
        for (int j = 0; j < 32; ++j) u[j] = __float_as_uint(__fmul_rn(__uint_as_float(u[j]), factor));
        tmem_st32(o_col + static_cast<uint32_t>(c * 32), u);
      }
    }
    const float mexp = m == -INFINITY ? 0.f : m;
#pragma unroll
    for (int c = 0; c < kGCols / 32; ++c) {
      uint32_t u[32];
      tmem_ld32(s_col + static_cast<uint32_t>(c * 32), u);
      tc_wait_ld32(u);
      uint32_t pk[16];
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float p0 = __expf(__fsub_rn(__uint_as_float(u[2 * j]), mexp));
        const float p1 = __expf(__fsub_rn(__uint_as_float(u[2 * j + 1]), mexp));
        sum = __fadd_rn(sum, __fadd_rn(p0, p1));
        pk[j] = pack2(p0, p1);
      }
      l = __fadd_rn(l, sum);
      tmem_st16(p_col + static_cast<uint32_t>(c * 16), pk);
    }
    tc_wait_st();
    tc_fence_before();
    __syncthreads();  // P and the rescaled O of every row are in TMEM
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kAttKeys / 16; ++kk) {
        const uint32_t off = static_cast<uint32_t>((kk >> 2) * (kF16Tile / 2) + (kk & 3) * 32);
        mma_f16_ts(tmem + kColO, tmem + kColP + static_cast<uint32_t>(kk * 8),
                   sw128_kmajor_desc(sbase + kOffV, off), idesc_f16(kAttRows, kAttD),
                   (t > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(smem_u32(&ctl->mma_o));
    }
  }
  wait(&ctl->mma_o, ph_o);
  tc_fence_after();

  // ---- the row's total sum and maximum, then O / l to the output rows
  red[cg * kAttRows + rloc] = l;
  __syncthreads();
  float lsum = 0.f;
#pragma unroll
  for (int g = 0; g < kCG; ++g) lsum = __fadd_rn(lsum, red[g * kAttRows + rloc]);
  __syncthreads();
  red[cg * kAttRows + rloc] = mt;
  __syncthreads();
#pragma unroll
  for (int g = 0; g < kCG; ++g) mt = fmaxf(mt, red[g * kAttRows + rloc]);
  const bool masked = !(mt >= -1e29f);  // the reference's fully masked rows -> 0
  const float inv_l = masked || !(lsum > 0.f) ? 0.f : __frcp_rn(lsum);
  float* orow = args.out + sg.q_off + static_cast<int64_t>(head) * kAttD + cg * kGCols +
                static_cast<int64_t>(row_ok ? row : 0) * args.q_stride;
#pragma unroll
  for (int c = 0; c < kGCols / 32; ++c) {
    uint32_t u[32];
    tmem_ld32(o_col + static_cast<uint32_t>(c * 32), u);
    tc_wait_ld32(u);
    if (row_ok) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(orow + c * 32 + j) =
            make_float4(__fmul_rn(__uint_as_float(u[j]), inv_l),
                        __fmul_rn(__uint_as_float(u[j + 1]), inv_l),
                        __fmul_rn(__uint_as_float(u[j + 2]), inv_l),
                        __fmul_rn(__uint_as_float(u[j + 3]), inv_l));
    }
  }
  if (amax > 65504.f) atomicOr(&g_status_att, kErrAttRange);
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && (!ok || *abort)) atomicOr(&g_status_att, kErrAttWait);
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================ fp16 operands
// attention_h_kernel: the same attention on fp16 q / k / v (written once per
// layer by the q/k-norm + RoPE kernel), warp-specialised so that the tensor
// core, the softmax and the loads overlap.
//
// One CTA per (segment, block of 128 query rows, kv head, pair of the query
// heads that share it): the two heads' Q tiles stay in shared memory and every
// K / V tile is loaded once for both.  352 threads:
//   warps 0-3  softmax of head A (thread = query row = TMEM lane),
//   warps 4-7  softmax of head B,
//   warp 8     TMA producer: Q_A, Q_B once, then K and V tiles into a
//              two-stage ring (fp16, 128-byte swizzle, two 64-column boxes
//              per tile),
//   warp 9     TMEM allocator and MMA issuer (one thread),
//   warp 10    watcher: waits on the mbarriers the MMA issuer needs and meets
//              it on a named barrier, so that the issuer never waits on an
//              mbarrier while its MMAs are in flight.
// TMEM: S_A [0, 128), S_B [128, 256), O_A [256, 384), O_B [384, 512) fp32
// columns; P (fp16 pairs) overwrites the first 64 columns of its head's S.
// The MMA issue order ping-pongs the heads,
//     S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) ...
// so the tensor core computes one head's next scores while the other head's
// softmax runs.  MMAs of the CTA complete in issue order, so a head's S(i)
// being complete (its commit) means its P V(i - 1) is complete too: the
// softmax then owns O for a rescale, and P(i - 1) has been read before S(i)
// overwrote it.  V is the B operand of P V in MN-major form (the keys are
// its K dimension), read straight from the TMA layout.
//
// Masks: an optional tile table (ovb_attention_tiles) classes every
// (segment, query block, key tile): 0 every key attended, 1 mixed (128 x 128
// bits, one 16-byte load per row), 3 nothing attended (the tile is skipped by
// every role).  Without a table, tiles read the segment's fp32 bias (or none).
// Scores are kept in base-2 units (x = s * scale * log2 e), the softmax
// reference point m moves only when a tile's maximum exceeds it by more than
// 8 (P <= 256), and a row whose scores are all below -1e29 (the reference's
// fully masked rows) gives zeros, as ov::attention_head_f32 does.
namespace {

constexpr int kHThreads = 352;
constexpr int kHBarW = 1;  // named barrier of the MMA warp and the watcher warp
constexpr int kHMaxTiles = 256;  // key tiles per segment (32768 rows)
constexpr uint32_t kHBox = 128 * 128;         // bytes of one 64-column fp16 box (128 rows)
constexpr uint32_t kHTile = 2 * kHBox;        // one 128 x 128 fp16 tile
constexpr uint32_t kHOffQ = 0;                // Q_A, Q_B
constexpr uint32_t kHOffKV = 2 * kHTile;      // stage s: K at +2s tiles, V at +2s+1
constexpr uint32_t kHOffCtl = kHOffKV + 4 * kHTile;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kHRescale = 8.f;              // base-2 units

struct AttnHCtl {
  uint64_t q_full;
  uint64_t q_empty;      // the item's last S has read Q (MMA commit)
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_final[2];
  uint64_t o_free[2];    // the epilogue of head h has read O_h (128 arrivals)
  uint64_t list_full[2];   // the key-tile list of list slot b is written
  uint64_t list_empty[2];  // ... and read by the watcher and the 8 softmax warps
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int wabort;  // set by the watcher warp only (see its loop)
  int n_act[2];
  int16_t act[2][kHMaxTiles];  // key tiles with something to attend, in order
  // how each active tile's scores are formed: 0 plain (every key attended and
  // inside the segment), 1 masked (class-1 bits and / or the segment's end),
  // 2 biased (the segment's fp32 bias, no table); + 4 when the tile has
  // class-1 mask bits to read
  int8_t kind[2][kHMaxTiles];
};
// Arrivals that release a list slot: the watcher warp and the 8 softmax warps.
constexpr int kHListUsers = 9;

// One work item: (segment, block of 128 query rows, kv head, pair of the
// query heads sharing it), numbered from its segment's cta0.
struct HItem {
  int si, qb, kv, nh, head0, S, row0, nkt, kx;
};
constexpr size_t kAttHSmem = 1024 + kHOffCtl + sizeof(AttnHCtl);
static_assert(kAttHSmem <= 227 * 1024, "attention_h shared memory");
static_assert(sizeof(AttnHArgs) <= 32764, "attention_h kernel parameters");

// Shared-memory descriptor of an MN-major operand written by TMA with the
// 128-byte swizzle: 64-element (128-byte) rows along MN, one row per K index,
// 8-row groups SBO bytes apart, the next 64 MN elements LBO bytes further.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(lbo >> 4) << 16;
  d |= static_cast<uint64_t>(sbo >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// max(a, b, c) in one instruction (the 3-input form of max.f32).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (y0, y1) = (x0, x1) * m + n, one packed f32x2 FFMA (each lane an fma.rn).
__device__ __forceinline__ void fma2(float x0, float x1, float m, float n, float& y0, float& y1) {
  asm("{\n\t.reg .b64 a, b, c, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %4};\n\t"
      "mov.b64 c, {%5, %5};\n\tfma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(y0), "=f"(y1)
      : "f"(x0), "f"(x1), "f"(m), "f"(n));
}

// (s0, s1) += (a, b), one packed f32x2 FADD.
__device__ __forceinline__ void add2(float& s0, float& s1, float a, float b) {
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "f"(a), "f"(b));
}

__device__ __forceinline__ void bar_sync_n(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ HItem decode_item(const AttnHArgs& args, int it) {
  // the last segment whose first item is <= it (cta0 increases with the
  // index): a binary search, six parameter loads for 64 segments instead of
  // a scan of all of them
  int si = 0, hi = args.n_segs - 1;
  while (si < hi) {
    const int mid = (si + hi + 1) >> 1;
    if (args.segs[mid].cta0 <= it) si = mid; else hi = mid - 1;
  }
  const AttnHSeg& sg = args.segs[si];
  int rem = it - sg.cta0;
  const int pair = rem % args.pairs;
  rem /= args.pairs;
  HItem w;
  w.si = si;
  w.kv = rem % args.n_kv;
  w.qb = rem / args.n_kv;
  w.S = sg.rows;
  w.row0 = w.qb * 128;
  w.head0 = w.kv * args.group + 2 * pair;
  w.nh = min(2, args.group - 2 * pair);
  w.nkt = (w.S + 127) / 128;
  w.kx = sg.kv_x + w.kv * 128;
  return w;
}

}  // namespace

__global__ void __launch_bounds__(kHThreads, 1)
    attention_h_kernel(const __grid_constant__ AttnHArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  AttnHCtl* ctl = reinterpret_cast<AttnHCtl*>(smem + kHOffCtl);
  const uint32_t sbase = smem_u32(smem);
  volatile int* abort = &ctl->abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_items = args.n_items;
  // This CTA's work items, the same sequence for every role: the host's
  // schedule, or every gridDim.x-th item.
  const int bid = static_cast<int>(blockIdx.x), grid = static_cast<int>(gridDim.x);
  const int n_mine = args.sched ? args.cta_first[bid + 1] - args.cta_first[bid]
                                : (n_items > bid ? (n_items - bid + grid - 1) / grid : 0);
  auto item_at = [&](int k) {
    return args.sched ? static_cast<int>(args.order[args.cta_first[bid] + k]) : bid + k * grid;
  };

  if (tid == 0) {
    mbar_init(smem_u32(&ctl->q_full), 1);
    mbar_init(smem_u32(&ctl->q_empty), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&ctl->kv_full[i]), 1);
      mbar_init(smem_u32(&ctl->kv_empty[i]), 1);
      mbar_init(smem_u32(&ctl->s_full[i]), 1);
      mbar_init(smem_u32(&ctl->p_full[i]), 128);
      mbar_init(smem_u32(&ctl->o_final[i]), 1);
      mbar_init(smem_u32(&ctl->o_free[i]), 128);
      mbar_init(smem_u32(&ctl->list_full[i]), 1);
      mbar_init(smem_u32(&ctl->list_empty[i]), kHListUsers);
    }
    mbar_init(smem_u32(&ctl->mma_done), 1);
    ctl->abort = 0;
    ctl->wabort = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(&ctl->tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    // Per item: the whole warp writes the item's key-tile list into list
    // slot c & 1 (once the item two back has released it); lane 0 then
    // loads Q (once the previous item's last S has read its Q) and the key
    // tiles into the two-stage ring.
    bool ok = true;
    int c = 0, q_loads = 0;
    int64_t g = 0;  // key tiles loaded by this CTA
    for (int k = 0; k < n_mine && ok; ++k, ++c) {
      const int it = item_at(k);
      const HItem w = decode_item(args, it);
      const AttnHSeg& sg = args.segs[w.si];
      const int b = c & 1;
      if (c >= 2 &&
          !__all_sync(0xffffffffu, ovb_wait(smem_u32(&ctl->list_empty[b]),
                                            static_cast<uint32_t>((c >> 1) - 1) & 1u, abort))) {
        if (lane == 0) *abort = 1;
        ok = false;
        break;
      }
      int n = 0;
      for (int j0 = 0; j0 < w.nkt; j0 += 32) {
        const int j = j0 + lane;
        int cls = 3;
        if (j < w.nkt)
          cls = args.tile_class ? args.tile_class[sg.tile0 + w.qb * w.nkt + j] : (sg.bias ? 2 : 0);
        const bool on = cls != 3;
        const unsigned m = __ballot_sync(0xffffffffu, on);
        if (on) {
          const int at = n + __popc(m & ((1u << lane) - 1u));
          ctl->act[b][at] = static_cast<int16_t>(j);
          ctl->kind[b][at] = static_cast<int8_t>(
              (cls == 2 ? 2 : (cls == 1 || j * 128 + 128 > w.S ? 1 : 0)) | (cls == 1 ? 4 : 0));
        }
        n += __popc(m);
      }
      if (lane == 0) ctl->n_act[b] = n;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&ctl->list_full[b]));
        if (c >= 1 &&
            !ovb_wait(smem_u32(&ctl->q_empty), static_cast<uint32_t>(c - 1) & 1u, abort)) {
          *abort = 1;
          ok = false;
        }
        if (ok) {
          mbar_arrive_expect_tx(smem_u32(&ctl->q_full), static_cast<uint32_t>(w.nh) * kHTile);
          for (int h = 0; h < w.nh; ++h)
            for (int bx = 0; bx < 2; ++bx)
              tma_load_2d(sbase + kHOffQ + h * kHTile + bx * kHBox, &args.tm_q,
                          sg.q_x + (w.head0 + h) * 128 + bx * 64, sg.q_y + w.row0,
                          smem_u32(&ctl->q_full));
          ++q_loads;
        }
        for (int i = 0; i < n && ok; ++i, ++g) {
          const int st = static_cast<int>(g & 1);
          if (g >= 2 && !ovb_wait(smem_u32(&ctl->kv_empty[st]),
                                  static_cast<uint32_t>((g >> 1) - 1) & 1u, abort)) {
            *abort = 1;
            ok = false;
            break;
          }
          const int ky = sg.kv_y + ctl->act[b][i] * 128;
          const uint32_t kb = sbase + kHOffKV + (2 * st) * kHTile, vb = kb + kHTile;
          mbar_arrive_expect_tx(smem_u32(&ctl->kv_full[st]), 2 * kHTile);
          for (int bx = 0; bx < 2; ++bx) {
            tma_load_2d(kb + bx * kHBox, &args.tm_k, w.kx + bx * 64, ky, smem_u32(&ctl->kv_full[st]));
            tma_load_2d(vb + bx * kHBox, &args.tm_v, w.kx + bx * 64, ky, smem_u32(&ctl->kv_full[st]));
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    // every load lane 0 issued has landed before the CTA can exit
    if (lane == 0) {
      volatile int no_abort = 0;
      if (q_loads > 0)
        ovb_wait(smem_u32(&ctl->q_full), static_cast<uint32_t>(q_loads - 1) & 1u, &no_abort);
      for (int st = 0; st < 2 && st < g; ++st) {
        const int64_t last = ((g - 1 - st) / 2) * 2 + st;  // last tile loaded into stage st
        ovb_wait(smem_u32(&ctl->kv_full[st]), static_cast<uint32_t>(last >> 1) & 1u, &no_abort);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp meets the watcher (warp 10) on named barrier kHBarW
    // before each step; lane 0 issues.  A thread with MMAs in flight would
    // pay ~400 clocks for each mbarrier wait of its own, so the MMA warp
    // never waits on an mbarrier until its last commit.
    const uint32_t id_s = idesc_f16(128, 128);
    const uint32_t id_o = idesc_f16(128, 128) | (1u << 16);  // B (V) MN-major
    auto issue_s = [&](int h, int st) {
      if (lane != 0) return;
      const uint32_t qa = sbase + kHOffQ + h * kHTile;
      const uint32_t kb = sbase + kHOffKV + (2 * st) * kHTile;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = static_cast<uint32_t>((kk >> 2) * kHBox + (kk & 3) * 32);
        mma_f16_ss(tmem + h * 128, sw128_kmajor_desc(qa, off), sw128_kmajor_desc(kb, off), id_s,
                   kk > 0 ? 1u : 0u);
      }
      tc_commit(smem_u32(&ctl->s_full[h]));
    };
    auto issue_pv = [&](int h, int st, bool first) {
      if (lane != 0) return;
      const uint32_t vb = sbase + kHOffKV + (2 * st + 1) * kHTile;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ts(tmem + 256 + h * 128, tmem + h * 128 + kk * 8,
                   sw128_mnmajor_desc(vb + kk * 2048, kHBox, 1024), id_o,
                   (!first || kk > 0) ? 1u : 0u);
    };
    auto commit = [&](uint64_t* bar) {
      if (lane == 0) tc_commit(smem_u32(bar));
    };
    // one step: the watcher has seen what the next MMAs need (or gave up)
    auto step = [&]() {
      bar_sync_n(kHBarW, 64);
      tc_fence_after();
      return ctl->wabort == 0;
    };
    int c = 0;
    int64_t g = 0;
    bool go = true;
    for (int k = 0; k < n_mine && go; ++k, ++c) {
      const int it = item_at(k);
      const int nh = decode_item(args, it).nh;
      if (!step()) break;  // the item's list, its Q and (if any) its first key tile
      const int n = ctl->n_act[c & 1];
      if (n == 0) {
        commit(&ctl->q_empty);
        continue;
      }
      for (int h = 0; h < nh; ++h) issue_s(h, static_cast<int>(g & 1));
      if (n == 1) commit(&ctl->q_empty);  // the item's last S has been issued
      for (int i = 0; i < n; ++i, ++g) {
        const int st = static_cast<int>(g & 1);
        const bool more = i + 1 < n;
        if (!step()) {  // P_A(i) (and, at i = 0, O_A read by the last epilogue)
          go = false;
          break;
        }
        issue_pv(0, st, i == 0);
        if (!more) commit(&ctl->o_final[0]);
        if (more) {
          if (!step()) {  // K / V(i + 1)
            go = false;
            break;
          }
          issue_s(0, st ^ 1);
          if (nh == 1 && i + 2 == n) commit(&ctl->q_empty);
        }
        if (nh == 2) {
          if (!step()) {  // P_B(i)
            go = false;
            break;
          }
          issue_pv(1, st, i == 0);
          if (!more) commit(&ctl->o_final[1]);
        }
        commit(&ctl->kv_empty[st]);
        if (nh == 2 && more) {
          issue_s(1, st ^ 1);
          if (i + 2 == n) commit(&ctl->q_empty);
        }
      }
    }
    __syncwarp();
    // every MMA issued has completed before TMEM is freed
    if (lane == 0) {
      tc_commit(smem_u32(&ctl->mma_done));
      volatile int no_abort = 0;
      ovb_wait(smem_u32(&ctl->mma_done), 0u, &no_abort);
    }
    __syncwarp();
  } else if (warp == 10) {
    // ------------------------------------------------------------ watcher
    // The MMA warp's waits, in the MMA warp's order; each step ends in
    // exactly one bar.sync on kHBarW, also after a failed wait (then wabort,
    // which only this warp writes, stops the MMA warp at the same step).
    auto seen = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, ovb_wait(smem_u32(bar), parity, abort));
    };
    auto release = [&](bool got) {
      if (!got && lane == 0) {
        ctl->wabort = 1;
        *abort = 1;
      }
      bar_sync_n(kHBarW, 64);
      return got;
    };
    int c = 0;
    int64_t g = 0;
    int tiles[2] = {0, 0}, items[2] = {0, 0};  // per head: P tiles and finished outputs
    bool go = true;
    for (int k = 0; k < n_mine && go; ++k, ++c) {
      const int it = item_at(k);
      const int nh = decode_item(args, it).nh;
      const int b = c & 1;
      bool got = seen(&ctl->list_full[b], static_cast<uint32_t>(c >> 1) & 1u) &&
                 seen(&ctl->q_full, static_cast<uint32_t>(c) & 1u);
      const int n = got ? ctl->n_act[b] : 0;
      if (got && n > 0) got = seen(&ctl->kv_full[g & 1], static_cast<uint32_t>(g >> 1) & 1u);
      if (!release(got)) break;
      for (int i = 0; i < n; ++i, ++g) {
        const bool more = i + 1 < n;
        // P_h(i); before an item's first P V_h, the last epilogue of head h
        // has read O_h
        auto p_ready = [&](int h) {
          return seen(&ctl->p_full[h], static_cast<uint32_t>(tiles[h]) & 1u) &&
                 (i > 0 || items[h] == 0 ||
                  seen(&ctl->o_free[h], static_cast<uint32_t>(items[h] - 1) & 1u));
        };
        if (!release(p_ready(0))) {
          go = false;
          break;
        }
        ++tiles[0];
        if (more && !release(seen(&ctl->kv_full[(g + 1) & 1],
                                  static_cast<uint32_t>((g + 1) >> 1) & 1u))) {
          go = false;
          break;
        }
        if (nh == 2) {
          if (!release(p_ready(1))) {
            go = false;
            break;
          }
          ++tiles[1];
        }
      }
      if (!go) break;
      if (n > 0) {
        ++items[0];
        if (nh == 2) ++items[1];
      }
      if (lane == 0) mbar_arrive(smem_u32(&ctl->list_empty[b]));
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int h = warp >> 2;          // head of this warpgroup
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_col = tmem + lane_off + static_cast<uint32_t>(h * 128);
    const uint32_t o_col = tmem + lane_off + static_cast<uint32_t>(256 + h * 128);
    const float sl2 = args.scale * kLog2e;
    bool ok = true;
    int c = 0, tiles = 0, items = 0;  // this head's P tiles and finished outputs
    for (int k = 0; k < n_mine && ok; ++k, ++c) {
      const int it = item_at(k);
      const HItem w = decode_item(args, it);
      const AttnHSeg& sg = args.segs[w.si];
      const int b = c & 1;
      if (!__all_sync(0xffffffffu, ovb_wait(smem_u32(&ctl->list_full[b]),
                                            static_cast<uint32_t>(c >> 1) & 1u, abort))) {
        if (lane == 0) *abort = 1;
        break;
      }
      const int n_act = ctl->n_act[b];
      const int row = w.row0 + r;
      const bool row_ok = row < w.S;
      const bool mine = h < w.nh;
      float m = -INFINITY, mt = -INFINITY, l = 0.f;
      for (int i = 0; i < n_act && mine; ++i, ++tiles) {
        const int j = ctl->act[b][i];
        const int key0 = j * 128;
        const int kind = ctl->kind[b][i] & 3;  // warp-uniform
        const bool has_bits = (ctl->kind[b][i] & 4) != 0;
        // this row's mask bits start towards L1 while S is computed
        const uint4* bits_at =
            has_bits ? reinterpret_cast<const uint4*>(args.tile_bits) +
                           (static_cast<int64_t>(sg.tile0 + w.qb * w.nkt + j) * 128 + r)
                     : nullptr;
        if (has_bits) asm volatile("prefetch.global.L1 [%0];" ::"l"(bits_at));
        // the warp leaves together: its TMEM accesses are warp-collective
        if (!__all_sync(0xffffffffu, ovb_wait(smem_u32(&ctl->s_full[h]),
                                              static_cast<uint32_t>(tiles) & 1u, abort))) {
          ok = false;
          if (lane == 0) *abort = 1;
          break;
        }
        tc_fence_after();
        uint32_t u[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(s_col + static_cast<uint32_t>(c * 32), u[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) tc_wait_ld32(u[c]);
        // Pass 1: the tile maximum in base-2 units.  A plain tile needs only the
        // maximum of the raw scores (scale > 0); the others form every score
        // x (masked keys -inf) in place.
        float tmax, mul;
        if (kind == 0) {
          // four independent chains of 3-input maxima (short dependency chains)
          float mr[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 2)
              mr[(e >> 1) & 3] =
                  max3f(mr[(e >> 1) & 3], __uint_as_float(u[c][e]), __uint_as_float(u[c][e + 1]));
          tmax = __fmul_rn(max3f(mr[0], mr[1], fmaxf(mr[2], mr[3])), sl2);
          mul = sl2;
        } else {
          uint32_t bw[4];
          if (has_bits) {
            const uint4 b4 = __ldg(bits_at);
            bw[0] = b4.x; bw[1] = b4.y; bw[2] = b4.z; bw[3] = b4.w;
          } else {
            bw[0] = bw[1] = bw[2] = bw[3] = 0xffffffffu;
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {  // keys past the segment's end
            const int vc = w.S - key0 - 32 * c;
            bw[c] &= vc >= 32 ? 0xffffffffu : (vc <= 0 ? 0u : (1u << vc) - 1u);
          }
          tmax = -INFINITY;
          if (kind == 1) {
            float mr[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                const float x = ((bw[c] >> e) & 1u) ? __fmul_rn(__uint_as_float(u[c][e]), sl2)
                                                    : -INFINITY;
                mr[e & 3] = fmaxf(mr[e & 3], x);
                u[c][e] = __float_as_uint(x);
              }
            tmax = max3f(mr[0], mr[1], fmaxf(mr[2], mr[3]));
          } else {
            const float* brow = sg.bias + static_cast<int64_t>(row_ok ? row : 0) * w.S + key0;
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                const bool on = row_ok && ((bw[c] >> e) & 1u);
                const float b = on ? brow[c * 32 + e] : 0.f;
                const float x =
                    on ? __fmul_rn(__fadd_rn(__fmul_rn(__uint_as_float(u[c][e]), args.scale), b),
                                   kLog2e)
                       : -INFINITY;
                tmax = fmaxf(tmax, x);
                u[c][e] = __float_as_uint(x);
              }
          }
          mul = 1.f;
        }
        mt = fmaxf(mt, tmax);
        float factor = 1.f;
        if (tmax > m + kHRescale) {  // also the first finite maximum (m = -inf)
          factor = m == -INFINITY ? 0.f : ex2_approx(m - tmax);
          l = __fmul_rn(l, factor);
          m = tmax;
        }
        if (i > 0 && __any_sync(0xffffffffu, factor != 1.f)) {
          // 16 columns at a time: the row's scores stay live in registers
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {
            uint32_t o[16];
            tmem_ld16(o_col + static_cast<uint32_t>(c * 16), o);
            tc_wait_ld16(o);
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__fmul_rn(__uint_as_float(o[e]), factor));
            tmem_st16(o_col + static_cast<uint32_t>(c * 16), o);
          }
        }
        // Pass 2: P = 2^(x - m), x = u * mul (the raw score times scale log2 e
        // on a plain tile, x itself otherwise), one FFMA and one ex2 each.
        // Pairs of elements go through the packed f32x2 FFMA and FADD; the row
        // sum is kept in four partial sums (two f32x2 accumulators).
        const float nm = m == -INFINITY ? 0.f : -m;
        float sa[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0, x1;
            fma2(__uint_as_float(u[c][2 * e]), __uint_as_float(u[c][2 * e + 1]), mul, nm, x0, x1);
            const float p0 = ex2_approx(x0);
            const float p1 = ex2_approx(x1);
            add2(sa[e & 1][0], sa[e & 1][1], p0, p1);
            pk[e] = pack2(p0, p1);
          }
          tmem_st16(s_col + static_cast<uint32_t>(c * 16), pk);
        }
        const float sum = __fadd_rn(__fadd_rn(sa[0][0], sa[0][1]), __fadd_rn(sa[1][0], sa[1][1]));
        l += sum;
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&ctl->p_full[h]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl->list_empty[b]));  // done with the list
      if (!ok || !mine) continue;
      // ---- O / l to the output row
      const bool have_o =
          n_act > 0 && __all_sync(0xffffffffu, ovb_wait(smem_u32(&ctl->o_final[h]),
                                                        static_cast<uint32_t>(items) & 1u, abort));
      if (n_act > 0 && !have_o) {
        ok = false;
        if (lane == 0) *abort = 1;
        break;
      }
      if (have_o) tc_fence_after();
      const bool masked = !(mt >= -1e29f * kLog2e);
      const float inv_l = masked || !(l > 0.f) ? 0.f : __frcp_rn(l);
      float* orow = args.out ? args.out + sg.q_off + static_cast<int64_t>(w.head0 + h) * 128 +
                                   static_cast<int64_t>(row_ok ? row : 0) * args.q_stride
                             : nullptr;
      // quantised output: the head's 128 values are four whole 32-k blocks of
      // the o projection's input row (q_x is 0: rows of the 2-D view)
      const int64_t qrow = static_cast<int64_t>(sg.q_y) + (row_ok ? row : 0);
      const int es = args.q_mode == 2 ? 2 : 1;
      bool range_bad = false;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        if (have_o) {
          tmem_ld32(o_col + static_cast<uint32_t>(c * 32), o);
          tc_wait_ld32(o);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (!row_ok) continue;
        if (args.q_out) {
          float vq[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) vq[e] = __fmul_rn(__uint_as_float(o[e]), inv_l);
          const int64_t blk = static_cast<int64_t>(w.head0 + h) * 4 + c;
          const float bs = quant_block32_fast(
              vq, args.q_out + (qrow * args.q_kb * 32 + blk * 32) * es, args.q_mode, &range_bad);
          args.q_asc[qrow * args.q_kb + blk] = bs;
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(orow + c * 32 + e) =
                make_float4(__fmul_rn(__uint_as_float(o[e]), inv_l),
                            __fmul_rn(__uint_as_float(o[e + 1]), inv_l),
                            __fmul_rn(__uint_as_float(o[e + 2]), inv_l),
                            __fmul_rn(__uint_as_float(o[e + 3]), inv_l));
        }
      }
      if (range_bad) atomicOr(&g_status_att, kErrAttRange);
      if (have_o) {  // O_h read: the next item's first P V_h may overwrite it
        tc_fence_before();
        mbar_arrive(smem_u32(&ctl->o_free[h]));
        ++items;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort) atomicOr(&g_status_att, kErrAttWait);
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Tile table of a segment list from its u8 masks (ovb_attention_tiles): one
// CTA of 128 threads per (segment, query block, key tile); thread r packs the
// 128 mask bits of query row r (keys past the segment count as attended, rows
// past it are not looked at) and the CTA classes the tile.
__global__ void __launch_bounds__(128) attn_tiles_kernel(const __grid_constant__ AttnTilesArgs a,
                                                         uint8_t* cls, uint32_t* bits) {
  const int t = blockIdx.x;
  int si = 0;
  for (int i = 1; i < a.n_segs; ++i)
    if (t >= a.tile0[i]) si = i;
  const int S = a.rows[si];
  const int nkt = (S + 127) / 128;
  const int qb = (t - a.tile0[si]) / nkt, kt = (t - a.tile0[si]) % nkt;
  const int r = threadIdx.x;
  const int row = qb * 128 + r;
  const uint8_t* mrow = a.masks + a.mask_off[si] + static_cast<int64_t>(row) * S;
  uint32_t w[4];
  bool any0 = false, any1 = false;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t v = 0;
    for (int e = 0; e < 32; ++e) {
      const int key = kt * 128 + c * 32 + e;
      bool on = true;
      if (row < S && key < S) {
        on = mrow[key] != 0;
        any0 |= !on;
        any1 |= on;
      }
      v |= static_cast<uint32_t>(on) << e;
    }
    w[c] = v;
  }
  reinterpret_cast<uint4*>(bits)[static_cast<int64_t>(t) * 128 + r] = make_uint4(w[0], w[1], w[2], w[3]);
  const int n0 = __syncthreads_or(any0), n1 = __syncthreads_or(any1);
  if (r == 0) cls[t] = static_cast<uint8_t>(!n0 ? 0 : (!n1 ? 3 : 1));
}

cudaError_t launch_attention_h(const AttnHArgs& args, int ctas, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev = -1;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(attention_h_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kAttHSmem));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  // persistent: at most one CTA per SM (the shared memory allows no more)
  AttnHArgs a = args;
  a.n_items = ctas;
  const int grid = std::min(ctas, num_sms(dev));
  a.sched = 0;
  if (ctas <= kAttSchedItems && grid <= kAttSchedCtas) {
    // Longest processing time first: the items in decreasing estimated work
    // (the segment's key tiles, plus two for the item's epilogue), each to
    // the CTA with the least work so far; a CTA runs its items in the order
    // they were given to it.  Round-robin left the busiest CTA with ~15 %
    // more work than the mean on config 4's 32 segments.
    std::vector<std::pair<int, int>> work;  // (work, item)
    work.reserve(static_cast<size_t>(ctas));
    for (int i = 0; i < a.n_segs; ++i) {
      const int nkt = (a.segs[i].rows + 127) / 128;
      const int n = nkt * a.n_kv * a.pairs;
      for (int j = 0; j < n; ++j) work.emplace_back(nkt + 2, a.segs[i].cta0 + j);
    }
    std::stable_sort(work.begin(), work.end(),
                     [](const std::pair<int, int>& x, const std::pair<int, int>& y) {
                       return x.first > y.first;
                     });
    using Load = std::pair<int64_t, int>;  // (work so far, CTA)
    std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
    for (int b = 0; b < grid; ++b) heap.emplace(0, b);
    std::vector<std::vector<uint16_t>> per(static_cast<size_t>(grid));
    for (const auto& wi : work) {
      Load l = heap.top();
      heap.pop();
      per[static_cast<size_t>(l.second)].push_back(static_cast<uint16_t>(wi.second));
      l.first += wi.first;
      heap.push(l);
    }
    int at = 0;
    for (int b = 0; b < grid; ++b) {
      a.cta_first[b] = static_cast<uint16_t>(at);
      for (uint16_t it : per[static_cast<size_t>(b)]) a.order[at++] = it;
    }
    a.cta_first[grid] = static_cast<uint16_t>(at);
    a.sched = 1;
  }
  return launch_plain(attention_h_kernel, dim3(static_cast<unsigned>(grid)), dim3(kHThreads),
                      kAttHSmem, s, a);
}

cudaError_t launch_attn_tiles(const AttnTilesArgs& a, int tiles, uint8_t* cls, uint32_t* bits,
                              cudaStream_t s) {
  return launch_plain(attn_tiles_kernel, dim3(static_cast<unsigned>(tiles)), dim3(128), 0, s, a,
                      cls, bits);
}

cudaError_t launch_attention(const AttnArgs& args, int total_qblocks, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev = -1;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kAttSmem));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  // Plain launch: TMEM is allocated at entry, before any wait on the
  // preceding grid could be placed.
  return launch_plain(attention_kernel, dim3(static_cast<unsigned>(total_qblocks * args.n_heads)),
                      dim3(kAttThreads), kAttSmem, s, args);
}

cudaError_t read_and_clear_status_att(int* out, cudaStream_t s) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_status_att, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_status_att, &zero, sizeof(int));
}

}  // namespace ovb
