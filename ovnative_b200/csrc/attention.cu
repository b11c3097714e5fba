// attention.cu -- the attention of one OVNative LM layer on the tensor cores:
// for every attention segment (one half of a CFG pair: its q/k/v rows, an
// additive bias [rows, rows] or none) and query head h (kv head h / group),
//
//   out = softmax(q k^T * scale + bias) v,  rows whose scores are all below
//   -1e29 (fully masked) -> 0,
//
// as ov::attention_head_f32 computes it (cpp/src/backend/cpu/ops_cpu.cpp:
// 907-943, called per (segment, head) by LM::run_layer, cpp/src/model/
// lm.cpp:256-274; the reference's CUDA runner uses a SIMT fp32 kernel,
// cpp/src/backend/cuda/cuda_lm.cu:434-606).  head_dim is 128.
//
// One CTA of 128 threads per (segment, head, block of 128 query rows); thread
// r owns query row r, i.e. TMEM lane r.  Q, K and V^T tiles are converted to
// fp16 and stored in shared memory in the 128-byte-swizzled K-major layout
// the MMA reads (two 64-wide K chunks per 128 x 128 tile).  Two passes over
// the key tiles (128 keys each):
//   1. S = Q K^T (tcgen05.mma kind::f16, fp32 in TMEM); each thread folds its
//      row into a running max and sum of exp (the softmax statistics);
//   2. S again (skipped with a single key tile), P = exp(S - max) / sum in
//      fp16 written into TMEM, O += P V with P as the A operand from TMEM.
// The two passes cost a second Q K^T instead of rescaling O in TMEM.  The
// fp16 inputs make the result agree with the fp32 reference to ~1e-3
// relative (the fp16 GEMM path's own rounding is 2^-11 per element).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "ovb_internal.h"
#include "ovb_ptx.cuh"

namespace ovb {

__device__ int g_status_att;

namespace {

constexpr int kErrAttWait = 32;  // an MMA-completion wait gave up
constexpr int kAttD = 128;
constexpr int kAttRows = 128;     // query rows per CTA = TMEM lanes
constexpr int kAttKeys = 128;     // keys per tile
constexpr int kAttThreads = 128;
constexpr uint32_t kTileBytes = 128 * 128 * 2;  // one fp16 operand tile
constexpr uint32_t kColS = 0, kColP = 128, kColO = 256, kTmemCols = 512;

struct AttnCtl {
  uint64_t mma;  // one arrival per committed MMA group
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 8 fp16 values of row r, K columns c8 .. c8+7 (c8 a multiple of 8) of a
// 128 x 128 operand stored as two K chunks of [128 rows][64 fp16] with the
// 128-byte swizzle (16-byte chunk j of row r at position j ^ (r % 8)).
__device__ __forceinline__ void put8(uint8_t* tile, int r, int c8, uint4 v) {
  const int chunk = c8 >> 6, j = (c8 & 63) >> 3;
  *reinterpret_cast<uint4*>(tile + chunk * (kTileBytes / 2) + r * 128 + ((j ^ (r & 7)) << 4)) = v;
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Rows [row0, row0 + 128) (beyond `rows`: zeros) x 128 columns of a
// row-major fp32 matrix (row stride `stride`) into `tile` as fp16.  Each warp
// reads two 512-byte rows per step.
__device__ __forceinline__ void stage_rows(uint8_t* tile, const float* src, int64_t stride,
                                           int row0, int rows) {
#pragma unroll 4
  for (int i = threadIdx.x; i < 128 * 16; i += kAttThreads) {
    const int r = i >> 4, c8 = (i & 15) * 8;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (row0 + r < rows) {
      const float* p = src + static_cast<int64_t>(row0 + r) * stride + c8;
      a = *reinterpret_cast<const float4*>(p);
      b = *reinterpret_cast<const float4*>(p + 4);
    }
    put8(tile, r, c8, make_uint4(pack2(a.x, a.y), pack2(a.z, a.w), pack2(b.x, b.y),
                                 pack2(b.z, b.w)));
  }
}

// V^T of key rows [row0, row0 + 128): tile row d holds v[row0 .. row0+127][d]
// (keys along K).  Lane l reads dimension 32*q + l of 8 consecutive keys, so
// every load instruction of a warp is one 128-byte segment of a key row.
__device__ __forceinline__ void stage_vt(uint8_t* tile, const float* v, int64_t stride, int row0,
                                         int rows) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int item = warp; item < 4 * 16; item += kAttThreads / 32) {
    const int q = item & 3, kg = item >> 2;  // dimension quarter, key group of 8
    const int d = 32 * q + lane;
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = row0 + kg * 8 + j;
      x[j] = t < rows ? v[static_cast<int64_t>(t) * stride + d] : 0.f;
    }
    put8(tile, d, kg * 8, make_uint4(pack2(x[0], x[1]), pack2(x[2], x[3]), pack2(x[4], x[5]),
                                     pack2(x[6], x[7])));
  }
}

}  // namespace

__global__ void __launch_bounds__(kAttThreads, 1)
    attention_kernel(const __grid_constant__ AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* qs = smem;
  uint8_t* ks = qs + kTileBytes;
  uint8_t* vt = ks + kTileBytes;
  AttnCtl* ctl = reinterpret_cast<AttnCtl*>(vt + kTileBytes);
  volatile int* abort = &ctl->abort;
  const int tid = threadIdx.x, warp = tid >> 5;

  // (segment, query block, head) of this CTA
  const int head = static_cast<int>(blockIdx.x % static_cast<unsigned>(args.n_heads));
  const int qb = static_cast<int>(blockIdx.x / static_cast<unsigned>(args.n_heads));
  int si = 0;
  for (int i = 1; i < args.n_segs; ++i)
    if (qb >= args.segs[i].qblock0) si = i;
  const AttnSeg sg = args.segs[si];
  const int row0 = (qb - sg.qblock0) * kAttRows;
  const int S = sg.rows;
  const int kv = head / args.group;
  const float* qbase = args.q + sg.q_off + static_cast<int64_t>(head) * kAttD;
  const float* kbase = args.k + sg.kv_off + static_cast<int64_t>(kv) * kAttD;
  const float* vbase = args.v + sg.kv_off + static_cast<int64_t>(kv) * kAttD;
  const int ntiles = (S + kAttKeys - 1) / kAttKeys;

  if (tid == 0) {
    mbar_init(smem_u32(&ctl->mma), 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  stage_rows(qs, qbase, args.q_stride, row0, S);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t idesc = idesc_f16(kAttRows, kAttKeys);
  uint32_t phase = 0;
  bool ok = true;
  // Wait for the last committed MMA group; after one wait gives up, every
  // later wait of the CTA returns at once (the outputs are then invalid and
  // status bit 32 is set).
  auto wait_mma = [&]() {
    if (!ovb_wait(smem_u32(&ctl->mma), phase, abort)) {
      ok = false;
      *abort = 1;
    }
    phase ^= 1u;
  };

  // S = Q K^T for the staged key tile, then wait for it (all threads).
  auto qk = [&]() {
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kAttD / 16; ++kk) {
        const uint32_t off = static_cast<uint32_t>((kk >> 2) * (kTileBytes / 2));
        const uint32_t kb = static_cast<uint32_t>((kk & 3) * 32);
        mma_f16_ss(tmem + kColS, sw128_kmajor_desc(smem_u32(qs) + off, kb),
                   sw128_kmajor_desc(smem_u32(ks) + off, kb), idesc, kk > 0 ? 1u : 0u);
      }
      tc_commit(smem_u32(&ctl->mma));
    }
    wait_mma();
    tc_fence_after();
  };

  // This thread's scores of key tile `t` (chunk c of 32 keys), scaled, biased
  // and masked past the segment.
  const int row = row0 + tid;
  const bool row_ok = row < S;
  const float* brow = sg.bias ? sg.bias + static_cast<int64_t>(row_ok ? row : 0) * S : nullptr;
  auto scores = [&](int t, int c, float (&x)[32]) {
    uint32_t u[32];
    tmem_ld32(tmem + lane_off + kColS + static_cast<uint32_t>(c * 32), u);
    tc_wait_ld32(u);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int key = t * kAttKeys + c * 32 + j;
      float s = __fmul_rn(__uint_as_float(u[j]), args.scale);
      if (brow && key < S) s = __fadd_rn(s, brow[key]);
      x[j] = key < S ? s : -INFINITY;
    }
  };

  // ---- pass 1: running max and sum of exp per row
  float m = -INFINITY, l = 0.f;
  for (int t = 0; t < ntiles; ++t) {
    stage_rows(ks, kbase, args.kv_stride, t * kAttKeys, S);
    fence_proxy_async();
    __syncthreads();
    qk();
    for (int c = 0; c < kAttKeys / 32; ++c) {
      float x[32];
      scores(t, c, x);
      float cm = m;
#pragma unroll
      for (int j = 0; j < 32; ++j) cm = fmaxf(cm, x[j]);
      if (cm > -INFINITY) {
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) sum = __fadd_rn(sum, __expf(__fsub_rn(x[j], cm)));
        l = __fadd_rn(__fmul_rn(l, __expf(__fsub_rn(m, cm))), sum);
        m = cm;
      }
    }
    tc_fence_before();
    __syncthreads();  // the key tile and S are reused
  }
  const bool masked = !(m >= -1e29f);  // the reference's fully masked rows -> 0
  const float inv_l = masked || l <= 0.f ? 0.f : __fdividef(1.f, l);

  // ---- pass 2: P = exp(S - m) / l into TMEM, O += P V
  for (int t = 0; t < ntiles; ++t) {
    if (ntiles > 1) stage_rows(ks, kbase, args.kv_stride, t * kAttKeys, S);
    stage_vt(vt, vbase, args.kv_stride, t * kAttKeys, S);
    fence_proxy_async();
    __syncthreads();
    if (ntiles > 1) qk();
    for (int c = 0; c < kAttKeys / 32; ++c) {
      float x[32];
      scores(t, c, x);
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        pk[j] = pack2(__fmul_rn(__expf(__fsub_rn(x[2 * j], m)), inv_l),
                      __fmul_rn(__expf(__fsub_rn(x[2 * j + 1], m)), inv_l));
      tmem_st16(tmem + lane_off + kColP + static_cast<uint32_t>(c * 16), pk);
    }
    tc_wait_st();
    tc_fence_before();
    __syncthreads();  // P of every row is in TMEM
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kAttKeys / 16; ++kk) {
        const uint32_t off = static_cast<uint32_t>((kk >> 2) * (kTileBytes / 2));
        const uint32_t kb = static_cast<uint32_t>((kk & 3) * 32);
        mma_f16_ts(tmem + kColO, tmem + kColP + static_cast<uint32_t>(kk * 8),
                   sw128_kmajor_desc(smem_u32(vt) + off, kb), idesc_f16(kAttRows, kAttD),
                   (t > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(smem_u32(&ctl->mma));
    }
    wait_mma();
    tc_fence_after();
    __syncthreads();  // V^T, the key tile, S and P are reused
  }

  // ---- O (already normalised) to the output rows
  if (tid == 0 && (!ok || *abort)) atomicOr(&g_status_att, kErrAttWait);
  float* orow = args.out + sg.q_off + static_cast<int64_t>(head) * kAttD +
                static_cast<int64_t>(row_ok ? row : 0) * args.q_stride;
  for (int c = 0; c < kAttD / 32; ++c) {
    uint32_t u[32];
    tmem_ld32(tmem + lane_off + kColO + static_cast<uint32_t>(c * 32), u);
    tc_wait_ld32(u);
    if (row_ok) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(orow + c * 32 + j) =
            masked ? make_float4(0.f, 0.f, 0.f, 0.f)
                   : make_float4(__uint_as_float(u[j]), __uint_as_float(u[j + 1]),
                                 __uint_as_float(u[j + 2]), __uint_as_float(u[j + 3]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

cudaError_t launch_attention(const AttnArgs& args, int total_qblocks, cudaStream_t s) {
  constexpr size_t kSmem = 1024 + 3 * kTileBytes + sizeof(AttnCtl) + 20 * 1024;  // 1 CTA / SM
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev = -1;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmem));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  // Plain launch: TMEM is allocated at entry, before any wait on the
  // preceding grid could be placed.
  return launch_plain(attention_kernel, dim3(static_cast<unsigned>(total_qblocks * args.n_heads)),
                    dim3(kAttThreads), kSmem, s, args);
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
