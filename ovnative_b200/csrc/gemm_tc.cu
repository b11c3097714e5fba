// gemm_tc.cu -- int8 x per-32-k-quantised-activation GEMM on the sm_100a
// tensor cores (tcgen05 kind::i8, accumulators in TMEM, operands staged by
// TMA), with the reference's per-block rescale epilogue.
//
// What it computes (gemm.cpp:432-504, linear_s8_nk_vnni_tile_at):
//   for every output (m, n):
//     f = 0
//     for b in 0 .. Kb-1:   P_b = sum_{k in block b} q[m,k] * w[n,k]    (exact int32)
//                           f   = fma((float)P_b, asc[m,b], f)
//     o = f * wscale[n];  if accumulate: o = o + C[m,n]
// so the fp32 result is bit-identical to the reference's.
//
// Mapping.  One quantisation block (32 k) is one tcgen05.mma.kind::i8 with
// K = 32, M = 128 rows of activations, N = 128 output channels.  Each block's
// int32 product lands in its own TMEM accumulator (a ring of four 128-column
// buffers = all 512 TMEM columns), so the tensor core runs up to four blocks
// ahead of the fp32 epilogue.  TMA moves 128-byte-wide boxes (four blocks of
// K, 128-byte swizzle); each MMA's descriptor points at its 32-byte K slice.
//
// Warp roles (608 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A box (128 B x 128 rows of aq) and B box (128 B
//               x 128 rows of the packed weight) per stage into a 4-stage ring;
//   warp 1      TMEM allocator + MMA issuer (lane 0 issues, the whole warp
//               takes part in the named barriers);
//   warps 2..17 epilogue: warp w reads TMEM lanes 32*(w%4).. (the lane quarter
//               it may access) and 32 of the 128 columns, converts each
//               block's int32 products and folds them into 32 fp32 running
//               sums per thread; at the end of the tile it stages the values
//               in shared memory and writes them row by row (coalesced) with
//               wscale and the optional residual applied.  Four epilogue
//               warps per SM sub-partition let one warp's barrier wait and
//               TMEM load overlap the others' arithmetic;
//   warp 18     stage watcher: waits for each TMA stage to land and hands it
//               to the MMA warp.
//
// Handshakes.  A thread that has tcgen05.mma operations in flight stalls on
// any shared-memory access of its own (an mbarrier wait included) until
// those MMAs have read their operands -- measured here at ~400 clocks per
// access, six times the 64-clock issue interval of a 128x128x32 int8 MMA.
// So the MMA warp never waits on an mbarrier inside its loop.  It meets the
// stage watcher on named barrier kBarFull (bar.sync, 64 threads, lockstep)
// once per stage.  TMEM holds four block accumulators as two slots of two
// (kGroup blocks per handshake): the MMA warp commits a slot's barrier once
// both of its blocks are issued, waits on named barrier kBarTmem + g
// (bar.sync, 544 threads) before refilling slot g, and the sixteen epilogue
// warps signal that slot with bar.arrive after reading it -- so while the
// epilogue drains one slot the tensor core fills the other.  Each slot's
// arrivals and syncs alternate strictly, and every participant executes its
// full count on every path (on an error it keeps signalling without doing
// work), so no named barrier can be left waiting.
//
#include "ovb_internal.h"
#include "ovb_ptx.cuh"

namespace ovb {

__device__ int g_status;

namespace {

constexpr int kBlocksPerStage = kStageK / 32;  // quantisation blocks per TMA box
constexpr int kStages = 4;
constexpr int kAccBufs = 4;
constexpr int kGroup = 2;                        // blocks per TMEM handshake
constexpr int kGroups = kAccBufs / kGroup;      // TMEM group slots
constexpr uint32_t kTmemCols = 512;
constexpr int kEpiWarps = 16;
constexpr int kWatcherWarp = 2 + kEpiWarps;
constexpr int kThreads = 32 * (3 + kEpiWarps);
// named barriers (0 is __syncthreads)
constexpr int kBarFull = 1;  // stage landed: watcher warp + MMA warp
constexpr int kBarTmem = 2;  // kBarTmem + g: TMEM group slot g free: epilogue warps + MMA warp
constexpr int kBarFullThreads = 64;
constexpr int kBarTmemThreads = 32 * (kEpiWarps + 1);
constexpr uint32_t kABytes = kBlockM * kStageK;
constexpr uint32_t kBBytes = kBlockN * kStageK;
constexpr uint32_t kStageBytes = kABytes + kBBytes;
// Per epilogue warp: its 32 rows x kEpiCols columns of the finished tile,
// rows padded by one float so both the row-wise writes and the column-wise
// reads are free of bank conflicts.
constexpr int kEpiCols = kBlockN / (kEpiWarps / 4);  // columns per epilogue warp
constexpr int kStgStride = kEpiCols + 1;
constexpr uint32_t kStgBytes = 32 * kStgStride * 4;
static_assert(kAccBufs * kBlockN <= static_cast<int>(kTmemCols), "TMEM ring too large");
static_assert(kEpiCols == 32, "the epilogue reads one 32-column TMEM slice per block");
static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "128B-swizzle tiles need 1 KB bases");

// status codes recorded in g_status (bit flags)
constexpr int kErrProducer = 1;
constexpr int kErrMma = 2;
constexpr int kErrEpilogue = 4;
constexpr int kErrDrain = 8;

struct Ctl {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[kGroups];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStages) * kStageBytes +
                              static_cast<size_t>(kEpiWarps) * kStgBytes + sizeof(Ctl);

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void named_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void fail(Ctl* ctl, int code) {
  atomicOr(&g_status, code);
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
}

// Block scales of rows m for blocks b0..b0+3 (zero past Kb or for rows >= M).
__device__ __forceinline__ float4 load_scales4(const float* asc_row, int64_t b0, int64_t Kb,
                                               bool row_ok, bool vec) {
  if (!row_ok) return make_float4(0.f, 0.f, 0.f, 0.f);
  if (vec) return __ldg(reinterpret_cast<const float4*>(asc_row + b0));
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = (b0 + i < Kb) ? __ldg(asc_row + b0 + i) : 0.f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

template <bool kProducts>
// 19 warps: five share one SM sub-partition's 16K registers, so at most 96
// registers per thread.
__global__ void __launch_bounds__(kThreads, 1)
    gemm_s8_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* stg_all = reinterpret_cast<float*>(smem + static_cast<size_t>(kStages) * kStageBytes);
  Ctl* ctl = reinterpret_cast<Ctl*>(reinterpret_cast<uint8_t*>(stg_all) +
                                    static_cast<size_t>(kEpiWarps) * kStgBytes);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int64_t M = args.M, N = args.N, Kb = args.Kb;
  const int64_t ksteps = (Kb + kBlocksPerStage - 1) / kBlocksPerStage;
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  const int64_t n_tiles = (N + kBlockN - 1) / kBlockN;
  const int64_t tiles = m_tiles * n_tiles;
  const int64_t my_tiles =
      tiles > blockIdx.x ? (tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int64_t tile_groups = (Kb + kGroup - 1) / kGroup;
  const int64_t my_groups = my_tiles * tile_groups;  // TMEM handshakes of this CTA

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int g = 0; g < kGroups; ++g) mbar_init(smem_u32(&ctl->tfull[g]), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One stage = kStageK bytes of K (kBlocksPerStage quantisation blocks)
    // of the A tile (128 activation rows) and the B tile (128 weight rows).
    if (lane == 0) {
      int64_t st = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int32_t m0 = static_cast<int32_t>((tile % m_tiles) * kBlockM);
        const int32_t n0 = static_cast<int32_t>((tile / m_tiles) * kBlockN);
        for (int64_t j = 0; j < ksteps; ++j, ++st) {
          const int s = static_cast<int>(st % kStages);
          const uint32_t ph = static_cast<uint32_t>((st / kStages) & 1);
          if (!ovb_wait(smem_u32(&ctl->empty[s]), ph ^ 1u, abort)) {
            fail(ctl, kErrProducer);
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&ctl->full[s]);
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * kStageBytes);
          mbar_arrive_expect_tx(full, kStageBytes);
          const int32_t x = static_cast<int32_t>(j * kStageK);
          tma_load_2d(sa, &tmap_a, x, m0, full);
          tma_load_2d(sa + kABytes, &tmap_b, x, n0, full);
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA's shared memory
        // is released: wait (bounded) on the last min(st, kStages) stages.
        const int64_t first = st > kStages ? st - kStages : 0;
        for (int64_t j = first; j < st; ++j) {
          const int s = static_cast<int>(j % kStages);
          const uint32_t ph = static_cast<uint32_t>((j / kStages) & 1);
          volatile int never = 0;
          ovb_wait(smem_u32(&ctl->full[s]), ph, &never);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    // One K = 32 MMA per quantisation block, each into its own TMEM buffer.
    // The whole warp walks the loop (named barriers count warps); lane 0
    // issues.  No shared-memory access happens here until the final drain.
    const uint32_t idesc = idesc_i8(kBlockM, kBlockN);
    int64_t st = 0, q = 0;
    for (int64_t t = 0; t < my_tiles; ++t) {
      uint32_t sa = 0;
      int s = 0;
      for (int64_t b = 0; b < Kb; ++b) {
        const int kk = static_cast<int>(b % kBlocksPerStage);
        if (kk == 0) {
          s = static_cast<int>(st % kStages);
          named_sync(kBarFull, kBarFullThreads);  // stage s has landed
          sa = smem_u32(smem + static_cast<size_t>(s) * kStageBytes);
        }
        const int g = static_cast<int>(q % kGroups);
        const int in_group = static_cast<int>(b % kGroup);
        if (in_group == 0 && q >= kGroups) named_sync(kBarTmem + g, kBarTmemThreads);  // slot g read
        if (lane == 0) {
          tc_fence_after();
          mma_i8(tmem_base + static_cast<uint32_t>((g * kGroup + in_group) * kBlockN),
                 sw128_kmajor_desc(sa, static_cast<uint32_t>(kk * 32)),
                 sw128_kmajor_desc(sa + kABytes, static_cast<uint32_t>(kk * 32)), idesc, 0u);
        }
        if (in_group == kGroup - 1 || b == Kb - 1) {
          if (lane == 0) tc_commit(smem_u32(&ctl->tfull[g]));
          ++q;
        }
        if (kk == kBlocksPerStage - 1 || b == Kb - 1) {
          if (lane == 0) tc_commit(smem_u32(&ctl->empty[s]));
          ++st;
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      // Drain: every MMA issued above has completed once this arrives.
      tc_commit(smem_u32(&ctl->drain));
      volatile int never = 0;
      if (!ovb_wait(smem_u32(&ctl->drain), 0u, &never)) atomicOr(&g_status, kErrDrain);
    }
    __syncwarp();
  } else if (warp == kWatcherWarp) {
    // ----------------------------------------------------- stage watcher
    // Exactly one bar.sync per stage, in lockstep with the MMA warp, even
    // after a failed wait (the MMA warp then reads stale data; the status
    // word reports the failure).
    int64_t st = 0;
    for (int64_t t = 0; t < my_tiles; ++t) {
      for (int64_t j = 0; j < ksteps; ++j, ++st) {
        const int s = static_cast<int>(st % kStages);
        const uint32_t ph = static_cast<uint32_t>((st / kStages) & 1);
        const bool got = ovb_wait(smem_u32(&ctl->full[s]), ph, abort);
        if (!__all_sync(0xffffffffu, got) && lane == 0) fail(ctl, kErrMma);
        named_sync(kBarFull, kBarFullThreads);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;          // TMEM lanes this warp may read
    const int group = (warp - 2) >> 2;     // which 32 of the 128 tile columns
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const bool vec_asc =
        ((Kb & 3) == 0) && ((reinterpret_cast<uintptr_t>(args.asc) & 15) == 0);
    float* stg = stg_all + (warp - 2) * (32 * kStgStride);
    int64_t q = 0;  // TMEM groups consumed
    bool ok = true;  // false after a failed wait: keep signalling, skip work
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int64_t m0 = (tile % m_tiles) * kBlockM;
      const int64_t n0 = (tile / m_tiles) * kBlockN;
      const int64_t m = m0 + quarter * 32 + lane;
      const bool row_ok = m < M;
      const float* asc_row = args.asc + (row_ok ? m : 0) * Kb;
      const int64_t nc = n0 + group * kEpiCols;  // first column of this warp's slice
      float f[kEpiCols];
#pragma unroll
      for (int j = 0; j < kEpiCols; ++j) f[j] = 0.f;
      float4 sv_next =
          kProducts ? make_float4(0.f, 0.f, 0.f, 0.f) : load_scales4(asc_row, 0, Kb, row_ok, vec_asc);
      for (int64_t b0 = 0; b0 < Kb; b0 += 4) {
        const float4 sv = sv_next;
        if (!kProducts && b0 + 4 < Kb) sv_next = load_scales4(asc_row, b0 + 4, Kb, row_ok, vec_asc);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          if (b0 + kk >= Kb) break;
          const int64_t b = b0 + kk;
          const float s = kk == 0 ? sv.x : kk == 1 ? sv.y : kk == 2 ? sv.z : sv.w;
          const int g = static_cast<int>(q % kGroups);
          const int in_group = static_cast<int>(b % kGroup);
          const bool last_in_group = in_group == kGroup - 1 || b == Kb - 1;
          if (ok && in_group == 0) {
            const uint32_t gph = static_cast<uint32_t>((q / kGroups) & 1);
            const bool got = ovb_wait(smem_u32(&ctl->tfull[g]), gph, abort);
            if (!__all_sync(0xffffffffu, got)) {
              if (lane == 0) fail(ctl, kErrEpilogue);
              ok = false;
            }
            if (ok) tc_fence_after();
          }
          uint32_t r[32];
          if (ok) {
            tmem_ld32(tmem_base + lane_off +
                          static_cast<uint32_t>((g * kGroup + in_group) * kBlockN + group * kEpiCols),
                      r);
            tc_wait_ld();
          }
          if (last_in_group) {
            tc_fence_before();
            // Slot g is free again; the MMA warp waits for this only when it
            // will reuse the slot, i.e. not for the last kGroups groups.
            if (q + kGroups < my_groups) named_arrive(kBarTmem + g, kBarTmemThreads);
            ++q;
          }
          if (!ok) continue;
          if constexpr (kProducts) {
            if (row_ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int64_t n = nc + j;
                if (n < N) args.products[(m * N + n) * Kb + b] = static_cast<int32_t>(r[j]);
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              f[j] = __fmaf_rn(__int2float_rn(static_cast<int>(r[j])), s, f[j]);
          }
        }
      }
      if (!ok) continue;
      if constexpr (!kProducts) {
        // Stage the warp's 32 x 32 block in shared memory, then write it out
        // row by row: each store instruction covers 128 contiguous bytes of
        // one output row instead of 32 scattered rows.
#pragma unroll
        for (int j = 0; j < kEpiCols; ++j) stg[lane * kStgStride + j] = f[j];
        __syncwarp();
        if (nc < N) {
          // The slice lies inside one output slice (slices are multiples of
          // 64 columns, or a single slice covering all N).
          int si = 0;
#pragma unroll
          for (int i = 1; i < kMaxSlices; ++i)
            if (i < args.n_slices && nc >= args.slices[i].n_begin) si = i;
          const SliceOut so = args.slices[si];
          const int64_t local = nc - so.n_begin;
          const bool col_ok = lane < so.n_count - local;
          const float ws = col_ok ? __ldg(args.wscale + nc + lane) : 0.f;
          const int64_t r0 = m0 + quarter * 32;
          const int rows = static_cast<int>(M - r0 < 32 ? M - r0 : 32);
          if (col_ok) {
            float* cbase = so.C + r0 * so.ldc + local + lane;
            for (int rr = 0; rr < rows; ++rr) {
              float o = __fmul_rn(stg[rr * kStgStride + lane], ws);
              float* cp = cbase + rr * so.ldc;
              if (args.accumulate) o = __fadd_rn(o, *cp);
              *cp = o;
            }
          }
        }
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <bool kProducts>
cudaError_t launch_impl(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b,
                        const GemmArgs& args, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev[2] = {-1, -1};
  if (configured_dev[kProducts] != dev) {
    cudaError_t e = cudaFuncSetAttribute(gemm_s8_tc_kernel<kProducts>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    configured_dev[kProducts] = dev;
  }
  const int64_t tiles = ((args.M + kBlockM - 1) / kBlockM) * ((args.N + kBlockN - 1) / kBlockN);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms(dev)));
  gemm_s8_tc_kernel<kProducts><<<grid, kThreads, kSmemBytes, s>>>(tmap_a, tmap_b, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b,
                        const GemmArgs& args, cudaStream_t s) {
  if (args.products) return launch_impl<true>(tmap_a, tmap_b, args, s);
  return launch_impl<false>(tmap_a, tmap_b, args, s);
}

cudaError_t read_and_clear_status(int* out, cudaStream_t s) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
}

}  // namespace ovb
