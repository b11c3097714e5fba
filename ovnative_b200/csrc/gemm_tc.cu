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
// int32 product lands in its own TMEM accumulator (four 128-column buffers =
// all 512 TMEM columns), so the tensor core runs ahead of the fp32 epilogue.
// TMA moves 128-byte-wide boxes (four blocks of K, 128-byte swizzle); each
// MMA's descriptor points at its 32-byte K slice.
//
// Warp roles (640 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A box (128 B x 128 rows of aq) and B box (128 B
//               x 128 rows of the packed weight) per stage into a 4-stage ring;
//   warp 1      TMEM allocator + MMA issuer (lane 0 issues, the whole warp
//               takes part in the named barriers);
//   warps 2..17 epilogue: warp w reads TMEM lanes 32*(w%4).. (the lane quarter
//               it may access) and 32 of the 128 columns, converts each
//               block's int32 products and folds them into 32 fp32 running
//               sums per thread; at the end of the tile it stages the values
//               in shared memory and writes them row by row (coalesced) with
//               wscale and the optional residual applied;
//   warp 18     stage watcher: waits for each TMA stage to land and hands it
//               to the MMA warp;
//   warp 19     TMEM poller: waits for each MMA to complete and releases
//               the epilogue warps.
//
// Handshakes.  A thread that has tcgen05.mma operations in flight stalls on
// any shared-memory access of its own (an mbarrier wait included) until
// those MMAs have read their operands -- measured here at ~400 clocks per
// access, six times the 64-clock issue interval of a 128x128x32 int8 MMA.
// So the MMA warp never waits on an mbarrier inside its loop: it meets the
// stage watcher on named barrier kBarFull (bar.sync, 64 threads, lockstep)
// once per stage.  TMEM holds four block accumulators (slots).  The MMA warp
// commits slot g's mbarrier after its MMA; the poller waits on that mbarrier
// and bar.arrives on kBarReady + g,
// on which the sixteen epilogue warps bar.sync -- so only one warp polls and
// the epilogue warps sleep until their data is there.  After reading slot g
// the epilogue warps bar.arrive on kBarTmem + g, on which the MMA warp
// bar.syncs before refilling it; the MMA warp in turn bar.arrives on
// kBarIssued + g after each MMA, on which the poller bar.syncs before waiting.  Each named barrier's arrivals and syncs
// alternate strictly, and every participant executes its full count on every
// path (after an error it keeps signalling without doing work), so no named
// barrier can be left waiting.
//
// Every mbarrier wait is bounded (ovb_wait); on a timeout the kernel records
// a non-zero status in g_status and the remaining waits return at once.
#include "ovb_internal.h"
#include "ovb_ptx.cuh"

namespace ovb {

__device__ int g_status;

namespace {

constexpr int kBlocksPerStage = kStageK / 32;  // quantisation blocks per TMA box
constexpr int kStages = 4;
constexpr int kAccBufs = 4;
constexpr int kSlots = kAccBufs;            // one block accumulator per TMEM slot
constexpr uint32_t kTmemCols = 512;
constexpr int kEpiWarps = 16;
constexpr int kWatcherWarp = 2 + kEpiWarps;
constexpr int kPollerWarp = kWatcherWarp + 1;
constexpr int kThreads = 32 * (kPollerWarp + 1);
// named barriers (0 is __syncthreads)
constexpr int kBarFull = 1;                    // stage landed: watcher + MMA warp
constexpr int kBarTmem = 2;                     // + g: slot g read: epilogue warps -> MMA warp
constexpr int kBarIssued = kBarTmem + kSlots;   // + g: slot g's MMA issued: MMA warp -> poller
constexpr int kBarReady = kBarIssued + kSlots;  // + g: slot g written: poller -> epilogue warps
constexpr int kBarFullThreads = 64;
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
static_assert(kBarReady + kSlots <= 16, "the hardware has 16 named barriers");

// status codes recorded in g_status (bit flags)
constexpr int kErrProducer = 1;
constexpr int kErrMma = 2;
constexpr int kErrEpilogue = 4;
constexpr int kErrDrain = 8;

struct Ctl {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[kSlots];
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

// Block scales of row m for blocks b0..b0+3 (zero past Kb or for rows >= M).
__device__ __forceinline__ float4 load_scales4(const float* asc_row, int b0, int Kb, bool row_ok,
                                               bool vec) {
  if (!row_ok) return make_float4(0.f, 0.f, 0.f, 0.f);
  if (vec) return __ldg(reinterpret_cast<const float4*>(asc_row + b0));
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = (b0 + i < Kb) ? __ldg(asc_row + b0 + i) : 0.f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

// f[j] = fma((float)P[j], s, f[j]) for one 16-column half of a block
// (columns 0..15 or 16..31 of the warp's slice) -- one exact int->fp32
// conversion and one fused multiply-add per output, as the reference does.
template <int kHalf>
__device__ __forceinline__ void fold_half(float (&f)[32], const uint32_t (&r)[16], float s) {
#pragma unroll
  for (int j = 0; j < 16; ++j)
    f[kHalf * 16 + j] = __fmaf_rn(__int2float_rn(static_cast<int>(r[j])), s, f[kHalf * 16 + j]);
}

// The slot barriers:
//   kBarTmem + g    the 16 epilogue warps arrive when slot g is read; the MMA
//                   warp syncs before refilling it;
//   kBarIssued + g  the MMA warp arrives once it has issued slot g's MMA; the
//                   poller syncs before waiting for that MMA to complete;
//   kBarReady + g   the poller arrives when slot g's MMA has completed; the
//                   16 epilogue warps sync before reading the slot.
// Every arrival on one of them happens after the previous generation of that
// barrier has completed (each arrive follows, through the other two, the sync
// of the generation before), so generations never merge -- also on the error
// path, where a failed mbarrier wait lets the poller go on without data.  The
// MMA warp never waits for the poller: an earlier version in which both synced
// on one "free" barrier held every MMA until the poller had seen the previous
// one complete, serialising them (~390 clocks per block).
constexpr int kBarSlotThreads = 32 * (kEpiWarps + 1);
constexpr int kBarIssuedThreads = 64;

template <bool kProducts>
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

  const int64_t M = args.M, N = args.N;
  const int Kb = static_cast<int>(args.Kb);
  const int ksteps = (Kb + kBlocksPerStage - 1) / kBlocksPerStage;
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  const int64_t n_tiles = (N + kBlockN - 1) / kBlockN;
  const int64_t tiles = m_tiles * n_tiles;
  const int64_t my_tiles =
      tiles > blockIdx.x ? (tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int64_t my_fills = my_tiles * Kb;  // TMEM slot fills (= MMAs) of this CTA

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int g = 0; g < kSlots; ++g) mbar_init(smem_u32(&ctl->tfull[g]), 1);
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
        for (int j = 0; j < ksteps; ++j, ++st) {
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
          tma_load_2d(sa, &tmap_a, j * kStageK, m0, full);
          tma_load_2d(sa + kABytes, &tmap_b, j * kStageK, n0, full);
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
    // One K = 32 MMA per quantisation block into TMEM slot g = fill % 4.
    // The whole warp walks the loop (named barriers count warps); lane 0
    // issues.  No shared-memory access here until the final drain.
    const uint32_t idesc = idesc_i8(kBlockM, kBlockN);
    int64_t st = 0, q = 0;
    for (int64_t t = 0; t < my_tiles; ++t) {
      for (int j = 0; j < ksteps; ++j, ++st) {
        const int s = static_cast<int>(st % kStages);
        named_sync(kBarFull, kBarFullThreads);  // stage s has landed
        const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * kStageBytes);
        const int nb = Kb - j * kBlocksPerStage < kBlocksPerStage ? Kb - j * kBlocksPerStage
                                                                  : kBlocksPerStage;
        for (int kk = 0; kk < nb; ++kk, ++q) {
          const int g = static_cast<int>(q & (kSlots - 1));
          if (q >= kSlots) named_sync(kBarTmem + g, kBarSlotThreads);  // slot g read
          if (lane == 0) {
            tc_fence_after();
            mma_i8(tmem_base + static_cast<uint32_t>(g * kBlockN),
                   sw128_kmajor_desc(sa, static_cast<uint32_t>(kk * 32)),
                   sw128_kmajor_desc(sa + kABytes, static_cast<uint32_t>(kk * 32)), idesc, 0u);
            tc_commit(smem_u32(&ctl->tfull[g]));
          }
          __syncwarp();
          named_arrive(kBarIssued + g, kBarIssuedThreads);
        }
        if (lane == 0) tc_commit(smem_u32(&ctl->empty[s]));
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
      for (int j = 0; j < ksteps; ++j, ++st) {
        const int s = static_cast<int>(st % kStages);
        const uint32_t ph = static_cast<uint32_t>((st / kStages) & 1);
        const bool got = ovb_wait(smem_u32(&ctl->full[s]), ph, abort);
        if (!__all_sync(0xffffffffu, got) && lane == 0) fail(ctl, kErrMma);
        named_sync(kBarFull, kBarFullThreads);
      }
    }
  } else if (warp == kPollerWarp) {
    // -------------------------------------------------------- TMEM poller
    for (int64_t q = 0; q < my_fills; ++q) {
      const int g = static_cast<int>(q & (kSlots - 1));
      named_sync(kBarIssued + g, kBarIssuedThreads);  // slot g's MMA has been issued
      const uint32_t ph = static_cast<uint32_t>((q / kSlots) & 1);
      const bool got = ovb_wait(smem_u32(&ctl->tfull[g]), ph, abort);
      if (!__all_sync(0xffffffffu, got) && lane == 0) fail(ctl, kErrEpilogue);
      named_arrive(kBarReady + g, kBarSlotThreads);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;       // TMEM lanes this warp may read
    const int cgroup = (warp - 2) >> 2;  // which 32 of the 128 tile columns
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const bool vec_asc =
        ((Kb & 3) == 0) && ((reinterpret_cast<uintptr_t>(args.asc) & 15) == 0);
    float* stg = stg_all + (warp - 2) * (32 * kStgStride);
    int64_t q = 0;  // TMEM slot fills consumed
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int64_t m0 = (tile % m_tiles) * kBlockM;
      const int64_t n0 = (tile / m_tiles) * kBlockN;
      const int64_t m = m0 + quarter * 32 + lane;
      const bool row_ok = m < M;
      const float* asc_row = args.asc + (row_ok ? m : 0) * static_cast<int64_t>(Kb);
      const int64_t nc = n0 + cgroup * kEpiCols;  // first column of this warp's slice
      float f[kEpiCols];
#pragma unroll
      for (int j = 0; j < kEpiCols; ++j) f[j] = 0.f;
      float4 sv_next = kProducts ? make_float4(0.f, 0.f, 0.f, 0.f)
                                 : load_scales4(asc_row, 0, Kb, row_ok, vec_asc);
      // Software pipeline over half-blocks: while the low 16 columns of block
      // b load from TMEM, the high 16 columns of block b-1 are folded in;
      // while the high half of b loads, its low half is folded in.  The fold
      // order per output is still b = 0, 1, 2, ...  (The TMEM load is as slow
      // as the arithmetic; done back to back they do not overlap, because all
      // epilogue warps reach each block at the same time.)
      uint32_t r_lo[16], r_hi[16];
      float s_prev = 0.f;
      for (int b0 = 0; b0 < Kb; b0 += 4) {
        const float4 sv = sv_next;
        if (!kProducts && b0 + 4 < Kb) sv_next = load_scales4(asc_row, b0 + 4, Kb, row_ok, vec_asc);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int b = b0 + kk;
          if (b >= Kb) break;
          const float s = kk == 0 ? sv.x : kk == 1 ? sv.y : kk == 2 ? sv.z : sv.w;
          const int g = static_cast<int>(q & (kSlots - 1));
          named_sync(kBarReady + g, kBarSlotThreads);  // slot g holds block b
          tc_fence_after();
          const uint32_t taddr =
              tmem_base + lane_off + static_cast<uint32_t>(g * kBlockN + cgroup * kEpiCols);
          tmem_ld16(taddr, r_lo);
          if constexpr (!kProducts) {
            if (b > 0) fold_half<1>(f, r_hi, s_prev);  // block b-1, columns 16..31
          }
          tc_wait_ld16(r_lo);
          if constexpr (kProducts) {
            if (row_ok) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int64_t n = nc + j;
                if (n < N) args.products[(m * N + n) * Kb + b] = static_cast<int32_t>(r_lo[j]);
              }
            }
          }
          tmem_ld16(taddr + 16, r_hi);
          if constexpr (!kProducts) fold_half<0>(f, r_lo, s);  // block b, columns 0..15
          tc_wait_ld16(r_hi);
          tc_fence_before();
          // Slot g is free again; the MMA warp waits for this only when it
          // will refill the slot, i.e. not for the last kSlots fills.
          if (q + kSlots < my_fills) named_arrive(kBarTmem + g, kBarSlotThreads);
          ++q;
          s_prev = s;
          if constexpr (kProducts) {
            if (row_ok) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int64_t n = nc + 16 + j;
                if (n < N) args.products[(m * N + n) * Kb + b] = static_cast<int32_t>(r_hi[j]);
              }
            }
          }
        }
      }
      if constexpr (!kProducts) fold_half<1>(f, r_hi, s_prev);  // last block, columns 16..31
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
