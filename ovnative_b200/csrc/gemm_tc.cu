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
// K = 32, M = 128 rows of activations and N = BN output channels, where the
// tile width BN is 128, 64 or 32 (one kernel instance per width; the host
// picks the widest that still gives every SM a tile, so the N = 1024 o/down
// projections at a few hundred rows use all SMs).  TMEM (512 columns) is
// split into four 128-column slots; a slot holds the int32 products of
// G = 128 / BN consecutive blocks, each block in its own BN columns, so the
// tensor core runs up to 4 G blocks ahead of the fp32 epilogue.  TMA moves
// 128-byte-wide boxes (four blocks of K, 128-byte swizzle); each MMA's
// descriptor points at its 32-byte K slice.
//
// Warp roles (640 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A box (128 B x 128 rows of aq) and B box (128 B
//               x BN rows of the packed weight) per stage into a 4-stage ring;
//   warp 1      TMEM allocator + MMA issuer (lane 0 issues, the whole warp
//               takes part in the named barriers);
//   warps 2..17 epilogue: warp w reads TMEM lanes 32*(w%4).. (the lane quarter
//               it may access) and BN/4 of the tile's columns, converts each
//               block's int32 products and folds them, block by block, into
//               BN/4 fp32 running sums per thread; at the end of the tile it
//               stages the values in shared memory and writes them row by row
//               (coalesced) with wscale and the optional residual applied;
//   warp 18     stage watcher: waits for each TMA stage to land and hands it
//               to the MMA warp;
//   warp 19     TMEM poller: waits for each slot's MMAs to complete and
//               releases the epilogue warps.
//
// Handshakes.  A thread that has tcgen05.mma operations in flight stalls on
// any shared-memory access of its own (an mbarrier wait included) until
// those MMAs have read their operands -- measured here at ~400 clocks per
// access, six times the 64-clock issue interval of a 128x128x32 int8 MMA.
// So the MMA warp never waits on an mbarrier inside its loop: it meets the
// stage watcher on named barrier kBarFull (bar.sync, 64 threads, lockstep)
// once per stage.  The MMA warp commits slot g's mbarrier after the slot's
// last MMA; the poller waits on that mbarrier and bar.arrives on
// kBarReady + g, on which the sixteen epilogue warps bar.sync -- so only one
// warp polls and the epilogue warps sleep until their data is there.  After
// reading slot g the epilogue warps bar.arrive on kBarTmem + g, on which the
// MMA warp bar.syncs before refilling it; the MMA warp in turn bar.arrives on
// kBarIssued + g after the slot's last MMA, on which the poller bar.syncs
// before waiting.  Each named barrier's arrivals and syncs alternate
// strictly, and every participant executes its full count on every path
// (after an error it keeps signalling without doing work), so no named
// barrier can be left waiting.
//
// Every mbarrier wait is bounded (ovb_wait); on a timeout the kernel records
// a non-zero status in g_status and the remaining waits return at once.
#include <cstdlib>

#include "ovb_internal.h"
#include "ovb_ptx.cuh"
#include "ovb_quant.cuh"

namespace ovb {

__device__ int g_status;

namespace {

constexpr int kBlocksPerStage = kStageK / 32;  // quantisation blocks per TMA box
constexpr int kStages = 4;
constexpr int kSlots = 4;                       // TMEM slots
constexpr uint32_t kTmemCols = 512;
constexpr int kSlotCols = static_cast<int>(kTmemCols) / kSlots;
constexpr int kEpiWarps = 16;
constexpr int kWatcherWarp = 2 + kEpiWarps;
constexpr int kPollerWarp = kWatcherWarp + 1;
constexpr int kThreads = 32 * (kPollerWarp + 1);
// named barriers (0 is __syncthreads)
constexpr int kBarFull = 1;                    // stage landed: watcher + MMA warp
constexpr int kBarTmem = 2;                     // + g: slot g read: epilogue warps -> MMA warp
constexpr int kBarIssued = kBarTmem + kSlots;   // + g: slot g's MMAs issued: MMA warp -> poller
constexpr int kBarReady = kBarIssued + kSlots;  // + g: slot g written: poller -> epilogue warps
constexpr int kBarFullThreads = 64;
constexpr uint32_t kABytes = kBlockM * kStageK;
static_assert(kABytes % 1024 == 0, "128B-swizzle tiles need 1 KB bases");
static_assert(kBarReady + kSlots <= 16, "the hardware has 16 named barriers");

// status codes recorded in g_status (bit flags)
constexpr int kErrProducer = 1;
constexpr int kErrMma = 2;
constexpr int kErrEpilogue = 4;
constexpr int kErrDrain = 8;
constexpr int kErrF16Range = 16;  // fused SiLU*up output beyond the fp16 range

// Kernel modes: C = wscale * sum (+ C), the int32 block products, or the
// fused SiLU*up + quantise epilogue of a gate|up weight (BN = 128 only).
constexpr int kModePlain = 0;
constexpr int kModeProducts = 1;
constexpr int kModeSilu = 2;
constexpr int kBarSilu = kBarReady + kSlots;  // all epilogue warps, fused SiLU*up
static_assert(kBarSilu < 16, "the hardware has 16 named barriers");

struct Ctl {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[kSlots];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// Everything that depends on the tile width BN.
template <int BN>
struct Tile {
  static_assert(BN == 128 || BN == 64 || BN == 32, "tile widths: 128, 64, 32");
  static constexpr int kG = kSlotCols / BN;    // quantisation blocks per TMEM slot
  static constexpr int kEpiCols = BN / 4;      // columns per epilogue warp (4 column groups)
  static constexpr uint32_t kBBytes = BN * kStageK;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  // Per epilogue warp: its 32 rows x kEpiCols columns of the finished tile,
  // rows padded by one float so the row-wise writes and the column-wise
  // reads are (nearly) free of bank conflicts.
  static constexpr int kStgStride = kEpiCols + 1;
  static constexpr uint32_t kStgBytes = 32 * kStgStride * 4;
  static constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStages) * kStageBytes +
                                       static_cast<size_t>(kEpiWarps) * kStgBytes + sizeof(Ctl);
  static_assert(kBBytes % 1024 == 0, "128B-swizzle tiles need 1 KB bases");
  static_assert(kEpiCols * kG == 32, "each warp reads 32 TMEM columns per slot");
  static_assert(kBlocksPerStage % kG == 0, "slots never straddle a stage");
};

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

// Scales of the blocks in slot `ps` of a group of four blocks (sv), first
// block in .x.
template <int G>
__device__ __forceinline__ float4 slot_scales(float4 sv, int ps) {
  if constexpr (G == 4) return sv;
  if constexpr (G == 2) return ps == 0 ? make_float4(sv.x, sv.y, 0.f, 0.f)
                                       : make_float4(sv.z, sv.w, 0.f, 0.f);
  const float s = ps == 0 ? sv.x : ps == 1 ? sv.y : ps == 2 ? sv.z : sv.w;
  return make_float4(s, 0.f, 0.f, 0.f);
}

// One slot holds 32 TMEM columns per epilogue warp, read in two halves of 16
// (so that one half loads while the other is folded):
//   BN = 128: half h = columns 16h..16h+15 of the slot's one block;
//   BN = 64:  half h = the warp's 16 columns of block h of the slot;
//   BN = 32:  half h = the warp's 8 columns of blocks 2h and 2h+1.
// `addr` is the slot's TMEM address for this warp's lanes and first column.
template <int BN, int H>
__device__ __forceinline__ void load_half(uint32_t addr, uint32_t (&r)[16]) {
  constexpr int G = Tile<BN>::kG;
  if constexpr (G == 1) {
    tmem_ld16(addr + 16 * H, r);
  } else if constexpr (G == 2) {
    tmem_ld16(addr + H * BN, r);
  } else {
    tmem_ld8(addr + (2 * H) * BN, *reinterpret_cast<uint32_t(*)[8]>(&r[0]));
    tmem_ld8(addr + (2 * H + 1) * BN, *reinterpret_cast<uint32_t(*)[8]>(&r[8]));
  }
}

// Folds half H of a slot into the running sums: f = fma((float)P, s, f) per
// output and block -- one exact int->fp32 conversion and one fused
// multiply-add, as the reference does -- blocks in increasing order.  `nv`
// is the number of the slot's blocks below Kb; `sc` their scales.
template <int BN, int H>
__device__ __forceinline__ void fold_half(float (&f)[BN / 4], const uint32_t (&r)[16], float4 sc,
                                          int nv) {
  constexpr int G = Tile<BN>::kG;
  if constexpr (G == 1) {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      f[16 * H + j] = __fmaf_rn(__int2float_rn(static_cast<int>(r[j])), sc.x, f[16 * H + j]);
  } else if constexpr (G == 2) {
    if (H < nv) {
      const float s = H == 0 ? sc.x : sc.y;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        f[j] = __fmaf_rn(__int2float_rn(static_cast<int>(r[j])), s, f[j]);
    }
  } else {
    if (2 * H < nv) {
      const float s = H == 0 ? sc.x : sc.z;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        f[j] = __fmaf_rn(__int2float_rn(static_cast<int>(r[j])), s, f[j]);
    }
    if (2 * H + 1 < nv) {
      const float s = H == 0 ? sc.y : sc.w;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        f[j] = __fmaf_rn(__int2float_rn(static_cast<int>(r[8 + j])), s, f[j]);
    }
  }
}

// Products mode: writes half H of a slot (first block b, nv valid blocks) as
// int32 P[m, n, block] for row m and the warp's first column nc.
template <int BN, int H>
__device__ __forceinline__ void store_products(int32_t* products, int64_t m, int64_t N, int Kb,
                                               int64_t nc, int b, int nv,
                                               const uint32_t (&r)[16]) {
  constexpr int G = Tile<BN>::kG;
  if constexpr (G == 1) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t n = nc + 16 * H + j;
      if (n < N) products[(m * N + n) * Kb + b] = static_cast<int32_t>(r[j]);
    }
  } else if constexpr (G == 2) {
    if (H < nv) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int64_t n = nc + j;
        if (n < N) products[(m * N + n) * Kb + b + H] = static_cast<int32_t>(r[j]);
      }
    }
  } else {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (2 * H + u < nv) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int64_t n = nc + j;
          if (n < N) products[(m * N + n) * Kb + b + 2 * H + u] = static_cast<int32_t>(r[8 * u + j]);
        }
      }
    }
  }
}

// The slot barriers:
//   kBarTmem + g    the 16 epilogue warps arrive when slot g is read; the MMA
//                   warp syncs before refilling it;
//   kBarIssued + g  the MMA warp arrives once it has issued slot g's MMAs;
//                   the poller syncs before waiting for them to complete;
//   kBarReady + g   the poller arrives when slot g's MMAs have completed; the
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

template <int BN, int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_s8_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ GemmArgs args) {
  using T = Tile<BN>;
  constexpr int G = T::kG;
  constexpr bool kProducts = kMode == kModeProducts;
  static_assert(kMode != kModeSilu || BN == 128, "the fused SiLU*up epilogue needs BN = 128");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* stg_all = reinterpret_cast<float*>(smem + static_cast<size_t>(kStages) * T::kStageBytes);
  Ctl* ctl = reinterpret_cast<Ctl*>(reinterpret_cast<uint8_t*>(stg_all) +
                                    static_cast<size_t>(kEpiWarps) * T::kStgBytes);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int64_t M = args.M, N = args.N;
  const int Kb = static_cast<int>(args.Kb);
  const int ksteps = (Kb + kBlocksPerStage - 1) / kBlocksPerStage;
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  const int64_t n_tiles = (N + BN - 1) / BN;
  const int64_t tiles = m_tiles * n_tiles;
  const int64_t my_tiles =
      tiles > blockIdx.x ? (tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  // TMEM slot fills of this CTA (each tile's last slot may hold < G blocks)
  const int64_t my_fills = my_tiles * ((Kb + G - 1) / G);

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
  pdl_wait();  // the preceding kernel's outputs (aq, asc, residual C) are complete
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One stage = kStageK bytes of K (kBlocksPerStage quantisation blocks)
    // of the A tile (128 activation rows) and the B tile (BN weight rows).
    if (lane == 0) {
      int64_t st = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int32_t m0 = static_cast<int32_t>((tile % m_tiles) * kBlockM);
        const int32_t n0 = static_cast<int32_t>((tile / m_tiles) * BN);
        for (int j = 0; j < ksteps; ++j, ++st) {
          const int s = static_cast<int>(st % kStages);
          const uint32_t ph = static_cast<uint32_t>((st / kStages) & 1);
          if (!ovb_wait(smem_u32(&ctl->empty[s]), ph ^ 1u, abort)) {
            fail(ctl, kErrProducer);
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&ctl->full[s]);
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * T::kStageBytes);
          mbar_arrive_expect_tx(full, T::kStageBytes);
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
    // One K = 32 MMA per quantisation block; block b of a tile goes to slot
    // g = fill % 4, columns (b % G) * BN.  The whole warp walks the loop
    // (named barriers count warps); lane 0 issues.  No shared-memory access
    // here until the final drain.
    const uint32_t idesc = idesc_i8(kBlockM, BN);
    int64_t st = 0, q = 0;  // stages consumed, slot fills issued
    for (int64_t t = 0; t < my_tiles; ++t) {
      for (int j = 0; j < ksteps; ++j, ++st) {
        const int s = static_cast<int>(st % kStages);
        named_sync(kBarFull, kBarFullThreads);  // stage s has landed
        const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * T::kStageBytes);
        const int b0 = j * kBlocksPerStage;
        const int nb = Kb - b0 < kBlocksPerStage ? Kb - b0 : kBlocksPerStage;
        for (int kk = 0; kk < nb; ++kk) {
          const int i = kk % G;  // position of block b0 + kk in its slot
          const int g = static_cast<int>(q & (kSlots - 1));
          if (i == 0 && q >= kSlots) named_sync(kBarTmem + g, kBarSlotThreads);  // slot g read
          const bool last = i == G - 1 || kk == nb - 1;
          if (lane == 0) {
            tc_fence_after();
            mma_i8(tmem_base + static_cast<uint32_t>(g * kSlotCols + i * BN),
                   sw128_kmajor_desc(sa, static_cast<uint32_t>(kk * 32)),
                   sw128_kmajor_desc(sa + kABytes, static_cast<uint32_t>(kk * 32)), idesc, 0u);
            if (last) tc_commit(smem_u32(&ctl->tfull[g]));
          }
          __syncwarp();
          if (last) {
            named_arrive(kBarIssued + g, kBarIssuedThreads);
            ++q;
          }
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
      named_sync(kBarIssued + g, kBarIssuedThreads);  // slot g's MMAs have been issued
      const uint32_t ph = static_cast<uint32_t>((q / kSlots) & 1);
      const bool got = ovb_wait(smem_u32(&ctl->tfull[g]), ph, abort);
      if (!__all_sync(0xffffffffu, got) && lane == 0) fail(ctl, kErrEpilogue);
      named_arrive(kBarReady + g, kBarSlotThreads);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr int E = T::kEpiCols;
    const int quarter = warp & 3;        // TMEM lanes this warp may read
    const int cgroup = (warp - 2) >> 2;  // which E of the BN tile columns
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const bool vec_asc =
        ((Kb & 3) == 0) && ((reinterpret_cast<uintptr_t>(args.asc) & 15) == 0);
    float* stg = stg_all + (warp - 2) * (32 * T::kStgStride);
    int64_t q = 0;  // TMEM slot fills consumed
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int64_t m0 = (tile % m_tiles) * kBlockM;
      const int64_t n0 = (tile / m_tiles) * BN;
      const int64_t m = m0 + quarter * 32 + lane;
      const bool row_ok = m < M;
      const float* asc_row = args.asc + (row_ok ? m : 0) * static_cast<int64_t>(Kb);
      const int64_t nc = n0 + cgroup * E;  // first column of this warp's slice
      // wscale of this lane's output column (see the stores below), fetched
      // now so its latency hides behind the K loop.
      const float ws_pre = (!kProducts && nc + lane % E < N) ? __ldg(args.wscale + nc + lane % E)
                                                            : 0.f;
      float f[E];
#pragma unroll
      for (int j = 0; j < E; ++j) f[j] = 0.f;
      float4 sv_next = kProducts ? make_float4(0.f, 0.f, 0.f, 0.f)
                                 : load_scales4(asc_row, 0, Kb, row_ok, vec_asc);
      // Software pipeline over half-slots: while half 0 of slot p loads from
      // TMEM, half 1 of slot p-1 is folded in; while half 1 of p loads, its
      // half 0 is folded in.  The fold order per output is still block
      // 0, 1, 2, ...  (The TMEM load is as slow as the arithmetic; done back
      // to back they do not overlap, because all epilogue warps reach each
      // slot at the same time.)
      uint32_t r_lo[16], r_hi[16];
      float4 sc_prev = make_float4(0.f, 0.f, 0.f, 0.f);
      int nv_prev = 0;
      for (int b0 = 0; b0 < Kb; b0 += 4) {
        const float4 sv = sv_next;
        if (!kProducts && b0 + 4 < Kb) sv_next = load_scales4(asc_row, b0 + 4, Kb, row_ok, vec_asc);
#pragma unroll
        for (int ps = 0; ps < 4 / G; ++ps) {
          const int b = b0 + ps * G;  // first block of the slot
          if (b >= Kb) break;
          const int nv = Kb - b < G ? Kb - b : G;
          const float4 sc = slot_scales<G>(sv, ps);
          const int g = static_cast<int>(q & (kSlots - 1));
          named_sync(kBarReady + g, kBarSlotThreads);  // slot g holds blocks b..b+nv-1
          tc_fence_after();
          const uint32_t taddr =
              tmem_base + lane_off + static_cast<uint32_t>(g * kSlotCols + cgroup * E);
          load_half<BN, 0>(taddr, r_lo);
          if constexpr (!kProducts) {
            if (b > 0) fold_half<BN, 1>(f, r_hi, sc_prev, nv_prev);  // previous slot, half 1
          }
          tc_wait_ld16(r_lo);
          if constexpr (kProducts) {
            if (row_ok) store_products<BN, 0>(args.products, m, N, Kb, nc, b, nv, r_lo);
          }
          load_half<BN, 1>(taddr, r_hi);
          if constexpr (!kProducts) fold_half<BN, 0>(f, r_lo, sc, nv);  // this slot, half 0
          tc_wait_ld16(r_hi);
          tc_fence_before();
          // Slot g is free again; the MMA warp waits for this only when it
          // will refill the slot, i.e. not for the last kSlots fills.
          if (q + kSlots < my_fills) named_arrive(kBarTmem + g, kBarSlotThreads);
          ++q;
          sc_prev = sc;
          nv_prev = nv;
          if constexpr (kProducts) {
            if (row_ok) store_products<BN, 1>(args.products, m, N, Kb, nc, b, nv, r_hi);
          }
        }
      }
      if constexpr (kMode == kModeSilu) {
        fold_half<BN, 1>(f, r_hi, sc_prev, nv_prev);  // last slot, half 1
        // Fused SiLU*up (silu_mul_quantize_f32, ops_cpu.cpp:144-198, on the
        // gate|up outputs).  Column group c of the tile is gate block (c even)
        // or up block (c odd) J = n0/64 + c/2 of the interleaved weight.  Each
        // warp forms its outputs o = f * wscale exactly as the plain GEMM
        // writes them; the up warp stages o, and the gate warp with the same
        // rows (warp + 4) forms v = silu(g) * u for its 32 columns -- one
        // whole quantisation block of the row -- and quantises it.
        float o[E];
#pragma unroll
        for (int j = 0; j < E; ++j) o[j] = __fmul_rn(f[j], __shfl_sync(0xffffffffu, ws_pre, j));
        if (cgroup & 1) {
#pragma unroll
          for (int j = 0; j < E; ++j) stg[lane * T::kStgStride + j] = o[j];
        }
        named_sync(kBarSilu, 32 * kEpiWarps);
        if (!(cgroup & 1) && nc < N && row_ok) {
          const float* ustg = stg + 4 * (32 * T::kStgStride);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = silu_up_vec(o[j], ustg[lane * T::kStgStride + j]);
          const int64_t J = n0 / 64 + cgroup / 2;
          const int64_t esz = args.silu_mode == 2 ? 2 : 1;
          bool bad = false;
          const float sc = quant_block32(v, args.silu_out + (m * args.silu_kp + J * 32) * esz,
                                         args.silu_mode, &bad);
          args.silu_asc[m * (args.silu_kp / 32) + J] = sc;
          if (bad) atomicOr(&g_status, kErrF16Range);
        }
        named_sync(kBarSilu, 32 * kEpiWarps);  // staging free for the next tile
      } else if constexpr (!kProducts) {
        fold_half<BN, 1>(f, r_hi, sc_prev, nv_prev);  // last slot, half 1
        // Stage the warp's 32 x E block in shared memory, then write it out
        // row-wise: each store instruction covers 32 / E rows of E
        // contiguous columns instead of 32 scattered rows.
#pragma unroll
        for (int j = 0; j < E; ++j) stg[lane * T::kStgStride + j] = f[j];
        __syncwarp();
        if (nc < N) {
          // The E columns lie inside one output slice (slices are multiples
          // of 64 columns, or a single slice covering all N).
          int si = 0;
#pragma unroll
          for (int i = 1; i < kMaxSlices; ++i)
            if (i < args.n_slices && nc >= args.slices[i].n_begin) si = i;
          const SliceOut so = args.slices[si];
          const int64_t local = nc - so.n_begin;
          const int cl = lane % E;       // column within the warp's slice
          const int rsub = lane / E;     // first row of this lane
          const bool col_ok = cl < so.n_count - local;
          const float ws = ws_pre;
          const int64_t r0 = m0 + quarter * 32;
          const int rows = static_cast<int>(M - r0 < 32 ? M - r0 : 32);
          if (col_ok) {
            // Rows rsub, rsub + 32/E, ...: the residual loads of 8 rows are
            // issued before their stores so their latencies overlap.
            constexpr int kStep = 32 / E;
            float* cbase = so.C + r0 * so.ldc + local + cl;
            for (int rr0 = rsub; rr0 < rows; rr0 += 8 * kStep) {
              float old[8];
              if (args.accumulate) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const int rr = rr0 + i * kStep;
                  old[i] = rr < rows ? cbase[rr * so.ldc] : 0.f;
                }
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int rr = rr0 + i * kStep;
                if (rr < rows) {
                  float o = __fmul_rn(stg[rr * T::kStgStride + cl], ws);
                  if (args.accumulate) o = __fadd_rn(o, old[i]);
                  cbase[rr * so.ldc] = o;
                }
              }
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

template <int BN, int kMode>
cudaError_t launch_impl(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b,
                        const GemmArgs& args, cudaStream_t s) {
  using T = Tile<BN>;
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev = -1;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(gemm_s8_tc_kernel<BN, kMode>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(T::kSmemBytes));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  const int64_t tiles = ((args.M + kBlockM - 1) / kBlockM) * ((args.N + BN - 1) / BN);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms(dev)));
  return launch_pdl(gemm_s8_tc_kernel<BN, kMode>, dim3(grid), dim3(kThreads), T::kSmemBytes, s,
                    tmap_a, tmap_b, args);
}

template <int kMode>
cudaError_t launch_width(int tile, const CUtensorMap& tmap_a, const CUtensorMap& tmap_b,
                         const GemmArgs& args, cudaStream_t s) {
  switch (tile) {
    case 0: return launch_impl<128, kMode>(tmap_a, tmap_b, args, s);
    case 1: return launch_impl<64, kMode>(tmap_a, tmap_b, args, s);
    case 2: return launch_impl<32, kMode>(tmap_a, tmap_b, args, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

// Cost of one output tile per quantisation block, by tile width, fitted to
// graph-timed runs on B200: ~430 clocks that do not depend on the width (an
// int8 K = 32 MMA takes ~64 clocks at any N; per-block handshakes) plus
// ~2.6 clocks per column (TMEM readout and conversion of the block's
// products).  The tile count sets how many rounds the persistent grid runs.
int pick_tile(int64_t M, int64_t N, int device) {
  if (const char* e = std::getenv("OVB_GEMM_TILE_N")) {
    const int v = std::atoi(e);
    for (int i = 0; i < 3; ++i)
      if (kTileN[i] == v) return i;
  }
  const int64_t sms = num_sms(device);
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  int best = 0;
  int64_t best_cost = -1;
  for (int i = 0; i < 3; ++i) {
    const int64_t tiles = m_tiles * ((N + kTileN[i] - 1) / kTileN[i]);
    const int64_t waves = (tiles + sms - 1) / sms;
    const int64_t cost = waves * (430 * 10 + 26 * kTileN[i]);
    if (best_cost < 0 || cost < best_cost) {
      best = i;
      best_cost = cost;
    }
  }
  return best;
}

cudaError_t launch_gemm(int tile, const CUtensorMap& tmap_a, const CUtensorMap& tmap_b,
                        const GemmArgs& args, cudaStream_t s) {
  if (args.silu_out) {
    if (tile != 0) return cudaErrorInvalidValue;  // the fused epilogue is built for BN = 128
    return launch_impl<128, kModeSilu>(tmap_a, tmap_b, args, s);
  }
  if (args.products) return launch_width<kModeProducts>(tile, tmap_a, tmap_b, args, s);
  return launch_width<kModePlain>(tile, tmap_a, tmap_b, args, s);
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
