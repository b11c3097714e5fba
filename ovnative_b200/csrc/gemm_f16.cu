// gemm_f16.cu -- the fp16 tensor-core mainloop for weight handles created
// with OVB_WEIGHT_F16: int8 x per-32-k-quantised activations, dequantised on
// chip and multiplied with tcgen05.mma kind::f16 into one fp32 accumulator
// per output tile.
//
// What it computes (the same contract as gemm.cpp:432-504, to tolerance):
//   C[m,n] = wscale[n] * sum_k A'[m,k] * w[n,k]      (+ C[m,n] if accumulate)
//   A'[m,k] = fp16(q[m,k] * asc[m, k/32])              (the dequantised activation)
// The weights are exact in fp16 (|w| <= 127) and the products and sums are
// exact-to-fp32 in the tensor core, so the only rounding beyond the
// reference's fp32 arithmetic is that of A' to fp16: relative error
// <= 2^-11 per element, ~3e-4 relative L2 on the outputs -- inside the
// rel-L2 <= 1e-3 / max-abs <= 1e-2 * rms contract, but not bit-exact.  The
// exact kernel (gemm_tc.cu) must read every 32-k block's int32 products out
// of TMEM to fold them in the reference's order; that readout competes with
// the MMAs for TMEM bandwidth and caps it near 700 clocks per 128x128 block.
// Here TMEM is read once per tile.
//
// Data flow per stage (64 k = two quantisation blocks):
//   TMA   A box: 64 B x 128 rows of aq (int8, 64-byte swizzle) and W box:
//         64 fp16 x BN rows of the fp16 weight copy (128-byte swizzle) into a
//         4-stage shared-memory ring (one mbarrier `full` per stage);
//   conv  eight converter warps: thread (quarter, lane) owns activation row
//         32*quarter + lane and one of the stage's two blocks; it reads its
//         32 int8 from shared memory, forms fp16(q * asc) and stores the 16
//         packed columns into the stage's A' slot in TMEM (tcgen05.st).
//         (Sixteen converter warps, each with half the work, measured slower:
//         the conversion is latency-bound, not bound by arithmetic);
//   MMA   one thread issues four K = 16 MMAs per stage with A from TMEM and
//         W from shared memory, accumulating into the tile's TMEM buffer;
//         tcgen05.commit on `empty` releases the stage (smem and A' slot);
//   epi   after the tile's last stage the MMA thread commits `tfull`; eight
//         epilogue warps read the accumulator (32 columns per tcgen05.ld),
//         stage it in shared memory and write rows coalesced with wscale and
//         the optional residual applied.
//
// TMEM (512 columns): kAcc accumulator buffers of BN columns (two when they
// fit beside the A' ring, so a tile's epilogue overlaps the next tile's
// MMAs), then the A' ring (four stages x 32 columns).
//
// Handshakes.  The MMA thread never waits on an mbarrier inside its loop (a
// thread with MMAs in flight stalls on its own shared-memory accesses):
//   kBarStage + s  the converter warps and the MMA warp bar.sync once stage
//                  s's A' is in TMEM (the converters waited on full[s], so
//                  the W box has landed too), then the MMA warp issues;
//   kBarDfree + d  the epilogue warps and the MMA warp bar.sync once
//                  accumulator d is read, before the MMA warp reuses it.
// Both sides of both barriers bar.sync (none only arrives), so no warp can
// enter a barrier's next generation before the current one completed -- on
// the error path too, where a failed mbarrier wait makes a warp skip its work
// but not its barrier.  Converters therefore run at most one stage ahead of
// the MMA warp, which is enough: a stage converts faster than its MMAs run.
// The converters overwrite A' slot s for stage st only after full[s] of
// stage st completed, and the producer issued that stage's copies only after
// empty[s] of stage st - 4 (whose MMAs read the slot) -- so a slot is never
// overwritten while an MMA may read it.  Every mbarrier wait is bounded
// (ovb_wait).
#include <cuda_fp16.h>

#include <cstdlib>

#include "ovb_internal.h"
#include "ovb_ptx.cuh"
#include "ovb_quant.cuh"

namespace ovb {

// Status word of this kernel's bounded waits (a device variable is private
// to its translation unit without relocatable device code, so the fp16
// mainloop keeps its own; ovb_device_status reports both).
__device__ int g_status_f16;

namespace {

constexpr int kStageKF = 64;      // k per stage: two quantisation blocks
constexpr int kStagesF = 4;
constexpr int kConvWarps = 8;     // warps 2..9
constexpr int kEpiWarpsF = 8;     // warps 10..17
constexpr int kFirstConv = 2;
constexpr int kFirstEpi = kFirstConv + kConvWarps;
constexpr int kThreadsF = 32 * (kFirstEpi + kEpiWarpsF);
constexpr uint32_t kTmemColsF = 512;
constexpr int kAColsPerStage = kStageKF / 2;  // fp16 pairs per row
constexpr uint32_t kABytesF = kBlockM * kStageKF;
// Epilogue staging row stride (floats): 16-byte rows, so that both the
// row-per-lane float4 writes and the 4-rows-per-instruction float4 reads of
// a 32x32 chunk are free of bank conflicts.
constexpr int kStgStrideF = 36;
// The plain fp16 epilogues' per-warp area: a 32 x 36-float staging chunk, or
// (TMA output) a 4 KB box with the 128-byte swizzle plus 1 KB of wscale.
constexpr int kStgTmaBytes = 32 * 128;
constexpr int kStgWarpBytes = 6144;
// Per epilogue warp of the fused q|k|v mode: one head's wscale and norm
// weights, staged for broadcast reads, and two 2 KB buffers of the RoPE
// table (32 rows x 8 pairs each).
constexpr int kRopeColFloats = 256;
constexpr int kRopeTabBufBytes = 2048;
// named barriers (0 is __syncthreads)
constexpr int kBarStage = 1;                    // + s: converters -> MMA warp
constexpr int kBarDfree = kBarStage + kStagesF;  // + d: epilogue -> MMA warp
constexpr int kBarStageThreads = 32 * (kConvWarps + 1);
constexpr int kBarDfreeThreads = 32 * (kEpiWarpsF + 1);
static_assert(kBarDfree + 2 <= 16, "the hardware has 16 named barriers");
static_assert(kABytesF % 1024 == 0, "stage bases stay 1 KB aligned");

// status bits (the same meaning as gemm_tc.cu's)
constexpr int kErrProducer = 1;
constexpr int kErrConvert = 2;
constexpr int kErrEpilogue = 4;
constexpr int kErrDrain = 8;
constexpr int kErrF16Range = 16;  // an activation block left the fp16 range

struct CtlF {
  uint64_t full[kStagesF];
  uint64_t empty[kStagesF];
  uint64_t tfull[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <int BN>
struct TileF {
  static_assert(BN == 256 || BN == 128 || BN == 64 || BN == 32, "tile widths: 256..32");
  static constexpr uint32_t kWBytes = BN * 128;  // 64 fp16 x BN rows
  static constexpr uint32_t kStageBytes = kABytesF + kWBytes;
  static constexpr int kAcc =
      2 * BN + kStagesF * kAColsPerStage <= static_cast<int>(kTmemColsF) ? 2 : 1;
  static constexpr int kACol0 = kAcc * BN;  // first column of the A' ring
  static constexpr int kChunks = BN / 32;   // 32-column epilogue chunks
  static constexpr uint32_t kStgBytes = 32 * kStgStrideF * 4;
  static constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStagesF) * kStageBytes +
                                       static_cast<size_t>(kEpiWarpsF) * kStgBytes +
                                       sizeof(CtlF);
  static_assert(kACol0 + kStagesF * kAColsPerStage <= static_cast<int>(kTmemColsF),
                "accumulators and A' ring exceed TMEM");
  static_assert(kStageBytes % 1024 == 0, "stage bases stay 1 KB aligned");
};

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// First row / column of output tile `tile` (tiles are numbered m-fastest).
// 32-bit arithmetic: a 64-bit division is a long dependent software
// sequence (~0.4 us on a kernel's critical path); the launchers keep the
// tile count below 2^31.
__device__ __forceinline__ void tile_origin(int64_t tile, int64_t m_tiles, int bn, int64_t* m0,
                                            int64_t* n0) {
  const uint32_t t = static_cast<uint32_t>(tile), mt = static_cast<uint32_t>(m_tiles);
  const uint32_t q = t / mt;
  *m0 = static_cast<int64_t>(t - q * mt) * kBlockM;
  *n0 = static_cast<int64_t>(q) * bn;
}

// The epilogues' walk over a CTA's output tiles.  Default: 128-row tiles
// with m fastest (tile_origin above).  pair_nfast (the CTA-pair kernel):
// tile 2p + rank is CTA `rank`'s half of pair tile p, and pair tiles run n
// fastest -- p covers rows [256 (p / n_tiles), + 256) and columns
// [bn (p % n_tiles), + bn), so the clusters working at the same time share
// their A rows (read from DRAM once, the W tiles from L2).
struct TileOrder {
  int64_t m_tiles;
  int64_t n_tiles = 0;
  bool pair_nfast = false;
  __host__ __device__ TileOrder(int64_t mt) : m_tiles(mt) {}
  __host__ __device__ TileOrder(int64_t mt, int64_t nt, bool nf)
      : m_tiles(mt), n_tiles(nt), pair_nfast(nf) {}
};

__device__ __forceinline__ void tile_origin(int64_t tile, const TileOrder& o, int bn, int64_t* m0,
                                            int64_t* n0) {
  if (!o.pair_nfast) {
    tile_origin(tile, o.m_tiles, bn, m0, n0);
    return;
  }
  const uint32_t p = static_cast<uint32_t>(tile) >> 1, rank = static_cast<uint32_t>(tile) & 1u;
  const uint32_t nt = static_cast<uint32_t>(o.n_tiles);
  const uint32_t pm = p / nt;
  *m0 = static_cast<int64_t>(2 * pm + rank) * kBlockM;
  *n0 = static_cast<int64_t>(p - pm * nt) * bn;
}

__device__ __forceinline__ void fail(CtlF* ctl, int code) {
  atomicOr(&g_status_f16, code);
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
}

// Four signed int8 (one 32-bit word) -> two fp16x2 words holding
// fp16(q * asc), asc given as hi + lo fp16 parts.  q is formed exactly:
// the byte q + 128 placed under the fp16 exponent of 1024 reads as
// 1024 + q + 128; subtracting 1152 leaves q.  Then q * hi + (q * lo) is
// rounded once (fma), i.e. fp16(q * asc) up to the ~2^-22 relative
// truncation of asc into hi + lo.
__device__ __forceinline__ void dequant4(uint32_t x, __half2 s_hi, __half2 s_lo, uint32_t& out0,
                                         uint32_t& out1) {
  const uint32_t u = x ^ 0x80808080u;  // q + 128 per byte
  const uint32_t b01 = __byte_perm(u, 0x64646464u, 0x4140);
  const uint32_t b23 = __byte_perm(u, 0x64646464u, 0x4342);
  const __half2 bias = __half2half2(__ushort_as_half(static_cast<unsigned short>(0x6480)));  // 1152
  const __half2 q01 = __hsub2(*reinterpret_cast<const __half2*>(&b01), bias);
  const __half2 q23 = __hsub2(*reinterpret_cast<const __half2*>(&b23), bias);
  const __half2 r01 = __hfma2(q01, s_hi, __hmul2(q01, s_lo));
  const __half2 r23 = __hfma2(q23, s_hi, __hmul2(q23, s_lo));
  out0 = *reinterpret_cast<const uint32_t*>(&r01);
  out1 = *reinterpret_cast<const uint32_t*>(&r23);
}

// Stage row `lane` of a warp's 32x32 accumulator chunk (one TMEM lane per
// thread) in shared memory, row stride kStgStrideF.
__device__ __forceinline__ void stage_chunk(float* stg, const uint32_t (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<float4*>(stg + lane * kStgStrideF + 4 * q) =
        make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                    __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
}

// Scalar path of store_chunk: lane l writes column l, row by row.  The
// residual loads of 8 rows are issued before their stores, so their
// latencies overlap (the compiler cannot reorder a load past a store it
// cannot prove distinct).
__device__ __forceinline__ void store_rows(const float* stg, int stride, float* cbase,
                                           int64_t ldc, int rows, float ws, int accumulate) {
  for (int r0 = 0; r0 < rows; r0 += 8) {
    float old[8];
    if (accumulate) {
#pragma unroll
      for (int i = 0; i < 8; ++i) old[i] = r0 + i < rows ? cbase[(r0 + i) * ldc] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (r0 + i < rows) {
        float o = __fmul_rn(stg[(r0 + i) * stride], ws);
        if (accumulate) o = __fadd_rn(o, old[i]);
        cbase[(r0 + i) * ldc] = o;
      }
    }
  }
}

// Lane l's residual values of a chunk for the float4 path: rows
// 4*it + l/8 (it in [it0, it0 + kN)), columns 4*(l%8) .. +3; zeros outside
// rows / ncols.  The whole-float4 loads are predicated, not branched, so that
// all of them are in flight together; ragged last columns load singly.
template <int kN>
__device__ __forceinline__ void load_residual(const float* cbase, int64_t ldc, int rows, int ncols,
                                              int it0, float4 (&old)[kN]) {
  const int lane = threadIdx.x & 31;
  const int c4 = (lane & 7) * 4;
  const bool full = c4 + 3 < ncols;
#pragma unroll
  for (int i = 0; i < kN; ++i) {
    const int r = (it0 + i) * 4 + (lane >> 3);
    const bool ok = full && r < rows;
    old[i] = ld_f4_if(cbase + (ok ? r * ldc + c4 : 0), ok);
  }
  if (!full && c4 < ncols) {
#pragma unroll
    for (int i = 0; i < kN; ++i) {
      const int r = (it0 + i) * 4 + (lane >> 3);
      if (r < rows) {
        const float* src = cbase + r * ldc + c4;
        old[i].x = src[0];
        if (c4 + 1 < ncols) old[i].y = src[1];
        if (c4 + 2 < ncols) old[i].z = src[2];
      }
    }
  }
}

// o = v * ws (+ old) for four columns, the reference's epilogue order.
__device__ __forceinline__ float4 scale_add4(float4 v, const float (&ws)[4], float4 old,
                                             int accumulate) {
  v.x = __fmul_rn(v.x, ws[0]);
  v.y = __fmul_rn(v.y, ws[1]);
  v.z = __fmul_rn(v.z, ws[2]);
  v.w = __fmul_rn(v.w, ws[3]);
  if (accumulate) {
    v.x = __fadd_rn(v.x, old.x);
    v.y = __fadd_rn(v.y, old.y);
    v.z = __fadd_rn(v.z, old.z);
    v.w = __fadd_rn(v.w, old.w);
  }
  return v;
}

// Write o (four columns of row r) to cbase + r * ldc + c4, clipped to ncols.
__device__ __forceinline__ void put4(float* cbase, int64_t ldc, int r, int c4, int ncols,
                                     float4 o) {
  float* dst = cbase + r * ldc + c4;
  if (c4 + 3 < ncols) {
    *reinterpret_cast<float4*>(dst) = o;
  } else {
    if (c4 < ncols) dst[0] = o.x;
    if (c4 + 1 < ncols) dst[1] = o.y;
    if (c4 + 2 < ncols) dst[2] = o.z;
  }
}

// Lane l's four wscale values (columns 4*(l%8) ..) from the per-lane values
// wl (lane l holds column l's).  All 32 lanes must call it.
__device__ __forceinline__ void gather_ws4(float wl, float (&ws)[4]) {
  const int c4 = ((threadIdx.x & 31) & 7) * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) ws[j] = __shfl_sync(0xffffffffu, wl, c4 + j);
}

// Write a warp's staged 32x32 chunk to C: o = acc * ws[col] (+ C_old) for
// the first `rows` rows and `ncols` columns at cbase (row stride ldc).
// Float4 path (C rows 16-byte aligned: vec): lane l handles rows 4*it + l/8
// and columns 4*(l%8) .. +3, i.e. four 128-byte row segments per warp
// instruction, with the whole residual chunk loaded before the first store.
// Otherwise the scalar path.  All 32 lanes must call it; wl as in gather_ws4.
__device__ __forceinline__ void store_chunk(const float* stg, float* cbase, int64_t ldc, int rows,
                                            int ncols, float wl, int accumulate, bool vec) {
  const int lane = threadIdx.x & 31;
  float ws[4];
  gather_ws4(wl, ws);
  if (!vec) {
    if (lane < ncols) store_rows(stg + lane, kStgStrideF, cbase + lane, ldc, rows, wl, accumulate);
    return;
  }
  const int c4 = (lane & 7) * 4;
  float4 old[8];
  if (accumulate) load_residual<8>(cbase, ldc, rows, ncols, 0, old);
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    if (r < rows && c4 < ncols) {
      const float4 v = *reinterpret_cast<const float4*>(stg + r * kStgStrideF + c4);
      put4(cbase, ldc, r, c4, ncols, scale_add4(v, ws, old[it], accumulate));
    }
  }
}

// True when every row of the slice's C is 16-byte aligned (float4 stores).
__device__ __forceinline__ bool rows_aligned(const SliceOut& so) {
  return (reinterpret_cast<uintptr_t>(so.C) & 15) == 0 && (so.ldc & 3) == 0;
}

// The epilogue warps' loop over this CTA's tiles (both fp16 mainloops).
// Warp (quarter, eh) reads TMEM lanes 32*quarter.. and the 32-column chunks
// eh, eh+2, ... of accumulator d = t % kAcc (none for eh = 1 at BN = 32;
// those warps still take part in every barrier).  Per tile: the chunks'
// wscale values are fetched before the accumulator is ready (tfull[d]), the
// TMEM load of the next chunk runs while the current one is stored, and
// after the last chunk the warps bar.sync on dfree_bar + d with the MMA warp
// (which syncs there before reusing accumulator d).  kPipe = false loads one
// chunk at a time (for kernels short of registers).
//
// TMA output (kTmaOk and args.out_tma; the warp's `stg` area is then
// kStgWarpBytes, 1 KB aligned): each lane scales its row of the chunk by the
// columns' wscale (read as shared-memory broadcasts from the area's last
// kilobyte), writes it into a 32 x 128-byte box with the 128-byte swizzle,
// and lane 0 hands the box to the TMA unit: a store, or with accumulate an
// element-wise add into C performed at L2 -- so the residual is never read
// into the SM.  fl(fl(acc * ws) + C) either way, as the register path.
// The TMA clips rows past M and columns past the slice.
template <int BN, int kAcc, bool kPipe = true, bool kTmaOk = false>
__device__ __forceinline__ void epilogue_loop(const GemmArgs& args, uint64_t* tfull,
                                              volatile int* abort, uint32_t tmem_base,
                                              float* stg, int quarter, int eh, int dfree_bar,
                                              int64_t tiles, TileOrder m_tiles, int64_t my_tiles,
                                              int64_t tile_first, int64_t tile_step) {
  constexpr int kChunks = BN / 32;
  constexpr int kMine = (kChunks + 1) / 2;  // chunks per warp (at most)
  const int lane = threadIdx.x & 31;
  const int64_t M = args.M, N = args.N;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const bool tma = kTmaOk && args.out_tma != 0;
  float* colv = stg + kStgTmaBytes / 4;  // TMA path: the chunks' wscale values
  int64_t t = 0;
  for (int64_t tile = tile_first; tile < tiles; tile += tile_step, ++t) {
    const int d = static_cast<int>(t % kAcc);
    const uint32_t ph = static_cast<uint32_t>((t / kAcc) & 1);
    int64_t m0, n0;
    tile_origin(tile, m_tiles, BN, &m0, &n0);
    float wsv[kMine];
#pragma unroll
    for (int i = 0; i < kMine; ++i) {
      const int64_t n = n0 + (eh + 2 * i) * 32 + lane;
      wsv[i] = (eh + 2 * i < kChunks && n < N) ? __ldg(args.wscale + n) : 0.f;
    }
    if (tma) {
#pragma unroll
      for (int i = 0; i < kMine; ++i) colv[32 * i + lane] = wsv[i];
    }
    const bool got = ovb_wait(smem_u32(&tfull[d]), ph, abort);
    if (!__all_sync(0xffffffffu, got)) {
      if (lane == 0) {
        atomicOr(&g_status_f16, kErrEpilogue);
        *abort = 1;
      }
    } else {
      tc_fence_after();
      const int64_t r0 = m0 + quarter * 32;
      const int rows = static_cast<int>(M - r0 < 32 ? M - r0 : 32);
      const uint32_t dcol = tmem_base + lane_off + static_cast<uint32_t>(d * BN);
      uint32_t va[32], vb[32];
      if (eh < kChunks) tmem_ld32(dcol + static_cast<uint32_t>(eh * 32), va);
#pragma unroll
      for (int i = 0; i < kMine; ++i) {
        const int c = eh + 2 * i;
        if (c >= kChunks) break;
        uint32_t(&cur)[32] = (kPipe && (i & 1)) ? vb : va;
        uint32_t(&nxt)[32] = (kPipe && (i & 1)) ? va : vb;
        if (!kPipe && i > 0) tmem_ld32(dcol + static_cast<uint32_t>(c * 32), cur);
        tc_wait_ld32(cur);
        if (kPipe && c + 2 < kChunks) tmem_ld32(dcol + static_cast<uint32_t>((c + 2) * 32), nxt);
        if (kTmaOk && tma) {
          const int64_t nc = n0 + c * 32;
          const float4* w4 = reinterpret_cast<const float4*>(colv + 32 * i);
          float4 o[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 w = w4[q];  // broadcast: every lane the same columns
            o[q] = make_float4(__fmul_rn(__uint_as_float(cur[4 * q]), w.x),
                               __fmul_rn(__uint_as_float(cur[4 * q + 1]), w.y),
                               __fmul_rn(__uint_as_float(cur[4 * q + 2]), w.z),
                               __fmul_rn(__uint_as_float(cur[4 * q + 3]), w.w));
          }
          // the previous chunk's box has left the staging area
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          float4* box = reinterpret_cast<float4*>(stg) + lane * 8;  // row `lane`
#pragma unroll
          for (int q = 0; q < 8; ++q) box[q ^ (lane & 7)] = o[q];
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && nc < N && rows > 0) {
            int si = 0;
#pragma unroll
            for (int k = 1; k < kMaxSlices; ++k)
              if (k < args.n_slices && nc >= args.slices[k].n_begin) si = k;
            const int32_t x = static_cast<int32_t>(nc - args.slices[si].n_begin);
            const int32_t y = static_cast<int32_t>(r0);
            if (args.accumulate)
              tma_reduce_add_2d(&args.out_map[si], smem_u32(stg), x, y);
            else
              tma_store_2d(&args.out_map[si], smem_u32(stg), x, y);
            bulk_commit();
          }
          continue;
        }
        stage_chunk(stg, cur);
        __syncwarp();
        const int64_t nc = n0 + c * 32;  // first column of the chunk
        if (nc < N && rows > 0) {
          // The chunk lies inside one output slice (slices are multiples of
          // 64 columns, or a single slice covering all N).
          int si = 0;
#pragma unroll
          for (int k = 1; k < kMaxSlices; ++k)
            if (k < args.n_slices && nc >= args.slices[k].n_begin) si = k;
          const SliceOut so = args.slices[si];
          const int64_t local = nc - so.n_begin;
          const int ncols = static_cast<int>(so.n_count - local < 32 ? so.n_count - local : 32);
          store_chunk(stg, so.C + r0 * so.ldc + local, so.ldc, rows, ncols, wsv[i],
                      args.accumulate, rows_aligned(so));
        }
        __syncwarp();
      }
    }
    tc_fence_before();
    if (t + kAcc < my_tiles) named_sync(dfree_bar + d, 32 * (kEpiWarpsF + 1));
  }
  if (tma && lane == 0) bulk_wait_all();  // the boxes are written before the CTA exits
}

// 16-byte asynchronous copy global -> shared (cp.async, L2 only), the group
// commit, and the wait until at most N of this thread's groups are pending.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_n() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Element e (0 .. 7) of two float4.
__device__ __forceinline__ float f4_at2(const float4 (&v)[2], int e) {
  const float4 q = v[e >> 2];
  return (e & 3) == 0 ? q.x : (e & 3) == 1 ? q.y : (e & 3) == 2 ? q.z : q.w;
}

// Two IEEE round-to-nearest products in one packed instruction:
// (a.x * b.x, a.y * b.y), rounded exactly as the scalar mul.rn.
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "mul.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
// (a.x + b.x, a.y + b.y), rounded as add.rn.
// Only for operands that are not products: ptxas contracts a packed mul.rn
// followed by a packed add.rn into one packed fma (measured on sm_100a: 16-25 %
// of such sums then differ from the two-rounding form, even with the product
// written as fma.rn(a, b, -0)), so a sum or difference of products stays two
// scalar add.rn / sub.rn, which ptxas leaves alone.
__device__ __forceinline__ float2 add2rn(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "add.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
// The running magnitude maximum of fp16 pairs: max(|acc|, |w|) per half, a
// NaN in either giving NaN.  An accumulator whose half has every exponent bit
// set has seen an fp16 infinity or NaN.
__device__ __forceinline__ uint32_t absmax_h2(uint32_t acc, uint32_t w) {
  uint32_t d;
  asm("max.NaN.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(d) : "r"(acc), "r"(w));
  return d;
}
__device__ __forceinline__ bool h2_inf_or_nan(uint32_t acc) {
  return (acc & 0x7c00u) == 0x7c00u || (acc & 0x7c000000u) == 0x7c000000u;
}

// Elements e, e + 1 (e even) of an 8-float register pair as a float2.
__device__ __forceinline__ float2 f4_pair(const float4 (&v)[2], int e) {
  const float4 q = v[e >> 2];
  return (e & 2) == 0 ? make_float2(q.x, q.y) : make_float2(q.z, q.w);
}

// The epilogue loop of the fused q|k|v mode (args.rope_q16 non-null; BN =
// 256, two 128-column heads per tile).  Warp (quarter, eh) takes head eh of
// the tile for TMEM lanes 32*quarter..: each thread holds one row of the
// head.  x = D * wscale per column is the plain epilogue's output value; q
// and k heads are then RMS-normalised and rotated exactly as
// qk_norm_rope_f16_kernel (lm_ops.cu) does -- the same sum of squares
// (s_l = (x_l^2 + x_{l+32}^2) + (x_{l+64}^2 + x_{l+96}^2), then pairwise sums
// at distances 16, 8, .., 1, the order of its warp tree), the same scale and
// rotation -- so the fp16 outputs equal the unfused sequence bit for bit; v
// heads are converted.  The per-column values (wscale, norm weight) are the
// same for every lane: they are read as float4 broadcasts; products and the
// sums of sums are packed two per instruction (f32x2), sums and differences
// of products stay scalar (add2rn), and an fp16 output's overflow is found
// from a running magnitude maximum of the packed outputs.  Two passes over
// TMEM, sixteen columns at a time: the sum of squares, then the rotation of
// set s (head elements 32s + i with 64 + 32s + i, s = 0, 1), whose 64 fp16
// outputs are staged in shared memory (32 rows x 128 bytes, 16-byte chunks
// XOR-swizzled by row: conflict-free both ways) and written as 64-byte row
// segments, 8 lanes per row.  The rows' RoPE table is staged in shared memory
// by coalesced asynchronous copies (loads of 16 bytes from 32 different rows
// per instruction cost the L1 far more than their bytes).
template <int BN, int kAcc>
__device__ __forceinline__ void epilogue_rope_loop(const GemmArgs& args, uint64_t* tfull,
                                                   volatile int* abort, uint32_t tmem_base,
                                                   float* stg, float* colv, uint8_t* tb,
                                                   int quarter, int eh,
                                                   int dfree_bar, int64_t tiles, TileOrder m_tiles,
                                                   int64_t my_tiles, int64_t tile_first,
                                                   int64_t tile_step) {
  static_assert(BN == 256, "two heads per tile, one per epilogue warp of a lane quarter");
  const int lane = threadIdx.x & 31;
  const int64_t M = args.M, N = args.N;
  const int64_t qd = args.rope_qd, kvd = args.rope_kvd;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  uint8_t* st8 = reinterpret_cast<uint8_t*>(stg);
  bool range_ok = true;
  int64_t t = 0;
  for (int64_t tile = tile_first; tile < tiles; tile += tile_step, ++t) {
    const int d = static_cast<int>(t % kAcc);
    const uint32_t ph = static_cast<uint32_t>((t / kAcc) & 1);
    int64_t m0, n0;
    tile_origin(tile, m_tiles, BN, &m0, &n0);
    const int64_t hc = n0 + 128 * eh;  // this warp's head: columns hc .. hc + 127
    const bool has = hc < N;           // uniform per warp
    const int kind = hc < qd ? 0 : (hc < qd + kvd ? 1 : 2);  // q, k or v head
    // The head's wscale (colv[0, 128)) and norm weights (colv[128, 256))
    // into this warp's shared area before the accumulator is ready; read
    // back as float4 broadcasts (every lane the same columns).
    if (has) {
      const float* nw = kind == 0 ? args.rope_qw : args.rope_kw;
      float wv[4], nv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        wv[j] = __ldg(args.wscale + hc + 32 * j + lane);
        nv[j] = kind < 2 ? __ldg(nw + 32 * j + lane) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        colv[32 * j + lane] = wv[j];
        colv[128 + 32 * j + lane] = nv[j];
      }
    }
    // The RoPE table of this warp's 32 rows reaches shared memory eight
    // elements (64 bytes per row) at a time, two steps ahead, by coalesced
    // asynchronous copies: step k (pairs 8k .. 8k + 7) into buffer k & 1.
    const int64_t r0 = m0 + quarter * 32;
    const int rows = static_cast<int>(M - r0 < 32 ? M - r0 : 32);
    const bool use_tab = has && rows > 0 && kind < 2;  // uniform per warp
    auto tab_copy = [&](int k) {
      uint8_t* dst = tb + (k & 1) * kRopeTabBufBytes;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int q = lane + 32 * j, row = q >> 2, part = q & 3;
        const int64_t src_row = r0 + row < M ? r0 + row : M - 1;
        cp_async16(dst + row * 64 + 16 * (part ^ ((row >> 1) & 3)),
                   args.rope_tab + src_row * 128 + 16 * k + 4 * part);
      }
      cp_async_commit();
    };
    if (use_tab) {
      tab_copy(0);
      tab_copy(1);
    }
    __syncwarp();
    const bool got = ovb_wait(smem_u32(&tfull[d]), ph, abort);
    if (!__all_sync(0xffffffffu, got)) {
      if (lane == 0) {
        atomicOr(&g_status_f16, kErrEpilogue);
        *abort = 1;
      }
      if (use_tab) cp_async_wait_n<0>();  // no copy stays in flight
    } else {
      tc_fence_after();
      if (has && rows > 0) {  // uniform per warp
        const uint32_t dcol =
            tmem_base + lane_off + static_cast<uint32_t>(d * BN + 128 * eh);
        const bool row_ok = lane < rows;
        uint32_t amax = 0u;  // this row's fp16 outputs' magnitude maximum (absmax_h2)
        const float4* ws4 = reinterpret_cast<const float4*>(colv);
        const float4* nw4 = reinterpret_cast<const float4*>(colv + 128);
        float scale = 0.f;
        if (kind < 2) {
          // pass 1: s01 = x0^2 + x1^2 (chunks 0 and 1), then + (x2^2 + x3^2),
          // element pairs (2i, 2i + 1) in s2[i]
          float2 s2[16];
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {  // chunks 2 pr and 2 pr + 1
              uint32_t va[16], vb[16];
              tmem_ld16(dcol + static_cast<uint32_t>(64 * pr + 16 * hf), va);
              tmem_ld16(dcol + static_cast<uint32_t>(64 * pr + 32 + 16 * hf), vb);
              tc_wait_ld16(va);
              tc_wait_ld16(vb);
#pragma unroll
              for (int gg = 0; gg < 2; ++gg) {
                float4 wa[2], wb[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                  wa[u] = *(ws4 + 16 * pr + 4 * hf + 2 * gg + u);
                  wb[u] = *(ws4 + 16 * pr + 8 + 4 * hf + 2 * gg + u);
                }
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                  const int iv = 8 * gg + e;
                  const float2 x = mul2(make_float2(__uint_as_float(va[iv]), __uint_as_float(va[iv + 1])),
                                        f4_pair(wa, e));
                  const float2 y = mul2(make_float2(__uint_as_float(vb[iv]), __uint_as_float(vb[iv + 1])),
                                        f4_pair(wb, e));
                  // a sum of two products stays scalar (add2rn would be
                  // contracted with the products); sums of sums are packed
                  const float2 xx = mul2(x, x), yy = mul2(y, y);
                  const float2 q = make_float2(__fadd_rn(xx.x, yy.x), __fadd_rn(xx.y, yy.y));
                  const int si = (16 * hf + iv) >> 1;
                  s2[si] = pr == 0 ? q : add2rn(s2[si], q);
                }
              }
            }
          }
          // s[i] += s[i + o] for o = 16, 8, 4, 2 (pairs), then 1
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) {
#pragma unroll
            for (int i = 0; i < o; ++i) s2[i] = add2rn(s2[i], s2[i + o]);
          }
          const float s01 = __fadd_rn(s2[0].x, s2[0].y);
          scale = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s01, 128.f), args.rope_eps)));
        }
        // The output rows of this head.
        __half* out;
        int64_t ld, col0;
        if (kind == 0) {
          out = static_cast<__half*>(args.rope_q16);
          ld = qd;
          col0 = hc;
        } else if (kind == 1) {
          out = static_cast<__half*>(args.rope_k16);
          ld = kvd;
          col0 = hc - qd;
        } else {
          out = static_cast<__half*>(args.rope_v16);
          ld = kvd;
          col0 = hc - qd - kvd;
        }
#pragma unroll
        for (int s = 0; s < 2; ++s) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            // set s, elements 16 hf .. 16 hf + 15: lo columns 32s + 16hf ..,
            // hi columns 64 + 32s + 16hf ..
            uint32_t va[16], vb[16];
            tmem_ld16(dcol + static_cast<uint32_t>(32 * s + 16 * hf), va);
            tmem_ld16(dcol + static_cast<uint32_t>(64 + 32 * s + 16 * hf), vb);
            tc_wait_ld16(va);
            tc_wait_ld16(vb);
#pragma unroll
            for (int gg = 0; gg < 2; ++gg) {
              const int g = 2 * hf + gg;  // 16-byte chunk g (lo) and 4 + g (hi)
              const int k = 4 * s + g;    // table step: pairs 8k .. 8k + 7
              float4 cs[4];               // this row's pairs 8k + 2p, 8k + 2p + 1
              if (use_tab) {
                if (k + 1 < 8) cp_async_wait_n<1>(); else cp_async_wait_n<0>();
                __syncwarp();
                const uint8_t* src = tb + (k & 1) * kRopeTabBufBytes + lane * 64;
#pragma unroll
                for (int p = 0; p < 4; ++p)
                  cs[p] = *reinterpret_cast<const float4*>(src + 16 * (p ^ ((lane >> 1) & 3)));
                __syncwarp();
                if (k + 2 < 8) tab_copy(k + 2);
              }
              // the eight elements' wscale and norm weights (broadcast reads)
              float4 wa[2], wb[2], na[2], nb[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                wa[u] = *(ws4 + 8 * s + 2 * g + u);
                wb[u] = *(ws4 + 16 + 8 * s + 2 * g + u);
                na[u] = kind < 2 ? *(nw4 + 8 * s + 2 * g + u) : make_float4(0.f, 0.f, 0.f, 0.f);
                nb[u] = kind < 2 ? *(nw4 + 16 + 8 * s + 2 * g + u)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
              }
              uint32_t lo_w[4], hi_w[4];
#pragma unroll
              for (int e = 0; e < 8; e += 2) {
                // elements e, e + 1 of the step (va / vb elements 8 gg + e ..);
                // products packed two per instruction, sums scalar
                const int iv = 8 * gg + e;
                const float2 x = mul2(make_float2(__uint_as_float(va[iv]), __uint_as_float(va[iv + 1])),
                                      f4_pair(wa, e));
                const float2 y = mul2(make_float2(__uint_as_float(vb[iv]), __uint_as_float(vb[iv + 1])),
                                      f4_pair(wb, e));
                float2 lo = x, hi = y;
                if (kind < 2) {
                  // pairs 8k + e, 8k + e + 1: (cos, cos, sin, sin) of both
                  // elements (rotation pairs are columns i and 64 + i: lo and hi)
                  const float4 c2 = cs[e >> 1];
                  const float2 cv = make_float2(c2.x, c2.y), sv = make_float2(c2.z, c2.w);
                  const float2 sc = make_float2(scale, scale);
                  const float2 a = mul2(mul2(x, sc), f4_pair(na, e));
                  const float2 b = mul2(mul2(y, sc), f4_pair(nb, e));
                  const float2 ac = mul2(a, cv), bs = mul2(b, sv);
                  const float2 bc = mul2(b, cv), as = mul2(a, sv);
                  lo = make_float2(__fsub_rn(ac.x, bs.x), __fsub_rn(ac.y, bs.y));
                  hi = make_float2(__fadd_rn(bc.x, as.x), __fadd_rn(bc.y, as.y));
                }
                const __half2 l2 = __floats2half2_rn(lo.x, lo.y);
                const __half2 h2 = __floats2half2_rn(hi.x, hi.y);
                lo_w[e >> 1] = *reinterpret_cast<const uint32_t*>(&l2);
                hi_w[e >> 1] = *reinterpret_cast<const uint32_t*>(&h2);
                amax = absmax_h2(absmax_h2(amax, lo_w[e >> 1]), hi_w[e >> 1]);
              }
              *reinterpret_cast<uint4*>(st8 + lane * 128 + 16 * (g ^ (lane & 7))) =
                  make_uint4(lo_w[0], lo_w[1], lo_w[2], lo_w[3]);
              *reinterpret_cast<uint4*>(st8 + lane * 128 + 16 * ((4 + g) ^ (lane & 7))) =
                  make_uint4(hi_w[0], hi_w[1], hi_w[2], hi_w[3]);
            }
          }
          __syncwarp();
          // chunk k of row r: columns 32s + 8k (k < 4) or 64 + 32s + 8(k - 4)
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int r = it * 4 + (lane >> 3);
            const int k = lane & 7;
            const int64_t col = col0 + (k < 4 ? 32 * s + 8 * k : 64 + 32 * s + 8 * (k - 4));
            if (r < rows)
              *reinterpret_cast<uint4*>(out + (r0 + r) * ld + col) =
                  *reinterpret_cast<const uint4*>(st8 + r * 128 + 16 * (k ^ (r & 7)));
          }
          __syncwarp();
        }
        if (row_ok && h2_inf_or_nan(amax)) range_ok = false;  // rows past M hold no outputs
      }
    }
    tc_fence_before();
    if (t + kAcc < my_tiles) named_sync(dfree_bar + d, 32 * (kEpiWarpsF + 1));
  }
  if (!range_ok) atomicOr(&g_status_f16, kErrF16Range);
}

// silu(g) * u for the fp16 mainloop's fused epilogue, which owes the
// contract's tolerance rather than the reference's bits: the hardware's
// approximate exponential and division (CUDA's __expf / __fdividef, relative
// error ~1e-6, far below the fp16 rounding of the activations).
__device__ __forceinline__ float silu_up_fast(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// Quantise the 32 SiLU outputs of one row's block with the block's absmax
// rule (gemm.cpp:379-430) into form kQMode (0 int8 q, 1 u8 q + 128, 2 fp16
// q * scale) at `dst` (shared memory, 32 or 64 bytes, 16-byte chunks
// XOR-swizzled by `sw`); returns the block scale.  |v * inv| <= 127 for finite
// v (inv = 127 / amax), so only NaN needs the x86 rule (-> -127), and an fp16
// value can overflow only if 127 * scale does.
template <int kQMode>
__device__ __forceinline__ float quant_row32(const float (&v)[32], uint8_t* dst, int sw,
                                            bool* range_bad) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  float scale, inv;
  block_scales(amax, &scale, &inv);
  int z[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float t = __fmul_rn(v[i], inv);
    int q = __float2int_rn(t);
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    z[i] = (t == t) ? q : -127;
  }
  if constexpr (kQMode == 2) {
    if (fabsf(__fmul_rn(127.0f, scale)) > 65504.f) *range_bad = true;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const __half2 x = __floats2half2_rn(__fmul_rn(static_cast<float>(z[8 * c + 2 * h]), scale),
                                            __fmul_rn(static_cast<float>(z[8 * c + 2 * h + 1]), scale));
        w[h] = *reinterpret_cast<const uint32_t*>(&x);
      }
      *reinterpret_cast<uint4*>(dst + 16 * (c ^ sw)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int q = z[16 * c + 4 * h + b];
          word |= (kQMode == 1 ? static_cast<uint32_t>(q + 128) : static_cast<uint32_t>(q & 0xFF))
                  << (8 * b);
        }
        w[h] = word;
      }
      *reinterpret_cast<uint4*>(dst + 16 * (c ^ (sw & 1))) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  return scale;
}

// The epilogue loop of the fused SiLU*up mode (gate|up weight, rows
// interleaved in 32-row blocks): chunk 2p of a tile is gate block
// J = n0/64 + p, chunk 2p+1 the up block J.  The kEpiW epilogue warps are
// kEpiW/4 per TMEM lane quarter; warp (quarter, eh) takes the pairs
// p = eh, eh + kEpiW/4, ...: each thread holds one row's 32 gate and 32 up
// accumulators, forms g = D_g * wscale and u = D_u * wscale per column, then
// v = silu(g) * u (silu_mul_quantize_f32's formula, ops_cpu.cpp:144-198, with
// fast exp/division) and quantises the whole 32-column block of its row into
// the warp's staging rows `stg` (32 rows x 64 bytes, 16-byte chunks swizzled
// so that both the row-per-lane writes and the reads below are free of bank
// conflicts), from where each store instruction writes whole row segments
// of 32 / (row bytes / 16) rows.  kQMode is the output form (silu_mode).
template <int BN, int kAcc, int kEpiW, int kQMode>
__device__ __forceinline__ void epilogue_silu_loop(const GemmArgs& args, uint64_t* tfull,
                                                   volatile int* abort, uint32_t tmem_base,
                                                   uint8_t* stg, int quarter, int eh,
                                                   int dfree_bar, int64_t tiles, TileOrder m_tiles,
                                                   int64_t my_tiles, int64_t tile_first,
                                                   int64_t tile_step) {
  constexpr int kPairs = BN / 64;
  constexpr int kPerQ = kEpiW / 4;  // warps per lane quarter
  constexpr int kMine = (kPairs + kPerQ - 1) / kPerQ;
  constexpr int kRowBytes = kQMode == 2 ? 64 : 32;  // one block of a row
  constexpr int kChunks = kRowBytes / 16;
  constexpr int kRowsPerStore = 32 / kChunks;
  const int lane = threadIdx.x & 31;
  const int64_t M = args.M, N = args.N;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const int64_t row_stride = args.silu_kp * (kQMode == 2 ? 2 : 1);  // bytes
  bool range_bad = false;
  int64_t t = 0;
  for (int64_t tile = tile_first; tile < tiles; tile += tile_step, ++t) {
    const int d = static_cast<int>(t % kAcc);
    const uint32_t ph = static_cast<uint32_t>((t / kAcc) & 1);
    int64_t m0, n0;
    tile_origin(tile, m_tiles, BN, &m0, &n0);
    float wsg[kMine], wsu[kMine];
#pragma unroll
    for (int i = 0; i < kMine; ++i) {
      const int64_t ng = n0 + (eh + kPerQ * i) * 64 + lane;
      const bool ok = eh + kPerQ * i < kPairs && ng + 32 < N;
      wsg[i] = ok ? __ldg(args.wscale + ng) : 0.f;
      wsu[i] = ok ? __ldg(args.wscale + ng + 32) : 0.f;
    }
    const bool got = ovb_wait(smem_u32(&tfull[d]), ph, abort);
    if (!__all_sync(0xffffffffu, got)) {
      if (lane == 0) {
        atomicOr(&g_status_f16, kErrEpilogue);
        *abort = 1;
      }
    } else {
      tc_fence_after();
      const int64_t rbase = m0 + quarter * 32;  // first row of this warp
      const uint32_t dcol = tmem_base + lane_off + static_cast<uint32_t>(d * BN);
#pragma unroll
      for (int i = 0; i < kMine; ++i) {
        const int p = eh + kPerQ * i;
        if (p >= kPairs) break;
        uint32_t vg[32], vu[32];
        tmem_ld32(dcol + static_cast<uint32_t>(p * 64), vg);
        tmem_ld32(dcol + static_cast<uint32_t>(p * 64 + 32), vu);
        tc_wait_ld32(vg);
        tc_wait_ld32(vu);
        // All lanes form v (the shuffles need the whole warp); rows past M
        // and columns past N are not stored.
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float g = __fmul_rn(__uint_as_float(vg[j]), __shfl_sync(0xffffffffu, wsg[i], j));
          const float u = __fmul_rn(__uint_as_float(vu[j]), __shfl_sync(0xffffffffu, wsu[i], j));
          v[j] = silu_up_fast(g, u);
        }
        if (n0 + p * 64 >= N) continue;  // uniform per warp
        const int64_t J = n0 / 64 + p;
        const float sc = quant_row32<kQMode>(v, stg + lane * 64, (lane >> 1) & 3, &range_bad);
        if (rbase + lane < M) args.silu_asc[(rbase + lane) * (args.silu_kp / 32) + J] = sc;
        __syncwarp();
        uint8_t* out = args.silu_out + rbase * row_stride + J * kRowBytes;
#pragma unroll
        for (int it = 0; it < 32 / kRowsPerStore; ++it) {
          const int r = it * kRowsPerStore + lane / kChunks;
          const int c = lane % kChunks;
          const int sw = kQMode == 2 ? ((r >> 1) & 3) : ((r >> 1) & 1);
          if (rbase + r < M)
            *reinterpret_cast<uint4*>(out + r * row_stride + 16 * c) =
                *reinterpret_cast<const uint4*>(stg + r * 64 + 16 * (c ^ sw));
        }
        __syncwarp();
      }
    }
    tc_fence_before();
    if (t + kAcc < my_tiles) named_sync(dfree_bar + d, 32 * (kEpiW + 1));
  }
  if (range_bad) atomicOr(&g_status_f16, kErrF16Range);
}

// epilogue_silu_loop with the output form args.silu_mode as a compile-time
// constant; the staging rows are the warp's 32 x 64 bytes at `stg`.
template <int BN, int kAcc, int kEpiW>
__device__ __forceinline__ void silu_epilogue(const GemmArgs& args, uint64_t* tfull,
                                              volatile int* abort, uint32_t tmem_base,
                                              uint8_t* stg, int quarter, int eh, int dfree_bar,
                                              int64_t tiles, TileOrder m_tiles, int64_t my_tiles,
                                              int64_t tile_first, int64_t tile_step) {
  switch (args.silu_mode) {
    case 0:
      epilogue_silu_loop<BN, kAcc, kEpiW, 0>(args, tfull, abort, tmem_base, stg, quarter, eh,
                                             dfree_bar, tiles, m_tiles, my_tiles, tile_first,
                                             tile_step);
      break;
    case 1:
      epilogue_silu_loop<BN, kAcc, kEpiW, 1>(args, tfull, abort, tmem_base, stg, quarter, eh,
                                             dfree_bar, tiles, m_tiles, my_tiles, tile_first,
                                             tile_step);
      break;
    default:
      epilogue_silu_loop<BN, kAcc, kEpiW, 2>(args, tfull, abort, tmem_base, stg, quarter, eh,
                                             dfree_bar, tiles, m_tiles, my_tiles, tile_first,
                                             tile_step);
      break;
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreadsF, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ GemmArgs args) {
  using T = TileF<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* stg_all = reinterpret_cast<float*>(smem + static_cast<size_t>(kStagesF) * T::kStageBytes);
  CtlF* ctl = reinterpret_cast<CtlF*>(reinterpret_cast<uint8_t*>(stg_all) +
                                      static_cast<size_t>(kEpiWarpsF) * T::kStgBytes);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int64_t M = args.M, N = args.N;
  const int Kb = static_cast<int>(args.Kb);
  const int ksteps = (Kb + 1) / 2;  // stages per tile
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  const int64_t n_tiles = (N + BN - 1) / BN;
  const int64_t tiles = m_tiles * n_tiles;
  const int64_t my_tiles =
      tiles > blockIdx.x ? (tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesF; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int d = 0; d < 2; ++d) mbar_init(smem_u32(&ctl->tfull[d]), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemColsF);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  pdl_wait();  // the preceding kernel's outputs (A, residual C) are complete
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int64_t st = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        int64_t m0l, n0l;
        tile_origin(tile, m_tiles, BN, &m0l, &n0l);
        const int32_t m0 = static_cast<int32_t>(m0l), n0 = static_cast<int32_t>(n0l);
        for (int j = 0; j < ksteps; ++j, ++st) {
          const int s = static_cast<int>(st % kStagesF);
          const uint32_t ph = static_cast<uint32_t>((st / kStagesF) & 1);
          if (!ovb_wait(smem_u32(&ctl->empty[s]), ph ^ 1u, abort)) {
            fail(ctl, kErrProducer);
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&ctl->full[s]);
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * T::kStageBytes);
          mbar_arrive_expect_tx(full, T::kStageBytes);
          tma_load_2d(sa, &tmap_a, j * kStageKF, m0, full);             // x in bytes (int8)
          tma_load_2d(sa + kABytesF, &tmap_w, j * kStageKF, n0, full);  // x in fp16 elements
        }
      }
      if (!ok) {
        const int64_t first = st > kStagesF ? st - kStagesF : 0;
        for (int64_t j = first; j < st; ++j) {
          const int s = static_cast<int>(j % kStagesF);
          const uint32_t ph = static_cast<uint32_t>((j / kStagesF) & 1);
          volatile int never = 0;
          ovb_wait(smem_u32(&ctl->full[s]), ph, &never);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_f16(kBlockM, BN);
    int64_t st = 0;
    for (int64_t t = 0; t < my_tiles; ++t) {
      const int d = static_cast<int>(t % T::kAcc);
      if (t >= T::kAcc) named_sync(kBarDfree + d, kBarDfreeThreads);  // accumulator d read
      const uint32_t dcol = tmem_base + static_cast<uint32_t>(d * BN);
      for (int j = 0; j < ksteps; ++j, ++st) {
        const int s = static_cast<int>(st % kStagesF);
        named_sync(kBarStage + s, kBarStageThreads);  // A' of stage s in TMEM, W landed
        if (lane == 0) {
          tc_fence_after();
          const uint32_t acol =
              tmem_base + static_cast<uint32_t>(T::kACol0 + s * kAColsPerStage);
          const uint32_t sw = smem_u32(smem + static_cast<size_t>(s) * T::kStageBytes + kABytesF);
#pragma unroll
          for (int kk = 0; kk < kStageKF / 16; ++kk)
            mma_f16_ts(dcol, acol + static_cast<uint32_t>(kk * 8),
                       sw128_kmajor_desc(sw, static_cast<uint32_t>(kk * 32)), idesc,
                       (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(smem_u32(&ctl->empty[s]));
          if (j == ksteps - 1) tc_commit(smem_u32(&ctl->tfull[d]));
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      tc_commit(smem_u32(&ctl->drain));
      volatile int never = 0;
      if (!ovb_wait(smem_u32(&ctl->drain), 0u, &never)) atomicOr(&g_status_f16, kErrDrain);
    }
    __syncwarp();
  } else if (warp < kFirstEpi) {
    // ---------------------------------------------------------- converters
    // TMEM lanes 32*quarter.. are the rows this warp may write; `half`
    // picks the stage's first or second quantisation block.
    const int quarter = warp & 3;
    const int half = (warp - kFirstConv) >> 2;
    const int r = quarter * 32 + lane;  // row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    int64_t st = 0;
    bool range_ok = true;
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int64_t m = static_cast<int64_t>(static_cast<uint32_t>(tile) % static_cast<uint32_t>(m_tiles)) * kBlockM + r;
      const bool row_ok = m < M;
      const float* asc_row = args.asc + (row_ok ? m : 0) * static_cast<int64_t>(Kb);
      auto scale_of = [&](int j) -> float {
        const int b = 2 * j + half;
        return (row_ok && j < ksteps && b < Kb) ? __ldg(asc_row + b) : 0.f;
      };
      // One stage: wait for its TMA, dequantise this thread's 32 values
      // into the stage's A' slot, meet the MMA warp.
      auto do_stage = [&](float sc) {
        const int s = static_cast<int>(st % kStagesF);
        const uint32_t ph = static_cast<uint32_t>((st / kStagesF) & 1);
        const bool got = ovb_wait(smem_u32(&ctl->full[s]), ph, abort);
        if (!__all_sync(0xffffffffu, got)) {
          if (lane == 0) fail(ctl, kErrConvert);
        } else {
          // Row r's 32 bytes of this block: 16-byte chunks 2*half and
          // 2*half+1 of its 64-byte row, placed by the 64-byte swizzle at
          // chunk c ^ ((r >> 1) & 3).
          const uint8_t* arow = smem + static_cast<size_t>(s) * T::kStageBytes + r * 64;
          const int sw = (r >> 1) & 3;
          const uint4 c0 = *reinterpret_cast<const uint4*>(arow + (((2 * half) ^ sw) << 4));
          const uint4 c1 = *reinterpret_cast<const uint4*>(arow + (((2 * half + 1) ^ sw) << 4));
          if (sc * 127.f > 65504.f) range_ok = false;
          const __half h_hi = __float2half_rn(sc);
          const __half h_lo = __float2half_rn(sc - __half2float(h_hi));
          const __half2 s_hi = __half2half2(h_hi), s_lo = __half2half2(h_lo);
          uint32_t v[16];
          dequant4(c0.x, s_hi, s_lo, v[0], v[1]);
          dequant4(c0.y, s_hi, s_lo, v[2], v[3]);
          dequant4(c0.z, s_hi, s_lo, v[4], v[5]);
          dequant4(c0.w, s_hi, s_lo, v[6], v[7]);
          dequant4(c1.x, s_hi, s_lo, v[8], v[9]);
          dequant4(c1.y, s_hi, s_lo, v[10], v[11]);
          dequant4(c1.z, s_hi, s_lo, v[12], v[13]);
          dequant4(c1.w, s_hi, s_lo, v[14], v[15]);
          tmem_st16(tmem_base + lane_off +
                        static_cast<uint32_t>(T::kACol0 + s * kAColsPerStage + half * 16),
                    v);
          tc_wait_st();
        }
        tc_fence_before();
        named_sync(kBarStage + s, kBarStageThreads);
        ++st;
      };
      // Block scales of a group of four stages are loaded one group ahead
      // into their own registers and indexed statically: no register with a
      // load in flight is ever copied (a copy would wait for the load).
      float cur[4], nxt[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) cur[u] = scale_of(u);
      for (int j0 = 0; j0 < ksteps; j0 += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) nxt[u] = scale_of(j0 + 4 + u);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j0 + u < ksteps) do_stage(cur[u]);
#pragma unroll
        for (int u = 0; u < 4; ++u) cur[u] = nxt[u];
      }
    }
    if (!range_ok) atomicOr(&g_status_f16, kErrF16Range);
  } else {
    // ------------------------------------------------------------ epilogue
    epilogue_loop<BN, T::kAcc, false>(args, ctl->tfull, abort, tmem_base,
                                      stg_all + (warp - kFirstEpi) * (32 * kStgStrideF), warp & 3,
                                      (warp - kFirstEpi) >> 2, kBarDfree, tiles, m_tiles,
                                      my_tiles, blockIdx.x, gridDim.x);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemColsF);
  }
}

// ---------------------------------------------------------------------------
// The plain fp16 mainloop (ovb_linear_h): the activations arrive already
// dequantised, fp16(q * asc) from a quantiser run with OVB_AQ_F16, so both
// operands come from shared memory and no warp converts anything.  Warps:
//   0  TMA producer: A box 64 fp16 x 128 rows and W box 64 fp16 x BN rows
//      (both 128-byte swizzle) per 64-k stage into a 4-stage ring;
//   1  TMEM allocator + MMA issuer: four K = 16 MMAs per stage;
//   2  stage watcher: waits `full[s]` and meets the MMA warp on kBarFullH
//      (bar.sync on both sides, so the MMA thread never waits on an
//      mbarrier while it has MMAs in flight);
//   3..10 epilogue (epilogue_loop), accumulators double-buffered in TMEM.
constexpr int kMaxStagesH = 8;
constexpr int kFirstEpiH = 3;
// Epilogue warps: 8 for plain outputs (each stages 32x32 chunks in shared
// memory); 16 for the fused SiLU*up epilogue, which is arithmetic-heavy and
// needs no staging.
template <bool kSilu>
constexpr int epi_warps_h() { return kSilu ? 16 : kEpiWarpsF; }
constexpr uint32_t kABytesH = kBlockM * kStageKF * 2;  // 16 KB
constexpr int kBarFullH = 1;
constexpr int kBarDfreeH = 2;  // + d

struct CtlH {
  uint64_t full[kMaxStagesH];
  uint64_t empty[kMaxStagesH];
  uint64_t tfull[2];
  uint64_t pfree[2];  // CTA pair: the peer's epilogue released accumulator d
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  uint32_t my_sm;  // split-K: %smid of this CTA (its workspace slot)
};

// kSplit > 1: the CTAs of a kSplit-CTA cluster share one output tile and
// split its k-stages; rank r owns the columns [r * kOwn, (r + 1) * kOwn) of
// the tile and receives the other ranks' partial accumulators for them in
// its SM's slot of the split-K workspace (global memory, L2-resident):
// [kSplit - 1 senders][128 rows][kOwn floats].  A split-K CTA needs more
// than half of the SM's shared memory, so no two of them share an SM (or a
// workspace slot).
template <int BN, bool kSilu, int kSplit = 1>
struct TileH {
  static_assert(kSplit == 1 || (!kSilu && (BN / kSplit) % 32 == 0), "split-K layout");
  static constexpr uint32_t kWBytes = BN * 128;
  static constexpr uint32_t kStageBytes = kABytesH + kWBytes;
  static constexpr int kAcc = 2;
  static constexpr int kEpiW = epi_warps_h<kSilu>();
  static constexpr int kThreads = 32 * (kFirstEpiH + kEpiW);
  // per epilogue warp: 32 x 64 bytes of quantised rows (SiLU*up), a 32 x 36
  // float chunk (split-K), or the plain epilogue's area
  static constexpr size_t kStgWarp =
      kSilu ? 32 * 64 : (kSplit > 1 ? 32 * kStgStrideF * 4 : kStgWarpBytes);
  static constexpr size_t kStgAll = static_cast<size_t>(kEpiW) * kStgWarp;
  static constexpr int kOwn = BN / kSplit;  // columns owned per rank
  static constexpr size_t kPartialFloats = static_cast<size_t>(kBlockM) * kOwn;  // per sender
  // As many stages as fit (a deeper ring hides more TMA latency; narrow
  // tiles have small stages), at most kMaxStagesH.
  static constexpr int kStagesFit =
      static_cast<int>((227 * 1024 - 1024 - kStgAll - sizeof(CtlH)) / kStageBytes);
  static constexpr int kStages = kStagesFit < kMaxStagesH ? kStagesFit : kMaxStagesH;
  static constexpr size_t kSmemBytes =
      1024 + static_cast<size_t>(kStages) * kStageBytes + kStgAll + sizeof(CtlH);
  static_assert(kStages >= 3, "too few pipeline stages");
  static_assert(kAcc * BN <= static_cast<int>(kTmemColsF), "accumulators exceed TMEM");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert((kStageBytes % 1024 == 0 && kStgWarp % 1024 == 0) || kSilu || kSplit > 1,
                "TMA output boxes stay 1 KB aligned");
  static_assert(kSplit == 1 || kSmemBytes > 116 * 1024, "a split-K CTA must have its SM alone");
  static_assert(kSplit == 1 || (kSplit - 1) * kPartialFloats * 4 <= kSplitSlotBytes,
                "split-K workspace slot");
};

// The split-K epilogue (one tile per cluster), in two phases around a
// cluster barrier that every thread of the cluster executes.  Warp
// (quarter, eh) handles the 32-column chunks c = eh, eh+2, ... of rows
// 32*quarter..; rank o = c*32 / kOwn owns chunk c.
// Phase 1 (split_send): a chunk another rank owns is staged in shared memory
// and written with coalesced float4 stores into the owner's workspace slot,
// sender slot (rank < o ? rank : rank - 1).
// Phase 2 (split_finish, after barrier.cluster arrive.release / wait.acquire,
// which makes those global stores visible cluster-wide): for an owned chunk
// the partials are summed in rank order 0, 1, ..., kSplit-1 (deterministic),
// then o = sum * wscale (+ C) as in the plain epilogue.
template <int BN, int kSplit>
__device__ __forceinline__ void split_send(const GemmArgs& args, CtlH* ctl, volatile int* abort,
                                           uint32_t tmem_base, float* stg, int quarter, int eh,
                                           int rank) {
  using T = TileH<BN, false, kSplit>;
  constexpr int kChunks = BN / 32;
  const int lane = threadIdx.x & 31;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  // The other ranks' SMs (workspace slots), read before the accumulator is
  // ready.  Every rank is alive until it has passed the cluster barrier,
  // which it cannot do before this rank arrives there.
  uint32_t peer[kSplit];
#pragma unroll
  for (int r = 0; r < kSplit; ++r)
    peer[r] = ld_cluster_u32(mapa_shared(smem_u32(&ctl->my_sm), static_cast<uint32_t>(r)));
  const bool got = ovb_wait(smem_u32(&ctl->tfull[0]), 0u, abort);
  if (!__all_sync(0xffffffffu, got) && lane == 0) {
    atomicOr(&g_status_f16, kErrEpilogue);
    *abort = 1;
  }
  tc_fence_after();
  const int c4 = (lane & 7) * 4;
#pragma unroll
  for (int c = eh; c < kChunks; c += 2) {
    const int o = (c * 32) / T::kOwn;
    if (o == rank) continue;
    uint32_t v[32];
    tmem_ld32(tmem_base + lane_off + static_cast<uint32_t>(c * 32), v);
    tc_wait_ld32(v);
    stage_chunk(stg, v);
    __syncwarp();
    uint32_t sm = 0;
#pragma unroll
    for (int r = 0; r < kSplit; ++r)
      if (r == o) sm = peer[r];
    if (sm < static_cast<uint32_t>(kSplitSlots)) {
      const int slot = rank < o ? rank : rank - 1;
      float* dst = args.split_ws + static_cast<size_t>(sm) * (kSplitSlotBytes / 4) +
                   static_cast<size_t>(slot) * T::kPartialFloats +
                   static_cast<size_t>(quarter * 32) * T::kOwn + (c * 32 - o * T::kOwn);
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + (lane >> 3);
        *reinterpret_cast<float4*>(dst + r * T::kOwn + c4) =
            *reinterpret_cast<const float4*>(stg + r * kStgStrideF + c4);
      }
    } else if (lane == 0) {
      atomicOr(&g_status_f16, kErrEpilogue);
    }
    __syncwarp();
  }
}

// Both warps of a lane quarter (eh = 0, 1) reduce each owned chunk, warp eh
// the rows 16*eh .. 16*eh + 15 of the quarter (row groups it = 4*eh ..
// 4*eh + 3), so that every residual and partial load of a thread is issued
// in one predicated batch before the sums.
template <int BN, int kSplit>
__device__ __forceinline__ void split_finish(const GemmArgs& args, CtlH* ctl,
                                             uint32_t tmem_base, float* stg, int quarter, int eh,
                                             int rank, int64_t tile, int64_t m_tiles) {
  using T = TileH<BN, false, kSplit>;
  constexpr int kOC = T::kOwn / 32;  // chunks owned per rank
  constexpr int kP = kSplit - 1;     // partials per element from the other ranks
  const int lane = threadIdx.x & 31;
  const int64_t M = args.M, N = args.N;
  int64_t m0, n0;
  tile_origin(tile, m_tiles, BN, &m0, &n0);
  const int64_t r0 = m0 + quarter * 32;
  const int rows = static_cast<int>(M - r0 < 32 ? M - r0 : 32);
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const uint32_t sm = ctl->my_sm;
  const bool have = sm < static_cast<uint32_t>(kSplitSlots);
  const int c4 = (lane & 7) * 4;
  const int it0 = eh * 4;
#pragma unroll
  for (int k = 0; k < kOC; ++k) {
    const int c = rank * kOC + k;  // chunk of the tile
    const int64_t nc = n0 + c * 32;
    if (nc >= N || rows <= 0) continue;  // uniform per warp
    int si = 0;
#pragma unroll
    for (int q = 1; q < kMaxSlices; ++q)
      if (q < args.n_slices && nc >= args.slices[q].n_begin) si = q;
    const SliceOut so = args.slices[si];
    const int64_t local = nc - so.n_begin;
    const int ncols = static_cast<int>(so.n_count - local < 32 ? so.n_count - local : 32);
    float* cbase = so.C + r0 * so.ldc + local;
    const bool vec = rows_aligned(so);
    const float* part = args.split_ws + static_cast<size_t>(have ? sm : 0) * (kSplitSlotBytes / 4) +
                        static_cast<size_t>(quarter * 32) * T::kOwn + k * 32 + c4;
    // One batch of loads: the residual (float4 path) and the partials.
    float4 old[4];
    if (vec && args.accumulate) {
      load_residual<4>(cbase, so.ldc, rows, ncols, it0, old);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) old[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float4 pr[kP][4];
#pragma unroll
    for (int sl = 0; sl < kP; ++sl)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        pr[sl][i] = ld_f4_cg_if(part + static_cast<size_t>(sl) * T::kPartialFloats +
                                    ((it0 + i) * 4 + (lane >> 3)) * T::kOwn,
                                have);
    const float wl = lane < ncols ? __ldg(args.wscale + nc + lane) : 0.f;
    float ws[4];
    gather_ws4(wl, ws);
    uint32_t v[32];
    tmem_ld32(tmem_base + lane_off + static_cast<uint32_t>(c * 32), v);
    tc_wait_ld32(v);
    stage_chunk(stg, v);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (it0 + i) * 4 + (lane >> 3);
      float* own_p = stg + r * kStgStrideF + c4;
      const float4 own = *reinterpret_cast<const float4*>(own_p);
      // Ranks in order 0 .. kSplit-1; rank q's partial is in sender slot
      // q (q < rank) or q - 1 (q > rank).
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kSplit; ++q) {
        float4 p = own;
        if (q < kP && q < rank) p = pr[q < kP ? q : 0][i];
        if (q >= 1 && q > rank) p = pr[q >= 1 ? q - 1 : 0][i];
        if (q == 0) {
          sum = p;
        } else {
          sum.x = __fadd_rn(sum.x, p.x);
          sum.y = __fadd_rn(sum.y, p.y);
          sum.z = __fadd_rn(sum.z, p.z);
          sum.w = __fadd_rn(sum.w, p.w);
        }
      }
      if (vec) {
        if (r < rows && c4 < ncols)
          put4(cbase, so.ldc, r, c4, ncols, scale_add4(sum, ws, old[i], args.accumulate));
      } else {
        *reinterpret_cast<float4*>(own_p) = sum;
      }
    }
    if (!vec) {  // scalar path: this warp's 16 rows, lane = column
      __syncwarp();
      const int rows_w = rows - 16 * eh < 16 ? rows - 16 * eh : 16;
      if (lane < ncols && rows_w > 0)
        store_rows(stg + 16 * eh * kStgStrideF + lane, kStgStrideF, cbase + 16 * eh * so.ldc + lane,
                   so.ldc, rows_w, wl, args.accumulate);
    }
    __syncwarp();
  }
}

template <int BN, bool kSilu, int kSplit>
__global__ void __launch_bounds__(TileH<BN, kSilu, kSplit>::kThreads, 1)
    gemm_h_kernel(const __grid_constant__ CUtensorMap tmap_a,
                  const __grid_constant__ CUtensorMap tmap_w,
                  const __grid_constant__ GemmArgs args) {
  using T = TileH<BN, kSilu, kSplit>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* stg_all = reinterpret_cast<float*>(smem + static_cast<size_t>(T::kStages) * T::kStageBytes);
  CtlH* ctl = reinterpret_cast<CtlH*>(reinterpret_cast<uint8_t*>(stg_all) + T::kStgAll);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t M = args.M, N = args.N;
  const int Kb = static_cast<int>(args.Kb);
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  const int64_t n_tiles = (N + BN - 1) / BN;
  const int64_t tiles = m_tiles * n_tiles;
  // Split-K: one tile per cluster (grid = tiles * kSplit); rank r runs the
  // k-stages [j_begin, j_end).  Otherwise a persistent grid over the tiles.
  const int rank = kSplit > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  // Rank r gets stages [r*S/kSplit, (r+1)*S/kSplit): at least one each,
  // since the host launches split-K only when S >= kSplit.
  const int all_steps = (Kb + 1) / 2;
  const int j_begin = kSplit > 1 ? (rank * all_steps) / kSplit : 0;
  const int j_end = kSplit > 1 ? ((rank + 1) * all_steps) / kSplit : all_steps;
  const int ksteps = j_end - j_begin;
  const int64_t tile0 = kSplit > 1 ? static_cast<int64_t>(blockIdx.x) / kSplit : blockIdx.x;
  const int64_t tile_step = kSplit > 1 ? tiles : static_cast<int64_t>(gridDim.x);
  const int64_t my_tiles =
      tiles > tile0 ? (kSplit > 1 ? 1 : (tiles - tile0 + tile_step - 1) / tile_step) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::kStages; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int d = 0; d < 2; ++d) mbar_init(smem_u32(&ctl->tfull[d]), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    ctl->my_sm = sm_id();  // read by the cluster's other ranks after cluster_sync
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemColsF);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kSplit > 1) cluster_sync();  // every rank has started; my_sm is set
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  pdl_wait();  // the preceding kernel's outputs (A, residual C) are complete
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int64_t st = 0;
      bool ok = true;
      for (int64_t tile = tile0; tile < tiles && ok; tile += tile_step) {
        int64_t m0l, n0l;
        tile_origin(tile, m_tiles, BN, &m0l, &n0l);
        const int32_t m0 = static_cast<int32_t>(m0l), n0 = static_cast<int32_t>(n0l);
        for (int jj = 0; jj < ksteps; ++jj, ++st) {
          const int j = j_begin + jj;
          const int s = static_cast<int>(st % T::kStages);
          const uint32_t ph = static_cast<uint32_t>((st / T::kStages) & 1);
          // The ring's first pass needs no wait: those stages were never used.
          if (st >= T::kStages && !ovb_wait(smem_u32(&ctl->empty[s]), ph ^ 1u, abort)) {
            atomicOr(&g_status_f16, kErrProducer);
            *abort = 1;
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&ctl->full[s]);
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * T::kStageBytes);
          mbar_arrive_expect_tx(full, T::kStageBytes);
          tma_load_2d(sa, &tmap_a, j * kStageKF, m0, full);            // x in fp16 elements
          tma_load_2d(sa + kABytesH, &tmap_w, j * kStageKF, n0, full);
        }
      }
      if (!ok) {
        const int64_t first = st > T::kStages ? st - T::kStages : 0;
        for (int64_t j = first; j < st; ++j) {
          volatile int never = 0;
          ovb_wait(smem_u32(&ctl->full[j % T::kStages]), static_cast<uint32_t>((j / T::kStages) & 1),
                   &never);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_f16(kBlockM, BN);
    int64_t st = 0;
    for (int64_t t = 0; t < my_tiles; ++t) {
      const int d = static_cast<int>(t % T::kAcc);
      if (t >= T::kAcc) named_sync(kBarDfreeH + d, 32 * (T::kEpiW + 1));  // accumulator d read
      const uint32_t dcol = tmem_base + static_cast<uint32_t>(d * BN);
      for (int j = 0; j < ksteps; ++j, ++st) {
        const int s = static_cast<int>(st % T::kStages);
        named_sync(kBarFullH, 64);  // stage s has landed
        if (lane == 0) {
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * T::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < kStageKF / 16; ++kk)
            mma_f16_ss(dcol, sw128_kmajor_desc(sa, static_cast<uint32_t>(kk * 32)),
                       sw128_kmajor_desc(sa + kABytesH, static_cast<uint32_t>(kk * 32)), idesc,
                       (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(smem_u32(&ctl->empty[s]));
          if (j == ksteps - 1) tc_commit(smem_u32(&ctl->tfull[d]));
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      tc_commit(smem_u32(&ctl->drain));
      volatile int never = 0;
      if (!ovb_wait(smem_u32(&ctl->drain), 0u, &never)) atomicOr(&g_status_f16, kErrDrain);
    }
    __syncwarp();
  } else if (warp == 2) {
    // ----------------------------------------------------- stage watcher
    // Exactly one bar.sync per stage, in lockstep with the MMA warp, also
    // after a failed wait (the status word reports it).
    int64_t st = 0;
    for (int64_t t = 0; t < my_tiles; ++t) {
      for (int j = 0; j < ksteps; ++j, ++st) {
        const int s = static_cast<int>(st % T::kStages);
        const uint32_t ph = static_cast<uint32_t>((st / T::kStages) & 1);
        const bool got = ovb_wait(smem_u32(&ctl->full[s]), ph, abort);
        if (!__all_sync(0xffffffffu, got) && lane == 0) {
          atomicOr(&g_status_f16, kErrConvert);
          *abort = 1;
        }
        named_sync(kBarFullH, 64);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    if constexpr (kSplit > 1) {
      if (my_tiles > 0)
        split_send<BN, kSplit>(args, ctl, abort, tmem_base,
                               stg_all + (warp - kFirstEpiH) * (32 * kStgStrideF), warp & 3,
                               (warp - kFirstEpiH) >> 2, rank);
    } else if constexpr (kSilu) {
      uint8_t* stg = reinterpret_cast<uint8_t*>(stg_all) + (warp - kFirstEpiH) * (32 * 64);
      silu_epilogue<BN, T::kAcc, T::kEpiW>(args, ctl->tfull, abort, tmem_base, stg, warp & 3,
                                           (warp - kFirstEpiH) >> 2, kBarDfreeH, tiles, m_tiles,
                                           my_tiles, blockIdx.x, gridDim.x);
    } else {
      epilogue_loop<BN, T::kAcc, true, true>(
          args, ctl->tfull, abort, tmem_base,
          reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(stg_all) +
                                   (warp - kFirstEpiH) * T::kStgWarp),
          warp & 3, (warp - kFirstEpiH) >> 2, kBarDfreeH, tiles, m_tiles, my_tiles, blockIdx.x,
          gridDim.x);
    }
  }

  if constexpr (kSplit > 1) {
    // Every rank's partials are in their owners' workspace slots (release /
    // acquire at cluster scope covers the global stores); then the owners
    // reduce.  Executed by every thread of the cluster.
    cluster_sync();
    if (warp >= kFirstEpiH && my_tiles > 0)
      split_finish<BN, kSplit>(args, ctl, tmem_base,
                               stg_all + (warp - kFirstEpiH) * (32 * kStgStrideF), warp & 3,
                               (warp - kFirstEpiH) >> 2, rank, tile0, m_tiles);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemColsF);
  }
}

template <int BN, bool kSilu, int kSplit = 1>
cudaError_t launch_h_impl(const CUtensorMap& tmap_a, const CUtensorMap& tmap_w,
                          const GemmArgs& args, cudaStream_t s) {
  using T = TileH<BN, kSilu, kSplit>;
  auto* kernel = gemm_h_kernel<BN, kSilu, kSplit>;
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev = -1;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(T::kSmemBytes));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  const int64_t tiles = ((args.M + kBlockM - 1) / kBlockM) * ((args.N + BN - 1) / BN);
  if (tiles * 4 > INT32_MAX) return cudaErrorInvalidValue;  // 32-bit tile arithmetic
  if constexpr (kSplit == 1) {
    const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms(dev)));
    return launch_pdl(kernel, dim3(grid), dim3(T::kThreads), T::kSmemBytes, s, tmap_a, tmap_w,
                      args);
  } else {
    // One tile per kSplit-CTA cluster; every rank needs at least one stage.
    if ((args.Kb + 1) / 2 < kSplit) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles * kSplit));
    cfg.blockDim = dim3(T::kThreads);
    cfg.dynamicSmemBytes = T::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kSplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, tmap_a, tmap_w, args);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair fp16 mainloop (tcgen05 cta_group::2), persistent.  The two CTAs
// of a 2-CTA cluster compute 256 x BN output tiles: rank r TMA-loads its 128
// rows of A' and rows [r * BN/2, (r + 1) * BN/2) of the W tile into its own
// shared memory; the leader (rank 0) issues tcgen05.mma.cta_group::2 with
// M = 256, which reads both CTAs' operands, and each CTA's TMEM receives its
// 128 rows x BN columns.  Each SM loads half of the W tile, so a stage
// moves 32 KB into an SM's shared memory for 128 x 256 outputs instead of
// 48 KB: the single-CTA mainloop's bound (shared-memory and L2-to-SM
// traffic) drops by a third.
//   - Cluster c takes the tile pairs c, c + clusters, ...; pair p covers
//     rows [256 * (p / n_tiles), + 256) and columns [BN * (p % n_tiles),
//     + BN): n fastest, so the clusters running at the same time share A
//     rows and each A row block is read from DRAM once (m fastest re-read A
//     from DRAM for every column of tiles once it outgrew L2: 357 MB instead
//     of ~165 MB for the down projection at 15,408 rows).  Seen from one CTA
//     these are the tiles blockIdx.x + t * gridDim.x of the TileOrder
//     {2 * m_pairs, n_tiles, pair_nfast}, which the single-CTA epilogues take.
//   - Both CTAs' loads complete on the leader's `full[s]` barrier, which
//     the leader alone arms with both CTAs' bytes; each producer waits on
//     its own `empty[s]`, which the leader's commits reach in both CTAs
//     (multicast to cluster ranks 0 and 1), as they reach `tfull[d]`.
//   - Two accumulators per CTA (2 x BN TMEM columns), so a tile's epilogue
//     overlaps the next tile's mainloop.  Before the MMA warp reuses
//     accumulator d it bar.syncs with its own CTA's epilogue (kBarDfreeH + d)
//     and with the stage watcher (kBarPeerH), which has waited for the
//     peer's release: the peer's warp 1 bar.syncs with the peer's epilogue
//     and arrives on the leader's `pfree[d]` (release / acquire at cluster
//     scope).  The MMA thread itself never waits on an mbarrier.
//   - TMEM is allocated and freed collectively by warp 1 of both CTAs.
// No load uses cluster multicast.
constexpr int kBarPeerH = 4;

template <int BN, bool kSilu, bool kRope = false>
struct TileH2 {
  static_assert(BN == 256 || BN == 128, "pair tile widths");
  static_assert(!kRope || (BN == 256 && !kSilu), "the norm + RoPE epilogue takes two heads");
  static constexpr uint32_t kWBytes = (BN / 2) * 128;  // this CTA's half of the W rows
  static constexpr uint32_t kStageBytes = kABytesH + kWBytes;
  static constexpr int kAcc = 2;
  static constexpr int kEpiW = epi_warps_h<kSilu>();
  static constexpr int kThreads = 32 * (kFirstEpiH + kEpiW);
  // per epilogue warp: 32 x 64 bytes of quantised rows (SiLU*up), a 32 x 36
  // float chunk (norm + RoPE, then its column values and table buffers), or
  // the plain epilogue's area
  static constexpr size_t kStgWarp =
      kSilu ? 32 * 64 : (kRope ? 32 * kStgStrideF * 4 : kStgWarpBytes);
  static constexpr size_t kStgAll =
      static_cast<size_t>(kEpiW) * kStgWarp +
      (kRope ? static_cast<size_t>(kEpiW) * (kRopeColFloats * 4 + 2 * kRopeTabBufBytes) : 0);
  static constexpr int kStagesFit =
      static_cast<int>((227 * 1024 - 1024 - kStgAll - sizeof(CtlH)) / kStageBytes);
  static constexpr int kStages = kStagesFit < kMaxStagesH ? kStagesFit : kMaxStagesH;
  static constexpr size_t kSmemBytes =
      1024 + static_cast<size_t>(kStages) * kStageBytes + kStgAll + sizeof(CtlH);
  static_assert(kStages >= 3, "too few pipeline stages");
  static_assert(kAcc * BN <= static_cast<int>(kTmemColsF), "accumulators exceed TMEM");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert(kStageBytes % 1024 == 0, "stage bases stay 1 KB aligned");
  static_assert(kRope || kSilu || kStgWarp % 1024 == 0, "TMA output boxes stay 1 KB aligned");
};

template <int BN, bool kSilu, bool kRope>
__global__ void __launch_bounds__(TileH2<BN, kSilu, kRope>::kThreads, 1)
    gemm_h2_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ GemmArgs args) {
  using T = TileH2<BN, kSilu, kRope>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* stg_all = reinterpret_cast<float*>(smem + static_cast<size_t>(T::kStages) * T::kStageBytes);
  CtlH* ctl = reinterpret_cast<CtlH*>(reinterpret_cast<uint8_t*>(stg_all) + T::kStgAll);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t M = args.M, N = args.N;
  const int Kb = static_cast<int>(args.Kb);
  const int rank = static_cast<int>(cluster_ctarank());  // 0: leader, 1: peer
  const int64_t m_pairs = (M + 2 * kBlockM - 1) / (2 * kBlockM);
  const int64_t n_tiles = (N + BN - 1) / BN;
  const int64_t pairs = m_pairs * n_tiles;
  const int64_t cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  const int64_t my_tiles = pairs > cluster ? (pairs - cluster + clusters - 1) / clusters : 0;
  const TileOrder order(2 * m_pairs, n_tiles, true);  // the epilogues' view of the tiles
  const int ksteps = (Kb + 1) / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::kStages; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int d = 0; d < 2; ++d) {
      mbar_init(smem_u32(&ctl->tfull[d]), 1);
      mbar_init(smem_u32(&ctl->pfree[d]), 1);
    }
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&ctl->tmem_base), kTmemColsF);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised and their TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  pdl_wait();  // the preceding kernel's outputs (A, residual C) are complete
  pdl_launch_dependents();

  if (warp == 0) {
    // --------------------------------------------------- producer (both CTAs)
    if (lane == 0) {
      bool ok = true;
      int64_t st = 0;
      for (int64_t p = cluster; p < pairs && ok; p += clusters) {
        const int64_t pm = p / n_tiles, pn = p - pm * n_tiles;  // n fastest (TileOrder)
        const int32_t a_row = static_cast<int32_t>((2 * pm + rank) * kBlockM);
        const int32_t w_row = static_cast<int32_t>(pn * BN + rank * (BN / 2));
        for (int j = 0; j < ksteps; ++j, ++st) {
          const int s = static_cast<int>(st % T::kStages);
          const uint32_t ph = static_cast<uint32_t>((st / T::kStages) & 1);
          // The ring's first pass needs no wait: those stages were never used.
          if (st >= T::kStages && !ovb_wait(smem_u32(&ctl->empty[s]), ph ^ 1u, abort)) {
            atomicOr(&g_status_f16, kErrProducer);
            *abort = 1;
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(smem_u32(&ctl->full[s]), 2 * T::kStageBytes);
          const uint32_t bar = mapa_shared(smem_u32(&ctl->full[s]), 0u);  // the leader's
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * T::kStageBytes);
          tma_load_2d_pair(sa, &tmap_a, j * kStageKF, a_row, bar);
          tma_load_2d_pair(sa + kABytesH, &tmap_w, j * kStageKF, w_row, bar);
        }
      }
      if (!ok && rank == 0) {  // let the loads in flight land before the CTA can exit
        const int64_t first = st > T::kStages ? st - T::kStages : 0;
        for (int64_t j = first; j < st; ++j) {
          volatile int never = 0;
          ovb_wait(smem_u32(&ctl->full[j % T::kStages]),
                   static_cast<uint32_t>((j / T::kStages) & 1), &never);
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ------------------------------------------------------ MMA (leader)
      const uint32_t idesc = idesc_f16(2 * kBlockM, BN);
      int64_t st = 0;
      for (int64_t t = 0; t < my_tiles; ++t) {
        const int d = static_cast<int>(t % T::kAcc);
        if (t >= T::kAcc) {
          named_sync(kBarDfreeH + d, 32 * (T::kEpiW + 1));  // this CTA's epilogue read d
          named_sync(kBarPeerH, 64);                        // and the peer's (watcher)
        }
        const uint32_t dcol = tmem_base + static_cast<uint32_t>(d * BN);
        for (int j = 0; j < ksteps; ++j, ++st) {
          const int s = static_cast<int>(st % T::kStages);
          named_sync(kBarFullH, 64);  // stage s of both CTAs has landed
          if (lane == 0) {
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * T::kStageBytes);
#pragma unroll
            for (int kk = 0; kk < kStageKF / 16; ++kk)
              mma_f16_ss_pair(dcol, sw128_kmajor_desc(sa, static_cast<uint32_t>(kk * 32)),
                              sw128_kmajor_desc(sa + kABytesH, static_cast<uint32_t>(kk * 32)),
                              idesc, (j > 0 || kk > 0) ? 1u : 0u);
            tc_commit_pair(smem_u32(&ctl->empty[s]), 0x3);
            if (j == ksteps - 1) tc_commit_pair(smem_u32(&ctl->tfull[d]), 0x3);
          }
          __syncwarp();
        }
      }
      if (lane == 0) {
        tc_commit_pair(smem_u32(&ctl->drain), 0x1);
        volatile int never = 0;
        if (!ovb_wait(smem_u32(&ctl->drain), 0u, &never)) atomicOr(&g_status_f16, kErrDrain);
      }
      __syncwarp();
    } else {
      // ------------------------------------------- peer: accumulator release
      // One bar.sync per tile with this CTA's epilogue, as the MMA warp does
      // in the leader, then an arrive on the leader's pfree[d].
      for (int64_t t = 0; t + T::kAcc < my_tiles; ++t) {
        const int d = static_cast<int>(t % T::kAcc);
        named_sync(kBarDfreeH + d, 32 * (T::kEpiW + 1));
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctl->pfree[d]), 0u));
        __syncwarp();
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------- stage watcher (leader)
    // In lockstep with the MMA warp: per tile (from the third on) one
    // bar.sync after the peer released the accumulator, per stage one after
    // the stage landed -- also after a failed wait (the status word reports
    // it).
    if (rank == 0) {
      int64_t st = 0;
      for (int64_t t = 0; t < my_tiles; ++t) {
        if (t >= T::kAcc) {
          const int d = static_cast<int>(t % T::kAcc);
          const uint32_t ph = static_cast<uint32_t>(((t - T::kAcc) / T::kAcc) & 1);
          const bool got = ovb_wait_cluster(smem_u32(&ctl->pfree[d]), ph, abort);
          if (!__all_sync(0xffffffffu, got) && lane == 0) {
            atomicOr(&g_status_f16, kErrEpilogue);
            *abort = 1;
          }
          named_sync(kBarPeerH, 64);
        }
        for (int j = 0; j < ksteps; ++j, ++st) {
          const int s = static_cast<int>(st % T::kStages);
          const uint32_t ph = static_cast<uint32_t>((st / T::kStages) & 1);
          const bool got = ovb_wait(smem_u32(&ctl->full[s]), ph, abort);
          if (!__all_sync(0xffffffffu, got) && lane == 0) {
            atomicOr(&g_status_f16, kErrConvert);
            *abort = 1;
          }
          named_sync(kBarFullH, 64);
        }
      }
    }
  } else {
    // ------------------------------------------------- epilogue (both CTAs)
    const int64_t vtiles = 2 * pairs;
    if constexpr (kRope) {
      epilogue_rope_loop<BN, T::kAcc>(args, ctl->tfull, abort, tmem_base,
                                      stg_all + (warp - kFirstEpiH) * (32 * kStgStrideF),
                                      stg_all + T::kEpiW * (32 * kStgStrideF) +
                                          (warp - kFirstEpiH) * kRopeColFloats,
                                      reinterpret_cast<uint8_t*>(stg_all + T::kEpiW * (32 * kStgStrideF +
                                                                                   kRopeColFloats)) +
                                          (warp - kFirstEpiH) * (2 * kRopeTabBufBytes),
                                      warp & 3, (warp - kFirstEpiH) >> 2, kBarDfreeH, vtiles,
                                      order, my_tiles, blockIdx.x, gridDim.x);
    } else if constexpr (kSilu) {
      uint8_t* stg = reinterpret_cast<uint8_t*>(stg_all) + (warp - kFirstEpiH) * (32 * 64);
      silu_epilogue<BN, T::kAcc, T::kEpiW>(args, ctl->tfull, abort, tmem_base, stg, warp & 3,
                                           (warp - kFirstEpiH) >> 2, kBarDfreeH, vtiles,
                                           order, my_tiles, blockIdx.x, gridDim.x);
    } else {
      epilogue_loop<BN, T::kAcc, true, true>(
          args, ctl->tfull, abort, tmem_base,
          reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(stg_all) +
                                   (warp - kFirstEpiH) * T::kStgWarp),
          warp & 3, (warp - kFirstEpiH) >> 2, kBarDfreeH, vtiles, order, my_tiles, blockIdx.x,
          gridDim.x);
    }
  }

  tc_fence_before();
  __syncthreads();
  // Neither CTA frees its TMEM or shared memory while the pair's MMAs or the
  // other CTA may still use them (the epilogues waited for the last MMA).
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemColsF);
  }
}

template <int BN, bool kSilu, bool kRope = false>
cudaError_t launch_h2_impl(const CUtensorMap& tmap_a, const CUtensorMap& tmap_w,
                           const GemmArgs& args, cudaStream_t s) {
  using T = TileH2<BN, kSilu, kRope>;
  auto* kernel = gemm_h2_kernel<BN, kSilu, kRope>;
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev = -1;
  static thread_local int max_clusters = 0;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(T::kThreads);
  cfg.dynamicSmemBytes = T::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(T::kSmemBytes));
    if (e != cudaSuccess) return e;
    // The persistent grid holds as many pairs as can be resident at once
    // (the GPCs' SM counts decide how many 2-CTA clusters fit).
    cfg.gridDim = dim3(2 * static_cast<unsigned>(num_sms(dev)));
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
    if (e != cudaSuccess) return e;
    if (n < 1) return cudaErrorInvalidConfiguration;
    max_clusters = n;
    configured_dev = dev;
  }
  const int64_t pairs = ((args.M + 2 * kBlockM - 1) / (2 * kBlockM)) * ((args.N + BN - 1) / BN);
  if (pairs * 8 > INT32_MAX) return cudaErrorInvalidValue;  // 32-bit tile arithmetic
  cfg.gridDim = dim3(2 * static_cast<unsigned>(std::min<int64_t>(pairs, max_clusters)));
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, tmap_a, tmap_w, args);
}

template <int BN>
cudaError_t launch_f16_impl(const CUtensorMap& tmap_a, const CUtensorMap& tmap_w,
                            const GemmArgs& args, cudaStream_t s) {
  using T = TileF<BN>;
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev = -1;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(gemm_f16_kernel<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(T::kSmemBytes));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  const int64_t tiles = ((args.M + kBlockM - 1) / kBlockM) * ((args.N + BN - 1) / BN);
  if (tiles * 4 > INT32_MAX) return cudaErrorInvalidValue;  // 32-bit tile arithmetic
  const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms(dev)));
  return launch_pdl(gemm_f16_kernel<BN>, dim3(grid), dim3(kThreadsF), T::kSmemBytes, s, tmap_a,
                    tmap_w, args);
}

}  // namespace

// Cost of one output tile per 32-k block, by width (clocks): the slower of
// the tensor core (a K = 16 fp16 MMA takes ~128 clocks at N = 256 and ~64 at
// N <= 128) and the TMA feed (~65 B/clock per SM from L2 for 4 KB of A and
// 64*BN B of fp16 weights per block), plus a fixed per-tile cost (pipeline
// fill, epilogue).
int pick_tile_f16(int64_t M, int64_t N, int64_t Kb, int device) {
  if (const char* e = std::getenv("OVB_GEMM_TILE_N")) {
    const int v = std::atoi(e);
    for (int i = 0; i < 4; ++i)
      if (kTileNF[i] == v) return i;
  }
  static constexpr int64_t kPerBlock[4] = {315, 189, 133, 133};
  const int64_t sms = num_sms(device);
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  int best = 0;
  int64_t best_cost = -1;
  for (int i = 0; i < 4; ++i) {
    const int64_t tiles = m_tiles * ((N + kTileNF[i] - 1) / kTileNF[i]);
    const int64_t waves = (tiles + sms - 1) / sms;
    const int64_t cost = waves * (2000 + Kb * kPerBlock[i]);
    if (best_cost < 0 || cost < best_cost) {
      best = i;
      best_cost = cost;
    }
  }
  return best;
}

// Split-K configurations need at least this many 64-k stages per rank to pay
// for the partial-sum exchange.
constexpr int kMinStagesPerRank = 4;

int pick_tile_h(int64_t M, int64_t N, int64_t Kb, int device, unsigned allowed) {
  const int64_t ksteps = (Kb + 1) / 2;
  const char* et = std::getenv("OVB_GEMM_TILE_N");
  const char* es = std::getenv("OVB_GEMM_SPLIT_K");
  const char* ep = std::getenv("OVB_GEMM_PAIR");
  if (et || es || ep) {
    const int bn = et ? std::atoi(et) : 0;
    const int sp = es ? std::atoi(es) : 1;
    const int pr = ep ? std::atoi(ep) : 0;
    for (int i = 0; i < kNumHConfigs; ++i)
      if (((allowed >> i) & 1u) && (bn == 0 || h_tile_n(i) == bn) && kHConfigs[i].split == sp &&
          kHConfigs[i].pair == pr && ksteps >= static_cast<int64_t>(kHConfigs[i].split))
        return i;
  }
  // Cost in SM clocks, fitted to graph timings at M = 400 and 1400: a fixed
  // part (launch, prologue, first load; more for a CTA pair), the epilogue
  // (per output column of the CTA; the fused SiLU*up one is heavier), and per
  // 64-k stage the slower of the tensor pipe (four K = 16 MMAs) and shared
  // memory at ~128 B per clock, which carries the stage twice (TMA write, MMA
  // read; a pair CTA writes half of W but serves it to both tensor cores),
  // plus the split-K exchange; whole waves of CTAs.  A CTA pair pays a
  // one-off ~3 us more (cluster launch, paired TMEM allocation, the peer's
  // handshakes), so it wins only with many 64-k stages per SM: measured at
  // 15,408 rows it is 3-17 % faster than the single-CTA 128 x 256 tiles, at
  // 400 and 1400 rows 1-2 us slower.
  const int64_t sms = num_sms(device);
  const bool silu = allowed == kHSilu;
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  int best = -1;
  int64_t best_cost = -1;
  for (int i = 0; i < kNumHConfigs; ++i) {
    if (!((allowed >> i) & 1u)) continue;
    const HConfig& c = kHConfigs[i];
    const int64_t bn = h_tile_n(i);
    if (c.split > 1 && ksteps < static_cast<int64_t>(c.split) * kMinStagesPerRank) continue;
    const int64_t n_tiles = (N + bn - 1) / bn;
    const int64_t ctas =
        c.pair ? 2 * ((m_tiles + 1) / 2) * n_tiles : m_tiles * n_tiles * c.split;
    const int64_t waves = (ctas + sms - 1) / sms;
    const int64_t box = kTileNF[c.width];  // W rows this CTA loads per stage
    const int64_t smem = c.pair ? (16384 + box * 128) + (16384 + bn * 128)
                                : 2 * (16384 + box * 128);
    const int64_t mma = 4 * (bn <= 128 ? 64 : 128);
    const int64_t per_stage = (mma > smem / 128 ? mma : smem / 128) + (c.pair ? 30 : 0);
    const int64_t stages = (ksteps + c.split - 1) / c.split;
    const int64_t cost = waves * (3000 + (silu ? 38 : 29) * (bn / c.split) + stages * per_stage +
                                  (c.split > 1 ? 4000 : 0)) +
                         (c.pair ? 5000 : 0);
    if (best_cost < 0 || cost < best_cost) {
      best = i;
      best_cost = cost;
    }
  }
  return best < 0 ? 0 : best;
}

cudaError_t launch_gemm_h(int config, const CUtensorMap& tmap_a, const CUtensorMap& tmap_w,
                          const GemmArgs& args, cudaStream_t s) {
  if (args.rope_q16)  // the fused q/k norm + RoPE epilogue: CTA pairs, two heads per CTA
    return config == 7 ? launch_h2_impl<256, false, true>(tmap_a, tmap_w, args, s)
                       : cudaErrorInvalidValue;
  if (args.silu_out) {
    switch (config) {  // the fused epilogue needs whole gate/up block pairs: BN >= 64
      case 0: return launch_h_impl<256, true>(tmap_a, tmap_w, args, s);
      case 1: return launch_h_impl<128, true>(tmap_a, tmap_w, args, s);
      case 2: return launch_h_impl<64, true>(tmap_a, tmap_w, args, s);
      case 7: return launch_h2_impl<256, true>(tmap_a, tmap_w, args, s);
      case 8: return launch_h2_impl<128, true>(tmap_a, tmap_w, args, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (config) {  // kHConfigs
    case 0: return launch_h_impl<256, false>(tmap_a, tmap_w, args, s);
    case 1: return launch_h_impl<128, false>(tmap_a, tmap_w, args, s);
    case 2: return launch_h_impl<64, false>(tmap_a, tmap_w, args, s);
    case 3: return launch_h_impl<32, false>(tmap_a, tmap_w, args, s);
    case 4: return launch_h_impl<64, false, 2>(tmap_a, tmap_w, args, s);
    case 5: return launch_h_impl<128, false, 2>(tmap_a, tmap_w, args, s);
    case 6: return launch_h_impl<128, false, 4>(tmap_a, tmap_w, args, s);
    case 7: return launch_h2_impl<256, false>(tmap_a, tmap_w, args, s);
    case 8: return launch_h2_impl<128, false>(tmap_a, tmap_w, args, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t read_and_clear_status_f16(int* out, cudaStream_t s) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_status_f16, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_status_f16, &zero, sizeof(int));
}

cudaError_t launch_gemm_f16(int tile, const CUtensorMap& tmap_a, const CUtensorMap& tmap_w,
                            const GemmArgs& args, cudaStream_t s) {
  switch (tile) {
    case 0: return launch_f16_impl<256>(tmap_a, tmap_w, args, s);
    case 1: return launch_f16_impl<128>(tmap_a, tmap_w, args, s);
    case 2: return launch_f16_impl<64>(tmap_a, tmap_w, args, s);
    case 3: return launch_f16_impl<32>(tmap_a, tmap_w, args, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ovb
