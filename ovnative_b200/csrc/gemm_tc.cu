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
// ahead of the fp32 epilogue.
//
// Warp roles (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A box (32 B x 128 rows of aq) and B box (32 B x
//               128 rows of the packed weight) per block into a 16-stage ring;
//   warp 1      TMEM allocator + MMA issuer (one thread);
//   warps 2..9  epilogue: warp w reads TMEM lanes 32*(w%4).. (the lane quarter
//               it may access) and 64 of the 128 columns, converts each
//               block's int32 products and folds them into 64 fp32 running
//               sums per thread; at the end of the tile it applies wscale,
//               the optional residual, and stores.
//
// Every mbarrier wait is bounded (ovb_wait); on a timeout the kernel records
// a non-zero status in g_status, stops its loops, waits (bounded) for its
// own outstanding copies and MMAs, frees TMEM and returns.
#include "ovb_internal.h"
#include "ovb_ptx.cuh"

namespace ovb {

__device__ int g_status;

namespace {

constexpr int kStages = 16;
constexpr int kAccBufs = 4;
constexpr uint32_t kTmemCols = 512;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kABytes = kBlockM * 32;
constexpr uint32_t kBBytes = kBlockN * 32;
constexpr uint32_t kStageBytes = kABytes + kBBytes;
static_assert(kAccBufs * kBlockN <= static_cast<int>(kTmemCols), "TMEM ring too large");

// status codes recorded in g_status (bit flags)
constexpr int kErrProducer = 1;
constexpr int kErrMma = 2;
constexpr int kErrEpilogue = 4;
constexpr int kErrDrain = 8;

struct Ctl {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[kAccBufs];
  uint64_t tempty[kAccBufs];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStages) * kStageBytes + sizeof(Ctl);

__device__ __forceinline__ void fail(Ctl* ctl, int code) {
  atomicOr(&g_status, code);
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
}

template <bool kProducts>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_s8_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + static_cast<size_t>(kStages) * kStageBytes);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int64_t M = args.M, N = args.N, Kb = args.Kb;
  const int64_t m_tiles = (M + kBlockM - 1) / kBlockM;
  const int64_t n_tiles = (N + kBlockN - 1) / kBlockN;
  const int64_t tiles = m_tiles * n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int a = 0; a < kAccBufs; ++a) {
      mbar_init(smem_u32(&ctl->tfull[a]), 1);
      mbar_init(smem_u32(&ctl->tempty[a]), kEpiWarps);
    }
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
    if (lane == 0) {
      int64_t it = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int32_t m0 = static_cast<int32_t>((tile % m_tiles) * kBlockM);
        const int32_t n0 = static_cast<int32_t>((tile / m_tiles) * kBlockN);
        for (int64_t b = 0; b < Kb; ++b, ++it) {
          const int s = static_cast<int>(it % kStages);
          const uint32_t ph = static_cast<uint32_t>((it / kStages) & 1);
          if (!ovb_wait(smem_u32(&ctl->empty[s]), ph ^ 1u, abort)) {
            fail(ctl, kErrProducer);
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&ctl->full[s]);
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * kStageBytes);
          mbar_arrive_expect_tx(full, kStageBytes);
          tma_load_2d(sa, &tmap_a, static_cast<int32_t>(b * 32), m0, full);
          tma_load_2d(sa + kABytes, &tmap_b, static_cast<int32_t>(b * 32), n0, full);
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA's shared memory
        // is released: wait (bounded) on the last min(it, kStages) stages.
        const int64_t first = it > kStages ? it - kStages : 0;
        for (int64_t j = first; j < it; ++j) {
          const int s = static_cast<int>(j % kStages);
          const uint32_t ph = static_cast<uint32_t>((j / kStages) & 1);
          volatile int never = 0;
          ovb_wait(smem_u32(&ctl->full[s]), ph, &never);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(kBlockM, kBlockN);
      int64_t it = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        for (int64_t b = 0; b < Kb; ++b, ++it) {
          const int s = static_cast<int>(it % kStages);
          const uint32_t ph = static_cast<uint32_t>((it / kStages) & 1);
          const int a = static_cast<int>(it % kAccBufs);
          const uint32_t aph = static_cast<uint32_t>((it / kAccBufs) & 1);
          if (!ovb_wait(smem_u32(&ctl->tempty[a]), aph ^ 1u, abort) ||
              !ovb_wait(smem_u32(&ctl->full[s]), ph, abort)) {
            fail(ctl, kErrMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * kStageBytes);
          mma_i8(tmem_base + static_cast<uint32_t>(a * kBlockN), sw32_kmajor_desc(sa),
                 sw32_kmajor_desc(sa + kABytes), idesc, 0u);
          tc_commit(smem_u32(&ctl->empty[s]));
          tc_commit(smem_u32(&ctl->tfull[a]));
        }
      }
      // Drain: every MMA issued above has completed once this arrives.
      tc_commit(smem_u32(&ctl->drain));
      volatile int never = 0;
      if (!ovb_wait(smem_u32(&ctl->drain), 0u, &never)) atomicOr(&g_status, kErrDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;      // TMEM lanes this warp may read
    const int half = (warp - 2) >> 2;  // which 64 of the 128 tile columns
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    int64_t it = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      const int64_t m0 = (tile % m_tiles) * kBlockM;
      const int64_t n0 = (tile / m_tiles) * kBlockN;
      const int64_t m = m0 + quarter * 32 + lane;
      const bool row_ok = m < M;
      const float* asc_row = args.asc + (row_ok ? m : 0) * Kb;
      const int64_t nc = n0 + half * 64;  // first column of this thread's chunk
      float f[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) f[j] = 0.f;
      for (int64_t b = 0; b < Kb; ++b, ++it) {
        const int a = static_cast<int>(it % kAccBufs);
        const uint32_t aph = static_cast<uint32_t>((it / kAccBufs) & 1);
        const float s = (!kProducts && row_ok) ? __ldg(asc_row + b) : 0.f;
        const bool got = ovb_wait(smem_u32(&ctl->tfull[a]), aph, abort);
        if (!__all_sync(0xffffffffu, got)) {
          if (lane == 0) fail(ctl, kErrEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r0[32], r1[32];
        const uint32_t taddr = tmem_base + lane_off + static_cast<uint32_t>(a * kBlockN + half * 64);
        tmem_ld32(taddr, r0);
        tmem_ld32(taddr + 32, r1);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl->tempty[a]));
        if constexpr (kProducts) {
          if (row_ok) {
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const int64_t n = nc + j;
              if (n < N)
                args.products[(m * N + n) * Kb + b] =
                    static_cast<int32_t>(j < 32 ? r0[j] : r1[j - 32]);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            f[j] = __fmaf_rn(__int2float_rn(static_cast<int>(r0[j])), s, f[j]);
            f[32 + j] = __fmaf_rn(__int2float_rn(static_cast<int>(r1[j])), s, f[32 + j]);
          }
        }
      }
      if (!ok) break;
      if constexpr (!kProducts) {
        if (row_ok && nc < N) {
          // The chunk lies inside one slice (slices are multiples of 64
          // columns, or a single slice covering all N).
          int si = 0;
#pragma unroll
          for (int i = 1; i < kMaxSlices; ++i)
            if (i < args.n_slices && nc >= args.slices[i].n_begin) si = i;
          const SliceOut so = args.slices[si];
          const int64_t local = nc - so.n_begin;
          const int64_t nvalid = so.n_count - local;  // >= 1
          float* crow = so.C + m * so.ldc + local;
          const float* ws = args.wscale + nc;
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            if (j < nvalid) {
              float o = __fmul_rn(f[j], __ldg(ws + j));
              if (args.accumulate) o = __fadd_rn(o, crow[j]);
              crow[j] = o;
            }
          }
        }
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
