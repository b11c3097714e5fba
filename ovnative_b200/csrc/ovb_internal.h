// ovb_internal.h -- declarations shared by the translation units of
// libovb200.so.  Not part of the public C ABI (include/ovb200.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <utility>

struct ovb_weight {
  int device = 0;
  int64_t N = 0;         // output channels
  int64_t K = 0;         // input features
  int64_t Kb = 0;        // ceil(K / 32)
  int64_t Kp = 0;        // Kb * 32: row stride of `w` in bytes
  int8_t* w = nullptr;   // device [N, Kp] int8, K-major, zero tail bytes
  float* scale = nullptr;  // device [N] per-output-channel scale
  // TMA descriptors of `w` for the GEMM's B tiles, one per tile width
  // (box kStageK B x kTileN[i] rows), built on first use.
  CUtensorMap tmap_b[3];
  bool tmap_ready[3] = {false, false, false};
  // Optional fp16 copy of `w` ([N, Kp], exact: |w| <= 127) for the fp16
  // tensor-core mainloop, with its TMA descriptors per tile width
  // (box 64 fp16 x kTileNF[i] rows).  Null unless created with OVB_WEIGHT_F16.
  uint16_t* w16 = nullptr;
  CUtensorMap tmap_w16[4];
  bool tmap16_ready[4] = {false, false, false, false};
  // Set for weights made by ovb_weight_create_batch: w, scale and w16 are
  // sub-ranges of one device allocation, freed with the batch's last weight.
  std::shared_ptr<void> arena;
  // Gate|up weight for the fused SiLU*up epilogue (ovb_weight_gate_up): rows
  // are gate and up interleaved in 32-row blocks (gate 32j.., up 32j.., ...);
  // glu_inter = N / 2 is the intermediate width.  0 for other weights.
  int64_t glu_inter = 0;
};

namespace ovb {

// Launch `kernel` on stream s with programmatic dependent launch (the kernel
// itself orders its memory accesses after the preceding grid with
// griddepcontrol.wait), unless the environment sets OVB_PDL=0.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same launch without the PDL attribute, for the quantisers: they
// start only after the preceding GEMM has finished.  (With PDL their blocks
// became resident and waited on the SMs while the GEMM ran, which slowed the
// RMSNorm-quantise + GEMM pair of the layer by ~3.8 us at M = 400.)  Their
// own griddepcontrol.launch_dependents still lets the next GEMM start early.
template <typename... KArgs, typename... Args>
cudaError_t launch_plain(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                         cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Rows / columns per GEMM output tile; bytes of K per TMA box (four 32-k
// quantisation blocks, one 128-byte swizzle row).
constexpr int kBlockM = 128;
constexpr int kStageK = 128;
// Output-tile widths the GEMM is built for (one kernel per width).
constexpr int kTileN[3] = {128, 64, 32};

// Output-tile widths of the fp16 mainloops.
constexpr int kTileNF[4] = {256, 128, 64, 32};
// Configurations of the plain fp16 mainloop: the W box (index into kTileNF:
// rows of W each CTA loads per stage), the split-K factor (a cluster of
// `split` CTAs per output tile) and CTA pairs (`pair`: a 2-CTA cluster runs
// cta_group::2 MMAs on a 256-row tile twice the box wide).
struct HConfig {
  int width;
  int split;
  int pair;
};
constexpr HConfig kHConfigs[9] = {{0, 1, 0}, {1, 1, 0}, {2, 1, 0}, {3, 1, 0}, {2, 2, 0},
                                  {1, 2, 0}, {1, 4, 0}, {1, 1, 1}, {2, 1, 1}};
constexpr int kNumHConfigs = 9;
// Output-tile width of configuration c.
constexpr int h_tile_n(int c) { return kTileNF[kHConfigs[c].width] * (kHConfigs[c].pair ? 2 : 1); }
// Allowed-configuration masks for pick_tile_h.
constexpr unsigned kHAll = (1u << kNumHConfigs) - 1;
constexpr unsigned kHNoSplit = 0x18Fu;  // 0-3 and the pairs 7, 8
constexpr unsigned kHSilu = 0x187u;     // BN >= 64 without split-K: 0-2, 7, 8
constexpr unsigned kHRope = 0x80u;      // the norm + RoPE epilogue: the 256-wide pair, 7

constexpr int kMaxSlices = 4;

struct SliceOut {
  int64_t n_begin;  // first global column of the slice
  int64_t n_count;
  float* C;
  int64_t ldc;
};

struct GemmArgs {
  int64_t M, N, Kb;
  const float* asc;     // [M, Kb]
  const float* wscale;  // [N]
  int accumulate;
  int n_slices;
  SliceOut slices[kMaxSlices];
  int32_t* products;    // when non-null: write P[m, n, b] instead of C
  // Fused SiLU*up epilogue (gate|up weights): when silu_out is non-null the
  // kernel writes quantise(silu(gate) * up) instead of C -- form silu_mode
  // (0 int8 q, 1 u8, 2 fp16 q*asc) into silu_out [M, silu_kp] and the block
  // scales into silu_asc [M, silu_kp / 32].
  uint8_t* silu_out;
  float* silu_asc;
  int silu_mode;
  int64_t silu_kp;
  // Split-K workspace of the device (fp16 mainloop, kSplit > 1 configs):
  // kSplitSlots slots of kSplitSlotBytes, slot i used only by the CTA
  // running on the SM with %smid == i.
  float* split_ws;
  // Fused q/k RMSNorm + RoPE epilogue (a q|k|v weight, plain fp16 mainloop):
  // when rope_q16 is non-null the kernel writes the q heads (columns
  // [0, rope_qd)) normalised with rope_qw and rotated, the k heads (the next
  // rope_kvd columns) likewise with rope_kw, and the v heads converted, all as
  // fp16 into rope_q16 [M, rope_qd], rope_k16 / rope_v16 [M, rope_kvd];
  // rope_tab is the RoPE table (launch_rope_table) of the M rows.  Head dim 128.
  void* rope_q16;
  void* rope_k16;
  void* rope_v16;
  const float* rope_qw;
  const float* rope_kw;
  const float* rope_tab;
  int64_t rope_qd, rope_kvd;
  float rope_eps;
  // Plain fp16-mainloop outputs written by TMA (out_tma != 0): out_map[i] is
  // slice i's C as fp32 [M, n_count] (row stride ldc), boxes of 32 x 32 with
  // 128-byte swizzle; stores, or element-wise adds when accumulating.
  int out_tma;
  alignas(64) CUtensorMap out_map[kMaxSlices];
};

// The split-K workspace: one slot per SM id (%smid < kSplitSlots), each large
// enough for the partial accumulators an owner CTA receives, (kSplit - 1) x
// 128 rows x (BN / kSplit) floats, at most 3 x 128 x 32 x 4 bytes.
constexpr int kSplitSlots = 256;
constexpr size_t kSplitSlotBytes = 48 * 1024;
// The device's split-K workspace (allocated with its first fp16 weight), or
// null when none could be allocated -- then no split-K config is launched.
float* split_workspace(int device);
bool ensure_split_workspace(int device);

// Thread-local error message (ovb_last_error).
void set_error(const std::string& msg);

// CUDA error -> message; returns true when `e` is an error.
bool cuda_failed(cudaError_t e, const char* what);

// Encode a 2-D uint8 tensor map [rows, row_bytes] with a (kStageK B x
// box_rows) box and 128-byte swizzle.  Returns false (and sets the error) on
// failure.
bool encode_tmap_u8(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
                    uint64_t stride_bytes, uint32_t box_rows);

int num_sms(int device);

// Launchers (stream-ordered, return a cudaError_t from the launch).
// Quantisers.  mode: 0 = int8 q, 1 = reference u8 q+128, 2 = fp16(q * asc).
cudaError_t launch_quantize(int64_t M, int64_t K, const float* A, int64_t lda, void* aq,
                            float* asc, int mode, cudaStream_t s);
cudaError_t launch_rmsnorm_quantize(int64_t rows, int64_t cols, const float* x, const float* w,
                                    float eps, void* aq, float* asc, int mode, cudaStream_t s);
cudaError_t launch_silu_mul_quantize(int64_t M, int64_t K, const float* gate, int64_t ldg,
                                     const float* up, int64_t ldu, void* aq, float* asc, int mode,
                                     cudaStream_t s);
cudaError_t read_and_clear_status_q(int* out, cudaStream_t s);
cudaError_t launch_pack_nk(const int8_t* src, int64_t N, int64_t K, int8_t* dst, int64_t Kp,
                           cudaStream_t s);
cudaError_t launch_pack_kn(const int8_t* src, int64_t N, int64_t K, int8_t* dst, int64_t Kp,
                           cudaStream_t s);
// General 2-D tensor map: dims {inner, rows} in elements, row stride in
// bytes, box {box_inner, box_rows} elements.  Returns false (and sets the
// error) on failure.
bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                    uint64_t inner, uint64_t rows, uint64_t stride_bytes, uint32_t box_inner,
                    uint32_t box_rows, CUtensorMapSwizzle swizzle);
// int8 [n] -> fp16 [n] (exact for |v| <= 2048).
cudaError_t launch_widen_f16(const int8_t* src, int64_t n, uint16_t* dst, cudaStream_t s);
// A kernel whose bounded wait cannot complete (status bit 64 after ~1 s).
cudaError_t launch_wait_selftest(cudaStream_t s);
// The guided argmax pass (sampler.cu): one warp per (codebook, frame) row.
//
// Up to kMaxGuidedPairs CFG pairs of V = 1025 in one launch: pair p's cond /
// uncond planes, cond sequence and target lengths, and its first output row
// out0[p] (out0[n] = all rows).
constexpr int kMaxGuidedPairs = 64;
struct GuidedBatch {
  const float* cond[kMaxGuidedPairs];
  const float* uncond[kMaxGuidedPairs];
  int cond_seq[kMaxGuidedPairs];
  int T[kMaxGuidedPairs];
  int64_t out0[kMaxGuidedPairs + 1];
  int n, C, mask_id;
  float guidance, penalty;
};
cudaError_t launch_guided_sample_batch(const GuidedBatch& g, int32_t* pred, float* scores,
                                       cudaStream_t s);
// One pair, any V.
cudaError_t launch_guided_sample(const float* cond, int cond_seq, const float* uncond, int C,
                                 int V, int T, float guidance, float penalty, int mask_id,
                                 int32_t* pred, float* scores, cudaStream_t s);
// Attention (attention.cu).  One segment as the kernel sees it: the
// reference's AttnSegment (bias, rows, q_off, kv_off; element offsets), the
// same offsets as (column, row) coordinates of the q and k/v tensor maps,
// and the index of its first 128-row query block in the launch.
constexpr int kAttMaxSegs = 64;
// Launches of at most this many attention work items on at most this many
// CTAs run a host-computed schedule (longest items first, each to the least
// loaded CTA); larger ones walk the items round-robin.
constexpr int kAttSchedItems = 4096;
constexpr int kAttSchedCtas = 256;
struct AttnSeg {
  const float* bias;  // [rows, rows] additive, or null
  int64_t q_off;      // element offset of the segment's first query row
  int rows;
  int qblock0;
  int q_x, q_y;       // q_off = q_y * q_stride + q_x
  int kv_x, kv_y;     // kv_off = kv_y * kv_stride + kv_x
};
struct AttnArgs {
  // fp32 2-D maps of q and k / v: {row stride, rows} elements, box 128 x 128
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  float* out;      // laid out like q: head h of row s at q_off + s * q_stride + h * 128
  int64_t q_stride;
  int n_heads;
  int group;       // query heads per kv head
  int n_segs;
  float scale;
  AttnSeg segs[kAttMaxSegs];
};
cudaError_t launch_attention(const AttnArgs& args, int total_qblocks, cudaStream_t s);
// The fp16-operand attention (attention_h_kernel): one work item per
// (segment, 128 query rows, kv head, pair of query heads), numbered from the
// segment's cta0.
struct AttnHSeg {
  const float* bias;  // [rows, rows] additive (no tile table), or null
  int64_t q_off;      // element offset of the segment's first query row (out)
  int rows;
  int cta0;
  int q_x, q_y;       // q_off = q_y * q_stride + q_x
  int kv_x, kv_y;
  int tile0;          // the segment's first entry in the tile table
};
struct AttnHArgs {
  // fp16 2-D maps {row stride, rows}, box 64 x 128, 128-byte swizzle
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  float* out;
  int64_t q_stride;
  int n_heads;
  int n_kv;
  int group;
  int pairs;          // CTAs per (query block, kv head): ceil(group / 2)
  int n_segs;
  float scale;
  const uint8_t* tile_class;  // [tiles] 0 / 1 / 3, or null (then the biases)
  const uint32_t* tile_bits;  // [tiles][128 rows][4 words]
  // When q_out is set, the output is written quantised instead of to `out`:
  // ovb_quantize's form q_mode (0 int8 q, 1 u8, 2 fp16 q*asc) into q_out
  // [rows, q_kb * 32] and the block scales into q_asc [rows, q_kb].
  uint8_t* q_out;
  float* q_asc;
  int q_mode;
  int q_kb;
  int n_items;        // work items (segment x query block x kv head x head pair)
  // The host's schedule (sched != 0): CTA b runs items order[cta_first[b] ..
  // cta_first[b + 1]) in that order; otherwise CTA b runs b, b + grid, ...
  int sched;
  uint16_t cta_first[kAttSchedCtas + 1];
  uint16_t order[kAttSchedItems];
  AttnHSeg segs[kAttMaxSegs];
};
// ctas = work items; the kernel runs persistent CTAs over them.
cudaError_t launch_attention_h(const AttnHArgs& args, int ctas, cudaStream_t s);
struct AttnTilesArgs {
  const uint8_t* masks;         // the segments' [rows, rows] u8 masks, concatenated
  int n_segs;
  int rows[kAttMaxSegs];
  int tile0[kAttMaxSegs];
  int64_t mask_off[kAttMaxSegs];
};
cudaError_t launch_attn_tiles(const AttnTilesArgs& a, int tiles, uint8_t* cls, uint32_t* bits,
                              cudaStream_t s);
// LM forward steps (lm_ops.cu).  An embedding table on the device: int8
// rows with one fp32 scale per row, or fp32 rows.
struct EmbTable {
  const int8_t* i8;
  const float* scale;
  const float* f32;
  int64_t rows;
  int64_t cols;
};
cudaError_t launch_embed(const int64_t* ids, const uint8_t* mask, const int64_t* offsets, int C,
                         int64_t rows, int seq, const EmbTable& tok, const EmbTable& aud,
                         float* out, int H, cudaStream_t s);
cudaError_t launch_permute_logits(const float* src, float* dst, int B, int S, int C, int V,
                                  cudaStream_t s);
// RoPE frequencies of head_dim 128: inv_freq[i] = (float) theta^(-2i/128).
struct RopeFreq {
  float inv_freq[64];
};
// The RoPE table of `rows` positions: tab [rows, 128] fp32, row r in groups
// (cos a_2j, cos a_2j+1, sin a_2j, sin a_2j+1) of its angles a_i, j < 32.
cudaError_t launch_rope_table(const int64_t* pos, const RopeFreq& f, int64_t rows, float* tab,
                              cudaStream_t s);
// q / k RMSNorm + RoPE written as fp16 (q16, k16) and v converted to fp16
// (v16): the operands of ovb_attention_h.  tab from launch_rope_table.
cudaError_t launch_qk_norm_rope_f16(const float* q, const float* k, const float* v, void* q16,
                                    void* k16, void* v16, const float* qw, const float* kw,
                                    const float* tab, int64_t rows, int n_heads, int n_kv,
                                    float eps, cudaStream_t s);
cudaError_t read_and_clear_status_lm(int* out, cudaStream_t s);
cudaError_t read_and_clear_status_att(int* out, cudaStream_t s);
// Index into kTileNF of the tile width used by the fp16 mainloop.
int pick_tile_f16(int64_t M, int64_t N, int64_t Kb, int device);
cudaError_t launch_gemm_f16(int tile, const CUtensorMap& tmap_a, const CUtensorMap& tmap_w,
                            const GemmArgs& args, cudaStream_t s);
cudaError_t read_and_clear_status_f16(int* out, cudaStream_t s);
// The plain fp16 mainloop: A is fp16 [M, Kp] (dequantised activations).
// Returns an index into kHConfigs among the configurations in `allowed`
// (a bit mask: kHAll, kHNoSplit without a split-K workspace, kHSilu for the
// fused SiLU*up epilogue).
int pick_tile_h(int64_t M, int64_t N, int64_t Kb, int device, unsigned allowed = kHAll);
cudaError_t launch_gemm_h(int tile, const CUtensorMap& tmap_a, const CUtensorMap& tmap_w,
                          const GemmArgs& args, cudaStream_t s);

// Index into kTileN of the tile width used for an M x N GEMM: the widest
// one that still gives every SM a tile (OVB_GEMM_TILE_N overrides it).
int pick_tile(int64_t M, int64_t N, int device);
cudaError_t launch_gemm(int tile, const CUtensorMap& tmap_a, const CUtensorMap& tmap_b,
                        const GemmArgs& args, cudaStream_t s);

// Device status word (0 = every bounded wait completed).
cudaError_t read_and_clear_status(int* out, cudaStream_t s);

}  // namespace ovb
