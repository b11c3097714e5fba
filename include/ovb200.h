/* ovb200.h -- C ABI of the B200-native int8 LM GEMM path for OVNative.
 *
 * This library replaces, for the int8 LM projections only, the per-GEMM
 * entry points of the reference's backend contract
 * (cpp/include/ovnative/ov_gemm.h, namespace ov) and the cuBLAS calls of
 * its CUDA LM runner (cpp/src/backend/cuda/cuda_lm.cu:984-989, :1023-1030).
 * Every compute entry point takes DEVICE pointers and a cudaStream_t (passed
 * as void*) and is stream-ordered; nothing here synchronises the device except
 * ovb_weight_create/ovb_weight_concat/ovb_weight_destroy.
 *
 * Numerics are those of the reference's CPU AVX-VNNI path
 * (cpp/src/backend/cpu/gemm.cpp:379-882, cpp/src/backend/cpu/ops_cpu.cpp:75-198):
 *   - activations are quantised per row per 32-k block:
 *       amax = max|a|, asc = amax/127, q = rne(a * (127/amax)) clamped to +-127;
 *   - each 32-k block product P_b = sum q*w is an exact int32;
 *   - the fp32 result is f = fma(P_b, asc_b, f) over b in order, then
 *     o = f * wscale[n], then o = o + C_old when accumulating.
 *   Following that order makes the fp32 output bit-identical to the
 *   reference's.
 * A weight created with OVB_WEIGHT_F16 instead runs the fp16 tensor-core
 * mainloop: the same quantised activations, dequantised on the GPU to
 * fp16(q * asc) and multiplied with the (exact) fp16 weights into one fp32
 * accumulator.  Its outputs agree with the reference within relative L2
 * ~3e-4 (contract: <= 1e-3, max-abs <= 1e-2 * rms), not bit for bit, and
 * need |activations| < 65504.  ovb_block_products always uses the int8 path.
 *
 * Activation buffers ("aq/asc"):
 *   aq  : int8 q, row-major [M, Kp], Kp = 32*ceil(K/32), tail bytes zero.
 *         With OVB_AQ_U8 a quantiser writes the reference's u8 form instead
 *         (q + 128, tail bytes zero; gemm.cpp:423-427) -- for byte comparison
 *         only, the GEMMs consume the int8 form.
 *   asc : fp32 row-major [M, Kb], Kb = ceil(K/32).
 *   Sizes: ovb_quant_bytes(M, K) bytes and ovb_quant_scales(M, K) floats
 *   (s8_nk_quant_bytes / s8_nk_quant_scales, ov_gemm.h:95-96).
 *
 * Error convention (mirrors ovnative.h:19-23): every call returns OVB_OK or
 * a negative status and leaves a message in ovb_last_error() (thread-local).
 * Like the reference, M, N or K <= 0 is a no-op that returns OVB_OK
 * (gemm.cpp:761, :779, :832).
 *
 * Thread safety: one weight handle may be used from several threads and
 * streams at once (it is read-only after creation).  Calls that share output
 * buffers must be ordered by the caller, as with the reference.
 */
#ifndef OVB200_H
#define OVB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OVB_ABI_VERSION 1

/* status codes: same values as OV_OK / OV_ERR_INVALID_ARG / OV_ERR_INTERNAL */
#define OVB_OK 0
#define OVB_ERR_INVALID_ARG (-1)
#define OVB_ERR_INTERNAL (-4)

/* weight layouts (OVW1 descriptor `layout`, weight-format.en.md / mat.cpp:69-106) */
#define OVB_LAYOUT_NK 0 /* [N, K], one scale per output row (layout=0) */
#define OVB_LAYOUT_KN 1 /* [K, N], one scale per output column (layout=1) */

/* flags */
#define OVB_SRC_DEVICE 1 /* ovb_weight_create: W and scale are device pointers */
#define OVB_WEIGHT_F16 2 /* ovb_weight_create: also keep an fp16 copy; GEMMs with this
                            handle run the fp16 mainloop (see above).  No counterpart
                            in the reference's CPU path; its CUDA runner multiplies
                            dequantised fp16 weights (cuda_lm.cu:840-873).  The first
                            such weight on a device also allocates the library's
                            split-K workspace there (12 MiB, one slot per SM, kept
                            until exit; safe for concurrent streams).  Without it the
                            fp16 GEMMs run without split-K. */
#define OVB_AQ_U8 1      /* quantisers: write reference u8 (q+128) instead of int8 */
#define OVB_AQ_F16 2     /* quantisers: write fp16(q * asc), [M, Kp] fp16 (2 bytes per
                            element, 16-byte aligned), the input of ovb_linear_h */
#define OVB_AQ_F16_RAW 4 /* quantisers: write fp16 of the (normalised) fp32 values
                            themselves, not quantised, [M, Kp] fp16 with a zero tail;
                            asc is not written and may be NULL.  The input of
                            ovb_linear_h with a weight from ovb_weight_create_f32: the
                            reference's fp32 activations x fp32 weights (linear_f32,
                            Mat::mul on an fp32 weight, mat.cpp:11-13).  Values beyond
                            the fp16 range set ovb_device_status bit 16. */

typedef struct ovb_weight ovb_weight;

/* One output slice of a concatenated weight (ov::S8NkSlice, ov_gemm.h:105-108),
 * with an explicit row stride for C. */
typedef struct ovb_slice {
  int64_t N;   /* columns of this slice, a positive multiple of 64 */
  float* C;    /* device [M, ldc] */
  int64_t ldc; /* >= N */
} ovb_slice;

int ovb_abi_version(void);
const char* ovb_last_error(void);

/* Device status of the GEMMs since the last call, on this thread's device:
 * 0 when every bounded wait inside the kernels completed.  Bits 1, 2, 4, 8:
 * a wait of the producer, stage watcher / converter, epilogue or drain gave
 * up (~1 s limit; the kernel then ends early and its outputs are invalid,
 * the context stays usable).  Bit 16 reports an activation block beyond the
 * fp16 range in the fp16 mainloop, or a q/k/v value beyond it in the
 * attention; bit 32 a wait of the attention kernel; bit 128 a token or
 * codebook id outside its embedding table (ovb_lm_*);
 * bit 64 the self-test below.  Reading it
 * synchronises the given stream and clears it. */
int ovb_device_status(void* stream);

/* Failure-detection self-test: launches a kernel whose bounded mbarrier
 * wait can never complete (nothing arrives on the barrier).  The wait gives
 * up after its limit (~1 s), the kernel ends normally and the next
 * ovb_device_status reports bit 64.  No GPU fault or hang is involved.  No
 * counterpart in the reference. */
int ovb_selftest_wait_timeout(void* stream);

/* --- sizes ------------------------------------------------------------ */
/* replaces ov::s8_nk_quant_bytes (ov_gemm.h:95) */
int64_t ovb_quant_bytes(int64_t M, int64_t K);
/* replaces ov::s8_nk_quant_scales (ov_gemm.h:96) */
int64_t ovb_quant_scales(int64_t M, int64_t K);

/* --- weights ---------------------------------------------------------- */
/* Build a device-resident weight from an int8 matrix in either OVW1 layout
 * and its per-output-channel fp32 scale (N floats).  Replaces the load-time
 * ov::s8_nk_pack (ov_gemm.h:60-63, gemm.cpp:584-621) and the CUDA runner's
 * dequantise-at-load (cuda_lm.cu:840-873).  Host sources (the OVW1 mmap) are
 * borrowed for the call only.  Synchronous. */
int ovb_weight_create(const int8_t* W, int layout, int64_t N, int64_t K, const float* scale,
                      int flags, void* stream, ovb_weight** out);
/* One host (or, with OVB_SRC_DEVICE, device) source of ovb_weight_create_batch. */
typedef struct ovb_weight_src {
  const int8_t* W;     /* layout 0: [N, K]; layout 1: [K, N] */
  int layout;
  int64_t N;
  int64_t K;
  const float* scale;  /* [N] per-output-channel scales */
} ovb_weight_src;

/* ovb_weight_create for n weights at once (a checkpoint's linear layers):
 * one device allocation holds all of them (freed with the last of the n
 * handles), every payload is copied and packed before a single
 * synchronisation.  flags: OVB_WEIGHT_F16 and/or OVB_SRC_DEVICE.  On error
 * no handle is returned.  No counterpart in the reference (its loader packs
 * tensor by tensor on the host, mat.cpp:69-106). */
int ovb_weight_create_batch(const ovb_weight_src* srcs, int n, int flags, void* stream,
                            ovb_weight** out);

/* An fp32 linear weight -- the reference's fp32 encoding of a linear layer
 * (OVW1 layout 1, [K, N], as tools/convert_weights.py:178-180 stores every
 * fp32 matrix, e.g. the default fp32 audio heads, :326-327; or layout 0,
 * [N, K]) consumed by Mat::mul -> linear_f32 (mat.cpp:11-13) -- held on the
 * device as fp16 [N, Kp] with one power-of-two scale per output channel
 * (2^(e-10), e the exponent of the channel's largest |w|: the scaling is
 * exact and the one rounding is W/s to fp16, relative error <= 2^-11).  Only
 * ovb_linear_h / ovb_linear_h_sliced accept it, with activations from a
 * quantiser run with OVB_AQ_F16_RAW: fp16 x fp16 products summed in fp32,
 * the precision of the reference CUDA runner's fp16 GEMMs (cuda_lm.cu:
 * 1023-1030).  The int8 entry points reject it (it has no int8 image).
 * W is a host pointer; synchronous; non-finite weights are rejected. */
int ovb_weight_create_f32(const float* W, int layout, int64_t N, int64_t K, void* stream,
                          ovb_weight** out);

/* Concatenate weights with the same K along N (q|k|v, gate|up).  Replaces
 * combine_packed (lm.cpp:57-94).  The parts stay valid.  The result has the
 * fp16 copy (OVB_WEIGHT_F16) when every part has it. */
int ovb_weight_concat(const ovb_weight* const* parts, int n_parts, void* stream,
                      ovb_weight** out);
/* Gate|up weight for the fused SiLU*up GEMMs below: the two projections'
 * rows interleaved in 32-row blocks (gate and up must have the same N, a
 * multiple of 32, and K).  It keeps the fp16 copy when both parts have one.
 * No counterpart in the reference (its gate_up is combine_packed, lm.cpp:57-94,
 * followed by a separate silu_mul_quantize_f32). */
int ovb_weight_gate_up(const ovb_weight* gate, const ovb_weight* up, void* stream,
                       ovb_weight** out);
int ovb_weight_destroy(ovb_weight* w);
int ovb_weight_shape(const ovb_weight* w, int64_t* N, int64_t* K);
/* Copy the device weight back as [N, K] int8 and its N scales (host pointers);
 * used by tests to check the packers. */
int ovb_weight_export(const ovb_weight* w, int8_t* W_nk, float* scale);

/* --- activation quantisers (device pointers) --------------------------- */
/* replaces ov::s8_nk_quantize (ov_gemm.h:97; gemm.cpp:379-430, :709-720).
 * A is [M, K] with row stride lda >= K. */
int ovb_quantize(int64_t M, int64_t K, const float* A, int64_t lda, void* aq, float* asc,
                 int flags, void* stream);
/* replaces ov::rmsnorm_quantize_f32 (ov_gemm.h:118-119; gemm.cpp:638-707) */
int ovb_rmsnorm_quantize(int64_t rows, int64_t cols, const float* x, const float* w, float eps,
                         void* aq, float* asc, int flags, void* stream);
/* replaces ov::silu_mul_quantize_f32 (ov_gemm.h:84-85; ops_cpu.cpp:144-198,
 * :1138-1168).  gate/up are [M, K] with row strides ldg / ldu. */
int ovb_silu_mul_quantize(int64_t M, int64_t K, const float* gate, int64_t ldg,
                          const float* up, int64_t ldu, void* aq, float* asc, int flags,
                          void* stream);

/* --- GEMMs (device pointers) ------------------------------------------ */
/* C[m, n] (+)= linear(aq, asc) with w.  accumulate = 0 replaces
 * ov::linear_s8_nk_packed_q (ov_gemm.h:98-100); accumulate = 1 replaces
 * ov::linear_s8_nk_packed_q_add (ov_gemm.h:78-80).  C is [M, ldc]. */
int ovb_linear_q(int64_t M, const ovb_weight* w, const int8_t* aq, const float* asc, float* C,
                 int64_t ldc, int accumulate, void* stream);
/* One launch over a concatenated weight writing each slice to its own C.
 * Replaces ov::linear_s8_nk_packed_q_sliced (ov_gemm.h:109-111). */
int ovb_linear_q_sliced(int64_t M, const ovb_weight* w, const int8_t* aq, const float* asc,
                        const ovb_slice* slices, int n_slices, void* stream);

/* gate|up GEMM fused with silu_mul_quantize_f32 (ov_gemm.h:84-85): computes
 * gate = x*Wg^T*sg and up = x*Wu^T*su exactly as ovb_linear_q would, then
 * writes quantise(silu(gate) * up) -- the down projection's input -- in the
 * form `flags` selects (0 int8 q / OVB_AQ_U8 / OVB_AQ_F16) into out
 * [M, Kp_inter] and its scales into out_asc [M, inter/32], without writing
 * gate and up.  w comes from ovb_weight_gate_up.  The _q form runs the int8
 * mainloop and is bit-identical to the reference's two calls; the _h form
 * takes fp16(q*asc) activations (OVB_WEIGHT_F16 weights) and runs the fp16
 * mainloop (tolerance numerics).  Replaces linear_s8_nk_packed_q_sliced on
 * gate|up plus silu_mul_quantize_f32 (lm.cpp:295-311). */
int ovb_linear_q_silu(int64_t M, const ovb_weight* w, const int8_t* aq, const float* asc,
                      void* out, float* out_asc, int flags, void* stream);
int ovb_linear_h_silu(int64_t M, const ovb_weight* w, const void* a16, void* out,
                      float* out_asc, int flags, void* stream);

/* The fp16 mainloop on already-dequantised activations: a16 is [M, Kp] fp16,
 * fp16(q * asc) as written by a quantiser with OVB_AQ_F16; w must have been
 * created with OVB_WEIGHT_F16.  Same outputs (slices, residual add) and
 * tolerance as ovb_linear_q on such a handle, without converting the int8
 * activations once per output tile.  No counterpart in the reference: it
 * splits the reference's quantise+GEMM pair (s8_nk_quantize +
 * linear_s8_nk_packed_q) at a different point. */
int ovb_linear_h(int64_t M, const ovb_weight* w, const void* a16, float* C, int64_t ldc,
                 int accumulate, void* stream);
int ovb_linear_h_sliced(int64_t M, const ovb_weight* w, const void* a16, const ovb_slice* slices,
                        int n_slices, void* stream);

/* The RoPE table of `rows` positions (device int64 pos): table [rows, 128]
 * fp32, cos / sin of the angles a_i = fl(fl(pos[r]) * inv_freq[i]), i < 64,
 * a row in 32 groups (cos a_2j, cos a_2j+1, sin a_2j, sin a_2j+1) so that a
 * kernel rotating two adjacent elements reads its cosines and its sines as
 * pairs; inv_freq[i] = (float) theta^(-2i/128) computed on the host as the
 * reference does.  The reference tabulates the same per row and keeps it
 * across layers (qk_norm_rope_f32, ops_cpu.cpp:945-986); the device LM
 * builds it once per forward.  head_dim must be 128; table 16-byte aligned. */
int ovb_rope_table(const int64_t* pos, int64_t rows, int head_dim, float theta, float* table,
                   void* stream);

/* The per-head q / k RMSNorm + RoPE of one layer (qk_norm_rope_f32,
 * ops_cpu.cpp:945-1013; the reference CUDA runner's norm_rope_heads_kernel,
 * cuda_lm.cu:117-147) written as fp16: q [rows, n_heads*128] and k [rows,
 * n_kv*128] (fp32, as the q|k|v GEMM writes them, read only) normalised with
 * q_norm / k_norm [128], rotated by `table` (ovb_rope_table) and stored into
 * q16 / k16; v [rows, n_kv*128] converted into v16 -- the operands of
 * ovb_attention_h.  A value beyond the fp16 range sets status bit 16. */
int ovb_qk_norm_rope_f16(int64_t rows, const float* q, const float* k, const float* v,
                         int n_heads, int n_kv, int head_dim, const float* q_norm,
                         const float* k_norm, float eps, const float* table, void* q16, void* k16,
                         void* v16, void* stream);

/* The q|k|v GEMM on the fp16 mainloop with ovb_qk_norm_rope_f16 fused into
 * its epilogue: w is the concatenation q|k|v (OVB_WEIGHT_F16, N = (n_heads +
 * 2 n_kv) * 128), a16 as for ovb_linear_h.  Writes the same bytes into q16 /
 * k16 / v16 as ovb_linear_h_sliced into fp32 q / k / v followed by
 * ovb_qk_norm_rope_f16, without the fp32 q / k / v.  No counterpart in the
 * reference (its q|k|v GEMM and norm + RoPE are separate calls, lm.cpp:
 * 228-253). */
int ovb_linear_h_qk_rope(int64_t M, const ovb_weight* w, const void* a16, int n_heads, int n_kv,
                         int head_dim, const float* q_norm, const float* k_norm, float eps,
                         const float* table, void* q16, void* k16, void* v16, void* stream);
/* fp32 activations in, quantised inside (two launches).  accumulate = 0
 * replaces ov::linear_s8_nk_packed (ov_gemm.h:67-69); accumulate = 1
 * replaces ov::linear_s8_nk_packed_add (ov_gemm.h:73-75).  `work` is a device
 * scratch of at least ovb_linear_workspace_bytes(M, K) bytes, 256-byte
 * aligned, owned by the caller (the reference's thread-local aq/asc vectors,
 * gemm.cpp:835-839). */
size_t ovb_linear_workspace_bytes(int64_t M, int64_t K);
int ovb_linear(int64_t M, const ovb_weight* w, const float* A, int64_t lda, float* C,
               int64_t ldc, int accumulate, void* work, size_t work_bytes, void* stream);

/* ovb_linear for callers that cannot allocate device memory (a host whose
 * device memory all belongs to its own pool, a latency-critical step that
 * must not pay for cudaMalloc's device synchronisation, an FFI binding that
 * cannot own a device buffer).  Same arguments and results as ovb_linear
 * without `work`: the quantised activations go to an 8 MiB device array
 * inside the library, one per device, held until the process exits.
 * Sizes with ovb_linear_workspace_bytes(M, K) above 8 MiB return
 * OVB_ERR_INVALID_ARG.  Arguments are checked before anything is enqueued.
 * Calls that overlap on the GPU race on the array.  The first call in each
 * CUDA context (the device's primary context, a context the host binds
 * through the driver API, or the new context after cudaDeviceReset) looks up
 * the array's address in that context and should come before any stream
 * capture in it.  No counterpart in the reference. */
int ovb_linear_static(int64_t M, const ovb_weight* w, const float* A, int64_t lda, float* C,
                      int64_t ldc, int accumulate, void* stream);

/* Exact per-32-k block products P[m, n, b] (int32 [M, N, Kb]) of the same
 * tensor-core mainloop, for parity checks of the integer arithmetic. */
int ovb_block_products(int64_t M, const ovb_weight* w, const int8_t* aq, int32_t* P,
                       void* stream);

/* The guided (classifier-free guidance) argmax pass of a TTS step, on device
 * pointers: for every codebook c < codebooks and target frame t < target_len,
 * with the cond row at token cond_seq - target_len + t of `cond` and the
 * uncond row at token t of `uncond` (both planes token-major [seq,
 * codebooks * vocab] fp32):
 *   lp_c, lp_u = log_softmax of the two rows;
 *   mix = log_softmax(lp_c + guidance * (lp_c - lp_u))   (mix = lp_c if guidance == 0);
 *   mix[mask_id] = -inf (no token is masked if mask_id is outside [0, vocab));
 *   pred[c * target_len + t] = first argmax of mix;
 *   scores[c * target_len + t] = max(mix) - c * layer_penalty.
 * Replaces the reference's CPU loop (cpp/src/model/tts.cpp:291-326, log_softmax
 * :91-101) and its CUDA guided_sample_kernel (cpp/src/backend/cuda/
 * cuda_lm.cu:679-758, called by LmRunnerSampleThunk :1228-1262) behind
 * LM::CudaSampleFn (cpp/src/model/lm.h:106-108; that hook copies pred/scores
 * back to the host).  pred and scores are device
 * arrays of codebooks * target_len.  target_len <= 0 or codebooks <= 0
 * returns OVB_OK without work; cond_seq / uncond_seq < target_len is
 * OVB_ERR_INVALID_ARG.  Log-probabilities agree with the CPU loop to a few
 * ulps (its sums run left to right, these in a warp tree), so pred agrees
 * except where two tokens' scores tie within rounding. */
int ovb_guided_sample(const float* cond, int cond_seq, const float* uncond, int uncond_seq,
                      int codebooks, int vocab, int target_len, float guidance,
                      float layer_penalty, int mask_id, int32_t* pred, float* scores,
                      void* stream);

/* One CFG pair of ovb_guided_sample_batch: its planes and lengths. */
typedef struct ovb_guided_pair {
  const float* cond;
  int cond_seq;
  const float* uncond;
  int uncond_seq;
  int target_len;
} ovb_guided_pair;

/* ovb_guided_sample for n_pairs CFG pairs (n_pairs <= 64) with the same
 * codebooks, vocab, guidance, layer_penalty and mask_id, in one launch when
 * vocab is 1025 (the LM's audio vocabulary; one launch per pair otherwise):
 * pair p's [codebooks, target_len] outputs follow pair p - 1's in pred and
 * scores.  The same values as one ovb_guided_sample per pair.  A serving
 * loop's TTS step calls it once for all the utterances of a packed forward
 * (the reference calls LM::CudaSampleFn once per utterance, tts.cpp:278-286). */
int ovb_guided_sample_batch(int n_pairs, const ovb_guided_pair* pairs, int codebooks, int vocab,
                            float guidance, float layer_penalty, int mask_id, int32_t* pred,
                            float* scores, void* stream);

/* One attention segment, as the reference's AttnSegment (cpp/src/model/
 * lm.h:46-51): `rows` query rows starting at element offset q_off of q/out,
 * attending to the `rows` keys / values starting at element offset kv_off of
 * k/v, with an optional additive bias [rows, rows] (row-major, device). */
typedef struct ovb_attn_segment {
  const float* bias;
  int32_t rows;
  int64_t q_off;
  int64_t kv_off;
} ovb_attn_segment;

/* The attention of one layer on device pointers: for each segment and query
 * head h < n_heads (kv head h / (n_heads / n_kv)),
 *   out[s, h] = softmax_t(q[s, h] . k[t, kv] * scale + bias[s, t]) v[t, kv],
 * a row whose scores are all below -1e29 (fully masked) giving zeros --
 * ov::attention_head_f32 (cpp/src/backend/cpu/ops_cpu.cpp:907-943) over the
 * loop of LM::run_layer (cpp/src/model/lm.cpp:256-274); the reference's CUDA
 * runner does the same with a SIMT kernel or TF32 cuBLAS (cpp/src/backend/
 * cuda/cuda_lm.cu:393-421, :423-606, dispatched at :1132-1145).  Row s of
 * head h of q and out is at element q_off + s * q_stride + h * head_dim; of
 * k / v at kv_off + t * kv_stride + kv * head_dim.  head_dim must be 128;
 * q/k/v/out 16-byte aligned; strides and offsets multiples of 4 elements;
 * every head of a segment's rows within one row of the 2-D view
 * ((q_off % q_stride) + n_heads * 128 <= q_stride, likewise for k/v); at
 * most 64 segments.  The products run on the tensor cores with fp16 inputs
 * and fp32 accumulation: the output agrees with the fp32 reference to ~1e-3
 * relative; a q/k/v value beyond the fp16 range sets ovb_device_status bit
 * 16.  n_segs == 0 (or only empty segments) returns OVB_OK without work. */
int ovb_attention(const float* q, const float* k, const float* v, float* out, int64_t q_stride,
                  int64_t kv_stride, int n_heads, int n_kv, int head_dim, float scale,
                  const ovb_attn_segment* segs, int n_segs, void* stream);

/* The same attention on fp16 q / k / v ([rows, q_stride] and [rows,
 * kv_stride] fp16, strides and offsets multiples of 8 elements), the form
 * the LM forward writes after its q/k norm + RoPE: two query heads of a kv
 * head per CTA sharing each K / V tile, the tensor core and the softmax
 * overlapped (S, P and O in tensor memory), V read in place as an MN-major
 * operand.  `tiles` is a table from ovb_attention_tiles for the same
 * segment list (the segments' masks; their bias fields are then ignored) or
 * NULL (each segment's fp32 bias, or none, read per element).  Output fp32
 * like ovb_attention; the same agreement with the fp32 reference (fp16
 * operands, fp32 accumulation and softmax).  Segment rows <= 32768.  No
 * counterpart in the reference beyond ovb_attention's. */
int ovb_attention_h(const void* q, const void* k, const void* v, float* out, int64_t q_stride,
                    int64_t kv_stride, int n_heads, int n_kv, int head_dim, float scale,
                    const ovb_attn_segment* segs, int n_segs, const void* tiles, void* stream);
/* ovb_attention_h followed by ovb_quantize of its output (the o
 * projection's input, LM::run_layer lm.cpp:281 quantising inside
 * linear_s8_nk_packed_add), in one kernel: every query row's head output is
 * four whole 32-k blocks, quantised as the output is formed and written in
 * the form `flags` selects (0 int8 q / OVB_AQ_U8 / OVB_AQ_F16) into aq
 * [rows, n_heads * head_dim] and its scales into asc [rows, n_heads *
 * head_dim / 32] -- bit-identical to the two calls, without the fp32
 * output.  Needs q_stride == n_heads * head_dim and segment offsets at whole
 * rows; rows are those of the q view.  No counterpart in the reference. */
int ovb_attention_h_q(const void* q, const void* k, const void* v, int64_t q_stride,
                      int64_t kv_stride, int n_heads, int n_kv, int head_dim, float scale,
                      const ovb_attn_segment* segs, int n_segs, const void* tiles, void* aq,
                      float* asc, int flags, void* stream);
/* Bytes of the tile table of a segment list (seg_rows: host array of the
 * segments' row counts): per (segment, 128-query block, 128-key tile) a
 * class byte and 2 KB of mask bits. */
size_t ovb_attention_tiles_bytes(const int32_t* seg_rows, int n_segs);
/* Build that table on the device from the segments' u8 attention masks
 * (1 = attend; [rows_i, rows_i] each, concatenated in segment order, the
 * reference's attn masks, lm.cpp:365): class 0 when every key of a tile is
 * attended (no mask is read), 1 when mixed (its bits are read), 3 when none
 * is (the tile is skipped) -- the same softmax as the additive bias
 * 0 / -1e30 the reference builds from the masks.  `tiles` 256-byte aligned,
 * tiles_bytes >= ovb_attention_tiles_bytes. */
int ovb_attention_tiles(const int32_t* seg_rows, int n_segs, const uint8_t* masks, void* tiles,
                        size_t tiles_bytes, void* stream);

/* ------------------------------------------------------------------ OVW1
 * The reference's weight file (docs/weight-format.en.md), read the way its
 * loader reads it (ov::WeightFile::Open, cpp/src/core/weight_file.cpp:124-206:
 * one read-only mapping, header and index validated, tensors by name), so
 * that int8 linear weights go from the mapping straight into the device
 * layout: ovb_ovw1_weight replaces make_linear's host repack into VNNI tiles
 * (cpp/src/model/mat.cpp:69-106, gemm.cpp:584-621) and the CUDA runner's
 * fp32 expansion of every int8 tensor (LmRunner::weight, cuda_lm.cu:840-873).
 * Pointers in ovb_ovw1_tensor point into the mapping and stay valid until
 * ovb_ovw1_close.  Errors are OVB_ERR_INVALID_ARG with the reference loader's
 * messages ("OVW1: bad magic (not an OVW1 file)", "... out of bounds",
 * "size mismatch for ...", "tensor not found: ..."). */
typedef struct ovb_ovw1 ovb_ovw1;

typedef struct ovb_ovw1_tensor {
  const char* name;     /* NUL-terminated copy, owned by the file handle */
  int32_t name_len;
  int32_t dtype;        /* 0 f32, 1 int8, 2 f16, 3 int64 */
  int32_t ndim;         /* 0..4 */
  int32_t layout;       /* 0 row-major as stored, 1 transposed linear weight [K, N] */
  int32_t quant;        /* 1: per-output-channel symmetric int8 with `scales` */
  int64_t dims[4];      /* shape in the stored layout */
  const void* data;     /* payload in the mapping */
  int64_t nbytes;
  const float* scales;  /* n_scales fp32 scales in the mapping, or NULL */
  int64_t n_scales;
  uint32_t crc;         /* stored CRC32 of the payload */
} ovb_ovw1_tensor;

/* WeightFile::Open (weight_file.cpp:124-206). */
int ovb_ovw1_open(const char* path, ovb_ovw1** out);
/* WeightFile::Release (weight_file.cpp:77-94); NULL is a no-op. */
int ovb_ovw1_close(ovb_ovw1* f);
/* Number of tensors (0 for NULL). */
int64_t ovb_ovw1_count(const ovb_ovw1* f);
/* The header's dtype_mode, flags and n_params (any output may be NULL). */
int ovb_ovw1_header(const ovb_ovw1* f, uint32_t* dtype_mode, uint64_t* flags, uint64_t* n_params);
/* Tensor i in file order. */
int ovb_ovw1_tensor_at(const ovb_ovw1* f, int64_t i, ovb_ovw1_tensor* out);
/* WeightFile::Get (weight_file.cpp:208-218): OVB_ERR_INVALID_ARG when absent. */
int ovb_ovw1_find(const ovb_ovw1* f, const char* name, ovb_ovw1_tensor* out);
/* WeightFile::ComputeCrc (weight_file.cpp:220-222): CRC32 (IEEE) of the
 * payload as mapped; compare with ovb_ovw1_tensor.crc. */
int ovb_ovw1_crc(const ovb_ovw1* f, const char* name, uint32_t* computed);
/* make_linear (mat.cpp:69-106) for an int8 weight with per-output-channel
 * scales, either layout (1: [K, N], 0: [N, K]), packed on the device by
 * ovb_weight_create; flags 0 or OVB_WEIGHT_F16.  Other tensors are
 * OVB_ERR_INVALID_ARG (fp32 linear weights are not on this path). */
int ovb_ovw1_weight(const ovb_ovw1* f, const char* name, int flags, void* stream,
                    ovb_weight** out);
/* ovb_ovw1_weight for n tensors at once through ovb_weight_create_batch (one
 * device allocation, one synchronisation).  This is the loader fast path: a
 * checkpoint's int8 linear layers go from the file to the device layout
 * without a host repack. */
int ovb_ovw1_weights(const ovb_ovw1* f, const char* const* names, int n, int flags,
                     void* stream, ovb_weight** out);

/* ------------------------------------------------------------------ LM
 * The whole LM forward on the device, built from an OVW1 checkpoint: the
 * reference's LM (cpp/src/model/lm.h:52-140, lm.cpp) for the accelerator
 * hook LM::CudaForwardFn (lm.h:91-96) and the ragged
 * CFG forward.  Linear weights (q/k/v/o, gate/up/down) must be int8 with
 * per-output-channel scales, either orientation; the audio heads int8 the
 * same way or fp32 (the reference converter's default, tools/
 * convert_weights.py:326-327, run through ovb_weight_create_f32 and fp16
 * activations of the final RMSNorm, OVB_AQ_F16_RAW); embeddings int8
 * with row scales or fp32; head_dim 128; LMConfig's rms_eps 1e-6 and
 * rope_theta 1e6.  flags: 0 runs the bit-exact int8 mainloop, OVB_WEIGHT_F16
 * the fp16 one.  One model per (thread, device); its forward buffers grow on
 * demand (ovb_lm_reserve sizes them ahead, e.g. before a stream capture). */
typedef struct ovb_lm ovb_lm;
int ovb_lm_create(const char* ovw1_path, int flags, void* stream, ovb_lm** out);
int ovb_lm_destroy(ovb_lm* m);
/* {n_layers, hidden, n_heads, n_kv_heads, head_dim, inter, vocab,
 *  audio_vocab, n_codebooks} */
int ovb_lm_config(const ovb_lm* m, int64_t* cfg);
int ovb_lm_reserve(ovb_lm* m, int64_t rows, int64_t mask_elems);
/* LM::forward_cfg (lm.cpp:403-454) on host buffers: input_ids [C, rows]
 * (rows = cond_seq + uncond_seq, codebook-major), audio_mask [rows],
 * cond_attn [cond_seq, cond_seq], uncond_attn [uncond_seq, uncond_seq],
 * position [rows]; logits [rows, C*V] token-major, or NULL to leave them on
 * the device only (ovb_lm_logits).  Synchronous. */
int ovb_lm_forward_cfg(ovb_lm* m, int cond_seq, int uncond_seq, const int64_t* ids,
                       const uint8_t* audio_mask, const uint8_t* cond_attn,
                       const uint8_t* uncond_attn, const int64_t* pos, float* logits,
                       void* stream);
/* The same on device inputs, stream-ordered (no synchronisation); the logits
 * stay on the device, at ovb_lm_logits(m) (LM::CudaLogitsFn, lm.h:95). */
int ovb_lm_forward_cfg_device(ovb_lm* m, int cond_seq, int uncond_seq, const int64_t* ids,
                              const uint8_t* audio_mask, const uint8_t* cond_attn,
                              const uint8_t* uncond_attn, const int64_t* pos, void* stream);
const float* ovb_lm_logits(const ovb_lm* m);
/* Several attention segments in one forward, on device inputs (stream-
 * ordered, no synchronisation): segment i has seg_rows[i] >= 1 rows (a HOST
 * array of n_segs <= 64 counts), packed one after another; ids [C, rows]
 * codebook-major, audio_mask [rows], pos [rows] and masks (each segment's
 * [seg_rows[i], seg_rows[i]] u8 attention mask, concatenated) are device
 * arrays; the logits [rows, C*V] stay at ovb_lm_logits(m).  Rows attend only
 * within their own segment, and every other step of the forward works row by
 * row, so each segment's logits are those of a forward over that segment
 * alone.  A CFG pair is two segments (LM::forward_cfg, lm.cpp:403-454, is
 * this call with n_segs = 2) and a batch of B rows B segments (LM::forward,
 * lm.cpp:343-401): the call packs several utterances' CFG pairs into one
 * forward -- the reference's AttnSegment list (cpp/src/model/lm.h:46-51)
 * with more than one utterance in it, which the reference never builds (it
 * runs one utterance at a time, cpp/src/model/tts.cpp:260-269). */
int ovb_lm_forward_segments_device(ovb_lm* m, int n_segs, const int32_t* seg_rows,
                                   const int64_t* ids, const uint8_t* audio_mask,
                                   const uint8_t* masks, const int64_t* pos, void* stream);
/* LM::forward (lm.cpp:343-401) with CudaForwardFn's arguments on host
 * buffers: input_ids [B, C, S], audio_mask [B, S], attn_mask [B, S, S],
 * position [B, S]; logits [B, C, S, V], or NULL to leave them on the device
 * only, token-major [B * S, C * V] at ovb_lm_logits -- the reference runner's
 * device-sampling mode (LmRunnerSetDeviceSampling, cuda_lm.h:48-50), whose
 * CFG planes LM::sample_guided then reads (tts.cpp:270-282).  batch <= 64.
 * Synchronous. */
int ovb_lm_forward(ovb_lm* m, int batch, int seq, const int64_t* ids, const uint8_t* audio_mask,
                   const uint8_t* attn_mask, const int64_t* pos, float* logits, void* stream);
/* LM::CudaSampleFn (lm.h:101-108) on the model's device: ovb_guided_sample on
 * the device planes cond / uncond (e.g. ovb_lm_logits and the plane after
 * it), then pred and scores ([C, target_len], HOST arrays) copied back,
 * synchronously; the device outputs are the model's own buffers.  The
 * contract of the reference's LmRunnerSampleThunk (cuda_lm.cu:1227-1262). */
int ovb_lm_sample(ovb_lm* m, const float* cond, int cond_seq, const float* uncond,
                  int uncond_seq, int target_len, float guidance, float layer_penalty,
                  int mask_id, int32_t* pred, float* scores, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OVB200_H */
