/* ovb200_ov_hooks.hpp -- the reference-side binding of libovb200.so into
 * OVNative: the code a maintainer of the reference adds (for example to
 * cpp/tools/ovtts.cpp, beside its own CUDA install at ovtts.cpp:119-150) so
 * that the reference's LM runs on the B200 path.  Header-only C++17, compiled
 * as part of the reference: it includes the reference's "model/lm.h" and
 * "model/mat.h" and this library's C ABI (ovb200.h), and needs no CUDA header.
 *
 * Two pieces:
 *
 *  - LmHook + install(): the LM's accelerator hooks (cpp/src/model/lm.h:
 *    91-110) over an ovb_lm made from the same OVW1 file:
 *        LM::CudaForwardFn  -> ovb_lm_forward (host logits [B, C, S, V]; with
 *                              device sampling on, the logits stay on the
 *                              device, as LmRunnerSetDeviceSampling does,
 *                              cuda_lm.h:48-50)
 *        LM::CudaLogitsFn   -> ovb_lm_logits (token-major [B * S, C * V])
 *        LM::CudaSampleFn   -> ovb_lm_sample (mask id 1024, as the
 *                              reference's LmRunnerSampleThunk passes it)
 *    They replace LmRunnerForwardThunk / LmRunnerLastLogitsThunk /
 *    LmRunnerSampleThunk (cuda_lm.h:33-45) and, unlike the reference's
 *    runner, accept the [N, K] int8 files (lm.h:60-63 rejects them on CUDA).
 *
 *  - Mat: the dispatch of the reference's Mat (mat.cpp:11-54) on the device:
 *    one ovb_weight built from a reference Mat (make_linear, mat.cpp:69-106:
 *    fp32 [K, N], int8 [K, N] with column scales, or int8 [N, K] with row
 *    scales) and mul / mul_add / mul_q / mul_q_add with the reference's
 *    argument meaning on DEVICE pointers, stream-ordered.  mul / mul_add take
 *    fp32 activations (quantised inside for int8 weights, the
 *    linear_s8_nk_packed[_add] semantics; converted to fp16 for fp32 weights,
 *    linear_f32's role); mul_q / mul_q_add take this library's quantised
 *    activations (int8 q [M, Kp] and fp32 scales from ovb_quantize /
 *    ovb_rmsnorm_quantize / ovb_silu_mul_quantize) where the reference takes
 *    its u8 form.  All four work for either int8 layout (the reference's
 *    mul_q / mul_add need its VNNI-packed [N, K] form; on the device both
 *    layouts pack to one image).
 *
 * Errors throw std::runtime_error with ovb_last_error(), as the reference's
 * own thunks throw on CUDA errors (cuda_lm.cu:19-26).
 */
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>

#include "model/lm.h"
#include "model/mat.h"
#include "ovb200.h"

namespace ovb_hooks {

inline void check(int status, const char* what) {
  if (status != OVB_OK)
    throw std::runtime_error(std::string("ovb200: ") + what + ": " + ovb_last_error());
}

// ------------------------------------------------------------------ LM hooks
struct LmHook {
  ovb_lm* lm = nullptr;
  void* stream = nullptr;        // cudaStream_t (NULL: the legacy default stream)
  bool device_sampling = false;  // forward leaves the logits on the device only
  LmHook() = default;
  LmHook(const LmHook&) = delete;
  LmHook& operator=(const LmHook&) = delete;
  ~LmHook() { ovb_lm_destroy(lm); }
};

inline void forward_thunk(void* ctx, int batch, int seq, const int64_t* ids,
                          const uint8_t* amask, const uint8_t* attn, const int64_t* pos,
                          float* logits) {
  auto* h = static_cast<LmHook*>(ctx);
  check(ovb_lm_forward(h->lm, batch, seq, ids, amask, attn, pos,
                       h->device_sampling ? nullptr : logits, h->stream),
        "LM forward");
}

inline const void* logits_thunk(void* ctx) {
  return ovb_lm_logits(static_cast<LmHook*>(ctx)->lm);
}

inline void sample_thunk(void* ctx, const void* cond, int cond_seq, const void* uncond,
                         int uncond_seq, int target_len, float guidance, float layer_penalty,
                         int32_t* pred, float* scores) {
  auto* h = static_cast<LmHook*>(ctx);
  check(ovb_lm_sample(h->lm, static_cast<const float*>(cond), cond_seq,
                      static_cast<const float*>(uncond), uncond_seq, target_len, guidance,
                      layer_penalty, /*mask_id=*/1024, pred, scores, h->stream),
        "guided sample");
}

// Create the device model from the OVW1 file `lm` was built from and install
// the hooks.  flags: 0 (bit-exact int8 mainloop) or OVB_WEIGHT_F16 (fp16
// mainloop).  With `sampler`, the sampling hook is installed too and the
// forward leaves its logits on the device (the reference's CUDA install does
// the same, ovtts.cpp:128-140).  The returned hook must outlive the LM's use.
inline std::unique_ptr<LmHook> install(ov::LM& lm, const std::string& ovw1_path, int flags,
                                       void* stream = nullptr, bool sampler = true) {
  auto h = std::make_unique<LmHook>();
  h->stream = stream;
  check(ovb_lm_create(ovw1_path.c_str(), flags, stream, &h->lm), "ovb_lm_create");
  int64_t c[9];
  check(ovb_lm_config(h->lm, c), "ovb_lm_config");
  const ov::LMConfig& k = lm.config();
  if (c[0] != k.n_layers || c[1] != k.hidden || c[2] != k.n_heads || c[3] != k.n_kv_heads ||
      c[4] != k.head_dim || c[5] != k.inter || c[7] != k.audio_vocab || c[8] != k.n_codebooks)
    throw std::runtime_error("ovb200: the file's LM shape differs from the LM's LMConfig");
  lm.set_cuda_backend(h.get(), forward_thunk, logits_thunk);
  if (sampler) {
    lm.set_cuda_sampler(h.get(), sample_thunk);
    h->device_sampling = true;
  }
  return h;
}

// ------------------------------------------------------------------ Mat
class Mat {
 public:
  // flags: 0 or OVB_WEIGHT_F16 (int8 weights); fp32 weights always run the
  // fp16 tensor cores (ovb_weight_create_f32).
  Mat(const ov::Mat& m, int flags = 0, void* stream = nullptr)
      : N_(m.N), K_(m.K), fp32_(m.w != nullptr), stream_(stream) {
    if (m.w) {
      check(ovb_weight_create_f32(m.w, OVB_LAYOUT_KN, N_, K_, stream, &w_), "fp32 weight");
    } else if (m.q) {
      check(ovb_weight_create(m.q, m.nk ? OVB_LAYOUT_NK : OVB_LAYOUT_KN, N_, K_, m.row_scale(),
                              flags, stream, &w_),
            "int8 weight");
    } else {
      throw std::runtime_error("ovb200 Mat: empty weight");
    }
  }
  Mat(const Mat&) = delete;
  Mat& operator=(const Mat&) = delete;
  ~Mat() { ovb_weight_destroy(w_); }

  int64_t N() const { return N_; }
  int64_t K() const { return K_; }
  const ovb_weight* handle() const { return w_; }
  bool add_supported() const { return true; }

  // Device scratch mul / mul_add need for M rows (caller-owned, 256-byte
  // aligned): the quantised activations of an int8 weight, or the fp16
  // activations of an fp32 weight.
  size_t workspace_bytes(int64_t M) const {
    const size_t f16 = static_cast<size_t>(M) * static_cast<size_t>((K_ + 31) / 32 * 32) * 2;
    return fp32_ ? f16 : ovb_linear_workspace_bytes(M, K_);
  }

  // Mat::mul (mat.cpp:11-27): C[M, N] = A[M, K] W, device pointers, row-major.
  void mul(int64_t M, const float* A, float* C, void* work, size_t work_bytes) const {
    run(M, A, C, 0, work, work_bytes);
  }
  // Mat::mul_add (mat.cpp:39-49): C += A W.
  void mul_add(int64_t M, const float* A, float* C, void* work, size_t work_bytes) const {
    run(M, A, C, 1, work, work_bytes);
  }
  // Mat::mul_q (mat.cpp:51-54): C = linear(aq, asc) for an int8 weight.
  void mul_q(int64_t M, const int8_t* aq, const float* asc, float* C) const {
    if (fp32_) throw std::runtime_error("Mat::mul_q: weight is not int8");
    check(ovb_linear_q(M, w_, aq, asc, C, N_, 0, stream_), "mul_q");
  }
  // Mat::mul_q_add (mat.cpp:31-37): C += linear(aq, asc).
  void mul_q_add(int64_t M, const int8_t* aq, const float* asc, float* C) const {
    if (fp32_) throw std::runtime_error("Mat::mul_q_add: weight is not int8");
    check(ovb_linear_q(M, w_, aq, asc, C, N_, 1, stream_), "mul_q_add");
  }

 private:
  void run(int64_t M, const float* A, float* C, int accumulate, void* work,
           size_t work_bytes) const {
    if (M <= 0) return;
    if (work_bytes < workspace_bytes(M)) throw std::runtime_error("ovb200 Mat: workspace too small");
    if (fp32_) {
      check(ovb_quantize(M, K_, A, K_, work, nullptr, OVB_AQ_F16_RAW, stream_), "fp16 activations");
      check(ovb_linear_h(M, w_, work, C, N_, accumulate, stream_), "fp32-weight GEMM");
    } else {
      check(ovb_linear(M, w_, A, K_, C, N_, accumulate, work, work_bytes, stream_), "int8 GEMM");
    }
  }

  int64_t N_, K_;
  bool fp32_;
  void* stream_;
  ovb_weight* w_ = nullptr;
};

}  // namespace ovb_hooks
