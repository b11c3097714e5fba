// ref_shim.cpp -- extern "C" entry points over the reference's own CPU GEMM
// path, so Python tests can call it through ctypes.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference sources cpp/src/backend/cpu/gemm.cpp, ops_cpu.cpp,
// cpp/src/core/weight_file.cpp and cpp/src/model/lm.cpp + mat.cpp (read in
// place from the reference checkout, never copied) into oracle/_ref/libovref.so.
// Each wrapper forwards to the ov:: function named in its comment
// (declared in cpp/include/ovnative/ov_gemm.h and cpp/src/model/ops.h) and turns
// C++ exceptions into a non-zero return.
#include <cstdint>
#include <cstring>
#include <exception>
#include <vector>

#include <xmmintrin.h>

#include <memory>

#include "model/lm.h"
#include "model/ops.h"
#include "ovnative/ov_gemm.h"
#include "ovnative/ov_weights.h"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {
template <class F>
int guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}
}  // namespace

REF_API int ref_vnni_available() { return ov::cpu_vnni_available() ? 1 : 0; }
REF_API const char* ref_kernel_name() { return ov::cpu_kernel_name(); }
REF_API int64_t ref_packed_bytes(int64_t N, int64_t K) { return ov::s8_nk_packed_bytes(N, K); }
REF_API int64_t ref_wsum_elems(int64_t N, int64_t K) { return ov::s8_nk_wsum_elems(N, K); }

// ov::s8_nk_pack (gemm.cpp:584-621)
REF_API int ref_s8_nk_pack(int64_t N, int64_t K, const int8_t* W, int8_t* packed, int32_t* wsum) {
  return guard([&] { ov::s8_nk_pack(N, K, W, packed, wsum); });
}
// ov::s8_nk_quantize (gemm.cpp:709-720)
REF_API int ref_s8_nk_quantize(int64_t M, int64_t K, const float* A, uint8_t* aq, float* asc) {
  return guard([&] { ov::s8_nk_quantize(M, K, A, aq, asc); });
}
// ov::rmsnorm_quantize_f32 (gemm.cpp:722-756)
REF_API int ref_rmsnorm_quantize(int64_t rows, int64_t cols, const float* x, const float* w,
                                 float eps, uint8_t* aq, float* asc) {
  return guard([&] { ov::rmsnorm_quantize_f32(rows, cols, x, w, eps, aq, asc); });
}
// ov::silu_mul_quantize_f32 (ops_cpu.cpp:1138-1168)
REF_API int ref_silu_mul_quantize(int64_t M, int64_t K, const float* gate, const float* up,
                                  uint8_t* aq, float* asc) {
  return guard([&] { ov::silu_mul_quantize_f32(M, K, gate, up, aq, asc); });
}
// ov::rmsnorm_into_f32 (ops_cpu.cpp:812-825)
REF_API int ref_rmsnorm_into(float* dst, const float* src, const float* w, int64_t rows,
                             int64_t cols, float eps) {
  return guard([&] { ov::rmsnorm_into_f32(dst, src, w, rows, cols, eps); });
}
// ov::silu_mul_f32 (ops_cpu.cpp:834-839)
REF_API int ref_silu_mul(float* out, const float* gate, const float* up, int64_t n) {
  return guard([&] { ov::silu_mul_f32(out, gate, up, n); });
}
// ov::linear_s8_nk_packed_q (gemm.cpp:758-774)
REF_API int ref_linear_packed_q(int64_t M, int64_t N, int64_t K, const uint8_t* aq,
                                const float* asc, const int8_t* packed, const int32_t* wsum,
                                const float* scale, float* C) {
  return guard([&] { ov::linear_s8_nk_packed_q(M, N, K, aq, asc, packed, wsum, scale, C); });
}
// ov::linear_s8_nk_packed_q_add (gemm.cpp:847-862)
REF_API int ref_linear_packed_q_add(int64_t M, int64_t N, int64_t K, const uint8_t* aq,
                                    const float* asc, const int8_t* packed, const int32_t* wsum,
                                    const float* scale, float* C) {
  return guard([&] { ov::linear_s8_nk_packed_q_add(M, N, K, aq, asc, packed, wsum, scale, C); });
}
// ov::linear_s8_nk_packed (gemm.cpp:829-845)
REF_API int ref_linear_packed(int64_t M, int64_t N, int64_t K, const float* A,
                              const int8_t* packed, const int32_t* wsum, const float* scale,
                              float* C) {
  return guard([&] { ov::linear_s8_nk_packed(M, N, K, A, packed, wsum, scale, C); });
}
// ov::linear_s8_nk_packed_add (gemm.cpp:864-882)
REF_API int ref_linear_packed_add(int64_t M, int64_t N, int64_t K, const float* A,
                                  const int8_t* packed, const int32_t* wsum, const float* scale,
                                  float* C) {
  return guard([&] { ov::linear_s8_nk_packed_add(M, N, K, A, packed, wsum, scale, C); });
}
// ov::linear_s8_nk_packed_q_sliced (gemm.cpp:776-827); slice i has Ns[i] columns -> Cs[i].
REF_API int ref_linear_packed_q_sliced(int64_t M, int64_t K, const uint8_t* aq, const float* asc,
                                       const int8_t* packed, const int32_t* wsum,
                                       const float* scale, const int64_t* Ns, float* const* Cs,
                                       int n_slices) {
  std::vector<ov::S8NkSlice> s(static_cast<size_t>(n_slices));
  for (int i = 0; i < n_slices; ++i) {
    s[static_cast<size_t>(i)].N = Ns[i];
    s[static_cast<size_t>(i)].C = Cs[i];
  }
  return guard([&] {
    ov::linear_s8_nk_packed_q_sliced(M, K, aq, asc, packed, wsum, scale, s.data(), n_slices);
  });
}
// ov::linear_s8_nk (gemm.cpp:923-940): the AVX2 path with unquantised activations
// that the reference runs on hosts without AVX-VNNI.
REF_API int ref_linear_s8_nk(int64_t M, int64_t N, int64_t K, const float* A, const int8_t* W,
                             const float* scale, float* C) {
  return guard([&] { ov::linear_s8_nk(M, N, K, A, W, scale, C); });
}

// ov::attention_head_f32 (ops_cpu.cpp:907-943): one head of one attention
// segment, softmax(q k^T * scale + bias) v with fully masked rows -> 0.  Its
// AVX2 kernels switch the calling thread to flush-to-zero / denormals-are-zero
// (ops_cpu.cpp:335, :738, as LM::forward does for every worker, lm.cpp:347-348);
// the caller's MXCSR is restored afterwards so that the checkers that run
// later in the same process keep IEEE denormals.
REF_API int ref_attention_head(const float* q, int64_t q_stride, const float* k, const float* v,
                               int64_t kv_stride, const float* bias, int S, int D, float scale,
                               float* out, int64_t out_stride) {
  const unsigned csr = _mm_getcsr();
  const int rc = guard([&] {
    ov::attention_head_f32(q, q_stride, k, v, kv_stride, bias, S, D, scale, out, out_stride);
  });
  _mm_setcsr(csr);
  return rc;
}

// ov::WeightFile::Open + Get + ComputeCrc (cpp/src/core/weight_file.cpp:124-222):
// the reference loader's view of one tensor of an OVW1 file.  info[] =
// {dtype, ndim, transposed, quantized, dims[0..3], nbytes, n_scales,
// data offset in the file, scales offset (or -1)}; crc[] = {stored,
// computed}.  Returns 0, or 1 with the loader's exception message in err.
REF_API int ref_ovw1_tensor(const char* path, const char* name, int64_t* info, uint32_t* crc,
                            char* err, int err_len) {
  try {
    ov::WeightFile wf = ov::WeightFile::Open(path);
    const ov::Tensor& t = wf.Get(name);
    info[0] = static_cast<int64_t>(t.dtype);
    info[1] = t.shape.ndim;
    info[2] = t.transposed ? 1 : 0;
    info[3] = t.quantized ? 1 : 0;
    for (int k = 0; k < 4; ++k) info[4 + k] = t.shape.dims[k];
    info[8] = t.nbytes;
    info[9] = t.n_scales;
    crc[0] = wf.StoredCrc(t);
    crc[1] = wf.ComputeCrc(t);
    return 0;
  } catch (const std::exception& e) {
    if (err && err_len > 0) {
      std::strncpy(err, e.what(), static_cast<size_t>(err_len) - 1);
      err[err_len - 1] = 0;
    }
    return 1;
  }
}

// The attention of one layer as LM::run_layer runs it (lm.cpp:256-274):
// ov::attention_head_f32 for every (segment, kv head, query head of the
// group) in one OpenMP loop, head h at column h*D of q/out, kv head h/group
// at column kv*D of k/v.  The worker threads' MXCSR is restored afterwards
// (the AVX2 kernels turn on flush-to-zero).
REF_API int ref_attention_layer(const float* q, const float* k, const float* v, float* out,
                                int64_t QD, int64_t KVD, int NH, int NKV, int D, float scale,
                                const float* const* bias, const int* rows, const int64_t* q_off,
                                const int64_t* kv_off, int n_segs) {
  const unsigned csr = _mm_getcsr();
  const int group = NH / NKV;
  int bad = 0;
#pragma omp parallel for collapse(3) schedule(static) reduction(| : bad)
  for (int seg = 0; seg < n_segs; ++seg) {
    for (int kv = 0; kv < NKV; ++kv) {
      for (int g = 0; g < group; ++g) {
        const int h = kv * group + g;
        const int64_t qo = q_off[seg] + static_cast<int64_t>(h) * D;
        const int64_t ko = kv_off[seg] + static_cast<int64_t>(kv) * D;
        bad |= guard([&] {
          ov::attention_head_f32(q + qo, QD, k + ko, v + ko, KVD, bias[seg], rows[seg], D, scale,
                                 out + qo, QD);
        });
      }
    }
  }
#pragma omp parallel
  { _mm_setcsr(csr); }
  _mm_setcsr(csr);
  return bad;
}

// The reference's LM (cpp/src/model/lm.h:52-140) over an OVW1 file: LMConfig
// defaults except n_layers.  The WeightFile outlives the LM (its tensors point
// into the mapping).  The forwards switch every OpenMP worker to flush-to-zero
// (lm.cpp:347-348, :412-413); the caller's MXCSR is put back on all of them
// afterwards so that later checkers keep IEEE denormals.
namespace {
struct RefLm {
  ov::WeightFile wf;
  std::unique_ptr<ov::LM> lm;
};
template <class F>
int with_csr(F&& f) {
  const unsigned csr = _mm_getcsr();
  const int rc = guard(f);
#pragma omp parallel
  { _mm_setcsr(csr); }
  _mm_setcsr(csr);
  return rc;
}
}  // namespace

REF_API void* ref_lm_create(const char* path, int n_layers, char* err, int err_len) {
  try {
    auto r = std::make_unique<RefLm>();
    r->wf = ov::WeightFile::Open(path);
    ov::LMConfig cfg;
    cfg.n_layers = n_layers;
    r->lm = std::make_unique<ov::LM>(r->wf, cfg);
    return r.release();
  } catch (const std::exception& e) {
    if (err && err_len > 0) {
      std::strncpy(err, e.what(), static_cast<size_t>(err_len) - 1);
      err[err_len - 1] = 0;
    }
    return nullptr;
  }
}

REF_API void ref_lm_destroy(void* h) { delete static_cast<RefLm*>(h); }

// LM::forward_cfg (lm.cpp:403-454)
REF_API int ref_lm_forward_cfg(void* h, int cond_seq, int uncond_seq, const int64_t* ids,
                               const uint8_t* amask, const uint8_t* cond_attn,
                               const uint8_t* uncond_attn, const int64_t* pos, float* logits) {
  return with_csr([&] {
    static_cast<RefLm*>(h)->lm->forward_cfg(cond_seq, uncond_seq, ids, amask, cond_attn,
                                            uncond_attn, pos, logits);
  });
}

// LM::forward (lm.cpp:343-401)
REF_API int ref_lm_forward(void* h, int batch, int seq, const int64_t* ids, const uint8_t* amask,
                           const uint8_t* attn, const int64_t* pos, float* logits) {
  return with_csr([&] {
    static_cast<RefLm*>(h)->lm->forward(batch, seq, ids, amask, attn, pos, logits);
  });
}
