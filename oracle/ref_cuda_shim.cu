// ref_cuda_shim.cu -- C entry point to the reference's own CUDA guided
// sampler, for the GPU parity tests.  TEST INFRASTRUCTURE ONLY: nothing in
// the product library (ovnative_b200/) links or loads it.
//
// The reference's guided_sample_kernel (cpp/src/backend/cuda/cuda_lm.cu:
// 679-758) lives in an anonymous namespace of that file, reachable only from
// inside its translation unit, so this shim includes the reference's source
// file where it lies (the include path is the reference checkout, given by
// oracle/Makefile; nothing is copied) and launches the kernel exactly as its
// own LmRunnerSampleThunk does (cuda_lm.cu:1227-1252): one block of 128
// threads per (codebook, target frame), (V + 128) floats of dynamic shared
// memory, mask id passed by the caller (1024 there).  Built with the
// reference's CUDA flags (--use_fast_math, src/backend/cuda/CMakeLists.txt:21)
// for sm_100a.
#include "backend/cuda/cuda_lm.cu"

extern "C" int ref_cuda_guided_sample(const float* cond, int cond_seq, const float* uncond,
                                      int uncond_seq, int codebooks, int vocab, int target_len,
                                      float guidance, float layer_penalty, int mask_id,
                                      int32_t* pred, float* scores, void* stream) {
  const int n = codebooks * target_len;
  if (n <= 0) return 0;
  const int threads = 128;
  const size_t smem = (static_cast<size_t>(vocab) + threads) * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(ov::cuda::guided_sample_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return 1;
  ov::cuda::guided_sample_kernel<<<n, threads, smem, static_cast<cudaStream_t>(stream)>>>(
      cond, cond_seq, uncond, uncond_seq, codebooks, vocab, target_len, guidance, layer_penalty,
      mask_id, pred, scores);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// The reference's own CUDA LM forward (LmRunner, cuda_lm.cu:790-1221: fp16
// cublasGemmEx on weights dequantised at load, TF32 attention from 160
// tokens) for the end-to-end parity tests: how far the reference's GPU path
// itself sits from its CPU path on the same checkpoint.  The file must use the
// [K, N] int8 encoding (lm.h:60-63).
namespace {
struct RefCudaLm {
  ov::WeightFile wf;
  ov::cuda::LmRunnerPtr runner{nullptr, &ov::cuda::LmRunnerDelete};
};

void put_err(const char* msg, char* err, int err_len) {
  if (err && err_len > 0) {
    std::strncpy(err, msg, static_cast<size_t>(err_len) - 1);
    err[err_len - 1] = 0;
  }
}
}  // namespace

extern "C" void* ref_cuda_lm_create(const char* path, int n_layers, char* err, int err_len) {
  try {
    auto r = std::make_unique<RefCudaLm>();
    r->wf = ov::WeightFile::Open(path);
    ov::LMConfig cfg;
    cfg.n_layers = n_layers;
    r->runner = ov::cuda::LmRunnerCreate(r->wf, cfg);
    if (!r->runner) {
      put_err("LmRunnerCreate failed", err, err_len);
      return nullptr;
    }
    return r.release();
  } catch (const std::exception& e) {
    put_err(e.what(), err, err_len);
    return nullptr;
  }
}

extern "C" void ref_cuda_lm_destroy(void* h) { delete static_cast<RefCudaLm*>(h); }

// LmRunner::forward with LM::forward's arguments (host buffers, synchronous).
extern "C" int ref_cuda_lm_forward(void* h, int batch, int seq, const int64_t* ids,
                                   const uint8_t* amask, const uint8_t* attn, const int64_t* pos,
                                   float* logits) {
  try {
    ov::cuda::LmRunnerForward(*static_cast<RefCudaLm*>(h)->runner, batch, seq, ids, amask, attn,
                              pos, logits);
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 3;
  } catch (const std::exception&) {
    return 1;
  }
}
