// ov_hooks_test.cpp -- the reference-side binding (include/ovb200_ov_hooks.hpp)
// compiled into a program built on the reference's own LM, Mat and WeightFile
// (oracle/_ref/libovref.so) and run against the reference's CPU path.  TEST
// INFRASTRUCTURE ONLY: built by oracle/Makefile into oracle/_ref/, run by
// tests/test_gpu_ov_hooks.py on a GPU.
//
//   ov_hooks_test <lm.ovw> <n_layers> <mats.ovw> <flags> <out_dir>
//
// 1. Two reference LMs on the same file; ovb_hooks::install() puts the B200
//    path behind one of them (LM::set_cuda_backend).  LM::forward over a B = 2
//    CFG batch built as Pipeline::run_sampling builds it for the CUDA path
//    (cpp/src/model/tts.cpp:172-204) runs through the hook and on the CPU; the
//    cosine, mean |delta| and argmax agreement of the logits are printed (the
//    reference's LM gate, cpp/tests/test_lm.cpp:198-230).
// 2. With the sampling hook installed (device sampling: the forward leaves
//    its logits on the device), the same forward and LM::sample_guided on the
//    two CFG planes of LM::last_logits_dev() (tts.cpp:270-282); pred, scores
//    and the host logits of step 1 go to <out_dir> for the caller to check
//    against the guided-sampling checker.
// 3. For every tensor of <mats.ovw>: ov::make_linear (mat.cpp:69-106), then
//    ovb_hooks::Mat::mul / mul_add on the device against Mat::mul / mul_add on
//    the host; max |delta| and relative L2 are printed, and whether the
//    outputs are bit-identical.
// One JSON object per line on stdout; exit code 0 unless something threw.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <random>
#include <string>
#include <vector>

#include "model/lm.h"
#include "model/mat.h"
#include "ovb200_ov_hooks.hpp"
#include "ovnative/ov_weights.h"

namespace {

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <class T>
void dump(const std::string& path, const std::vector<T>& v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
}

struct Stats {
  double cos, mean, maxd, rel_l2, agree;
  bool identical;
};

Stats compare(const std::vector<float>& got, const std::vector<float>& want, int V) {
  double dot = 0, na = 0, nb = 0, sumd = 0, maxd = 0, d2 = 0;
  bool same = true;
  for (size_t i = 0; i < want.size(); ++i) {
    const double a = got[i], b = want[i], d = std::fabs(a - b);
    dot += a * b;
    na += a * a;
    nb += b * b;
    sumd += d;
    d2 += d * d;
    maxd = std::max(maxd, d);
    same = same && std::memcmp(&got[i], &want[i], 4) == 0;
  }
  size_t agree = 0, n = V > 0 ? want.size() / static_cast<size_t>(V) : 0;
  for (size_t p = 0; p < n; ++p) {
    const float* a = got.data() + p * V;
    const float* b = want.data() + p * V;
    int ia = 0, ib = 0;
    for (int v = 1; v < V; ++v) {
      if (a[v] > a[ia]) ia = v;
      if (b[v] > b[ib]) ib = v;
    }
    agree += ia == ib;
  }
  return {dot / (std::sqrt(na) * std::sqrt(nb) + 1e-30), sumd / static_cast<double>(want.size()),
          maxd, std::sqrt(d2 / (nb + 1e-30)), n ? static_cast<double>(agree) / n : 0.0, same};
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 6) {
    std::fprintf(stderr, "usage: %s <lm.ovw> <n_layers> <mats.ovw> <flags> <out_dir>\n", argv[0]);
    return 2;
  }
  try {
    const std::string lm_path = argv[1], mats_path = argv[3], out = argv[5];
    const int flags = std::atoi(argv[4]);
    ov::WeightFile wf = ov::WeightFile::Open(lm_path);
    ov::LMConfig cfg;
    cfg.n_layers = std::atoi(argv[2]);
    ov::LM cpu(wf, cfg), dev(wf, cfg);
    auto hook = ovb_hooks::install(dev, lm_path, flags, nullptr, /*sampler=*/false);
    if (!dev.cuda_enabled()) throw std::runtime_error("the forward hook is not installed");

    // ---- the B = 2 CFG batch of run_sampling's CUDA path (tts.cpp:172-204)
    const int C = cfg.n_codebooks, V = cfg.audio_vocab, S = 96, T = 70, kMask = 1024;
    std::mt19937 rng(1234);
    std::vector<int64_t> ids(static_cast<size_t>(2) * C * S, kMask);
    std::vector<uint8_t> amask(2 * S, 0), attn(static_cast<size_t>(2) * S * S, 0);
    std::vector<int64_t> pos(2 * S);
    std::uniform_int_distribution<int> text(0, 2000), audio(0, 1023);
    for (int c = 0; c < C; ++c)
      for (int i = 0; i < S; ++i) {
        // prompt: S - T text ids in every codebook row, then target frames,
        // half of them already unmasked with audio ids
        int64_t v = i < S - T ? text(rng) : (i % 2 ? audio(rng) : kMask);
        if (c > 0 && i < S - T) v = ids[static_cast<size_t>(i)];
        ids[static_cast<size_t>(c) * S + i] = v;
      }
    for (int c = 0; c < C; ++c)
      for (int t = 0; t < T; ++t)
        ids[static_cast<size_t>(C + c) * S + t] = ids[static_cast<size_t>(c) * S + (S - T + t)];
    for (int i = S - T; i < S; ++i) amask[i] = 1;
    for (int i = 0; i < S * S; ++i) attn[i] = 1;
    for (int t = 0; t < T; ++t) {
      amask[S + t] = 1;
      for (int j = 0; j < T; ++j) attn[static_cast<size_t>(S + t) * S + j] = 1;
    }
    for (int t = T; t < S; ++t) attn[static_cast<size_t>(S + t) * S + t] = 1;
    for (int b = 0; b < 2; ++b)
      for (int i = 0; i < S; ++i) pos[static_cast<size_t>(b) * S + i] = i;

    std::vector<float> want(static_cast<size_t>(2) * C * S * V), got(want.size());
    cpu.forward(2, S, ids.data(), amask.data(), attn.data(), pos.data(), want.data());
    dev.forward(2, S, ids.data(), amask.data(), attn.data(), pos.data(), got.data());
    Stats st = compare(got, want, V);
    std::printf("{\"check\": \"forward_hook\", \"cos\": %.9f, \"mean\": %.4e, \"max\": %.4e, "
                "\"agree\": %.5f}\n", st.cos, st.mean, st.maxd, st.agree);
    dump(out + "/logits_cpu.f32", want);
    dump(out + "/logits_dev.f32", got);

    // ---- the sampling hook with device sampling
    dev.set_cuda_sampler(hook.get(), ovb_hooks::sample_thunk);
    hook->device_sampling = true;
    std::vector<float> unused(want.size(), -7.f);
    dev.forward(2, S, ids.data(), amask.data(), attn.data(), pos.data(), unused.data());
    const bool untouched = unused[0] == -7.f && unused.back() == -7.f;
    const float* d = static_cast<const float*>(dev.last_logits_dev());
    if (!d) throw std::runtime_error("no device logits");
    std::vector<int32_t> pred(static_cast<size_t>(C) * T);
    std::vector<float> scores(pred.size());
    if (!dev.sample_guided(d, S, d + static_cast<size_t>(S) * C * V, S, T, 2.0f, 5.0f, pred.data(),
                           scores.data()))
      throw std::runtime_error("the sampling hook is not installed");
    std::vector<float> planes(static_cast<size_t>(2) * S * C * V);
    cuda_check(cudaMemcpy(planes.data(), d, planes.size() * 4, cudaMemcpyDeviceToHost),
               "copy device logits");
    dump(out + "/planes_dev.f32", planes);
    dump(out + "/pred.i32", pred);
    dump(out + "/scores.f32", scores);
    std::printf("{\"check\": \"sample_hook\", \"S\": %d, \"T\": %d, \"C\": %d, \"V\": %d, "
                "\"host_logits_untouched\": %s}\n", S, T, C, V, untouched ? "true" : "false");

    // ---- the Mat shim against the reference's Mat, every tensor of mats.ovw
    ov::WeightFile mw = ov::WeightFile::Open(mats_path);
    for (const ov::Tensor& t : mw.tensors()) {
      const ov::Mat m = ov::make_linear(mw, t.name);
      ovb_hooks::Mat om(m, flags);
      const int64_t M = 77;
      std::vector<float> A(static_cast<size_t>(M * m.K)), C0(static_cast<size_t>(M * m.N));
      std::normal_distribution<float> nd(0.f, 1.f);
      for (float& x : A) x = nd(rng);
      for (float& x : C0) x = nd(rng);
      std::vector<float> ref_mul(C0.size()), ref_add = C0;
      m.mul(M, A.data(), ref_mul.data());
      const bool add = m.add_supported();
      if (add) m.mul_add(M, A.data(), ref_add.data());
      float *dA = nullptr, *dC = nullptr;
      void* work = nullptr;
      const size_t wb = om.workspace_bytes(M);
      cuda_check(cudaMalloc(&dA, A.size() * 4), "cudaMalloc");
      cuda_check(cudaMalloc(&dC, C0.size() * 4), "cudaMalloc");
      cuda_check(cudaMalloc(&work, wb), "cudaMalloc");
      cuda_check(cudaMemcpy(dA, A.data(), A.size() * 4, cudaMemcpyHostToDevice), "copy");
      om.mul(M, dA, dC, work, wb);
      std::vector<float> got_mul(C0.size()), got_add(C0.size());
      cuda_check(cudaMemcpy(got_mul.data(), dC, C0.size() * 4, cudaMemcpyDeviceToHost), "copy");
      cuda_check(cudaMemcpy(dC, C0.data(), C0.size() * 4, cudaMemcpyHostToDevice), "copy");
      om.mul_add(M, dA, dC, work, wb);
      cuda_check(cudaMemcpy(got_add.data(), dC, C0.size() * 4, cudaMemcpyDeviceToHost), "copy");
      cudaFree(dA);
      cudaFree(dC);
      cudaFree(work);
      const Stats a = compare(got_mul, ref_mul, 0);
      const Stats b = add ? compare(got_add, ref_add, 0) : Stats{1, 0, 0, 0, 0, true};
      const char* kind = m.w ? "fp32" : (m.nk ? "int8_nk" : "int8_kn");
      std::printf("{\"check\": \"mat\", \"name\": \"%s\", \"kind\": \"%s\", \"packed\": %s, "
                  "\"mul_rel_l2\": %.4e, \"mul_max\": %.4e, \"mul_identical\": %s, "
                  "\"add_supported\": %s, \"add_rel_l2\": %.4e, \"add_identical\": %s}\n",
                  t.name.c_str(), kind, m.vnni_packed() ? "true" : "false", a.rel_l2, a.maxd,
                  a.identical ? "true" : "false", add ? "true" : "false", b.rel_l2,
                  b.identical ? "true" : "false");
    }
    std::printf("{\"check\": \"done\"}\n");
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ov_hooks_test: %s\n", e.what());
    return 1;
  }
}
