// capi.cpp -- the extern "C" entry points declared in include/ovb200.h:
// argument checks, weight handles, TMA descriptors, and kernel launches.
//
// Error behaviour mirrors the reference contract (ov_gemm.h / gemm.cpp):
// M, N or K <= 0 is a silent no-op (gemm.cpp:761, :779, :832); a bad
// argument that the reference rejects with std::invalid_argument /
// std::runtime_error (e.g. gemm.cpp:786-788 for slice widths) returns
// OVB_ERR_INVALID_ARG here; CUDA failures return OVB_ERR_INTERNAL.  The
// message is kept per thread for ovb_last_error().
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ovb200.h"
#include "ovb_internal.h"

namespace ovb {

namespace {
thread_local std::string t_error;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}
}  // namespace

void set_error(const std::string& msg) { t_error = msg; }

bool cuda_failed(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return false;
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return true;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("OVB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int num_sms(int device) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lock(mu);
  if (device >= static_cast<int>(cache.size())) cache.resize(static_cast<size_t>(device) + 1, 0);
  if (cache[static_cast<size_t>(device)] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cache[static_cast<size_t>(device)] = n;
  }
  return cache[static_cast<size_t>(device)];
}

namespace {
std::mutex g_ws_mu;
std::vector<float*> g_split_ws;  // per device; kept for the life of the process
}  // namespace

bool ensure_split_workspace(int device) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  if (device >= static_cast<int>(g_split_ws.size()))
    g_split_ws.resize(static_cast<size_t>(device) + 1, nullptr);
  float*& ws = g_split_ws[static_cast<size_t>(device)];
  if (ws) return true;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(kSplitSlots) * kSplitSlotBytes) != cudaSuccess) {
    cudaGetLastError();  // without a workspace the GEMMs run without split-K
    return false;
  }
  ws = static_cast<float*>(p);
  return true;
}

float* split_workspace(int device) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  return device < static_cast<int>(g_split_ws.size()) ? g_split_ws[static_cast<size_t>(device)]
                                                      : nullptr;
}

bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                    uint64_t inner, uint64_t rows, uint64_t stride_bytes, uint32_t box_inner,
                    uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
    return false;
  }
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t elem_strides[2] = {1u, 1u};
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    std::snprintf(buf, sizeof buf,
                  "cuTensorMapEncodeTiled failed (%d): rows=%llu inner=%llu stride=%llu",
                  static_cast<int>(r), static_cast<unsigned long long>(rows),
                  static_cast<unsigned long long>(inner),
                  static_cast<unsigned long long>(stride_bytes));
    set_error(buf);
    return false;
  }
  return true;
}

bool encode_tmap_u8(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
                    uint64_t stride_bytes, uint32_t box_rows) {
  return encode_tmap_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, row_bytes, rows, stride_bytes,
                        static_cast<uint32_t>(kStageK), box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace ovb

using ovb::cuda_failed;
using ovb::set_error;

namespace {

inline int64_t kblocks(int64_t K) { return (K + 31) / 32; }
inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// Output form of a quantiser from its flags (0 int8, 1 u8, 2 fp16), or -1.
int quant_mode(int flags) {
  const int f = flags & (OVB_AQ_U8 | OVB_AQ_F16 | OVB_AQ_F16_RAW);
  switch (f) {
    case 0: return 0;
    case OVB_AQ_U8: return 1;
    case OVB_AQ_F16: return 2;
    case OVB_AQ_F16_RAW: return 3;
    default: return -1;  // the forms are exclusive
  }
}

int invalid(const std::string& msg) {
  set_error(msg);
  return OVB_ERR_INVALID_ARG;
}

int internal_err() { return OVB_ERR_INTERNAL; }

// Tensor maps of the packed weight for every GEMM tile width.
bool ensure_weight_tmap(ovb_weight* w) {
  for (int i = 0; i < 3; ++i) {
    if (w->tmap_ready[i]) continue;
    if (!ovb::encode_tmap_u8(&w->tmap_b[i], w->w, static_cast<uint64_t>(w->Kp),
                             static_cast<uint64_t>(w->N), static_cast<uint64_t>(w->Kp),
                             static_cast<uint32_t>(ovb::kTileN[i])))
      return false;
    w->tmap_ready[i] = true;
  }
  return true;
}

// Tensor maps of the fp16 weight copy for every fp16-mainloop tile width.
bool ensure_weight_tmap16(ovb_weight* w) {
  if (!w->w16) return true;
  for (int i = 0; i < 4; ++i) {
    if (w->tmap16_ready[i]) continue;
    if (!ovb::encode_tmap_2d(&w->tmap_w16[i], w->w16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             static_cast<uint64_t>(w->Kp), static_cast<uint64_t>(w->N),
                             static_cast<uint64_t>(w->Kp) * 2, 64u,
                             static_cast<uint32_t>(ovb::kTileNF[i]), CU_TENSOR_MAP_SWIZZLE_128B))
      return false;
    w->tmap16_ready[i] = true;
  }
  return true;
}

// Allocate and fill the fp16 copy of a packed weight.
bool make_weight_f16(ovb_weight* w, cudaStream_t s) {
  const size_t n = static_cast<size_t>(w->N * w->Kp);
  ovb::ensure_split_workspace(w->device);  // optional: split-K configs need it
  return !cuda_failed(cudaMalloc(&w->w16, n * 2), "cudaMalloc(fp16 weight)") &&
         !cuda_failed(ovb::launch_widen_f16(w->w, static_cast<int64_t>(n), w->w16, s),
                      "widen weight") &&
         !cuda_failed(cudaStreamSynchronize(s), "widen sync") && ensure_weight_tmap16(w);
}

void free_weight(ovb_weight* w) {
  if (!w->arena) {
    cudaFree(w->w);
    cudaFree(w->scale);
    cudaFree(w->w16);
  }
  delete w;  // a batch's arena is freed with its last weight
}

// Common checks of a pre-quantised GEMM call.  Returns OVB_OK or a status.
int check_q_args(int64_t M, const ovb_weight* w, const int8_t* aq, const float* asc) {
  if (!w) return invalid("weight handle is null");
  if (!w->w) return invalid("weight has no int8 image (made by ovb_weight_create_f32): use ovb_linear_h");
  if (!aq || !asc) return invalid("aq/asc must be non-null");
  if (!aligned(aq, 16)) return invalid("aq must be 16-byte aligned (TMA source)");
  if (!aligned(asc, 4)) return invalid("asc must be 4-byte aligned");
  if (M > (int64_t{1} << 31) - 1) return invalid("M exceeds 2^31-1");
  int dev = 0;
  if (cuda_failed(cudaGetDevice(&dev), "cudaGetDevice")) return OVB_ERR_INTERNAL;
  if (dev != w->device) return invalid("weight lives on another device than the current one");
  return OVB_OK;
}

// Fused SiLU*up output of a gate|up GEMM (null: none).
struct SiluOut {
  void* out;
  float* asc;
  int mode;
};

int run_gemm(int64_t M, const ovb_weight* wc, const int8_t* aq, const float* asc,
             const ovb::SliceOut* slices, int n_slices, int accumulate, int32_t* products,
             cudaStream_t s, const SiluOut* silu = nullptr) {
  ovb_weight* w = const_cast<ovb_weight*>(wc);
  if (!ensure_weight_tmap(w)) return OVB_ERR_INTERNAL;
  CUtensorMap tmap_a;
  if (!ovb::encode_tmap_u8(&tmap_a, aq, static_cast<uint64_t>(w->Kp), static_cast<uint64_t>(M),
                           static_cast<uint64_t>(w->Kp), ovb::kBlockM))
    return OVB_ERR_INTERNAL;
  ovb::GemmArgs args{};
  // The fused SiLU*up epilogue and the block products run the int8 mainloop.
  const bool f16 = w->w16 != nullptr && products == nullptr && silu == nullptr;
  CUtensorMap tmap_a16;
  if (f16 && !ovb::encode_tmap_2d(&tmap_a16, aq, CU_TENSOR_MAP_DATA_TYPE_UINT8,
                                  static_cast<uint64_t>(w->Kp), static_cast<uint64_t>(M),
                                  static_cast<uint64_t>(w->Kp), 64u,
                                  static_cast<uint32_t>(ovb::kBlockM), CU_TENSOR_MAP_SWIZZLE_64B))
    return OVB_ERR_INTERNAL;
  args.M = M;
  args.N = w->N;
  args.Kb = w->Kb;
  args.asc = asc;
  args.wscale = w->scale;
  args.accumulate = accumulate;
  args.n_slices = n_slices;
  for (int i = 0; i < n_slices; ++i) args.slices[i] = slices[i];
  args.products = products;
  if (silu) {
    args.silu_out = static_cast<uint8_t*>(silu->out);
    args.silu_asc = silu->asc;
    args.silu_mode = silu->mode;
    args.silu_kp = w->glu_inter;
    if (cuda_failed(ovb::launch_gemm(0, tmap_a, w->tmap_b[0], args, s), "gemm launch"))
      return OVB_ERR_INTERNAL;
    return OVB_OK;
  }
  if (f16) {
    if (!ensure_weight_tmap16(w)) return OVB_ERR_INTERNAL;
    const int tile = ovb::pick_tile_f16(M, w->N, w->Kb, w->device);
    if (cuda_failed(ovb::launch_gemm_f16(tile, tmap_a16, w->tmap_w16[tile], args, s),
                    "gemm launch"))
      return OVB_ERR_INTERNAL;
    return OVB_OK;
  }
  const int tile = ovb::pick_tile(M, w->N, w->device);
  if (cuda_failed(ovb::launch_gemm(tile, tmap_a, w->tmap_b[tile], args, s), "gemm launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

// Outputs of the fused q/k RMSNorm + RoPE epilogue (null: none).
struct RopeOut {
  void *q16, *k16, *v16;
  const float *qw, *kw, *tab;
  int64_t qd, kvd;
  float eps;
};

// OVB_GEMM_TMA_OUT=0 keeps the plain fp16 epilogue on register stores (and
// residual loads), =1 uses TMA boxes whenever the output allows; unset, the
// launch shape decides.  A tuning and comparison switch.
int tma_out_mode() {
  const char* e = std::getenv("OVB_GEMM_TMA_OUT");
  return e ? (e[0] == '0' ? 0 : 1) : -1;
}

// The plain fp16 mainloop on dequantised activations a16 [M, Kp] fp16.
int run_gemm_h(int64_t M, const ovb_weight* wc, const void* a16, const ovb::SliceOut* slices,
               int n_slices, int accumulate, cudaStream_t s, const SiluOut* silu = nullptr,
               const RopeOut* rope = nullptr) {
  ovb_weight* w = const_cast<ovb_weight*>(wc);
  if (!ensure_weight_tmap16(w)) return OVB_ERR_INTERNAL;
  CUtensorMap tmap_a;
  if (!ovb::encode_tmap_2d(&tmap_a, a16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           static_cast<uint64_t>(w->Kp), static_cast<uint64_t>(M),
                           static_cast<uint64_t>(w->Kp) * 2, 64u,
                           static_cast<uint32_t>(ovb::kBlockM), CU_TENSOR_MAP_SWIZZLE_128B))
    return OVB_ERR_INTERNAL;
  ovb::GemmArgs args{};
  args.M = M;
  args.N = w->N;
  args.Kb = w->Kb;
  args.asc = nullptr;
  args.wscale = w->scale;
  args.accumulate = accumulate;
  args.n_slices = n_slices;
  for (int i = 0; i < n_slices; ++i) args.slices[i] = slices[i];
  args.products = nullptr;
  if (silu) {
    args.silu_out = static_cast<uint8_t*>(silu->out);
    args.silu_asc = silu->asc;
    args.silu_mode = silu->mode;
    args.silu_kp = w->glu_inter;
  }
  if (rope) {
    args.rope_q16 = rope->q16;
    args.rope_k16 = rope->k16;
    args.rope_v16 = rope->v16;
    args.rope_qw = rope->qw;
    args.rope_kw = rope->kw;
    args.rope_tab = rope->tab;
    args.rope_qd = rope->qd;
    args.rope_kvd = rope->kvd;
    args.rope_eps = rope->eps;
  }
  args.split_ws = ovb::split_workspace(w->device);
  // split-K configurations need the workspace; the fused SiLU*up epilogue
  // takes BN >= 64 without split-K; the fused q/k norm + RoPE epilogue
  // 256-column tiles per CTA (two whole heads): configurations 0 and 7
  const int config = ovb::pick_tile_h(
      M, w->N, w->Kb, w->device,
      rope ? ovb::kHRope
           : (silu ? ovb::kHSilu : (args.split_ws ? ovb::kHAll : ovb::kHNoSplit)));
  // Plain outputs leave through the TMA (stores, or adds into C when
  // accumulating) when every slice's rows are 16-byte aligned and the CTAs
  // have several tiles each (the epilogue then runs beside the next tile's
  // mainloop, and C's traffic no longer passes through the SM; with one tile
  // per CTA the register stores finish sooner: 0.2 us at 400 rows).
  const int64_t out_tiles = ((M + ovb::kBlockM - 1) / ovb::kBlockM) *
                            ((w->N + ovb::h_tile_n(config) - 1) / ovb::h_tile_n(config));
  const int tma_mode = tma_out_mode();
  if (!silu && !rope &&
      (tma_mode == 1 || (tma_mode < 0 && out_tiles > 2 * ovb::num_sms(w->device)))) {
    bool ok = true;
    for (int i = 0; i < n_slices; ++i)
      ok = ok && (reinterpret_cast<uintptr_t>(slices[i].C) & 15) == 0 && (slices[i].ldc & 3) == 0;
    for (int i = 0; ok && i < n_slices; ++i)
      if (!ovb::encode_tmap_2d(&args.out_map[i], slices[i].C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                               static_cast<uint64_t>(slices[i].n_count), static_cast<uint64_t>(M),
                               static_cast<uint64_t>(slices[i].ldc) * 4, 32u, 32u,
                               CU_TENSOR_MAP_SWIZZLE_128B))
        return OVB_ERR_INTERNAL;
    args.out_tma = ok ? 1 : 0;
  }
  const int width = ovb::kHConfigs[config].width;
  if (cuda_failed(ovb::launch_gemm_h(config, tmap_a, w->tmap_w16[width], args, s), "gemm launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

// Validate a slice list against a concatenated weight and convert it to
// the kernels' form (first column of each slice).  Returns OVB_OK or a status.
int build_slices(const ovb_weight* w, const ovb_slice* slices, int n_slices,
                 ovb::SliceOut (&so)[ovb::kMaxSlices]) {
  if (!slices) return invalid("slices is null");
  if (n_slices > ovb::kMaxSlices) return invalid("at most 4 slices");
  int64_t total = 0;
  for (int i = 0; i < n_slices; ++i) {
    // gemm.cpp:786-788: each slice N must be a positive multiple of 64.
    if (slices[i].N <= 0 || slices[i].N % 64 != 0 || !slices[i].C)
      return invalid("sliced GEMM: each slice N must be a positive multiple of 64");
    if (slices[i].ldc < slices[i].N) return invalid("sliced GEMM: ldc < N");
    so[i] = ovb::SliceOut{total, slices[i].N, slices[i].C, slices[i].ldc};
    total += slices[i].N;
  }
  if (total != w->N) return invalid("sliced GEMM: slice widths do not add up to the weight's N");
  return OVB_OK;
}

// Checks of a fused gate|up + SiLU*up call's weight and outputs.
int check_silu_out(const ovb_weight* w, void* out, float* out_asc, int flags, int* mode) {
  if (!w) return invalid("weight handle is null");
  if (w->glu_inter <= 0) return invalid("the fused SiLU*up GEMM needs a gate|up weight (ovb_weight_gate_up)");
  if (!out || !out_asc) return invalid("out/out_asc must be non-null");
  *mode = quant_mode(flags);
  if (*mode < 0) return invalid("OVB_AQ_U8, OVB_AQ_F16 and OVB_AQ_F16_RAW are exclusive");
  if (*mode == 3) return invalid("the fused SiLU*up GEMM writes quantised activations (no OVB_AQ_F16_RAW)");
  if (!aligned(out, 16) || !aligned(out_asc, 4)) return invalid("misaligned output buffer");
  return OVB_OK;
}

// Common checks of an ovb_linear_h call.
int check_h_args(int64_t M, const ovb_weight* w, const void* a16) {
  if (!w) return invalid("weight handle is null");
  if (!w->w16) return invalid("ovb_linear_h needs a weight created with OVB_WEIGHT_F16");
  if (!a16) return invalid("a16 is null");
  if (!aligned(a16, 16)) return invalid("a16 must be 16-byte aligned (TMA source)");
  if (M > (int64_t{1} << 31) - 1) return invalid("M exceeds 2^31-1");
  int dev = 0;
  if (cuda_failed(cudaGetDevice(&dev), "cudaGetDevice")) return OVB_ERR_INTERNAL;
  if (dev != w->device) return invalid("weight lives on another device than the current one");
  return OVB_OK;
}

int check_rope(int n_heads, int n_kv, int head_dim, const float* q_norm, const float* k_norm,
               const void* q16, const void* k16, const void* v16) {
  if (head_dim != 128) return invalid("head_dim must be 128");
  if (n_heads <= 0 || n_kv <= 0) return invalid("n_heads and n_kv must be positive");
  if (!q_norm || !k_norm || !q16 || !k16 || !v16)
    return invalid("q_norm/k_norm/q16/k16/v16 must be non-null");
  if (!aligned(q16, 16) || !aligned(k16, 16) || !aligned(v16, 16))
    return invalid("q16/k16/v16 must be 16-byte aligned");
  return OVB_OK;
}

}  // namespace

extern "C" {

int ovb_abi_version(void) { return OVB_ABI_VERSION; }

const char* ovb_last_error(void) { return ovb::t_error.c_str(); }

int ovb_device_status(void* stream) {
  int st = 0, st16 = 0, stq = 0, sta = 0, stl = 0;
  if (cuda_failed(ovb::read_and_clear_status(&st, as_stream(stream)), "read device status") ||
      cuda_failed(ovb::read_and_clear_status_f16(&st16, as_stream(stream)), "read device status") ||
      cuda_failed(ovb::read_and_clear_status_q(&stq, as_stream(stream)), "read device status") ||
      cuda_failed(ovb::read_and_clear_status_att(&sta, as_stream(stream)), "read device status") ||
      cuda_failed(ovb::read_and_clear_status_lm(&stl, as_stream(stream)), "read device status"))
    return OVB_ERR_INTERNAL;
  st |= st16 | stq | sta | stl;
  return st;
}

int64_t ovb_quant_bytes(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  return M * kblocks(K) * 32;
}

int64_t ovb_quant_scales(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  return M * kblocks(K);
}

// ---------------------------------------------------------------- weights
int ovb_weight_create(const int8_t* W, int layout, int64_t N, int64_t K, const float* scale,
                      int flags, void* stream, ovb_weight** out) {
  if (!out) return invalid("out is null");
  *out = nullptr;
  if (N <= 0 || K <= 0) return invalid("weight shape must be positive");
  if (!W || !scale) return invalid("W/scale must be non-null");
  if (layout != OVB_LAYOUT_NK && layout != OVB_LAYOUT_KN) return invalid("unknown layout");
  if (N > (int64_t{1} << 31) - 1 || K > (int64_t{1} << 30))
    return invalid("weight dimensions too large");
  cudaStream_t s = as_stream(stream);
  auto* w = new ovb_weight();
  if (cuda_failed(cudaGetDevice(&w->device), "cudaGetDevice")) {
    delete w;
    return OVB_ERR_INTERNAL;
  }
  w->N = N;
  w->K = K;
  w->Kb = kblocks(K);
  w->Kp = w->Kb * 32;
  const size_t wbytes = static_cast<size_t>(N * w->Kp);
  const size_t sbytes = static_cast<size_t>(N) * sizeof(float);
  const size_t src_bytes = static_cast<size_t>(N * K);
  int8_t* src_dev = nullptr;
  bool ok = !cuda_failed(cudaMalloc(&w->w, wbytes), "cudaMalloc(weight)") &&
            !cuda_failed(cudaMalloc(&w->scale, sbytes), "cudaMalloc(scale)");
  const bool on_device = (flags & OVB_SRC_DEVICE) != 0;
  if (ok) {
    if (on_device) {
      src_dev = const_cast<int8_t*>(W);
      ok = !cuda_failed(cudaMemcpyAsync(w->scale, scale, sbytes, cudaMemcpyDeviceToDevice, s),
                        "copy scale");
    } else {
      ok = !cuda_failed(cudaMalloc(&src_dev, src_bytes), "cudaMalloc(staging)") &&
           !cuda_failed(cudaMemcpyAsync(src_dev, W, src_bytes, cudaMemcpyHostToDevice, s),
                        "copy weight") &&
           !cuda_failed(cudaMemcpyAsync(w->scale, scale, sbytes, cudaMemcpyHostToDevice, s),
                        "copy scale");
    }
  }
  if (ok) {
    cudaError_t e = layout == OVB_LAYOUT_NK ? ovb::launch_pack_nk(src_dev, N, K, w->w, w->Kp, s)
                                            : ovb::launch_pack_kn(src_dev, N, K, w->w, w->Kp, s);
    ok = !cuda_failed(e, "pack weight") &&
         !cuda_failed(cudaStreamSynchronize(s), "weight pack sync");
  }
  if (!on_device && src_dev) cudaFree(src_dev);
  if (ok) ok = ensure_weight_tmap(w);
  if (ok && (flags & OVB_WEIGHT_F16)) ok = make_weight_f16(w, s);
  if (!ok) {
    free_weight(w);
    return OVB_ERR_INTERNAL;
  }
  *out = w;
  return OVB_OK;
}

int ovb_weight_create_f32(const float* W, int layout, int64_t N, int64_t K, void* stream,
                          ovb_weight** out) {
  if (!out) return invalid("out is null");
  *out = nullptr;
  if (N <= 0 || K <= 0) return invalid("weight shape must be positive");
  if (!W) return invalid("W must be non-null");
  if (layout != OVB_LAYOUT_NK && layout != OVB_LAYOUT_KN) return invalid("unknown layout");
  if (N > (int64_t{1} << 31) - 1 || K > (int64_t{1} << 30))
    return invalid("weight dimensions too large");
  const int64_t Kb = kblocks(K), Kp = Kb * 32;
  // Per output channel n: a power-of-two scale s[n] = 2^(e - 10), e the
  // exponent of max_k |W[n, k]|, so that W / s is exact in fp32 and lies
  // below 2048 in magnitude (well inside fp16), then one rounding to fp16.
  // The GEMM's epilogue multiplies by s[n] again (exact).
  std::vector<float> sc(static_cast<size_t>(N));
  std::vector<__half> h(static_cast<size_t>(N * Kp), __float2half_rn(0.f));
  auto at = [&](int64_t n, int64_t k) {
    return layout == OVB_LAYOUT_NK ? W[n * K + k] : W[k * N + n];
  };
  for (int64_t n = 0; n < N; ++n) {
    float amax = 0.f;
    for (int64_t k = 0; k < K; ++k) {
      const float v = at(n, k);
      if (!std::isfinite(v)) return invalid("ovb_weight_create_f32: non-finite weight");
      amax = std::fmax(amax, std::fabs(v));
    }
    const float s_n = amax > 0.f ? std::ldexp(1.f, std::ilogb(amax) - 10) : 1.f;
    sc[static_cast<size_t>(n)] = s_n;
    const float inv = 1.f / s_n;  // a power of two: exact
    for (int64_t k = 0; k < K; ++k) h[static_cast<size_t>(n * Kp + k)] = __float2half_rn(at(n, k) * inv);
  }
  cudaStream_t s = as_stream(stream);
  auto* w = new ovb_weight();
  if (cuda_failed(cudaGetDevice(&w->device), "cudaGetDevice")) {
    delete w;
    return OVB_ERR_INTERNAL;
  }
  w->N = N;
  w->K = K;
  w->Kb = Kb;
  w->Kp = Kp;
  const size_t hbytes = h.size() * sizeof(__half), sbytes = sc.size() * sizeof(float);
  bool ok = !cuda_failed(cudaMalloc(&w->w16, hbytes), "cudaMalloc(fp16 weight)") &&
            !cuda_failed(cudaMalloc(&w->scale, sbytes), "cudaMalloc(scale)") &&
            !cuda_failed(cudaMemcpyAsync(w->w16, h.data(), hbytes, cudaMemcpyHostToDevice, s),
                         "copy fp16 weight") &&
            !cuda_failed(cudaMemcpyAsync(w->scale, sc.data(), sbytes, cudaMemcpyHostToDevice, s),
                         "copy scale") &&
            !cuda_failed(cudaStreamSynchronize(s), "fp32 weight upload sync") &&
            ensure_weight_tmap16(w);
  if (ok) ovb::ensure_split_workspace(w->device);  // optional: split-K configs need it
  if (!ok) {
    free_weight(w);
    return OVB_ERR_INTERNAL;
  }
  *out = w;
  return OVB_OK;
}

int ovb_weight_create_batch(const ovb_weight_src* srcs, int n, int flags, void* stream,
                            ovb_weight** out) {
  if (!out) return invalid("out is null");
  if (n <= 0) return n == 0 ? OVB_OK : invalid("n must be >= 0");
  if (!srcs) return invalid("srcs is null");
  for (int i = 0; i < n; ++i) out[i] = nullptr;
  if ((flags & ~(OVB_WEIGHT_F16 | OVB_SRC_DEVICE)) != 0) return invalid("unknown flags");
  const bool f16 = (flags & OVB_WEIGHT_F16) != 0;
  const bool on_device = (flags & OVB_SRC_DEVICE) != 0;
  auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  size_t arena_bytes = 0, staging_bytes = 0;
  for (int i = 0; i < n; ++i) {
    const ovb_weight_src& w = srcs[i];
    if (!w.W || !w.scale) return invalid("W/scale must be non-null");
    if (w.N <= 0 || w.K <= 0) return invalid("weight shape must be positive");
    if (w.layout != OVB_LAYOUT_NK && w.layout != OVB_LAYOUT_KN) return invalid("unknown layout");
    if (w.N > (int64_t{1} << 31) - 1 || w.K > (int64_t{1} << 30))
      return invalid("weight dimensions too large");
    const size_t wb = static_cast<size_t>(w.N * kblocks(w.K) * 32);
    arena_bytes += up(wb) + up(static_cast<size_t>(w.N) * 4) + (f16 ? up(wb * 2) : 0);
    if (!on_device) staging_bytes += up(static_cast<size_t>(w.N * w.K));
  }
  int device = 0;
  if (cuda_failed(cudaGetDevice(&device), "cudaGetDevice")) return OVB_ERR_INTERNAL;
  cudaStream_t s = as_stream(stream);
  uint8_t* arena = nullptr;
  uint8_t* staging = nullptr;
  if (cuda_failed(cudaMalloc(&arena, arena_bytes), "cudaMalloc(weight arena)")) return OVB_ERR_INTERNAL;
  std::shared_ptr<void> hold(arena, [device](void* p) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaFree(p);
    cudaSetDevice(prev);
  });
  if (staging_bytes && cuda_failed(cudaMalloc(&staging, staging_bytes), "cudaMalloc(staging)"))
    return OVB_ERR_INTERNAL;
  if (f16) ovb::ensure_split_workspace(device);  // optional: split-K configs need it
  // Copies first (host payloads, as stored), then every pack / widen kernel;
  // one synchronisation at the end.
  std::vector<ovb_weight*> ws(static_cast<size_t>(n), nullptr);
  bool ok = true;
  size_t a_off = 0, s_off = 0;
  std::vector<const int8_t*> src_dev(static_cast<size_t>(n));
  for (int i = 0; i < n && ok; ++i) {
    const ovb_weight_src& src = srcs[i];
    auto* w = new ovb_weight();
    ws[static_cast<size_t>(i)] = w;
    w->device = device;
    w->arena = hold;
    w->N = src.N;
    w->K = src.K;
    w->Kb = kblocks(src.K);
    w->Kp = w->Kb * 32;
    const size_t wb = static_cast<size_t>(w->N * w->Kp);
    w->w = reinterpret_cast<int8_t*>(arena + a_off);
    a_off += up(wb);
    w->scale = reinterpret_cast<float*>(arena + a_off);
    a_off += up(static_cast<size_t>(w->N) * 4);
    if (f16) {
      w->w16 = reinterpret_cast<uint16_t*>(arena + a_off);
      a_off += up(wb * 2);
    }
    const size_t sb = static_cast<size_t>(w->N) * sizeof(float);
    if (on_device) {
      src_dev[static_cast<size_t>(i)] = src.W;
      ok = !cuda_failed(cudaMemcpyAsync(w->scale, src.scale, sb, cudaMemcpyDeviceToDevice, s),
                        "copy scale");
    } else {
      int8_t* d = reinterpret_cast<int8_t*>(staging + s_off);
      s_off += up(static_cast<size_t>(src.N * src.K));
      src_dev[static_cast<size_t>(i)] = d;
      ok = !cuda_failed(cudaMemcpyAsync(d, src.W, static_cast<size_t>(src.N * src.K),
                                        cudaMemcpyHostToDevice, s), "copy weight") &&
           !cuda_failed(cudaMemcpyAsync(w->scale, src.scale, sb, cudaMemcpyHostToDevice, s),
                        "copy scale");
    }
  }
  for (int i = 0; i < n && ok; ++i) {
    ovb_weight* w = ws[static_cast<size_t>(i)];
    const int8_t* d = src_dev[static_cast<size_t>(i)];
    cudaError_t e = srcs[i].layout == OVB_LAYOUT_NK
                        ? ovb::launch_pack_nk(d, w->N, w->K, w->w, w->Kp, s)
                        : ovb::launch_pack_kn(d, w->N, w->K, w->w, w->Kp, s);
    ok = !cuda_failed(e, "pack weight");
    if (ok && f16)
      ok = !cuda_failed(ovb::launch_widen_f16(w->w, w->N * w->Kp, w->w16, s), "widen weight");
  }
  if (ok) ok = !cuda_failed(cudaStreamSynchronize(s), "weight batch sync");
  if (staging) cudaFree(staging);
  for (int i = 0; i < n && ok; ++i) {
    ovb_weight* w = ws[static_cast<size_t>(i)];
    ok = ensure_weight_tmap(w) && ensure_weight_tmap16(w);
  }
  if (!ok) {
    for (ovb_weight* w : ws)
      if (w) free_weight(w);
    return OVB_ERR_INTERNAL;
  }
  for (int i = 0; i < n; ++i) out[i] = ws[static_cast<size_t>(i)];
  return OVB_OK;
}

int ovb_weight_concat(const ovb_weight* const* parts, int n_parts, void* stream,
                      ovb_weight** out) {
  if (!out) return invalid("out is null");
  *out = nullptr;
  if (!parts || n_parts <= 0) return invalid("no parts");
  int64_t total = 0;
  for (int i = 0; i < n_parts; ++i) {
    if (!parts[i]) return invalid("null part");
    if (!parts[i]->w) return invalid("concat: a part has no int8 image (ovb_weight_create_f32)");
    if (parts[i]->K != parts[0]->K) return invalid("concat: parts differ in K");
    if (parts[i]->device != parts[0]->device) return invalid("concat: parts on different devices");
    total += parts[i]->N;
  }
  cudaStream_t s = as_stream(stream);
  auto* w = new ovb_weight();
  w->device = parts[0]->device;
  w->N = total;
  w->K = parts[0]->K;
  w->Kb = parts[0]->Kb;
  w->Kp = parts[0]->Kp;
  bool ok = !cuda_failed(cudaMalloc(&w->w, static_cast<size_t>(total * w->Kp)), "cudaMalloc") &&
            !cuda_failed(cudaMalloc(&w->scale, static_cast<size_t>(total) * 4), "cudaMalloc");
  int64_t row = 0;
  for (int i = 0; ok && i < n_parts; ++i) {
    const ovb_weight* p = parts[i];
    ok = !cuda_failed(cudaMemcpyAsync(w->w + row * w->Kp, p->w, static_cast<size_t>(p->N * p->Kp),
                                      cudaMemcpyDeviceToDevice, s),
                      "concat copy") &&
         !cuda_failed(cudaMemcpyAsync(w->scale + row, p->scale, static_cast<size_t>(p->N) * 4,
                                      cudaMemcpyDeviceToDevice, s),
                      "concat copy");
    row += p->N;
  }
  if (ok) ok = !cuda_failed(cudaStreamSynchronize(s), "concat sync") && ensure_weight_tmap(w);
  bool all_f16 = true;
  for (int i = 0; i < n_parts; ++i) all_f16 = all_f16 && parts[i]->w16 != nullptr;
  if (ok && all_f16) ok = make_weight_f16(w, s);
  if (!ok) {
    free_weight(w);
    return OVB_ERR_INTERNAL;
  }
  *out = w;
  return OVB_OK;
}

int ovb_weight_gate_up(const ovb_weight* gate, const ovb_weight* up, void* stream,
                       ovb_weight** out) {
  if (!out) return invalid("out is null");
  *out = nullptr;
  if (!gate || !up) return invalid("gate/up handle is null");
  if (!gate->w || !up->w) return invalid("gate_up: a part has no int8 image (ovb_weight_create_f32)");
  if (gate->N != up->N || gate->K != up->K) return invalid("gate_up: gate and up differ in shape");
  if (gate->N % 32 != 0) return invalid("gate_up: N must be a multiple of 32");
  if (gate->device != up->device) return invalid("gate_up: parts on different devices");
  cudaStream_t s = as_stream(stream);
  auto* w = new ovb_weight();
  w->device = gate->device;
  w->N = 2 * gate->N;
  w->K = gate->K;
  w->Kb = gate->Kb;
  w->Kp = gate->Kp;
  w->glu_inter = gate->N;
  const int64_t blocks = gate->N / 32;
  // Rows interleaved in 32-row blocks: out block 2j = gate block j, 2j+1 = up block j.
  auto interleave = [&](void* dst, const void* g, const void* u, size_t row_bytes) {
    const size_t blk = 32 * row_bytes;
    return !cuda_failed(cudaMemcpy2DAsync(dst, 2 * blk, g, blk, blk, static_cast<size_t>(blocks),
                                          cudaMemcpyDeviceToDevice, s),
                        "gate_up interleave") &&
           !cuda_failed(cudaMemcpy2DAsync(static_cast<uint8_t*>(dst) + blk, 2 * blk, u, blk, blk,
                                          static_cast<size_t>(blocks), cudaMemcpyDeviceToDevice, s),
                        "gate_up interleave");
  };
  bool ok = !cuda_failed(cudaMalloc(&w->w, static_cast<size_t>(w->N * w->Kp)), "cudaMalloc") &&
            !cuda_failed(cudaMalloc(&w->scale, static_cast<size_t>(w->N) * 4), "cudaMalloc");
  if (ok) ok = interleave(w->w, gate->w, up->w, static_cast<size_t>(w->Kp));
  if (ok) ok = interleave(w->scale, gate->scale, up->scale, 4);
  if (ok && gate->w16 && up->w16) {
    ok = !cuda_failed(cudaMalloc(&w->w16, static_cast<size_t>(w->N * w->Kp) * 2), "cudaMalloc") &&
         interleave(w->w16, gate->w16, up->w16, static_cast<size_t>(w->Kp) * 2);
  }
  if (ok) ok = !cuda_failed(cudaStreamSynchronize(s), "gate_up sync") && ensure_weight_tmap(w) &&
               ensure_weight_tmap16(w);
  if (!ok) {
    free_weight(w);
    return OVB_ERR_INTERNAL;
  }
  *out = w;
  return OVB_OK;
}

int ovb_weight_destroy(ovb_weight* w) {
  if (!w) return OVB_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(w->device);
  free_weight(w);
  cudaSetDevice(prev);
  return OVB_OK;
}

int ovb_weight_shape(const ovb_weight* w, int64_t* N, int64_t* K) {
  if (!w) return invalid("weight handle is null");
  if (N) *N = w->N;
  if (K) *K = w->K;
  return OVB_OK;
}

int ovb_weight_export(const ovb_weight* w, int8_t* W_nk, float* scale) {
  if (!w || !W_nk || !scale) return invalid("null argument");
  if (!w->w) return invalid("weight has no int8 image (made by ovb_weight_create_f32)");
  if (cuda_failed(cudaMemcpy2D(W_nk, static_cast<size_t>(w->K), w->w, static_cast<size_t>(w->Kp),
                               static_cast<size_t>(w->K), static_cast<size_t>(w->N),
                               cudaMemcpyDeviceToHost),
                  "export weight") ||
      cuda_failed(cudaMemcpy(scale, w->scale, static_cast<size_t>(w->N) * 4,
                             cudaMemcpyDeviceToHost),
                  "export scale"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

// ------------------------------------------------------------- quantisers
int ovb_quantize(int64_t M, int64_t K, const float* A, int64_t lda, void* aq, float* asc,
                 int flags, void* stream) {
  if (M <= 0 || K <= 0) return OVB_OK;
  const int mode = quant_mode(flags);
  if (mode < 0) return invalid("OVB_AQ_U8, OVB_AQ_F16 and OVB_AQ_F16_RAW are exclusive");
  if (!A || !aq || (!asc && mode != 3)) return invalid("A/aq/asc must be non-null");
  if (lda < K) return invalid("lda < K");
  if (!aligned(aq, mode >= 2 ? 16 : 8) || !aligned(asc, 4) || !aligned(A, 4))
    return invalid("misaligned buffer");
  if (cuda_failed(ovb::launch_quantize(M, K, A, lda, aq, asc, mode, as_stream(stream)),
                  "quantize launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

int ovb_rmsnorm_quantize(int64_t rows, int64_t cols, const float* x, const float* w, float eps,
                         void* aq, float* asc, int flags, void* stream) {
  if (rows <= 0 || cols <= 0) return OVB_OK;
  const int mode = quant_mode(flags);
  if (mode < 0) return invalid("OVB_AQ_U8, OVB_AQ_F16 and OVB_AQ_F16_RAW are exclusive");
  if (!x || !w || !aq || (!asc && mode != 3)) return invalid("x/w/aq/asc must be non-null");
  if (cols > 24 * 1024) return invalid("rmsnorm_quantize: cols > 24576 not supported");
  if (!aligned(aq, mode >= 2 ? 16 : 8) || !aligned(asc, 4) || !aligned(x, 4) || !aligned(w, 4))
    return invalid("misaligned buffer");
  if (cuda_failed(ovb::launch_rmsnorm_quantize(rows, cols, x, w, eps, aq, asc, mode,
                                               as_stream(stream)),
                  "rmsnorm_quantize launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

int ovb_silu_mul_quantize(int64_t M, int64_t K, const float* gate, int64_t ldg,
                          const float* up, int64_t ldu, void* aq, float* asc, int flags,
                          void* stream) {
  if (M <= 0 || K <= 0) return OVB_OK;
  const int mode = quant_mode(flags);
  if (mode < 0) return invalid("OVB_AQ_U8, OVB_AQ_F16 and OVB_AQ_F16_RAW are exclusive");
  if (!gate || !up || !aq || (!asc && mode != 3)) return invalid("gate/up/aq/asc must be non-null");
  if (ldg < K || ldu < K) return invalid("ldg/ldu < K");
  if (!aligned(aq, mode >= 2 ? 16 : 8) || !aligned(asc, 4) || !aligned(gate, 4) ||
      !aligned(up, 4))
    return invalid("misaligned buffer");
  if (cuda_failed(ovb::launch_silu_mul_quantize(M, K, gate, ldg, up, ldu, aq, asc, mode,
                                                as_stream(stream)),
                  "silu_mul_quantize launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

// ------------------------------------------------------------------ GEMMs
int ovb_linear_q(int64_t M, const ovb_weight* w, const int8_t* aq, const float* asc, float* C,
                 int64_t ldc, int accumulate, void* stream) {
  if (M <= 0) return OVB_OK;
  int st = check_q_args(M, w, aq, asc);
  if (st != OVB_OK) return st;
  if (!C) return invalid("C is null");
  if (ldc < w->N) return invalid("ldc < N");
  const ovb::SliceOut so{0, w->N, C, ldc};
  return run_gemm(M, w, aq, asc, &so, 1, accumulate ? 1 : 0, nullptr, as_stream(stream));
}

int ovb_linear_q_sliced(int64_t M, const ovb_weight* w, const int8_t* aq, const float* asc,
                        const ovb_slice* slices, int n_slices, void* stream) {
  if (M <= 0 || n_slices <= 0) return OVB_OK;
  int st = check_q_args(M, w, aq, asc);
  if (st != OVB_OK) return st;
  ovb::SliceOut so[ovb::kMaxSlices];
  st = build_slices(w, slices, n_slices, so);
  if (st != OVB_OK) return st;
  return run_gemm(M, w, aq, asc, so, n_slices, 0, nullptr, as_stream(stream));
}

int ovb_linear_q_silu(int64_t M, const ovb_weight* w, const int8_t* aq, const float* asc,
                      void* out, float* out_asc, int flags, void* stream) {
  if (M <= 0) return OVB_OK;
  int st = check_q_args(M, w, aq, asc);
  if (st != OVB_OK) return st;
  int mode = 0;
  st = check_silu_out(w, out, out_asc, flags, &mode);
  if (st != OVB_OK) return st;
  const ovb::SliceOut so{0, w->N, nullptr, 0};
  const SiluOut silu{out, out_asc, mode};
  return run_gemm(M, w, aq, asc, &so, 1, 0, nullptr, as_stream(stream), &silu);
}

int ovb_linear_h_silu(int64_t M, const ovb_weight* w, const void* a16, void* out,
                      float* out_asc, int flags, void* stream) {
  if (M <= 0) return OVB_OK;
  int st = check_h_args(M, w, a16);
  if (st != OVB_OK) return st;
  int mode = 0;
  st = check_silu_out(w, out, out_asc, flags, &mode);
  if (st != OVB_OK) return st;
  const ovb::SliceOut so{0, w->N, nullptr, 0};
  const SiluOut silu{out, out_asc, mode};
  return run_gemm_h(M, w, a16, &so, 1, 0, as_stream(stream), &silu);
}

int ovb_linear_h(int64_t M, const ovb_weight* w, const void* a16, float* C, int64_t ldc,
                 int accumulate, void* stream) {
  if (M <= 0) return OVB_OK;
  int st = check_h_args(M, w, a16);
  if (st != OVB_OK) return st;
  if (!C) return invalid("C is null");
  if (ldc < w->N) return invalid("ldc < N");
  const ovb::SliceOut so{0, w->N, C, ldc};
  return run_gemm_h(M, w, a16, &so, 1, accumulate ? 1 : 0, as_stream(stream));
}

int ovb_linear_h_sliced(int64_t M, const ovb_weight* w, const void* a16, const ovb_slice* slices,
                        int n_slices, void* stream) {
  if (M <= 0 || n_slices <= 0) return OVB_OK;
  int st = check_h_args(M, w, a16);
  if (st != OVB_OK) return st;
  ovb::SliceOut so[ovb::kMaxSlices];
  st = build_slices(w, slices, n_slices, so);
  if (st != OVB_OK) return st;
  return run_gemm_h(M, w, a16, so, n_slices, 0, as_stream(stream));
}

int ovb_rope_table(const int64_t* pos, int64_t rows, int head_dim, float theta, float* table,
                   void* stream) {
  if (rows <= 0) return OVB_OK;
  if (head_dim != 128) return invalid("head_dim must be 128");
  if (!pos || !table) return invalid("pos/table must be non-null");
  if (!aligned(table, 16)) return invalid("table must be 16-byte aligned");
  if (!aligned(pos, 8)) return invalid("pos must be 8-byte aligned");
  if (rows > (int64_t{1} << 31) - 1) return invalid("rows exceeds 2^31-1");
  // inv_freq as qk_norm_rope_f32 computes it (ops_cpu.cpp:953-962)
  ovb::RopeFreq f;
  for (int i = 0; i < 64; ++i)
    f.inv_freq[i] = static_cast<float>(std::pow(static_cast<double>(theta), -2.0 * i / 128.0));
  if (cuda_failed(ovb::launch_rope_table(pos, f, rows, table, as_stream(stream)), "rope table launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

int ovb_qk_norm_rope_f16(int64_t rows, const float* q, const float* k, const float* v,
                         int n_heads, int n_kv, int head_dim, const float* q_norm,
                         const float* k_norm, float eps, const float* table, void* q16, void* k16,
                         void* v16, void* stream) {
  if (rows <= 0) return OVB_OK;
  int st = check_rope(n_heads, n_kv, head_dim, q_norm, k_norm, q16, k16, v16);
  if (st != OVB_OK) return st;
  if (!table) return invalid("table must be non-null");
  if (!aligned(table, 16)) return invalid("table must be 16-byte aligned");
  if (!q || !k || !v) return invalid("q/k/v must be non-null");
  if (rows > (int64_t{1} << 31) - 1) return invalid("rows exceeds 2^31-1");
  if (cuda_failed(ovb::launch_qk_norm_rope_f16(q, k, v, q16, k16, v16, q_norm, k_norm, table, rows,
                                               n_heads, n_kv, eps, as_stream(stream)),
                  "qk norm / rope launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

int ovb_linear_h_qk_rope(int64_t M, const ovb_weight* w, const void* a16, int n_heads, int n_kv,
                         int head_dim, const float* q_norm, const float* k_norm, float eps,
                         const float* table, void* q16, void* k16, void* v16, void* stream) {
  if (M <= 0) return OVB_OK;
  int st = check_h_args(M, w, a16);
  if (st != OVB_OK) return st;
  st = check_rope(n_heads, n_kv, head_dim, q_norm, k_norm, q16, k16, v16);
  if (st != OVB_OK) return st;
  if (!table) return invalid("table must be non-null");
  if (!aligned(table, 16)) return invalid("table must be 16-byte aligned");
  const int64_t qd = int64_t{n_heads} * 128, kvd = int64_t{n_kv} * 128;
  if (w->N != qd + 2 * kvd)
    return invalid("the weight's N must be (n_heads + 2 n_kv) * head_dim (a q|k|v weight)");
  const ovb::SliceOut so{0, w->N, nullptr, w->N};
  const RopeOut r{q16, k16, v16, q_norm, k_norm, table, qd, kvd, eps};
  return run_gemm_h(M, w, a16, &so, 1, 0, as_stream(stream), nullptr, &r);
}

size_t ovb_linear_workspace_bytes(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  const size_t qb = static_cast<size_t>(ovb_quant_bytes(M, K));
  return ((qb + 255) / 256) * 256 + static_cast<size_t>(ovb_quant_scales(M, K)) * 4;
}

int ovb_linear(int64_t M, const ovb_weight* w, const float* A, int64_t lda, float* C,
               int64_t ldc, int accumulate, void* work, size_t work_bytes, void* stream) {
  if (M <= 0) return OVB_OK;
  if (!w) return invalid("weight handle is null");
  if (!A || !C) return invalid("A/C must be non-null");
  if (!work || !aligned(work, 256)) return invalid("work must be non-null and 256-byte aligned");
  if (work_bytes < ovb_linear_workspace_bytes(M, w->K)) return invalid("work buffer too small");
  if (lda < w->K) return invalid("lda < K");
  if (ldc < w->N) return invalid("ldc < N");
  const size_t qb = static_cast<size_t>(ovb_quant_bytes(M, w->K));
  auto* aq = static_cast<int8_t*>(work);
  auto* asc = reinterpret_cast<float*>(static_cast<uint8_t*>(work) + ((qb + 255) / 256) * 256);
  int st = ovb_quantize(M, w->K, A, lda, aq, asc, 0, stream);
  if (st != OVB_OK) return st;
  return ovb_linear_q(M, w, aq, asc, C, ldc, accumulate, stream);
}

int ovb_block_products(int64_t M, const ovb_weight* w, const int8_t* aq, int32_t* P,
                       void* stream) {
  if (M <= 0) return OVB_OK;
  if (!w) return invalid("weight handle is null");
  if (!w->w) return invalid("weight has no int8 image (made by ovb_weight_create_f32)");
  if (!aq || !P) return invalid("aq/P must be non-null");
  if (!aligned(aq, 16)) return invalid("aq must be 16-byte aligned (TMA source)");
  const ovb::SliceOut so{0, w->N, nullptr, w->N};
  // asc is not read in this mode; pass a valid dummy pointer.
  return run_gemm(M, w, aq, reinterpret_cast<const float*>(aq), &so, 1, 0, P,
                  as_stream(stream));
}

int ovb_selftest_wait_timeout(void* stream) {
  if (cuda_failed(ovb::launch_wait_selftest(as_stream(stream)), "wait self-test launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

int ovb_guided_sample(const float* cond, int cond_seq, const float* uncond, int uncond_seq,
                      int codebooks, int vocab, int target_len, float guidance,
                      float layer_penalty, int mask_id, int32_t* pred, float* scores,
                      void* stream) {
  if (target_len <= 0 || codebooks <= 0) return OVB_OK;
  if (!cond || !uncond || !pred || !scores) return invalid("cond/uncond/pred/scores must be non-null");
  if (vocab <= 0) return invalid("vocab must be positive");
  if (cond_seq < target_len || uncond_seq < target_len)
    return invalid("cond_seq and uncond_seq must be >= target_len");
  if (!aligned(cond, 4) || !aligned(uncond, 4) || !aligned(pred, 4) || !aligned(scores, 4))
    return invalid("misaligned sampler buffer");
  if (static_cast<int64_t>(codebooks) * target_len > (int64_t{1} << 31) - 1)
    return invalid("codebooks * target_len exceeds 2^31-1");
  if (cuda_failed(ovb::launch_guided_sample(cond, cond_seq, uncond, codebooks, vocab, target_len,
                                            guidance, layer_penalty, mask_id, pred, scores,
                                            as_stream(stream)),
                  "guided sample launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

int ovb_guided_sample_batch(int n_pairs, const ovb_guided_pair* pairs, int codebooks, int vocab,
                            float guidance, float layer_penalty, int mask_id, int32_t* pred,
                            float* scores, void* stream) {
  if (n_pairs == 0) return OVB_OK;
  if (n_pairs < 0 || n_pairs > ovb::kMaxGuidedPairs) return invalid("n_pairs must be in [0, 64]");
  if (!pairs || !pred || !scores) return invalid("pairs/pred/scores must be non-null");
  if (codebooks <= 0 || vocab <= 0) return invalid("codebooks and vocab must be positive");
  if (!aligned(pred, 4) || !aligned(scores, 4)) return invalid("misaligned sampler buffer");
  ovb::GuidedBatch g = {};
  int64_t rows = 0;
  for (int p = 0; p < n_pairs; ++p) {
    const ovb_guided_pair& x = pairs[p];
    if (!x.cond || !x.uncond) return invalid("cond/uncond must be non-null");
    if (x.target_len < 0 || x.cond_seq < x.target_len || x.uncond_seq < x.target_len)
      return invalid("cond_seq and uncond_seq must be >= target_len >= 0");
    if (!aligned(x.cond, 4) || !aligned(x.uncond, 4)) return invalid("misaligned sampler buffer");
    g.cond[p] = x.cond;
    g.uncond[p] = x.uncond;
    g.cond_seq[p] = x.cond_seq;
    g.T[p] = x.target_len;
    g.out0[p] = rows;
    rows += static_cast<int64_t>(codebooks) * x.target_len;
    if (rows > (int64_t{1} << 31) - 1) return invalid("total output rows exceed 2^31-1");
  }
  g.out0[n_pairs] = rows;
  g.n = n_pairs;
  g.C = codebooks;
  g.mask_id = mask_id;
  g.guidance = guidance;
  g.penalty = layer_penalty;
  cudaStream_t s = as_stream(stream);
  if (vocab == 1025) {
    if (cuda_failed(ovb::launch_guided_sample_batch(g, pred, scores, s), "guided sample launch"))
      return OVB_ERR_INTERNAL;
    return OVB_OK;
  }
  for (int p = 0; p < n_pairs; ++p) {
    if (g.T[p] == 0) continue;
    if (cuda_failed(ovb::launch_guided_sample(g.cond[p], g.cond_seq[p], g.uncond[p], codebooks,
                                              vocab, g.T[p], guidance, layer_penalty, mask_id,
                                              pred + g.out0[p], scores + g.out0[p], s),
                    "guided sample launch"))
      return OVB_ERR_INTERNAL;
  }
  return OVB_OK;
}

int ovb_attention(const float* q, const float* k, const float* v, float* out, int64_t q_stride,
                  int64_t kv_stride, int n_heads, int n_kv, int head_dim, float scale,
                  const ovb_attn_segment* segs, int n_segs, void* stream) {
  if (n_segs == 0) return OVB_OK;
  if (n_segs < 0 || n_segs > ovb::kAttMaxSegs) return invalid("n_segs must be in [0, 64]");
  if (!segs || !q || !k || !v || !out) return invalid("q/k/v/out/segs must be non-null");
  if (head_dim != 128) return invalid("head_dim must be 128");
  if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0)
    return invalid("n_heads must be a positive multiple of n_kv");
  if (q_stride < int64_t{n_heads} * head_dim || kv_stride < int64_t{n_kv} * head_dim)
    return invalid("row strides must cover every head");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16) ||
      q_stride % 4 != 0 || kv_stride % 4 != 0)
    return invalid("q/k/v/out must be 16-byte aligned with strides a multiple of 4");
  if (q_stride > (int64_t{1} << 30) || kv_stride > (int64_t{1} << 30))
    return invalid("row strides too large");
  ovb::AttnArgs a = {};
  a.out = out;
  a.q_stride = q_stride;
  a.n_heads = n_heads;
  a.group = n_heads / n_kv;
  a.scale = scale;
  int64_t blocks = 0, q_rows = 1, kv_rows = 1;
  for (int i = 0; i < n_segs; ++i) {
    const ovb_attn_segment& g = segs[i];
    if (g.rows < 0 || g.q_off < 0 || g.kv_off < 0) return invalid("negative segment field");
    if (g.q_off % 4 != 0 || g.kv_off % 4 != 0)
      return invalid("segment offsets must be multiples of 4");
    if (g.rows == 0) continue;
    const int64_t qx = g.q_off % q_stride, qy = g.q_off / q_stride;
    const int64_t kx = g.kv_off % kv_stride, ky = g.kv_off / kv_stride;
    // every head of every row must lie within one row of the 2-D view
    if (qx + int64_t{n_heads} * head_dim > q_stride || kx + int64_t{n_kv} * head_dim > kv_stride)
      return invalid("segment offset leaves no room for every head within a row");
    if (qy + g.rows > (int64_t{1} << 31) - 1 - 128 || ky + g.rows > (int64_t{1} << 31) - 1 - 128)
      return invalid("segment rows too large");
    ovb::AttnSeg& d = a.segs[a.n_segs++];
    d.bias = g.bias;
    d.q_off = g.q_off;
    d.rows = g.rows;
    d.qblock0 = static_cast<int>(blocks);
    d.q_x = static_cast<int>(qx);
    d.q_y = static_cast<int>(qy);
    d.kv_x = static_cast<int>(kx);
    d.kv_y = static_cast<int>(ky);
    q_rows = std::max(q_rows, qy + g.rows);
    kv_rows = std::max(kv_rows, ky + g.rows);
    blocks += (g.rows + 127) / 128;
    if (blocks * n_heads > (int64_t{1} << 31) - 1) return invalid("too many query blocks");
  }
  if (blocks == 0) return OVB_OK;
  // fp32 views {row stride, rows} with a 128 x 128 box; rows past the last
  // segment read as zeros.
  if (!ovb::encode_tmap_2d(&a.tm_q, q, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, q_stride, q_rows,
                           q_stride * 4, 128, 128, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !ovb::encode_tmap_2d(&a.tm_k, k, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, kv_stride, kv_rows,
                           kv_stride * 4, 128, 128, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !ovb::encode_tmap_2d(&a.tm_v, v, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, kv_stride, kv_rows,
                           kv_stride * 4, 128, 128, CU_TENSOR_MAP_SWIZZLE_NONE))
    return OVB_ERR_INTERNAL;
  if (cuda_failed(ovb::launch_attention(a, static_cast<int>(blocks), as_stream(stream)),
                  "attention launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

// ------------------------------------------------- fp16-operand attention
namespace {
// Tile count of a segment list: per segment ceil(rows/128) query blocks x as
// many key tiles.
int64_t attn_tile_count(const int32_t* seg_rows, int n_segs) {
  int64_t t = 0;
  for (int i = 0; i < n_segs; ++i) {
    const int64_t b = (int64_t{seg_rows[i]} + 127) / 128;
    t += b * b;
  }
  return t;
}
size_t attn_class_bytes(int64_t tiles) { return static_cast<size_t>((tiles + 255) / 256 * 256); }
}  // namespace

size_t ovb_attention_tiles_bytes(const int32_t* seg_rows, int n_segs) {
  if (!seg_rows || n_segs <= 0) return 0;
  for (int i = 0; i < n_segs; ++i)
    if (seg_rows[i] < 0) return 0;
  const int64_t t = attn_tile_count(seg_rows, n_segs);
  return attn_class_bytes(t) + static_cast<size_t>(t) * 2048;
}

int ovb_attention_tiles(const int32_t* seg_rows, int n_segs, const uint8_t* masks, void* tiles,
                        size_t tiles_bytes, void* stream) {
  if (n_segs == 0) return OVB_OK;
  if (n_segs < 0 || n_segs > ovb::kAttMaxSegs) return invalid("n_segs must be in [0, 64]");
  if (!seg_rows || !masks || !tiles) return invalid("seg_rows/masks/tiles must be non-null");
  if (!aligned(tiles, 256)) return invalid("tiles must be 256-byte aligned");
  ovb::AttnTilesArgs a = {};
  a.masks = masks;
  a.n_segs = n_segs;
  int64_t t = 0, off = 0;
  for (int i = 0; i < n_segs; ++i) {
    if (seg_rows[i] < 0 || seg_rows[i] > 128 * 256) return invalid("segment rows must be in [0, 32768]");
    const int64_t b = (int64_t{seg_rows[i]} + 127) / 128;
    a.rows[i] = seg_rows[i];
    a.tile0[i] = static_cast<int>(t);
    a.mask_off[i] = off;
    t += b * b;
    off += int64_t{seg_rows[i]} * seg_rows[i];
  }
  if (tiles_bytes < ovb_attention_tiles_bytes(seg_rows, n_segs)) return invalid("tiles buffer too small");
  if (t == 0) return OVB_OK;
  if (t > (int64_t{1} << 30)) return invalid("too many tiles");
  auto* cls = static_cast<uint8_t*>(tiles);
  auto* bits = reinterpret_cast<uint32_t*>(cls + attn_class_bytes(t));
  if (cuda_failed(ovb::launch_attn_tiles(a, static_cast<int>(t), cls, bits, as_stream(stream)),
                  "attention tile table launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}

}  // extern "C"

namespace {
// ovb_attention_h and ovb_attention_h_q: `out` (fp32) or the quantised
// output (q_out / q_asc in form q_mode) is written.
int attention_h_impl(const void* q, const void* k, const void* v, float* out, int64_t q_stride,
                     int64_t kv_stride, int n_heads, int n_kv, int head_dim, float scale,
                     const ovb_attn_segment* segs, int n_segs, const void* tiles, void* q_out,
                     float* q_asc, int q_mode, void* stream) {
  if (n_segs == 0) return OVB_OK;
  if (n_segs < 0 || n_segs > ovb::kAttMaxSegs) return invalid("n_segs must be in [0, 64]");
  if (!segs || !q || !k || !v || (!out && !q_out)) return invalid("q/k/v/out/segs must be non-null");
  if (head_dim != 128) return invalid("head_dim must be 128");
  if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0)
    return invalid("n_heads must be a positive multiple of n_kv");
  if (q_stride < int64_t{n_heads} * head_dim || kv_stride < int64_t{n_kv} * head_dim)
    return invalid("row strides must cover every head");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16) ||
      q_stride % 8 != 0 || kv_stride % 8 != 0)
    return invalid("q/k/v/out must be 16-byte aligned with strides a multiple of 8");
  if (tiles && !aligned(tiles, 256)) return invalid("tiles must be 256-byte aligned");
  if (q_out) {
    if (!q_asc || !aligned(q_out, 16) || !aligned(q_asc, 4)) return invalid("misaligned aq/asc");
    if (q_stride != int64_t{n_heads} * head_dim)
      return invalid("the quantised output needs q_stride == n_heads * head_dim");
  }
  if (q_stride > (int64_t{1} << 30) || kv_stride > (int64_t{1} << 30))
    return invalid("row strides too large");
  ovb::AttnHArgs a = {};
  a.out = out;
  a.q_stride = q_stride;
  a.n_heads = n_heads;
  a.n_kv = n_kv;
  a.group = n_heads / n_kv;
  a.pairs = (a.group + 1) / 2;
  a.scale = scale;
  std::vector<int32_t> rows(static_cast<size_t>(n_segs));
  for (int i = 0; i < n_segs; ++i) rows[static_cast<size_t>(i)] = segs[i].rows;
  // Longer segments' CTAs first (they run longest), the table in segment order.
  std::vector<int> order(static_cast<size_t>(n_segs));
  for (int i = 0; i < n_segs; ++i) order[static_cast<size_t>(i)] = i;
  std::stable_sort(order.begin(), order.end(),
                   [&](int x, int y) { return segs[x].rows > segs[y].rows; });
  std::vector<int64_t> tile0(static_cast<size_t>(n_segs));
  int64_t t = 0;
  for (int i = 0; i < n_segs; ++i) {
    if (segs[i].rows < 0 || segs[i].rows > 128 * 256) return invalid("segment rows must be in [0, 32768]");
    tile0[static_cast<size_t>(i)] = t;
    const int64_t b = (int64_t{segs[i].rows} + 127) / 128;
    t += b * b;
  }
  int64_t ctas = 0, q_rows = 1, kv_rows = 1;
  for (int oi = 0; oi < n_segs; ++oi) {
    const ovb_attn_segment& g = segs[order[static_cast<size_t>(oi)]];
    if (g.q_off < 0 || g.kv_off < 0) return invalid("negative segment field");
    if (g.q_off % 8 != 0 || g.kv_off % 8 != 0)
      return invalid("segment offsets must be multiples of 8");
    if (g.rows == 0) continue;
    const int64_t qx = g.q_off % q_stride, qy = g.q_off / q_stride;
    const int64_t kx = g.kv_off % kv_stride, ky = g.kv_off / kv_stride;
    if (qx + int64_t{n_heads} * head_dim > q_stride || kx + int64_t{n_kv} * head_dim > kv_stride)
      return invalid("segment offset leaves no room for every head within a row");
    if (qy + g.rows > (int64_t{1} << 31) - 1 - 128 || ky + g.rows > (int64_t{1} << 31) - 1 - 128)
      return invalid("segment rows too large");
    if (q_out && qx != 0) return invalid("the quantised output needs row-aligned segment offsets");
    ovb::AttnHSeg& d = a.segs[a.n_segs++];
    d.bias = tiles ? nullptr : g.bias;
    d.q_off = g.q_off;
    d.rows = g.rows;
    d.cta0 = static_cast<int>(ctas);
    d.q_x = static_cast<int>(qx);
    d.q_y = static_cast<int>(qy);
    d.kv_x = static_cast<int>(kx);
    d.kv_y = static_cast<int>(ky);
    d.tile0 = static_cast<int>(tile0[static_cast<size_t>(order[static_cast<size_t>(oi)])]);
    q_rows = std::max(q_rows, qy + g.rows);
    kv_rows = std::max(kv_rows, ky + g.rows);
    ctas += (g.rows + 127) / 128 * n_kv * a.pairs;
    if (ctas > (int64_t{1} << 31) - 1) return invalid("too many query blocks");
  }
  if (ctas == 0) return OVB_OK;
  if (tiles) {
    a.tile_class = static_cast<const uint8_t*>(tiles);
    a.tile_bits = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(tiles) +
                                                    attn_class_bytes(t));
  }
  if (!ovb::encode_tmap_2d(&a.tm_q, q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, q_stride, q_rows,
                           q_stride * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !ovb::encode_tmap_2d(&a.tm_k, k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kv_stride, kv_rows,
                           kv_stride * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !ovb::encode_tmap_2d(&a.tm_v, v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kv_stride, kv_rows,
                           kv_stride * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return OVB_ERR_INTERNAL;
  if (q_out) {
    a.q_out = static_cast<uint8_t*>(q_out);
    a.q_asc = q_asc;
    a.q_mode = q_mode;
    a.q_kb = n_heads * head_dim / 32;
    a.out = nullptr;
  }
  if (cuda_failed(ovb::launch_attention_h(a, static_cast<int>(ctas), as_stream(stream)),
                  "attention_h launch"))
    return OVB_ERR_INTERNAL;
  return OVB_OK;
}
}  // namespace

extern "C" {

int ovb_attention_h(const void* q, const void* k, const void* v, float* out, int64_t q_stride,
                    int64_t kv_stride, int n_heads, int n_kv, int head_dim, float scale,
                    const ovb_attn_segment* segs, int n_segs, const void* tiles, void* stream) {
  if (n_segs > 0 && !out) return invalid("out must be non-null");
  return attention_h_impl(q, k, v, out, q_stride, kv_stride, n_heads, n_kv, head_dim, scale,
                          segs, n_segs, tiles, nullptr, nullptr, 0, stream);
}

int ovb_attention_h_q(const void* q, const void* k, const void* v, int64_t q_stride,
                      int64_t kv_stride, int n_heads, int n_kv, int head_dim, float scale,
                      const ovb_attn_segment* segs, int n_segs, const void* tiles, void* aq,
                      float* asc, int flags, void* stream) {
  const int mode = quant_mode(flags);
  if (mode < 0 || mode == 3) return invalid("flags: 0, OVB_AQ_U8 or OVB_AQ_F16");
  if (n_segs > 0 && (!aq || !asc)) return invalid("aq/asc must be non-null");
  return attention_h_impl(q, k, v, nullptr, q_stride, kv_stride, n_heads, n_kv, head_dim, scale,
                          segs, n_segs, tiles, aq, asc, mode, stream);
}

}  // extern "C"
