// lm.cpp -- the whole LM forward on one device (ovb_lm_*): the reference's
// LM (cpp/src/model/lm.h:52-140, lm.cpp) with every step on the GPU, built
// from an OVW1 checkpoint, for the accelerator hook LM::CudaForwardFn
// (lm.h:91-96) and the ragged CFG forward (LM::forward_cfg, lm.cpp:403-454).
//
// Per layer (LM::run_layer, lm.cpp:217-322): RMSNorm + quantise -> q|k|v
// GEMM -> per-head RMSNorm + RoPE (written as fp16 q / k, with v as fp16; on
// the fp16 path fused into the q|k|v GEMM's epilogue, ovb_linear_h_qk_rope)
// -> attention over the segments with the o projection's quantiser in its
// epilogue (ovb_attention_h_q; the masks as a tile table and the RoPE
// angles as a table, both built once per forward)
// -> o GEMM += x -> RMSNorm + quantise -> gate|up GEMM fused with SiLU*up +
// quantise -> down GEMM += x.  Then the final RMSNorm + quantise and the
// audio-heads GEMM.  The linear weights are int8 (either OVW1 orientation)
// and run the bit-exact int8 mainloop, or the fp16 mainloop when the model is
// created with OVB_WEIGHT_F16.  Everything between the host copies of the
// inputs and of the logits is stream-ordered device work.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "ovb200.h"
#include "ovb_internal.h"

namespace {

struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  bool grow(size_t bytes) {
    if (bytes <= n) return true;
    cudaFree(p);
    p = nullptr;
    n = 0;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return false;
    n = bytes;
    return true;
  }
  ~DevBuf() { cudaFree(p); }
  template <class T>
  T* as() const { return static_cast<T*>(p); }
};

int fail(const std::string& msg) {
  ovb::set_error("ovb_lm: " + msg);
  return OVB_ERR_INVALID_ARG;
}

int internal(const std::string& msg) {
  ovb::set_error("ovb_lm: " + msg);
  return OVB_ERR_INTERNAL;
}

}  // namespace

struct ovb_lm {
  int device = 0;
  bool f16 = false;
  int n_layers = 0, hidden = 0, n_heads = 0, n_kv = 0, head_dim = 0, inter = 0;
  int64_t vocab = 0;
  int audio_vocab = 0, n_codebooks = 0;
  float eps = 1e-6f, theta = 1e6f;  // LMConfig defaults (lm.h:16-28)
  struct Layer {
    ovb_weight* qkv = nullptr;
    ovb_weight* o = nullptr;
    ovb_weight* gate_up = nullptr;
    ovb_weight* down = nullptr;
    const float* in_ln = nullptr;
    const float* post_ln = nullptr;
    const float* q_norm = nullptr;
    const float* k_norm = nullptr;
  };
  std::vector<Layer> layers;
  ovb_weight* heads = nullptr;
  bool heads_f32 = false;  // the reference's default fp32 audio heads (ovb_weight_create_f32)
  const float* final_norm = nullptr;
  DevBuf norms, emb, offsets;
  ovb::EmbTable tok{}, aud{};
  // forward buffers (grown on demand)
  DevBuf x, aq, asc, q, k, v, qi, asci, logits, logits_perm, ids, amask, pos, masks;
  DevBuf q16, k16, v16;  // fp16 q / k (normalised, rotated) and v: the attention's operands
  DevBuf rope;           // the RoPE table of the forward's positions (ovb_rope_table)
  DevBuf tiles;          // the attention's mask tile table (ovb_attention_tiles)
  DevBuf pred, scores;  // ovb_lm_sample's device outputs
  // pinned host staging of the logits for the host-buffer forwards: one
  // device-to-host copy at full link speed, then a host copy into the
  // caller's (pageable) array
  void* stage = nullptr;
  size_t stage_n = 0;
  int64_t last_rows = 0;

  ~ovb_lm() {
    if (stage) cudaFreeHost(stage);
    for (Layer& L : layers)
      for (ovb_weight* w : {L.qkv, L.o, L.gate_up, L.down})
        if (w) ovb_weight_destroy(w);
    if (heads) ovb_weight_destroy(heads);
  }
};

namespace {

// An fp32 vector tensor of `n` elements (norm weights).
int vec_f32(const ovb_ovw1* f, const std::string& name, int64_t n, const float** out) {
  ovb_ovw1_tensor t;
  if (ovb_ovw1_find(f, name.c_str(), &t) != OVB_OK) return OVB_ERR_INVALID_ARG;
  if (t.dtype != 0 || t.nbytes != n * 4) return fail(name + ": expected fp32 [" + std::to_string(n) + "]");
  *out = static_cast<const float*>(t.data);
  return OVB_OK;
}

// make_emb (mat.cpp:108-128): an int8 table with one scale per row, or fp32.
int emb_info(const ovb_ovw1* f, const char* name, int64_t cols, ovb_ovw1_tensor* t) {
  if (ovb_ovw1_find(f, name, t) != OVB_OK) return OVB_ERR_INVALID_ARG;
  if (t->ndim != 2 || t->dims[1] != cols) return fail(std::string(name) + ": expected [rows, hidden]");
  if (t->dtype == 1 && t->quant == 1 && t->scales && t->n_scales == t->dims[0]) return OVB_OK;
  if (t->dtype == 0) return OVB_OK;
  return fail(std::string(name) + ": expected an fp32 or row-scaled int8 table");
}

// Shape of a linear weight as make_linear reads it (mat.cpp:69-106): int8
// with per-output-channel scales in either orientation, or -- when
// `allow_f32` -- the fp32 encoding ([K, N], layout 1, or [N, K]).
int linear_nk(const ovb_ovw1* f, const std::string& name, int64_t* N, int64_t* K,
              bool allow_f32 = false, bool* is_f32 = nullptr) {
  ovb_ovw1_tensor t;
  if (ovb_ovw1_find(f, name.c_str(), &t) != OVB_OK) return OVB_ERR_INVALID_ARG;
  const bool f32 = t.ndim == 2 && t.dtype == 0 && t.quant == 0;
  if (is_f32) *is_f32 = f32;
  if (!(t.ndim == 2 && t.dtype == 1 && t.quant == 1) && !(allow_f32 && f32))
    return fail(name + (allow_f32 ? ": expected an int8 or fp32 linear weight"
                                   : ": expected an int8 linear weight"));
  *N = t.layout == 1 ? t.dims[1] : t.dims[0];
  *K = t.layout == 1 ? t.dims[0] : t.dims[1];
  return OVB_OK;
}

std::string lname(int i, const char* part) {
  return "llm.layers." + std::to_string(i) + "." + part;
}

int load(ovb_lm* m, const ovb_ovw1* f, cudaStream_t s) {
  // ---- shapes (LM::LM's checks, lm.cpp:96-141)
  while (true) {
    ovb_ovw1_tensor t;
    if (ovb_ovw1_find(f, lname(m->n_layers, "input_layernorm.weight").c_str(), &t) != OVB_OK) break;
    ++m->n_layers;
  }
  if (m->n_layers == 0) return fail("no llm.layers.0.input_layernorm.weight in the file");
  if (m->n_layers > 64) return fail("too many layers");
  ovb_ovw1_tensor t;
  int rc = ovb_ovw1_find(f, "llm.norm.weight", &t);
  if (rc != OVB_OK) return rc;
  m->hidden = static_cast<int>(t.dims[0]);
  rc = ovb_ovw1_find(f, lname(0, "self_attn.q_norm.weight").c_str(), &t);
  if (rc != OVB_OK) return rc;
  m->head_dim = static_cast<int>(t.dims[0]);
  if (m->head_dim != 128) return fail("head_dim must be 128");
  int64_t N = 0, K = 0;
  if ((rc = linear_nk(f, lname(0, "self_attn.q_proj.weight"), &N, &K)) != OVB_OK) return rc;
  m->n_heads = static_cast<int>(N / m->head_dim);
  if ((rc = linear_nk(f, lname(0, "self_attn.k_proj.weight"), &N, &K)) != OVB_OK) return rc;
  m->n_kv = static_cast<int>(N / m->head_dim);
  if ((rc = linear_nk(f, lname(0, "mlp.gate_proj.weight"), &N, &K)) != OVB_OK) return rc;
  m->inter = static_cast<int>(N);
  if (m->n_kv <= 0 || m->n_heads % m->n_kv != 0) return fail("n_heads must be a multiple of n_kv_heads");
  rc = ovb_ovw1_find(f, "codebook_layer_offsets", &t);
  if (rc != OVB_OK) return rc;
  if (t.dtype != 3 || t.ndim != 1) return fail("codebook_layer_offsets: expected int64 [C]");
  m->n_codebooks = static_cast<int>(t.dims[0]);
  const int64_t* offs = static_cast<const int64_t*>(t.data);
  ovb_ovw1_tensor tt, ta;
  if ((rc = emb_info(f, "llm.embed_tokens.weight", m->hidden, &tt)) != OVB_OK) return rc;
  if ((rc = emb_info(f, "audio_embeddings.weight", m->hidden, &ta)) != OVB_OK) return rc;
  m->vocab = tt.dims[0];
  if (ta.dims[0] % m->n_codebooks != 0) return fail("audio embedding rows mismatch");
  m->audio_vocab = static_cast<int>(ta.dims[0] / m->n_codebooks);
  if ((rc = linear_nk(f, "audio_heads.weight", &N, &K, true, &m->heads_f32)) != OVB_OK) return rc;
  if (N != static_cast<int64_t>(m->n_codebooks) * m->audio_vocab || K != m->hidden)
    return fail("audio head shape mismatch");
  const int64_t H = m->hidden, QD = int64_t(m->n_heads) * 128, KVD = int64_t(m->n_kv) * 128;
  for (int i = 0; i < m->n_layers; ++i) {
    struct { const char* n; int64_t N, K; } want[7] = {
        {"self_attn.q_proj.weight", QD, H}, {"self_attn.k_proj.weight", KVD, H},
        {"self_attn.v_proj.weight", KVD, H}, {"self_attn.o_proj.weight", H, QD},
        {"mlp.gate_proj.weight", m->inter, H}, {"mlp.up_proj.weight", m->inter, H},
        {"mlp.down_proj.weight", H, m->inter}};
    for (auto& w : want) {
      if ((rc = linear_nk(f, lname(i, w.n), &N, &K)) != OVB_OK) return rc;
      if (N != w.N || K != w.K)
        return fail("layer " + std::to_string(i) + ": projection shape mismatch");
    }
  }
  if (QD % 64 || KVD % 64 || m->inter % 64) return fail("projection widths must be multiples of 64");

  // ---- linear weights: q|k|v and gate|up parts in one batch (freed once
  // concatenated), o / down / heads in another.
  const int wflags = m->f16 ? OVB_WEIGHT_F16 : 0;
  const int L = m->n_layers;
  std::vector<std::string> na, nb;
  for (int i = 0; i < L; ++i)
    for (const char* p : {"self_attn.q_proj.weight", "self_attn.k_proj.weight",
                          "self_attn.v_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight"})
      na.push_back(lname(i, p));
  for (int i = 0; i < L; ++i)
    for (const char* p : {"self_attn.o_proj.weight", "mlp.down_proj.weight"}) nb.push_back(lname(i, p));
  if (!m->heads_f32) nb.push_back("audio_heads.weight");
  auto cstrs = [](const std::vector<std::string>& v) {
    std::vector<const char*> c;
    for (const auto& x : v) c.push_back(x.c_str());
    return c;
  };
  std::vector<ovb_weight*> wa(na.size(), nullptr), wb(nb.size(), nullptr);
  const auto ca = cstrs(na), cb = cstrs(nb);
  if ((rc = ovb_ovw1_weights(f, ca.data(), static_cast<int>(ca.size()), wflags, s, wa.data())) != OVB_OK)
    return rc;
  if ((rc = ovb_ovw1_weights(f, cb.data(), static_cast<int>(cb.size()), wflags, s, wb.data())) != OVB_OK) {
    for (ovb_weight* w : wa) ovb_weight_destroy(w);
    return rc;
  }
  m->layers.resize(static_cast<size_t>(L));
  for (int i = 0; i < L && rc == OVB_OK; ++i) {
    ovb_weight** p = &wa[static_cast<size_t>(i) * 5];
    ovb_lm::Layer& Ly = m->layers[static_cast<size_t>(i)];
    const ovb_weight* qkv[3] = {p[0], p[1], p[2]};
    rc = ovb_weight_concat(qkv, 3, s, &Ly.qkv);
    if (rc == OVB_OK) rc = ovb_weight_gate_up(p[3], p[4], s, &Ly.gate_up);
    Ly.o = wb[static_cast<size_t>(i) * 2];
    Ly.down = wb[static_cast<size_t>(i) * 2 + 1];
    wb[static_cast<size_t>(i) * 2] = wb[static_cast<size_t>(i) * 2 + 1] = nullptr;
  }
  if (!m->heads_f32) {
    m->heads = wb.back();
    wb.back() = nullptr;
  }
  for (ovb_weight* w : wa) ovb_weight_destroy(w);
  for (ovb_weight* w : wb)
    if (w) ovb_weight_destroy(w);
  if (rc != OVB_OK) return rc;
  if (m->heads_f32) {
    // The reference's default checkpoint keeps the audio heads in fp32
    // (tools/convert_weights.py:326-327), consumed by Mat::mul -> linear_f32
    // (lm.cpp:449-451, mat.cpp:11-13): fp16 tensor-core GEMM on fp16
    // activations (ovb_weight_create_f32, OVB_AQ_F16_RAW).
    ovb_ovw1_tensor th;
    if ((rc = ovb_ovw1_find(f, "audio_heads.weight", &th)) != OVB_OK) return rc;
    const bool kn = th.layout == 1;
    rc = ovb_weight_create_f32(static_cast<const float*>(th.data),
                               kn ? OVB_LAYOUT_KN : OVB_LAYOUT_NK, kn ? th.dims[1] : th.dims[0],
                               kn ? th.dims[0] : th.dims[1], s, &m->heads);
    if (rc != OVB_OK) return rc;
  }

  // ---- norms (fp32), one device buffer: per layer in / post (H), q / k (D); final (H)
  const int64_t per = 2 * H + 2 * 128;
  std::vector<float> hn(static_cast<size_t>(per * L + H));
  for (int i = 0; i < L; ++i) {
    const float* v[4];
    if ((rc = vec_f32(f, lname(i, "input_layernorm.weight"), H, &v[0])) != OVB_OK ||
        (rc = vec_f32(f, lname(i, "post_attention_layernorm.weight"), H, &v[1])) != OVB_OK ||
        (rc = vec_f32(f, lname(i, "self_attn.q_norm.weight"), 128, &v[2])) != OVB_OK ||
        (rc = vec_f32(f, lname(i, "self_attn.k_norm.weight"), 128, &v[3])) != OVB_OK)
      return rc;
    float* d = hn.data() + per * i;
    std::memcpy(d, v[0], H * 4);
    std::memcpy(d + H, v[1], H * 4);
    std::memcpy(d + 2 * H, v[2], 128 * 4);
    std::memcpy(d + 2 * H + 128, v[3], 128 * 4);
  }
  const float* fn = nullptr;
  if ((rc = vec_f32(f, "llm.norm.weight", H, &fn)) != OVB_OK) return rc;
  std::memcpy(hn.data() + per * L, fn, H * 4);
  if (!m->norms.grow(hn.size() * 4) ||
      cudaMemcpy(m->norms.p, hn.data(), hn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return internal("norm upload failed");
  const float* dn = m->norms.as<float>();
  for (int i = 0; i < L; ++i) {
    ovb_lm::Layer& Ly = m->layers[static_cast<size_t>(i)];
    Ly.in_ln = dn + per * i;
    Ly.post_ln = dn + per * i + H;
    Ly.q_norm = dn + per * i + 2 * H;
    Ly.k_norm = dn + per * i + 2 * H + 128;
  }
  m->final_norm = dn + per * L;

  // ---- embeddings as stored (int8 + row scales, or fp32)
  auto tab_bytes = [](const ovb_ovw1_tensor& x) {
    return static_cast<size_t>((x.nbytes + 255) / 256 * 256) +
           (x.dtype == 1 ? static_cast<size_t>((x.n_scales * 4 + 255) / 256 * 256) : 0);
  };
  if (!m->emb.grow(tab_bytes(tt) + tab_bytes(ta))) return internal("cudaMalloc(embeddings) failed");
  uint8_t* e = m->emb.as<uint8_t>();
  auto put = [&](const ovb_ovw1_tensor& x, ovb::EmbTable* out) {
    out->rows = x.dims[0];
    out->cols = x.dims[1];
    out->i8 = nullptr;
    out->scale = nullptr;
    out->f32 = nullptr;
    if (cudaMemcpy(e, x.data, static_cast<size_t>(x.nbytes), cudaMemcpyHostToDevice) != cudaSuccess)
      return false;
    if (x.dtype == 1) {
      out->i8 = reinterpret_cast<const int8_t*>(e);
      uint8_t* sc = e + (x.nbytes + 255) / 256 * 256;
      if (cudaMemcpy(sc, x.scales, static_cast<size_t>(x.n_scales) * 4, cudaMemcpyHostToDevice) !=
          cudaSuccess)
        return false;
      out->scale = reinterpret_cast<const float*>(sc);
    } else {
      out->f32 = reinterpret_cast<const float*>(e);
    }
    e += tab_bytes(x);
    return true;
  };
  if (!put(tt, &m->tok) || !put(ta, &m->aud)) return internal("embedding upload failed");
  if (!m->offsets.grow(static_cast<size_t>(m->n_codebooks) * 8) ||
      cudaMemcpy(m->offsets.p, offs, static_cast<size_t>(m->n_codebooks) * 8,
                 cudaMemcpyHostToDevice) != cudaSuccess)
    return internal("offset upload failed");
  return OVB_OK;
}

// Bytes of the mask tile table for any segment list of `rows` rows in total
// whose masks hold `mask_elems` entries (sum of rows_i^2): sum of
// ceil(r_i / 128)^2 <= mask_elems / 16384 + rows / 64 + n_segs (n_segs <= 64).
size_t tiles_bound(int64_t rows, int64_t mask_elems) {
  const int64_t t = mask_elems / 16384 + rows / 64 + 128;
  return static_cast<size_t>((t + 255) / 256 * 256 + t * 2048);
}

// Size every forward buffer for `rows` packed rows and `mask_elems` attention
// mask entries.
bool reserve(ovb_lm* m, int64_t rows, int64_t mask_elems) {
  const int64_t H = m->hidden, QD = int64_t(m->n_heads) * 128, KVD = int64_t(m->n_kv) * 128;
  const int64_t KM = std::max<int64_t>(std::max<int64_t>(H, QD), m->inter);
  const int64_t CV = int64_t(m->n_codebooks) * m->audio_vocab;
  const size_t ab = m->f16 ? 2 : 1;
  const size_t r = static_cast<size_t>(rows);
  // fp32 q / k / v only on the int8 path (the fp16 path's q|k|v GEMM writes
  // the fp16 operands directly)
  const bool qkv32 = !m->f16;
  return m->x.grow(r * H * 4) && m->aq.grow(r * std::max<int64_t>(KM * ab, H * 2)) &&
         m->asc.grow(r * (KM / 32) * 4) &&
         (!qkv32 || (m->q.grow(r * QD * 4) && m->k.grow(r * KVD * 4) && m->v.grow(r * KVD * 4))) &&
         m->rope.grow(r * 128 * 4) &&
         m->qi.grow(r * m->inter * ab) &&
         m->asci.grow(r * (m->inter / 32) * 4) && m->logits.grow(r * CV * 4) &&
         m->ids.grow(r * m->n_codebooks * 8) && m->amask.grow(r) && m->pos.grow(r * 8) &&
         m->masks.grow(static_cast<size_t>(mask_elems)) && m->q16.grow(r * QD * 2) &&
         m->k16.grow(r * KVD * 2) && m->v16.grow(r * KVD * 2) &&
         m->tiles.grow(tiles_bound(rows, mask_elems));
}

// The layers and heads on device buffers already holding ids / amask / pos
// and the attention's tile table: x <- embed; per layer; logits <- heads.
int run(ovb_lm* m, int64_t rows, int seq, const ovb_attn_segment* segs, int n_segs,
        const void* tiles, cudaStream_t s) {
  const int64_t H = m->hidden, QD = int64_t(m->n_heads) * 128, KVD = int64_t(m->n_kv) * 128;
  const int64_t CV = int64_t(m->n_codebooks) * m->audio_vocab;
  const int qf = m->f16 ? OVB_AQ_F16 : 0;
  float* x = m->x.as<float>();
  int8_t* aq = m->aq.as<int8_t>();
  float* asc = m->asc.as<float>();
  if (ovb::launch_embed(m->ids.as<int64_t>(), m->amask.as<uint8_t>(), m->offsets.as<int64_t>(),
                        m->n_codebooks, rows, seq, m->tok, m->aud, x, m->hidden, s) != cudaSuccess)
    return internal("embed launch failed");
  const float scale = 1.f / std::sqrt(static_cast<float>(m->head_dim));
  const float* rope = m->rope.as<float>();
  int rc = OVB_OK;
#define OVB_LM_TRY(call) \
  if ((rc = (call)) != OVB_OK) return rc
  OVB_LM_TRY(ovb_rope_table(m->pos.as<int64_t>(), rows, 128, m->theta, m->rope.as<float>(), s));
  for (const ovb_lm::Layer& L : m->layers) {
    OVB_LM_TRY(ovb_rmsnorm_quantize(rows, H, x, L.in_ln, m->eps, aq, asc, qf, s));
    if (m->f16) {
      OVB_LM_TRY(ovb_linear_h_qk_rope(rows, L.qkv, aq, m->n_heads, m->n_kv, 128, L.q_norm,
                                      L.k_norm, m->eps, rope, m->q16.p, m->k16.p, m->v16.p, s));
    } else {
      const ovb_slice sl[3] = {{QD, m->q.as<float>(), QD}, {KVD, m->k.as<float>(), KVD},
                               {KVD, m->v.as<float>(), KVD}};
      OVB_LM_TRY(ovb_linear_q_sliced(rows, L.qkv, aq, asc, sl, 3, s));
      OVB_LM_TRY(ovb_qk_norm_rope_f16(rows, m->q.as<float>(), m->k.as<float>(), m->v.as<float>(),
                                      m->n_heads, m->n_kv, 128, L.q_norm, L.k_norm, m->eps, rope,
                                      m->q16.p, m->k16.p, m->v16.p, s));
    }
    // attention with the o projection's quantiser in its epilogue
    OVB_LM_TRY(ovb_attention_h_q(m->q16.p, m->k16.p, m->v16.p, QD, KVD, m->n_heads, m->n_kv, 128,
                                 scale, segs, n_segs, tiles, aq, asc, qf, s));
    OVB_LM_TRY(m->f16 ? ovb_linear_h(rows, L.o, aq, x, H, 1, s)
                      : ovb_linear_q(rows, L.o, aq, asc, x, H, 1, s));
    OVB_LM_TRY(ovb_rmsnorm_quantize(rows, H, x, L.post_ln, m->eps, aq, asc, qf, s));
    OVB_LM_TRY(m->f16 ? ovb_linear_h_silu(rows, L.gate_up, aq, m->qi.p, m->asci.as<float>(), qf, s)
                      : ovb_linear_q_silu(rows, L.gate_up, aq, asc, m->qi.p, m->asci.as<float>(),
                                          qf, s));
    OVB_LM_TRY(m->f16 ? ovb_linear_h(rows, L.down, m->qi.p, x, H, 1, s)
                      : ovb_linear_q(rows, L.down, m->qi.as<int8_t>(), m->asci.as<float>(), x, H,
                                     1, s));
  }
  // final RMSNorm + the audio heads (rmsnorm_f32 + audio_heads_.mul, lm.cpp:446-447:
  // byte-identical to rmsnorm_quantize_f32 + linear_s8_nk_packed_q)
  if (m->heads_f32) {
    // rmsnorm_f32 + linear_f32 on fp32 heads: fp16 of the normalised rows
    // (not quantised) times the fp16 heads, fp32 accumulation.
    OVB_LM_TRY(ovb_rmsnorm_quantize(rows, H, x, m->final_norm, m->eps, aq, nullptr,
                                    OVB_AQ_F16_RAW, s));
    OVB_LM_TRY(ovb_linear_h(rows, m->heads, aq, m->logits.as<float>(), CV, 0, s));
  } else {
    OVB_LM_TRY(ovb_rmsnorm_quantize(rows, H, x, m->final_norm, m->eps, aq, asc, qf, s));
    OVB_LM_TRY(m->f16 ? ovb_linear_h(rows, m->heads, aq, m->logits.as<float>(), CV, 0, s)
                      : ovb_linear_q(rows, m->heads, aq, asc, m->logits.as<float>(), CV, 0, s));
  }
#undef OVB_LM_TRY
  m->last_rows = rows;
  return OVB_OK;
}

// The forward over packed segments whose u8 masks are in m->masks (in
// segment order): the attention's tile table from the masks, then run().
int run_segments(ovb_lm* m, const int32_t* seg_rows, int n_segs, int64_t rows, int seq,
                 cudaStream_t s) {
  const int64_t QD = int64_t(m->n_heads) * 128, KVD = int64_t(m->n_kv) * 128;
  int rc = ovb_attention_tiles(seg_rows, n_segs, m->masks.as<uint8_t>(), m->tiles.p, m->tiles.n, s);
  if (rc != OVB_OK) return rc;
  ovb_attn_segment segs[ovb::kAttMaxSegs];
  int64_t r0 = 0;
  for (int i = 0; i < n_segs; ++i) {
    segs[i] = {nullptr, seg_rows[i], r0 * QD, r0 * KVD};
    r0 += seg_rows[i];
  }
  return run(m, rows, seq, segs, n_segs, m->tiles.p, s);
}

}  // namespace

namespace {

// Sets the model's device for the duration of a call.
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Device logits -> the caller's host array through the pinned staging
// buffer (grown on demand), synchronising the stream.
int copy_logits_out(ovb_lm* m, const float* dev, size_t bytes, float* host, cudaStream_t s) {
  if (bytes > m->stage_n) {
    if (m->stage) cudaFreeHost(m->stage);
    m->stage = nullptr;
    m->stage_n = 0;
    if (cudaHostAlloc(&m->stage, bytes, cudaHostAllocDefault) != cudaSuccess)
      return internal("cudaHostAlloc(logits staging) failed");
    m->stage_n = bytes;
  }
  if (cudaMemcpyAsync(m->stage, dev, bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return internal("logits copy failed");
  std::memcpy(host, m->stage, bytes);
  return OVB_OK;
}

int finish(ovb_lm* m, cudaStream_t s) {
  (void)m;
  if (cudaStreamSynchronize(s) != cudaSuccess) return internal("forward failed on the device");
  const int st = ovb_device_status(s);
  if (st < 0) return st;
  if (st != 0) return internal("a bounded device check failed (status " + std::to_string(st) + ")");
  return OVB_OK;
}

}  // namespace

extern "C" {

int ovb_lm_create(const char* path, int flags, void* stream, ovb_lm** out) {
  if (!out) return fail("out is null");
  *out = nullptr;
  if ((flags & ~OVB_WEIGHT_F16) != 0) return fail("flags: only OVB_WEIGHT_F16 applies");
  ovb_ovw1* f = nullptr;
  int rc = ovb_ovw1_open(path, &f);
  if (rc != OVB_OK) return rc;
  auto* m = new ovb_lm();
  cudaGetDevice(&m->device);
  m->f16 = (flags & OVB_WEIGHT_F16) != 0;
  rc = load(m, f, static_cast<cudaStream_t>(stream));
  ovb_ovw1_close(f);
  if (rc != OVB_OK) {
    delete m;
    return rc;
  }
  *out = m;
  return OVB_OK;
}

int ovb_lm_destroy(ovb_lm* m) {
  if (!m) return OVB_OK;
  DeviceScope d(m->device);
  delete m;
  return OVB_OK;
}

int ovb_lm_config(const ovb_lm* m, int64_t* cfg) {
  if (!m || !cfg) return fail("model/cfg is null");
  const int64_t v[9] = {m->n_layers, m->hidden, m->n_heads, m->n_kv, m->head_dim,
                        m->inter, m->vocab, m->audio_vocab, m->n_codebooks};
  std::memcpy(cfg, v, sizeof v);
  return OVB_OK;
}

int ovb_lm_reserve(ovb_lm* m, int64_t rows, int64_t mask_elems) {
  if (!m) return fail("model is null");
  if (rows <= 0 || mask_elems < 0) return fail("rows must be positive");
  DeviceScope d(m->device);
  return reserve(m, rows, mask_elems) ? OVB_OK : internal("cudaMalloc(forward buffers) failed");
}

const float* ovb_lm_logits(const ovb_lm* m) { return m ? m->logits.as<float>() : nullptr; }

int ovb_lm_forward_cfg_device(ovb_lm* m, int cond_seq, int uncond_seq, const int64_t* ids,
                              const uint8_t* audio_mask, const uint8_t* cond_attn,
                              const uint8_t* uncond_attn, const int64_t* pos, void* stream) {
  if (!m) return fail("model is null");
  if (cond_seq <= 0 || uncond_seq <= 0) return fail("forward_cfg: both segments must be non-empty");
  if (!ids || !audio_mask || !cond_attn || !uncond_attn || !pos) return fail("null input");
  DeviceScope d(m->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t rows = int64_t(cond_seq) + uncond_seq;
  const int64_t cm = int64_t(cond_seq) * cond_seq, um = int64_t(uncond_seq) * uncond_seq;
  if (!reserve(m, rows, cm + um)) return internal("cudaMalloc(forward buffers) failed");
  const auto dd = cudaMemcpyDeviceToDevice;
  if (cudaMemcpyAsync(m->ids.p, ids, rows * m->n_codebooks * 8, dd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->amask.p, audio_mask, rows, dd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->pos.p, pos, rows * 8, dd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->masks.p, cond_attn, cm, dd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->masks.as<uint8_t>() + cm, uncond_attn, um, dd, s) != cudaSuccess)
    return internal("input copies failed");
  const int32_t seg_rows[2] = {cond_seq, uncond_seq};
  return run_segments(m, seg_rows, 2, rows, static_cast<int>(rows), s);
}

int ovb_lm_forward_segments_device(ovb_lm* m, int n_segs, const int32_t* seg_rows,
                                   const int64_t* ids, const uint8_t* audio_mask,
                                   const uint8_t* masks, const int64_t* pos, void* stream) {
  if (!m) return fail("model is null");
  if (n_segs <= 0) return OVB_OK;
  if (n_segs > ovb::kAttMaxSegs) return fail("at most 64 segments per forward");
  if (!seg_rows || !ids || !audio_mask || !masks || !pos) return fail("null input");
  int64_t rows = 0, mask_elems = 0;
  for (int i = 0; i < n_segs; ++i) {
    if (seg_rows[i] <= 0) return fail("every segment must have at least one row");
    rows += seg_rows[i];
    mask_elems += int64_t(seg_rows[i]) * seg_rows[i];
  }
  if (rows > (int64_t{1} << 30)) return fail("too many rows");
  DeviceScope d(m->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!reserve(m, rows, mask_elems)) return internal("cudaMalloc(forward buffers) failed");
  const auto dd = cudaMemcpyDeviceToDevice;
  if (cudaMemcpyAsync(m->ids.p, ids, rows * m->n_codebooks * 8, dd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->amask.p, audio_mask, rows, dd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->pos.p, pos, rows * 8, dd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->masks.p, masks, mask_elems, dd, s) != cudaSuccess)
    return internal("input copies failed");
  return run_segments(m, seg_rows, n_segs, rows, static_cast<int>(rows), s);
}

int ovb_lm_forward_cfg(ovb_lm* m, int cond_seq, int uncond_seq, const int64_t* ids,
                       const uint8_t* audio_mask, const uint8_t* cond_attn,
                       const uint8_t* uncond_attn, const int64_t* pos, float* logits,
                       void* stream) {
  if (!m) return fail("model is null");
  if (cond_seq <= 0 || uncond_seq <= 0) return fail("forward_cfg: both segments must be non-empty");
  if (!ids || !audio_mask || !cond_attn || !uncond_attn || !pos) return fail("null input");
  DeviceScope d(m->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t rows = int64_t(cond_seq) + uncond_seq;
  const int64_t cm = int64_t(cond_seq) * cond_seq, um = int64_t(uncond_seq) * uncond_seq;
  if (!reserve(m, rows, cm + um)) return internal("cudaMalloc(forward buffers) failed");
  const auto hd = cudaMemcpyHostToDevice;
  if (cudaMemcpyAsync(m->ids.p, ids, rows * m->n_codebooks * 8, hd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->amask.p, audio_mask, rows, hd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->pos.p, pos, rows * 8, hd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->masks.p, cond_attn, cm, hd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->masks.as<uint8_t>() + cm, uncond_attn, um, hd, s) != cudaSuccess)
    return internal("input copies failed");
  const int32_t seg_rows[2] = {cond_seq, uncond_seq};
  int rc = run_segments(m, seg_rows, 2, rows, static_cast<int>(rows), s);
  if (rc != OVB_OK) return rc;
  const int64_t CV = int64_t(m->n_codebooks) * m->audio_vocab;
  if (logits) {
    rc = copy_logits_out(m, m->logits.as<float>(), static_cast<size_t>(rows * CV * 4), logits, s);
    if (rc != OVB_OK) return rc;
  }
  return finish(m, s);
}

int ovb_lm_forward(ovb_lm* m, int batch, int seq, const int64_t* ids, const uint8_t* audio_mask,
                   const uint8_t* attn_mask, const int64_t* pos, float* logits, void* stream) {
  if (!m) return fail("model is null");
  if (batch <= 0 || seq <= 0) return OVB_OK;
  if (batch > 64) return fail("batch must be <= 64");
  if (!ids || !audio_mask || !attn_mask || !pos) return fail("null input");
  DeviceScope d(m->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t rows = int64_t(batch) * seq, mm = rows * seq;
  const int64_t CV = int64_t(m->n_codebooks) * m->audio_vocab;
  if (!reserve(m, rows, mm) || !m->logits_perm.grow(static_cast<size_t>(rows * CV * 4)))
    return internal("cudaMalloc(forward buffers) failed");
  const auto hd = cudaMemcpyHostToDevice;
  if (cudaMemcpyAsync(m->ids.p, ids, rows * m->n_codebooks * 8, hd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->amask.p, audio_mask, rows, hd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->pos.p, pos, rows * 8, hd, s) != cudaSuccess ||
      cudaMemcpyAsync(m->masks.p, attn_mask, mm, hd, s) != cudaSuccess)
    return internal("input copies failed");
  std::vector<int32_t> seg_rows(static_cast<size_t>(batch), seq);
  int rc = run_segments(m, seg_rows.data(), batch, rows, seq, s);
  if (rc != OVB_OK) return rc;
  if (logits) {
    if (ovb::launch_permute_logits(m->logits.as<float>(), m->logits_perm.as<float>(), batch, seq,
                                   m->n_codebooks, m->audio_vocab, s) != cudaSuccess)
      return internal("logits permute failed");
    rc = copy_logits_out(m, m->logits_perm.as<float>(), static_cast<size_t>(rows * CV * 4),
                         logits, s);
    if (rc != OVB_OK) return rc;
  }
  return finish(m, s);
}

int ovb_lm_sample(ovb_lm* m, const float* cond, int cond_seq, const float* uncond,
                  int uncond_seq, int target_len, float guidance, float layer_penalty,
                  int mask_id, int32_t* pred, float* scores, void* stream) {
  if (!m) return fail("model is null");
  if (target_len <= 0) return OVB_OK;
  if (!pred || !scores) return fail("pred/scores must be non-null");
  DeviceScope d(m->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t n = static_cast<size_t>(m->n_codebooks) * static_cast<size_t>(target_len);
  if (!m->pred.grow(n * 4) || !m->scores.grow(n * 4))
    return internal("cudaMalloc(sampler outputs) failed");
  int rc = ovb_guided_sample(cond, cond_seq, uncond, uncond_seq, m->n_codebooks, m->audio_vocab,
                             target_len, guidance, layer_penalty, mask_id, m->pred.as<int32_t>(),
                             m->scores.as<float>(), stream);
  if (rc != OVB_OK) return rc;
  if (cudaMemcpyAsync(pred, m->pred.p, n * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyAsync(scores, m->scores.p, n * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return internal("sampler output copy failed");
  return finish(m, s);
}

}  // extern "C"
