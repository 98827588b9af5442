// OpenThai forward on one GPU (Model::forward, src/models/openthai/model.rs:
// 192-241): embedding rows; per layer x += mixer(rms(x, n1, 1)) with the
// gated attention or the gated DeltaNet mixer, x += down(silu(gate h) * up h)
// with h = rms(x, n2, 1); the slot head (+ bias) on rms(x[positions], norm, 1).
//
// Built from the decoder path's pieces: the tcgen05 GEMM for every
// projection (F16 operands, F32 accumulation; the attention output, out_proj
// and down GEMMs add into the F32 residual; gate/up interleaved per 128 rows
// for the SwiGLU epilogue), the RMSNorm kernel with the offset-1 weights
// stored as 1 + w, and the two mixer kernels (gated_attn.cu, deltanet.cu).
// The model shape comes parsed from the file's `openthai.config` by the
// caller (the host's config checks); tensors are read from the GGUF here.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "engine.h"
#include "gemm.h"
#include "gguf.h"
#include "kernels.h"

namespace laya {

struct OtLayer {
  bool full = false;
  const float *n1 = nullptr, *n2 = nullptr;  // 1 + w
  const half *gu = nullptr, *down = nullptr;
  const half *q = nullptr, *o = nullptr;  // q: [q | gate] rows, then k, then v rows, stacked
  const float *qn = nullptr, *kn = nullptr;
  const half *qkv = nullptr, *out = nullptr;  // qkv: in_proj_qkv, z, a, b rows, stacked
  const float *conv = nullptr, *dt = nullptr, *alog = nullptr, *normw = nullptr;
};

}  // namespace laya

struct laya_ot_model {
  laya_ot_config cfg{};
  int device = 0, num_sms = 148;
  cudaStream_t st = nullptr;
  std::vector<laya::OtLayer> layers;
  laya::QTensor embd{};
  const float* norm = nullptr;  // 1 + w
  const half* head = nullptr;
  const float* head_bias = nullptr;
  unsigned* err = nullptr;
  std::vector<void*> allocs;
  // forward scratch, grown on demand and kept between passes
  laya::DevBuf dids, dpos, x, h, big, att, att16, act, logits, gscr, kpart;
  // several sequences per forward: each one's DeltaNet mixer runs on a side
  // stream, so the token-sequential recurrences of the sequences overlap
  static constexpr int kSide = 4;
  cudaStream_t side[kSide] = {};
  cudaEvent_t fork = nullptr, join[kSide] = {};
  std::mutex mu;
};

namespace laya {
namespace {

using Model = laya_ot_model;

int dalloc(Model& m, size_t bytes, void** p) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (OpenThai weights)");
  m.allocs.push_back(*p);
  return 0;
}

// Decodes a block-quantised tensor (Q8_0, Q4_0, Q4_K, Q6_K) into `dst`, a
// device buffer of t->count() floats, with the reference decoder's block
// arithmetic (gguf::decode, src/gguf.rs:250-336; the values are bit-identical).
int decode_on_device(const Gguf& g, const TensorInfo* t, const std::string& name, float* dst) {
  int block = 0, size = 0;
  if (!ggml_layout(t->kind, &block, &size) || t->count() % block)
    return fail(LAYA_E_FORMAT, name + ": unsupported tensor type for OpenThai");
  void* raw = nullptr;
  LAYA_CK(cudaMalloc(&raw, t->len ? t->len : 16));
  cudaError_t e = cudaMemcpy(raw, g.data(*t), t->len, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = dequant_raw((int)t->kind, static_cast<const uint8_t*>(raw), t->count() / block, dst, 0);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(raw);
  if (e != cudaSuccess) return cuda_fail(e, "OpenThai tensor decode");
  return 0;
}

// The tensor's elements as F32 on the host: F32 / F16 read directly, the
// block-quantised types decoded as the reference decodes them when it
// loads the model (g.floats, src/models/openthai/model.rs:61).
int host_f32(const Gguf& g, const std::string& name, size_t count, std::vector<float>* out) {
  const TensorInfo* t = g.tensor(name);
  if (!t) return fail(LAYA_E_FORMAT, "missing tensor " + name);
  if (t->count() != count) return fail(LAYA_E_FORMAT, name + ": unexpected shape");
  out->resize(count);
  const uint8_t* d = g.data(*t);
  if (t->kind == K_F32) {
    std::memcpy(out->data(), d, count * 4);
  } else if (t->kind == K_F16) {
    for (size_t i = 0; i < count; i++) (*out)[i] = half_bits((uint16_t)(d[2 * i] | (d[2 * i + 1] << 8)));
  } else {
    void* f = nullptr;
    LAYA_CK(cudaMalloc(&f, count * 4));
    int rc = decode_on_device(g, t, name, static_cast<float*>(f));
    cudaError_t e = rc ? cudaSuccess : cudaMemcpy(out->data(), f, count * 4, cudaMemcpyDeviceToHost);
    cudaFree(f);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail(e, "OpenThai tensor read-back");
  }
  return 0;
}

int upload_vec(Model& m, const Gguf& g, const std::string& name, size_t n, float offset, const float** out) {
  std::vector<float> v;
  if (int rc = host_f32(g, name, n, &v)) return rc;
  for (float& x : v) x = offset + x;
  void* p;
  if (int rc = dalloc(m, n * 4, &p)) return rc;
  LAYA_CK(cudaMemcpy(p, v.data(), n * 4, cudaMemcpyHostToDevice));
  *out = static_cast<const float*>(p);
  return 0;
}

// Matrix [rows][cols] as F16 (GGUF dims [cols, rows]).
int upload_mat(Model& m, const Gguf& g, const std::string& name, int rows, int cols, const half** out) {
  const TensorInfo* t = g.tensor(name);
  if (!t) return fail(LAYA_E_FORMAT, "missing tensor " + name);
  if (t->dims.size() != 2 || t->dims[0] != (uint64_t)cols || t->dims[1] != (uint64_t)rows)
    return fail(LAYA_E_FORMAT, name + ": unexpected matrix shape");
  std::vector<float> v;
  if (int rc = host_f32(g, name, (size_t)rows * cols, &v)) return rc;
  std::vector<half> h(v.size());
  for (size_t i = 0; i < v.size(); i++) h[i] = __float2half_rn(v[i]);
  void* p;
  if (int rc = dalloc(m, h.size() * 2, &p)) return rc;
  LAYA_CK(cudaMemcpy(p, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
  *out = static_cast<const half*>(p);
  return 0;
}

// Several matrices [rows_i][cols] stacked row-wise into one F16 operand, so
// the projections that read the same normed rows run as one GEMM.
int upload_stack(Model& m, const Gguf& g, const std::vector<std::pair<std::string, int>>& parts, int cols,
                 const half** out) {
  size_t total = 0;
  for (const auto& pr : parts) total += (size_t)pr.second * cols;
  std::vector<half> h(total);
  size_t at = 0;
  for (const auto& pr : parts) {
    const TensorInfo* t = g.tensor(pr.first);
    if (!t) return fail(LAYA_E_FORMAT, "missing tensor " + pr.first);
    if (t->dims.size() != 2 || t->dims[0] != (uint64_t)cols || t->dims[1] != (uint64_t)pr.second)
      return fail(LAYA_E_FORMAT, pr.first + ": unexpected matrix shape");
    std::vector<float> v;
    if (int rc = host_f32(g, pr.first, (size_t)pr.second * cols, &v)) return rc;
    for (size_t i = 0; i < v.size(); i++) h[at + i] = __float2half_rn(v[i]);
    at += v.size();
  }
  void* p;
  if (int rc = dalloc(m, h.size() * 2, &p)) return rc;
  LAYA_CK(cudaMemcpy(p, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
  *out = static_cast<const half*>(p);
  return 0;
}

// gate and up [ffn][d] interleaved per 128 rows into one [2 ffn][d] operand
int upload_gate_up(Model& m, const Gguf& g, const std::string& p, int ffn, int d, const half** out) {
  std::vector<float> gt, up;
  if (int rc = host_f32(g, p + ".mlp.gate_proj.weight", (size_t)ffn * d, &gt)) return rc;
  if (int rc = host_f32(g, p + ".mlp.up_proj.weight", (size_t)ffn * d, &up)) return rc;
  std::vector<half> h((size_t)2 * ffn * d);
  for (int r = 0; r < ffn; r++) {
    const size_t blk = r / 128, off = r % 128;
    for (int c = 0; c < d; c++) {
      h[((blk * 256) + off) * d + c] = __float2half_rn(gt[(size_t)r * d + c]);
      h[((blk * 256) + 128 + off) * d + c] = __float2half_rn(up[(size_t)r * d + c]);
    }
  }
  void* q;
  if (int rc = dalloc(m, h.size() * 2, &q)) return rc;
  LAYA_CK(cudaMemcpy(q, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
  *out = static_cast<const half*>(q);
  return 0;
}

int load(Model& m, const Gguf& g, const uint8_t* layer_full) {
  const laya_ot_config& c = m.cfg;
  const int d = c.d, H = c.heads, KV = c.kv_heads, hd = c.head_dim, nh = c.lin_heads, hk = c.lin_dim;
  const int w = nh * hk;
  const TensorInfo* e = g.tensor("model.embed_tokens.weight");
  if (!e || e->dims.size() != 2 || e->dims[0] != (uint64_t)d || e->dims[1] != (uint64_t)c.vocab)
    return fail(LAYA_E_FORMAT, "OpenThai embeddings must have shape [vocab, hidden]");
  void* pe;
  m.embd = QTensor{};
  if (e->kind == K_F32 || e->kind == K_F16) {
    if (int rc = dalloc(m, e->len, &pe)) return rc;
    LAYA_CK(cudaMemcpy(pe, g.data(*e), e->len, cudaMemcpyHostToDevice));
    m.embd.kind = (int)e->kind;
  } else {
    // a block-quantised table is decoded once to F32, the rows the reference gathers
    if (int rc = dalloc(m, (size_t)c.vocab * d * 4, &pe)) return rc;
    if (int rc = decode_on_device(g, e, "model.embed_tokens.weight", static_cast<float*>(pe))) return rc;
    m.embd.kind = K_F32;
  }
  m.embd.rows = c.vocab;
  m.embd.cols = d;
  m.embd.q = static_cast<const uint8_t*>(pe);
  m.layers.resize(c.n_layers);
  int rc;
  for (int l = 0; l < c.n_layers; l++) {
    OtLayer& L = m.layers[l];
    const std::string p = "model.layers." + std::to_string(l);
    L.full = layer_full[l] != 0;
    if ((rc = upload_vec(m, g, p + ".input_layernorm.weight", d, 1.f, &L.n1)) ||
        (rc = upload_vec(m, g, p + ".post_attention_layernorm.weight", d, 1.f, &L.n2)) ||
        (rc = upload_gate_up(m, g, p, c.ffn, d, &L.gu)) ||
        (rc = upload_mat(m, g, p + ".mlp.down_proj.weight", d, c.ffn, &L.down)))
      return rc;
    if (L.full) {
      // q | k | v stacked: one projection GEMM
      if ((rc = upload_stack(m, g, {{p + ".self_attn.q_proj.weight", 2 * H * hd}, {p + ".self_attn.k_proj.weight", KV * hd},
                                    {p + ".self_attn.v_proj.weight", KV * hd}}, d, &L.q)) ||
          (rc = upload_mat(m, g, p + ".self_attn.o_proj.weight", d, H * hd, &L.o)) ||
          (rc = upload_vec(m, g, p + ".self_attn.q_norm.weight", hd, 0.f, &L.qn)) ||
          (rc = upload_vec(m, g, p + ".self_attn.k_norm.weight", hd, 0.f, &L.kn)))
        return rc;
    } else {
      // qkv | z | a | b stacked: one projection GEMM
      if ((rc = upload_stack(m, g, {{p + ".linear_attn.in_proj_qkv.weight", 3 * w}, {p + ".linear_attn.in_proj_z.weight", w},
                                    {p + ".linear_attn.in_proj_a.weight", nh}, {p + ".linear_attn.in_proj_b.weight", nh}},
                             d, &L.qkv)) ||
          (rc = upload_mat(m, g, p + ".linear_attn.out_proj.weight", d, w, &L.out)) ||
          (rc = upload_vec(m, g, p + ".linear_attn.conv1d.weight", (size_t)3 * w * 4, 0.f, &L.conv)) ||
          (rc = upload_vec(m, g, p + ".linear_attn.dt_bias", nh, 0.f, &L.dt)) ||
          (rc = upload_vec(m, g, p + ".linear_attn.A_log", nh, 0.f, &L.alog)) ||
          (rc = upload_vec(m, g, p + ".linear_attn.norm.weight", hk, 0.f, &L.normw)))
        return rc;
    }
  }
  if ((rc = upload_vec(m, g, "model.norm.weight", d, 1.f, &m.norm)) ||
      (rc = upload_mat(m, g, "slot_head.weight", c.slots, d, &m.head)) ||
      (rc = upload_vec(m, g, "slot_head.bias", c.slots, 0.f, &m.head_bias)))
    return rc;
  void* pe2;
  if ((rc = dalloc(m, 16, &pe2))) return rc;
  m.err = static_cast<unsigned*>(pe2);
  LAYA_CK(cudaMemset(m.err, 0, 16));
  return 0;
}

// Prefill GEMMs launch with programmatic dependent launch unless
// LAYA_GEMM_PDL=0 (their first weight tiles come into L2 while the previous
// kernel drains).
bool gemm_pdl() {
  static const bool on = [] {
    const char* e = std::getenv("LAYA_GEMM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// ksplit > 1 (residual GEMMs only): partial sums into planes of `part`,
// merged by the RMSNorm that next reads the residual.
int gemm(Model& m, int epi, const half* A, int lda, const half* B, int N, int K, int M, void* out, int ldo,
         float* resid, const float* bias, int ksplit = 1, float* part = nullptr) {
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.out = out;
  a.ldo = ldo;
  a.resid = resid;
  a.bias = bias;
  a.ksplit = ksplit;
  a.part = part;
  a.err = m.err;
  a.budget = 4000000000ll;
  LAYA_CK(gemm_launch(epi, A, lda, B, K, a, m.num_sms, m.st, gemm_pdl()));
  return 0;
}

int check_shape(const laya_ot_config& c) {
  if (c.d < 32 || c.d % 32 || c.ffn < 128 || c.ffn % 128 || c.heads < 1 || c.kv_heads < 1 || c.heads % c.kv_heads ||
      (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256) || c.rot < 0 || c.rot > c.head_dim ||
      c.rot % 2 || c.lin_heads < 1 || (c.lin_dim != 64 && c.lin_dim != 128) || c.vocab < 1 || c.slots < 1 ||
      c.n_layers < 1 || c.n_layers > 256)
    return fail(LAYA_E_INVALID, "unsupported OpenThai shape for the GPU forward");
  return 0;
}

// The model on `device` from a parsed GGUF (the tensors are read from it
// during this call only).
int open_parsed(const Gguf& g, int device, const laya_ot_config& c, laya_ot_model** out) {
  auto m = std::make_unique<laya_ot_model>();
  m->cfg = c;
  m->cfg.layer_full = nullptr;  // read only here: the flags go into the layers
  m->device = device;
  LAYA_CK(cudaSetDevice(device));
  cudaDeviceProp prop;
  LAYA_CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return fail(LAYA_E_CUDA, "not an sm_100 GPU");
  m->num_sms = prop.multiProcessorCount;
  LAYA_CK(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking));
  if (int rc = load(*m, g, c.layer_full)) {
    laya_openthai_close(m.release());
    return rc;
  }
  *out = m.release();
  return 0;
}

}  // namespace
}  // namespace laya

namespace laya {
namespace {

// The forward of nseq sequences of lens[i] tokens, concatenated in ids;
// positions index the concatenated rows.  Every row-wise step (norms,
// projections, MLP, head) runs once over all rows; the sequence mixers run
// per sequence (causal within it).
int forward_seqs(laya_ot_model* m, const int32_t* ids, const int* lens, int nseq, const int32_t* positions, int npos,
                 float* out) {
  const laya_ot_config& c = m->cfg;
  int s = 0;
  for (int i = 0; i < nseq; i++) {
    if (lens[i] < 1) return fail(LAYA_E_INVALID, "invalid forward arguments");
    s += lens[i];
  }
  for (int i = 0; i < s; i++)
    if (ids[i] < 0 || ids[i] >= c.vocab) return fail(LAYA_E_INVALID, "invalid OpenThai token sequence");
  for (int i = 0; i < npos; i++)
    if (positions[i] < 0 || positions[i] >= s) return fail(LAYA_E_INVALID, "invalid OpenThai token sequence");
  LAYA_CK(cudaSetDevice(m->device));
  LAYA_CK(cudaMemsetAsync(m->err, 0, 4, m->st));
  const int d = c.d, H = c.heads, KV = c.kv_heads, hd = c.head_dim, nh = c.lin_heads, hk = c.lin_dim;
  const int w = nh * hk, qd = H * hd, ffn = c.ffn;
  const size_t S = (size_t)s;
  DevBuf &dids = m->dids, &dpos = m->dpos, &x = m->x, &h = m->h, &big = m->big,
         &att = m->att, &att16 = m->att16, &act = m->act, &logits = m->logits;
  // big: the stacked projection output of either layer kind, then each
  // sequence's DeltaNet mixer scratch (16-byte aligned)
  const int nfull = 2 * qd + 2 * KV * hd, ndelta = 4 * w + 2 * nh;
  const int ldd = (ndelta + 3) / 4 * 4;  // DeltaNet projection rows padded to 16 bytes (vector loads)
  const size_t pw = ((size_t)std::max(nfull, ldd) + 63) / 64 * 64;
  std::vector<size_t> scr_off(nseq);
  size_t scr_f = 0, gscr_b = 16;
  for (int i = 0; i < nseq; i++) {
    scr_off[i] = scr_f;
    scr_f += (gated_delta_mixer_scratch(lens[i], nh, hk) / 4 + 63) / 64 * 64;
    gscr_b = std::max(gscr_b, gated_attention_scratch(lens[i], H, KV, hd));
  }
  const size_t bigf = S * pw + scr_f + 64;
  int rc;
  if ((rc = dids.ensure(S * 4)) || (rc = dpos.ensure((size_t)npos * 4)) || (rc = x.ensure(S * d * 4)) ||
      (rc = h.ensure(std::max(S, (size_t)npos) * d * 2)) || (rc = big.ensure(bigf * 4)) ||
      (rc = att.ensure(S * std::max(qd, w) * 4)) ||
      (rc = att16.ensure(S * std::max(qd, w) * 2)) || (rc = act.ensure(S * ffn * 2)) ||
      (rc = logits.ensure((size_t)npos * c.slots * 4)) || (rc = m->gscr.ensure(gscr_b)))
    return rc;
  if (nseq > 1 && !m->fork) {
    LAYA_CK(cudaEventCreateWithFlags(&m->fork, cudaEventDisableTiming));
    for (int i = 0; i < laya_ot_model::kSide; i++) {
      LAYA_CK(cudaStreamCreateWithFlags(&m->side[i], cudaStreamNonBlocking));
      LAYA_CK(cudaEventCreateWithFlags(&m->join[i], cudaEventDisableTiming));
    }
  }
  // Residual GEMMs with few output tiles split K (as in the decoder forward);
  // the RMSNorm that next reads the residual adds the planes in split order.
  const char* ke = std::getenv("LAYA_KSPLIT");
  const bool ks_on = !(ke && ke[0] == '0');
  const int ks_full = ks_on ? gemm_ksplit(s, d, qd, m->num_sms) : 1;
  const int ks_delta = ks_on ? gemm_ksplit(s, d, w, m->num_sms) : 1;
  const int ks_down = ks_on ? gemm_ksplit(s, d, ffn, m->num_sms) : 1;
  const int ks_max = std::max(std::max(ks_full, ks_delta), ks_down);
  if (ks_max > 1 && (rc = m->kpart.ensure((size_t)ks_max * S * d * 4))) return rc;
  float* PART = ks_max > 1 ? m->kpart.as<float>() : nullptr;
  int pend = 0;  // K splits of X not yet merged
  auto norm = [&](const int* rows, int n, const float* wn) -> cudaError_t {
    const int ns = pend;
    pend = 0;
    if (ns > 1)
      return rmsnorm_merge(x.as<float>(), rows, n, PART, ns, S * d, wn, d, c.eps, h.as<half>(), nullptr, m->st,
                           gemm_pdl());
    return rmsnorm(x.as<float>(), rows, n, wn, d, c.eps, h.as<half>(), nullptr, m->st, gemm_pdl(), m->err);
  };
  cudaStream_t st = m->st;
  LAYA_CK(cudaMemcpyAsync(dids.p, ids, S * 4, cudaMemcpyHostToDevice, st));
  LAYA_CK(cudaMemcpyAsync(dpos.p, positions, (size_t)npos * 4, cudaMemcpyHostToDevice, st));
  float* X = x.as<float>();
  half* Hh = h.as<half>();
  float* P = big.as<float>();  // stacked projection outputs, rows of nfull / ndelta
  float* SCR = P + S * pw;     // DeltaNet mixer scratch, one region per sequence
  LAYA_CK(rows_f32(m->embd, dids.as<int>(), s, X, st));
  for (int l = 0; l < c.n_layers; l++) {
    const OtLayer& L = m->layers[l];
    LAYA_CK(norm(nullptr, s, L.n1));
    if (L.full) {
      // one GEMM: rows [q | gate per head] (2 qd), k (KV hd), v (KV hd)
      if ((rc = gemm(*m, EPI_F32, Hh, d, L.q, nfull, d, s, P, nfull, nullptr, nullptr))) return rc;
      for (int i = 0, r0 = 0; i < nseq; r0 += lens[i], i++) {
        const float* Pi = P + (size_t)r0 * nfull;
        LAYA_CK(gated_attention(Pi, nfull, Pi + 2 * qd, Pi + 2 * qd + KV * hd, nfull, L.qn, L.kn, lens[i], H, KV, hd,
                                c.rot, c.theta, m->gscr.p, att16.as<half>() + (size_t)r0 * qd, m->err, st));
      }
      if ((rc = gemm(*m, EPI_RESID, att16.as<half>(), qd, L.o, d, qd, s, nullptr, d, X, nullptr, ks_full, PART)))
        return rc;
      pend = ks_full;
    } else {
      // one GEMM: rows in_proj_qkv (3w), z (w), a (nh), b (nh)
      if ((rc = gemm(*m, EPI_F32, Hh, d, L.qkv, ndelta, d, s, P, ldd, nullptr, nullptr))) return rc;
      // the mixer writes its normalised, gated rows as F16 straight into
      // the output projection's operand; with several sequences each one's
      // mixer runs on a side stream (fork after the projection, join before
      // the output projection)
      if (nseq > 1) LAYA_CK(cudaEventRecord(m->fork, st));
      for (int i = 0, r0 = 0; i < nseq; r0 += lens[i], i++) {
        cudaStream_t ms = st;
        if (nseq > 1) {
          ms = m->side[i % laya_ot_model::kSide];
          LAYA_CK(cudaStreamWaitEvent(ms, m->fork, 0));
        }
        const float* Pi = P + (size_t)r0 * ldd;
        LAYA_CK(gated_delta_mixer(Pi, ldd, Pi + 3 * w, ldd, Pi + 4 * w, Pi + 4 * w + nh, ldd, L.conv, L.dt,
                                  L.alog, L.normw, lens[i], nh, hk, SCR + scr_off[i],
                                  att.as<float>() + (size_t)r0 * w, att16.as<half>() + (size_t)r0 * w, ms));
      }
      if (nseq > 1)
        for (int k = 0; k < std::min(nseq, laya_ot_model::kSide); k++) {
          LAYA_CK(cudaEventRecord(m->join[k], m->side[k]));
          LAYA_CK(cudaStreamWaitEvent(st, m->join[k], 0));
        }
      if ((rc = gemm(*m, EPI_RESID, att16.as<half>(), w, L.out, d, w, s, nullptr, d, X, nullptr, ks_delta, PART)))
        return rc;
      pend = ks_delta;
    }
    LAYA_CK(norm(nullptr, s, L.n2));
    if ((rc = gemm(*m, EPI_SWIGLU, Hh, d, L.gu, 2 * ffn, d, s, act.p, ffn, nullptr, nullptr)) ||
        (rc = gemm(*m, EPI_RESID, act.as<half>(), ffn, L.down, d, ffn, s, nullptr, d, X, nullptr, ks_down, PART)))
      return rc;
    pend = ks_down;
  }
  LAYA_CK(norm(dpos.as<int>(), npos, m->norm));
  if ((rc = gemm(*m, EPI_F32, Hh, d, m->head, c.slots, d, npos, logits.p, c.slots, nullptr, m->head_bias))) return rc;
  LAYA_CK(cudaMemcpyAsync(out, logits.p, (size_t)npos * c.slots * 4, cudaMemcpyDeviceToHost, st));
  LAYA_CK(cudaStreamSynchronize(st));
  unsigned err = 0;
  LAYA_CK(cudaMemcpy(&err, m->err, 4, cudaMemcpyDeviceToHost));
  if (err) return fail(LAYA_E_TIMEOUT, "a device-side wait ran out of its budget");
  for (size_t i = 0; i < (size_t)npos * c.slots; i++)
    if (!std::isfinite(out[i])) return fail(LAYA_E_NONFINITE, "non-finite model output");
  return 0;
}

}  // namespace
}  // namespace laya

using namespace laya;

extern "C" {

int laya_openthai_open(const char* path, int device, const laya_ot_config* cfg, laya_ot_model** out) {
  if (!path || !cfg || !out || !cfg->layer_full) return fail(LAYA_E_INVALID, "null argument");
  *out = nullptr;
  if (int rc = check_shape(*cfg)) return rc;
  Gguf g;
  std::string e = g.open_file(path);
  if (!e.empty()) return fail(g.bytes() ? LAYA_E_FORMAT : LAYA_E_IO, e);
  return open_parsed(g, device, *cfg, out);
}

int laya_openthai_open_memory(const uint8_t* gguf, size_t len, int device, const laya_ot_config* cfg,
                              laya_ot_model** out) {
  if (!gguf || !cfg || !out || !cfg->layer_full) return fail(LAYA_E_INVALID, "null argument");
  *out = nullptr;
  if (int rc = check_shape(*cfg)) return rc;
  Gguf g;
  std::string e = g.open_memory(gguf, len);
  if (!e.empty()) return fail(LAYA_E_FORMAT, e);
  return open_parsed(g, device, *cfg, out);
}

int laya_openthai_forward(laya_ot_model* m, const int32_t* ids, int s, const int32_t* positions, int npos,
                          float* out) {
  if (!m || !ids || !positions || !out || s < 1 || npos < 1) return fail(LAYA_E_INVALID, "invalid forward arguments");
  std::lock_guard<std::mutex> lk(m->mu);
  return forward_seqs(m, ids, &s, 1, positions, npos, out);
}

int laya_openthai_forward_batch(laya_ot_model* m, const int32_t* ids, const int32_t* lens, int nseq,
                                const int32_t* positions, int npos, float* out) {
  if (!m || !ids || !lens || !positions || !out || nseq < 1 || nseq > 256 || npos < 1)
    return fail(LAYA_E_INVALID, "invalid forward arguments");
  std::lock_guard<std::mutex> lk(m->mu);
  return forward_seqs(m, ids, lens, nseq, positions, npos, out);
}

void laya_openthai_close(laya_ot_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->st) cudaStreamSynchronize(m->st);
  for (void* p : m->allocs) cudaFree(p);
  for (DevBuf* b : {&m->dids, &m->dpos, &m->x, &m->h, &m->big, &m->att, &m->att16, &m->act, &m->logits,
                     &m->gscr, &m->kpart})
    b->release();
  for (int i = 0; i < laya_ot_model::kSide; i++) {
    if (m->side[i]) cudaStreamDestroy(m->side[i]);
    if (m->join[i]) cudaEventDestroy(m->join[i]);
  }
  if (m->fork) cudaEventDestroy(m->fork);
  if (m->st) cudaStreamDestroy(m->st);
  delete m;
}

}  // extern "C"
