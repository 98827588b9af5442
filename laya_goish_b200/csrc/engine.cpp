// Host engine: model load, batched prefill + shared-prefix branch forward,
// heads and decision rules.  All device work of one replica runs on that
// replica's stream; the host plans each wave of requests, uploads the plan
// and enqueues the layer kernels.
#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "gemm.h"

namespace laya {

thread_local std::string g_err;
int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();
  return fail(e == cudaErrorMemoryAllocation ? LAYA_E_NOMEM : LAYA_E_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

const char* kProfNames[P_NCAT] = {"gemm_qkv",  "gemm_o",      "gemm_gate_up", "gemm_down",       "gemm_head",
                                  "attention", "dequant_f16", "gemv",         "attention_decode"};

static constexpr long long kWaitBudget = 4000000000ll;  // SM cycles (~2-3 s) per device-side wait

int DevBuf::ensure(size_t bytes) {
  if (bytes <= cap) return 0;
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
  size_t want = bytes + bytes / 8 + 256;
  cudaError_t e = cudaMalloc(&p, want);
  if (e != cudaSuccess) {
    p = nullptr;
    return cuda_fail(e, "cudaMalloc (scratch)");
  }
  cap = want;
  return 0;
}
void DevBuf::release() {
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
}
int HostBuf::ensure(size_t bytes) {
  if (bytes <= cap) return 0;
  if (p) cudaFreeHost(p);
  p = nullptr;
  cap = 0;
  size_t want = bytes + bytes / 4 + 4096;
  cudaError_t e = cudaMallocHost(&p, want);
  if (e != cudaSuccess) {
    p = nullptr;
    return cuda_fail(e, "cudaMallocHost");
  }
  cap = want;
  return 0;
}
void HostBuf::release() {
  if (p) cudaFreeHost(p);
  p = nullptr;
  cap = 0;
}

// ---------------------------------------------------------------- profiling

void prof_begin(Replica& r, int, cudaEvent_t* a) {
  *a = nullptr;
  if (!r.prof) return;
  if (r.event_pool.empty()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return;
    r.event_pool.push_back(e);
  }
  *a = r.event_pool.back();
  r.event_pool.pop_back();
  cudaEventRecord(*a, r.stream);
}
void prof_end(Replica& r, int cat, cudaEvent_t a) {
  if (!r.prof || !a) return;
  cudaEvent_t b;
  if (r.event_pool.empty()) {
    if (cudaEventCreate(&b) != cudaSuccess) return;
  } else {
    b = r.event_pool.back();
    r.event_pool.pop_back();
  }
  cudaEventRecord(b, r.stream);
  r.prof_events.push_back({cat, a, b});
}
void prof_collect(Replica& r) {
  for (auto& e : r.prof_events) {
    float ms = 0;
    if (cudaEventElapsedTime(&ms, e.a, e.b) == cudaSuccess) {
      auto& acc = r.prof_acc[kProfNames[e.cat]];
      acc.first += 1;
      acc.second += ms;
    }
    r.event_pool.push_back(e.a);
    r.event_pool.push_back(e.b);
  }
  r.prof_events.clear();
}

int timing_begin_call(Replica& r) {
  r.call_ms = 0;
  r.launches = r.h2d = r.d2h = 0;
  r.arm_start = false;
  if (!r.ev_start) LAYA_CK(cudaEventCreate(&r.ev_start));
  if (!r.ev_end) LAYA_CK(cudaEventCreate(&r.ev_end));
  return 0;
}
int timing_mark_start(Replica& r) {
  r.arm_start = false;
  LAYA_CK(cudaEventRecord(r.ev_start, r.stream));
  return 0;
}
// Records the end event, waits for it and adds the start..end device time.
int timing_mark_end(Replica& r) {
  LAYA_CK(cudaEventRecord(r.ev_end, r.stream));
  LAYA_CK(cudaEventSynchronize(r.ev_end));
  float ms = 0;
  LAYA_CK(cudaEventElapsedTime(&ms, r.ev_start, r.ev_end));
  r.call_ms += ms;
  return 0;
}

struct ProfScope {
  Replica& r;
  int cat;
  cudaEvent_t a;
  ProfScope(Replica& rr, int c) : r(rr), cat(c) { prof_begin(r, cat, &a); }
  ~ProfScope() { prof_end(r, cat, a); }
};

// ---------------------------------------------------------------- config

static void parse_temperature(const Gguf& g, Config* c) {
  // laya.temperature: JSON array [choice, score, noul];
  // laya.temperature_by_options: {"kind:bucket": t}
  // (src/models/laya/decision.rs:181-213)
  std::string t = g.str("laya.temperature");
  size_t p = t.find('[');
  for (int i = 0; p != std::string::npos && i < 3; i++) {
    const char* s = t.c_str() + p + 1;
    char* e;
    double v = std::strtod(s, &e);
    if (e == s) break;
    c->temperature[i] = (float)v;
    p = t.find(',', e - t.c_str());
  }
  std::string b = g.str("laya.temperature_by_options");
  static const char* kinds[3] = {"choice", "score", "noul"};
  static const char* buckets[4] = {"2", "3-5", "6-10", "11+"};
  for (int k = 0; k < 3; k++)
    for (int j = 0; j < 4; j++) {
      std::string key = std::string("\"") + kinds[k] + ":" + buckets[j] + "\"";
      size_t q = b.find(key);
      if (q == std::string::npos) continue;
      q = b.find(':', q + key.size());
      if (q == std::string::npos) continue;
      c->bucket[k][j] = (float)std::strtod(b.c_str() + q + 1, nullptr);
      c->has_bucket[k][j] = true;
    }
}

std::string read_config(const Gguf& g, Config* c) {
  c->arch = g.str("general.architecture");
  if (c->arch != "llama" && c->arch != "qwen2") return "unsupported GGUF architecture " + c->arch;
  auto k = [&](const char* s) { return c->arch + "." + s; };
  c->L = (int)g.num(k("block_count"), 0);
  c->d = (int)g.num(k("embedding_length"), 0);
  c->H = (int)g.num(k("attention.head_count"), 0);
  c->KV = (int)g.num(k("attention.head_count_kv"), c->H);
  c->ffn = (int)g.num(k("feed_forward_length"), 0);
  c->eps = (float)g.num(k("attention.layer_norm_rms_epsilon"), 1e-5);
  c->theta = (float)g.num(k("rope.freq_base"), 10000.0);
  c->ctx = (int)g.num(k("context_length"), 4096);
  if (c->L < 1 || c->d < 1 || c->H < 1 || c->KV < 1 || c->H % c->KV || c->d % c->H || c->ffn < 1)
    return "invalid decoder hyperparameters";
  c->hd = c->d / c->H;
  if (c->hd != 64 && c->hd != 128) return "head_dim must be 64 or 128";
  if (c->d % 32 || c->ffn % 128) return "embedding_length must be a multiple of 32 and feed_forward_length of 128";
  if (c->ctx < 1 || c->ctx > (1 << 20)) return "invalid context_length";
  const TensorInfo* e = g.tensor("token_embd.weight");
  if (!e || e->dims.size() != 2 || e->dims[0] != (uint64_t)c->d) return "missing or malformed token_embd.weight";
  c->V = (int)e->dims[1];
  const TensorInfo* o = g.tensor("output.weight");
  if (!o || o->dims.size() != 2 || o->dims[0] != (uint64_t)c->d || o->dims[1] != (uint64_t)c->V)
    return "missing or malformed output.weight (untied lm_head)";
  const TensorInfo* q = g.tensor("blk.0.attn_q.weight");
  if (!q) return "missing tensor blk.0.attn_q.weight";
  c->wkind = (int)q->kind;
  c->bias = g.tensor("blk.0.attn_q.bias") != nullptr;
  c->quantized = false;
  for (int l = 0; l < c->L; l++)
    for (const char* t : {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"}) {
      const TensorInfo* ti = g.tensor("blk." + std::to_string(l) + "." + t + ".weight");
      if (ti && ti->kind != K_F16 && ti->kind != K_F32) c->quantized = true;
    }
  parse_temperature(g, c);
  return "";
}

// ---------------------------------------------------------------- load

static int dmalloc(Replica& r, size_t bytes, void** p) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (weights)");
  r.allocs.push_back(*p);
  if (r.loading) r.wmap.emplace_back(*p, bytes ? bytes : 16);
  r.weight_bytes += bytes;
  return 0;
}

// Host -> device weight copy.  The source is mostly the mmap'd GGUF file;
// the driver's pageable copy pins and streams it (a pinned staging ring
// filled by host threads measured no faster: the page faults on the mapping
// bound both).
static cudaError_t h2d(void* dst, const void* src, size_t n) {
  return cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice);
}

static int upload(Replica& r, const void* src, size_t bytes, void** p) {
  if (int rc = dmalloc(r, bytes, p)) return rc;
  LAYA_CK(h2d(*p, src, bytes));
  return 0;
}

static void f32_to_f16_host(const float* x, size_t n, uint16_t* y) {
  for (size_t i = 0; i < n; i++) {
    __half h = __float2half_rn(x[i]);
    std::memcpy(&y[i], &h, 2);
  }
}

static const TensorInfo* matrix_info(const Gguf& g, const std::string& name, int rows, int cols, int* rc) {
  const TensorInfo* t = g.tensor(name);
  if (!t) {
    *rc = fail(LAYA_E_FORMAT, "missing tensor " + name);
    return nullptr;
  }
  if (t->dims.size() != 2 || t->dims[0] != (uint64_t)cols || t->dims[1] != (uint64_t)rows) {
    *rc = fail(LAYA_E_FORMAT, name + ": unexpected matrix shape");
    return nullptr;
  }
  return t;
}

// Uploads one matrix in its HBM layout (see QTensor), transcoding GGUF blocks
// into structure-of-arrays streams where the block size is not 16-byte aligned.
static int upload_matrix(Replica& r, const Gguf& g, const std::string& name, int rows, int cols, QTensor* out) {
  int rc = 0;
  const TensorInfo* t = matrix_info(g, name, rows, cols, &rc);
  if (!t) return rc;
  const uint8_t* src = g.data(*t);
  const size_t n = (size_t)rows * cols;
  QTensor q{};
  q.kind = (int)t->kind;
  q.rows = rows;
  q.cols = cols;
  void* p = nullptr;
  switch (t->kind) {
    case K_F32:
    case K_F16:
    case K_Q4_K:
      if ((rc = upload(r, src, t->len, &p))) return rc;
      q.q = static_cast<const uint8_t*>(p);
      break;
    case K_Q8_0:
    case K_Q4_0: {
      const int bs = t->kind == K_Q8_0 ? 34 : 18, qb = t->kind == K_Q8_0 ? 32 : 16;
      const size_t nb = n / 32;
      std::vector<uint8_t> qs(nb * qb);
      std::vector<uint16_t> d(nb);
      for (size_t i = 0; i < nb; i++) {
        const uint8_t* c = src + i * bs;
        d[i] = (uint16_t)(c[0] | (c[1] << 8));
        std::memcpy(&qs[i * qb], c + 2, qb);
      }
      void* pq;
      void* pd;
      if ((rc = upload(r, qs.data(), qs.size(), &pq)) || (rc = upload(r, d.data(), d.size() * 2, &pd))) return rc;
      q.q = static_cast<const uint8_t*>(pq);
      q.s = static_cast<const uint16_t*>(pd);
    } break;
    case K_Q6_K: {
      const size_t nb = n / 256;
      std::vector<uint8_t> ql(nb * 128), qh(nb * 64), sc(nb * 16);
      std::vector<uint16_t> d(nb);
      for (size_t i = 0; i < nb; i++) {
        const uint8_t* c = src + i * 210;
        std::memcpy(&ql[i * 128], c, 128);
        std::memcpy(&qh[i * 64], c + 128, 64);
        std::memcpy(&sc[i * 16], c + 192, 16);
        d[i] = (uint16_t)(c[208] | (c[209] << 8));
      }
      void *a, *b, *cc, *dd;
      if ((rc = upload(r, ql.data(), ql.size(), &a)) || (rc = upload(r, qh.data(), qh.size(), &b)) ||
          (rc = upload(r, sc.data(), sc.size(), &cc)) || (rc = upload(r, d.data(), d.size() * 2, &dd)))
        return rc;
      q.q = static_cast<const uint8_t*>(a);
      q.qh = static_cast<const uint8_t*>(b);
      q.sc = static_cast<const int8_t*>(cc);
      q.s = static_cast<const uint16_t*>(dd);
    } break;
    default:
      return fail(LAYA_E_FORMAT, name + ": unsupported tensor type");
  }
  *out = q;
  r.named[name] = q;
  return 0;
}

// Copies an F16/F32 matrix into rows of a resident F16 operand:
// destination row of source row n = (n / grp) * gstride + goff + n % grp.
static int place_f16(const Gguf& g, const std::string& name, int rows, int cols, half* dst, int grp, int gstride,
                     int goff) {
  int rc = 0;
  const TensorInfo* t = matrix_info(g, name, rows, cols, &rc);
  if (!t) return rc;
  std::vector<uint16_t> conv;
  const uint16_t* src;
  if (t->kind == K_F16) {
    src = reinterpret_cast<const uint16_t*>(g.data(*t));
  } else if (t->kind == K_F32) {
    conv.resize((size_t)rows * cols);
    std::vector<float> tmp((size_t)rows * cols);
    std::memcpy(tmp.data(), g.data(*t), tmp.size() * 4);
    f32_to_f16_host(tmp.data(), tmp.size(), conv.data());
    src = conv.data();
  } else {
    return fail(LAYA_E_FORMAT, name + ": expected F16/F32");
  }
  const size_t row_bytes = (size_t)cols * 2;
  const int nblk = (rows + grp - 1) / grp;
  for (int bidx = 0; bidx < nblk; bidx++) {
    const int r0 = bidx * grp, cnt = std::min(grp, rows - r0);
    LAYA_CK(h2d(dst + ((size_t)bidx * gstride + goff) * cols, src + (size_t)r0 * cols, row_bytes * cnt));
  }
  return 0;
}

static int upload_vector(Replica& r, const Gguf& g, const std::string& name, int n, const float** out,
                         bool required = true) {
  const TensorInfo* t = g.tensor(name);
  if (!t) {
    if (!required) return 0;
    return fail(LAYA_E_FORMAT, "missing tensor " + name);
  }
  if (t->count() != (uint64_t)n) return fail(LAYA_E_FORMAT, name + ": unexpected vector shape");
  std::vector<float> v(n);
  if (t->kind == K_F32)
    std::memcpy(v.data(), g.data(*t), (size_t)n * 4);
  else if (t->kind == K_F16)
    for (int i = 0; i < n; i++) v[i] = half_bits(g.data(*t)[2 * i] | (g.data(*t)[2 * i + 1] << 8));
  else
    return fail(LAYA_E_FORMAT, name + ": norm/bias tensors must be F32 or F16");
  void* p;
  if (int rc = upload(r, v.data(), (size_t)n * 4, &p)) return rc;
  *out = static_cast<const float*>(p);
  return 0;
}

static int init_device(int device, Replica& r) {
  r.device = device;
  LAYA_CK(cudaSetDevice(device));
  cudaDeviceProp prop;
  LAYA_CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return fail(LAYA_E_CUDA, std::string("device ") + prop.name + " is not an sm_100 GPU");
  r.num_sms = prop.multiProcessorCount;
  LAYA_CK(cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking));
  return 0;
}

static int load_weights(Model& m, const Gguf& g, Replica& r);

int load_replica(Model& m, const Gguf& g, int device, Replica& r) {
  if (int rc = init_device(device, r)) return rc;
  r.loading = true;
  const int rc = load_weights(m, g, r);
  r.loading = false;
  if (rc) return rc;
  LAYA_CK(cudaMemsetAsync(r.err, 0, 16, r.stream));
  LAYA_CK(cudaStreamSynchronize(r.stream));
  return 0;
}

static int load_weights(Model& m, const Gguf& g, Replica& r) {
  const Config& c = m.cfg;
  const int qd = c.H * c.hd, kd = c.KV * c.hd, d = c.d;
  int rc;
  r.layers.resize(c.L);
  for (int l = 0; l < c.L; l++) {
    Layer& L = r.layers[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    if ((rc = upload_vector(r, g, p + "attn_norm.weight", d, &L.attn_norm)) ||
        (rc = upload_vector(r, g, p + "ffn_norm.weight", d, &L.ffn_norm)))
      return rc;
    if (c.bias) {
      std::vector<float> b(qd + 2 * kd, 0.f);
      const char* names[3] = {"attn_q.bias", "attn_k.bias", "attn_v.bias"};
      const int off[3] = {0, qd, qd + kd}, len[3] = {qd, kd, kd};
      for (int i = 0; i < 3; i++) {
        const TensorInfo* t = g.tensor(p + names[i]);
        if (!t) continue;
        if (t->count() != (uint64_t)len[i] || (t->kind != K_F32 && t->kind != K_F16))
          return fail(LAYA_E_FORMAT, p + names[i] + ": unexpected bias");
        for (int j = 0; j < len[i]; j++)
          b[off[i] + j] = t->kind == K_F32 ? reinterpret_cast<const float*>(g.data(*t))[j]
                                           : half_bits(g.data(*t)[2 * j] | (g.data(*t)[2 * j + 1] << 8));
      }
      void* bp;
      if ((rc = upload(r, b.data(), b.size() * 4, &bp))) return rc;
      L.bqkv = static_cast<const float*>(bp);
    }
    if (!c.quantized) {
      // Resident F16 operands: q|k|v stacked, gate/up interleaved per 128 rows.
      void *pqkv, *pgu, *po, *pd;
      if ((rc = dmalloc(r, (size_t)(qd + 2 * kd) * d * 2, &pqkv)) || (rc = dmalloc(r, (size_t)2 * c.ffn * d * 2, &pgu)) ||
          (rc = dmalloc(r, (size_t)d * qd * 2, &po)) || (rc = dmalloc(r, (size_t)d * c.ffn * 2, &pd)))
        return rc;
      half* qkv = static_cast<half*>(pqkv);
      half* gu = static_cast<half*>(pgu);
      const int big = 1 << 30;
      if ((rc = place_f16(g, p + "attn_q.weight", qd, d, qkv, big, 0, 0)) ||
          (rc = place_f16(g, p + "attn_k.weight", kd, d, qkv, big, 0, qd)) ||
          (rc = place_f16(g, p + "attn_v.weight", kd, d, qkv, big, 0, qd + kd)) ||
          (rc = place_f16(g, p + "ffn_gate.weight", c.ffn, d, gu, 128, 256, 0)) ||
          (rc = place_f16(g, p + "ffn_up.weight", c.ffn, d, gu, 128, 256, 128)) ||
          (rc = place_f16(g, p + "attn_output.weight", d, qd, static_cast<half*>(po), big, 0, 0)) ||
          (rc = place_f16(g, p + "ffn_down.weight", d, c.ffn, static_cast<half*>(pd), big, 0, 0)))
        return rc;
      L.wqkv16 = qkv;
      L.wgu16 = gu;
      L.wo16 = static_cast<half*>(po);
      L.wd16 = static_cast<half*>(pd);
      auto view = [&](const half* base, int rows, int cols) {
        QTensor q{};
        q.kind = K_F16;
        q.rows = rows;
        q.cols = cols;
        q.q = reinterpret_cast<const uint8_t*>(base);
        return q;
      };
      L.wq = view(qkv, qd, d);
      L.wk = view(qkv + (size_t)qd * d, kd, d);
      L.wv = view(qkv + (size_t)(qd + kd) * d, kd, d);
      L.wo = view(L.wo16, d, qd);
      L.wd = view(L.wd16, d, c.ffn);
      L.wg = view(gu, 2 * c.ffn, d);  // interleaved gate/up operand
      L.wu = QTensor{};
      r.named[p + "attn_q.weight"] = L.wq;
      r.named[p + "attn_k.weight"] = L.wk;
      r.named[p + "attn_v.weight"] = L.wv;
      r.named[p + "attn_output.weight"] = L.wo;
      r.named[p + "ffn_down.weight"] = L.wd;
    } else {
      if ((rc = upload_matrix(r, g, p + "attn_q.weight", qd, d, &L.wq)) ||
          (rc = upload_matrix(r, g, p + "attn_k.weight", kd, d, &L.wk)) ||
          (rc = upload_matrix(r, g, p + "attn_v.weight", kd, d, &L.wv)) ||
          (rc = upload_matrix(r, g, p + "attn_output.weight", d, qd, &L.wo)) ||
          (rc = upload_matrix(r, g, p + "ffn_gate.weight", c.ffn, d, &L.wg)) ||
          (rc = upload_matrix(r, g, p + "ffn_up.weight", c.ffn, d, &L.wu)) ||
          (rc = upload_matrix(r, g, p + "ffn_down.weight", d, c.ffn, &L.wd)))
        return rc;
    }
  }
  if ((rc = upload_vector(r, g, "output_norm.weight", d, &r.out_norm))) return rc;
  if ((rc = upload_matrix(r, g, "token_embd.weight", c.V, d, &r.embd))) return rc;
  if ((rc = upload_matrix(r, g, "output.weight", c.V, d, &r.head))) return rc;
  if (r.head.kind == K_F16) r.head16 = reinterpret_cast<const half*>(r.head.q);
  // RoPE table: angle = pos / theta^(2j/hd), rotate-half pairs (j, j + hd/2)
  // (src/models/openthai/model.rs:264 with rotary dim = head_dim).
  {
    const int half_hd = c.hd / 2;
    std::vector<float2> tab((size_t)c.ctx * half_hd);
    for (int pos = 0; pos < c.ctx; pos++)
      for (int j = 0; j < half_hd; j++) {
        float angle = (float)pos / powf(c.theta, (float)(2 * j) / (float)c.hd);
        tab[(size_t)pos * half_hd + j] = make_float2(cosf(angle), sinf(angle));
      }
    void* p;
    if ((rc = upload(r, tab.data(), tab.size() * sizeof(float2), &p))) return rc;
    r.rope = static_cast<const float2*>(p);
  }
  void* e;
  if ((rc = dmalloc(r, 16, &e))) return rc;
  r.err = static_cast<unsigned*>(e);
  return 0;
}

// Pointer relocation from a source replica's weight buffers to a copy's.
class Reloc {
 public:
  Reloc(const std::vector<std::pair<void*, size_t>>& src, const std::vector<void*>& dst) {
    for (size_t i = 0; i < src.size(); i++) map_.push_back({static_cast<char*>(src[i].first), src[i].second,
                                                            static_cast<char*>(dst[i])});
    std::sort(map_.begin(), map_.end(), [](const E& a, const E& b) { return a.s < b.s; });
  }
  bool ok = true;
  template <class T>
  T* operator()(T* p) {
    if (!p) return p;
    const char* c = reinterpret_cast<const char*>(p);
    auto it = std::upper_bound(map_.begin(), map_.end(), c, [](const char* v, const E& e) { return v < e.s; });
    if (it == map_.begin() || c >= (it - 1)->s + (it - 1)->n) {
      ok = false;
      return nullptr;
    }
    --it;
    return reinterpret_cast<T*>(it->d + (c - it->s));
  }
  QTensor operator()(QTensor t) {
    t.q = (*this)(t.q);
    t.s = (*this)(t.s);
    t.qh = (*this)(t.qh);
    t.sc = (*this)(t.sc);
    return t;
  }

 private:
  struct E {
    char* s;
    size_t n;
    char* d;
  };
  std::vector<E> map_;
};

// Allocates src's weight buffers on r's device and queues their copies on
// r's stream; the pointers of r are src's, relocated.
static int mirror_from(const Replica& src, Replica& r) {
  LAYA_CK(cudaSetDevice(r.device));
  std::vector<void*> dst(src.wmap.size());
  r.loading = true;
  for (size_t i = 0; i < src.wmap.size(); i++) {
    if (int rc = dmalloc(r, src.wmap[i].second, &dst[i])) {
      r.loading = false;
      return rc;
    }
    LAYA_CK(cudaMemcpyPeerAsync(dst[i], r.device, src.wmap[i].first, src.device, src.wmap[i].second, r.stream));
  }
  r.loading = false;
  Reloc rl(src.wmap, dst);
  r.layers.resize(src.layers.size());
  for (size_t l = 0; l < src.layers.size(); l++) {
    const Layer& a = src.layers[l];
    Layer& b = r.layers[l];
    b.attn_norm = rl(a.attn_norm);
    b.ffn_norm = rl(a.ffn_norm);
    b.wq = rl(a.wq);
    b.wk = rl(a.wk);
    b.wv = rl(a.wv);
    b.wo = rl(a.wo);
    b.wg = rl(a.wg);
    b.wu = rl(a.wu);
    b.wd = rl(a.wd);
    b.bqkv = rl(a.bqkv);
    b.wqkv16 = rl(a.wqkv16);
    b.wgu16 = rl(a.wgu16);
    b.wo16 = rl(a.wo16);
    b.wd16 = rl(a.wd16);
  }
  r.embd = rl(src.embd);
  r.head = rl(src.head);
  r.out_norm = rl(src.out_norm);
  r.head16 = rl(src.head16);
  r.rope = rl(src.rope);
  r.err = rl(src.err);
  for (const auto& kv : src.named) r.named[kv.first] = rl(kv.second);
  if (!rl.ok) return fail(LAYA_E_CUDA, "replica copy: a weight pointer lies outside the loaded buffers");
  LAYA_CK(cudaMemsetAsync(r.err, 0, 16, r.stream));
  return 0;
}

int mirror_replicas(Model& m, const std::vector<int>& devices) {
  std::vector<int> have = {0};
  size_t next = 1;
  while (next < devices.size()) {
    std::vector<int> fresh;
    for (int s : std::vector<int>(have)) {
      if (next >= devices.size()) break;
      Replica& r = m.reps[next];
      if (int rc = init_device(devices[next], r)) return rc;
      // the copy reads the source device's buffers: wait for them to be filled
      LAYA_CK(cudaSetDevice(m.reps[s].device));
      LAYA_CK(cudaStreamSynchronize(m.reps[s].stream));
      if (int rc = mirror_from(m.reps[s], r)) return rc;
      fresh.push_back((int)next++);
    }
    for (int i : fresh) {
      LAYA_CK(cudaSetDevice(m.reps[i].device));
      LAYA_CK(cudaStreamSynchronize(m.reps[i].stream));
      have.push_back(i);
    }
  }
  return 0;
}

void free_replica(Replica& r) {
  if (r.stream) {
    cudaSetDevice(r.device);
    cudaStreamSynchronize(r.stream);
  }
  for (void* p : r.allocs) cudaFree(p);
  r.allocs.clear();
  for (DevBuf* b : {&r.ids, &r.pos, &r.slot, &r.x, &r.h, &r.qb, &r.att, &r.act, &r.items, &r.tables, &r.rows, &r.hid32,
                    &r.hid16, &r.cand, &r.row_of, &r.clog, &r.flog, &r.lse, &r.cow, &r.wqkv_s, &r.wo_s, &r.wgu_s,
                    &r.wd_s, &r.kpart, &r.kc, &r.vc, &r.dx16, &r.dlogits, &r.dargmax, &r.dpart})
    b->release();
  r.pin.release();
  for (auto& e : r.prof_events) {
    cudaEventDestroy(e.a);
    cudaEventDestroy(e.b);
  }
  for (auto e : r.event_pool) cudaEventDestroy(e);
  if (r.ev_start) cudaEventDestroy(r.ev_start);
  if (r.ev_end) cudaEventDestroy(r.ev_end);
  r.ev_start = r.ev_end = nullptr;
  r.prof_events.clear();
  r.event_pool.clear();
  if (r.stream) cudaStreamDestroy(r.stream);
  r.stream = nullptr;
}

int ensure_head16(Model& m, Replica& r) {
  if (r.head16) return 0;
  void* p;
  if (int rc = dmalloc(r, (size_t)m.cfg.V * m.cfg.d * 2, &p)) return rc;
  LAYA_CK(dequant_f16(r.head, static_cast<half*>(p), m.cfg.d, 1 << 30, 0, 0, r.stream));
  r.head16 = static_cast<const half*>(p);
  return 0;
}

int ensure_f16_cache(Model& m, Replica& r) {
  const Config& c = m.cfg;
  const char* e = std::getenv("LAYA_F16_CACHE");
  if (!c.quantized || (e && e[0] == '0') || r.layers.empty() || r.layers[0].rqkv16 || r.f16_cache_failed) return 0;
  const int qd = c.H * c.hd, kd = c.KV * c.hd, d = c.d, ffn = c.ffn, big = 1 << 30;
  const size_t sizes[4] = {(size_t)(qd + 2 * kd) * d * 2, (size_t)2 * ffn * d * 2, (size_t)d * qd * 2,
                           (size_t)d * ffn * 2};
  std::vector<void*> bufs;
  for (int l = 0; l < c.L && !r.f16_cache_failed; l++)
    for (int i = 0; i < 4; i++) {
      void* p = nullptr;
      if (cudaMalloc(&p, sizes[i]) != cudaSuccess) {
        cudaGetLastError();
        r.f16_cache_failed = true;  // keep staging before each GEMM
        break;
      }
      bufs.push_back(p);
    }
  if (r.f16_cache_failed) {
    for (void* p : bufs) cudaFree(p);
    return 0;
  }
  for (int l = 0; l < c.L; l++) {
    Layer& L = r.layers[l];
    half* qkv = static_cast<half*>(bufs[4 * l]);
    half* gu = static_cast<half*>(bufs[4 * l + 1]);
    half* o = static_cast<half*>(bufs[4 * l + 2]);
    half* dn = static_cast<half*>(bufs[4 * l + 3]);
    // the layouts of the per-GEMM staging: q|k|v stacked, gate/up interleaved per 128 rows
    LAYA_CK(dequant_f16(L.wq, qkv, d, big, 0, 0, r.stream));
    LAYA_CK(dequant_f16(L.wk, qkv, d, big, 0, qd, r.stream));
    LAYA_CK(dequant_f16(L.wv, qkv, d, big, 0, qd + kd, r.stream));
    LAYA_CK(dequant_f16(L.wg, gu, d, 128, 256, 0, r.stream));
    LAYA_CK(dequant_f16(L.wu, gu, d, 128, 256, 128, r.stream));
    LAYA_CK(dequant_f16(L.wo, o, qd, big, 0, 0, r.stream));
    LAYA_CK(dequant_f16(L.wd, dn, ffn, big, 0, 0, r.stream));
    r.launches += 7;
    L.rqkv16 = qkv;
    L.rgu16 = gu;
    L.ro16 = o;
    L.rd16 = dn;
  }
  for (void* p : bufs) r.allocs.push_back(p);
  return 0;
}

bool use_q8_gemm(const Model& m, const Replica& r, int M) {
  const Config& c = m.cfg;
  if (!c.quantized || r.layers.empty() || M < 1) return false;
  const char* on = std::getenv("LAYA_Q8_FUSED");
  if (on && on[0] == '0') return false;
  const char* mx = std::getenv("LAYA_Q8_FUSED_MAX_M");
  const int max_m = mx ? std::atoi(mx) : 256;
  if (M > max_m) return false;
  const int qd = c.H * c.hd, kd = c.KV * c.hd;
  if (c.d % 128 || qd % 128 || kd % 128 || c.ffn % 128) return false;
  for (const Layer& L : r.layers)
    for (const QTensor* t : {&L.wq, &L.wk, &L.wv, &L.wo, &L.wg, &L.wu, &L.wd})
      if (t->kind != K_Q8_0) return false;
  return true;
}

int ensure_q8_scales(Model& m, Replica& r) {
  const Config& c = m.cfg;
  if (r.layers.empty() || r.layers.back().sqkv_t) return 0;  // the last layer is built last
  const int qd = c.H * c.hd, kd = c.KV * c.hd, d = c.d, ffn = c.ffn, big = 1 << 30;
  const int nqkv = qd + 2 * kd;
  // [K/32][N] F16 per operand
  const size_t sizes[4] = {(size_t)(d / 32) * nqkv * 2, (size_t)(d / 32) * 2 * ffn * 2, (size_t)(qd / 32) * d * 2,
                           (size_t)(ffn / 32) * d * 2};
  for (int l = 0; l < c.L; l++) {
    Layer& L = r.layers[l];
    half* p[4];
    for (int i = 0; i < 4; i++) {
      void* v = nullptr;
      LAYA_CK(cudaMalloc(&v, sizes[i]));
      r.allocs.push_back(v);
      p[i] = static_cast<half*>(v);
    }
    LAYA_CK(q8_scales_t(L.wq, p[0], nqkv, big, 0, 0, r.stream));
    LAYA_CK(q8_scales_t(L.wk, p[0], nqkv, big, 0, qd, r.stream));
    LAYA_CK(q8_scales_t(L.wv, p[0], nqkv, big, 0, qd + kd, r.stream));
    LAYA_CK(q8_scales_t(L.wg, p[1], 2 * ffn, 128, 256, 0, r.stream));
    LAYA_CK(q8_scales_t(L.wu, p[1], 2 * ffn, 128, 256, 128, r.stream));
    LAYA_CK(q8_scales_t(L.wo, p[2], d, big, 0, 0, r.stream));
    LAYA_CK(q8_scales_t(L.wd, p[3], d, big, 0, 0, r.stream));
    r.launches += 7;
    L.sqkv_t = p[0];
    L.sgu_t = p[1];
    L.so_t = p[2];
    L.sd_t = p[3];
  }
  if (r.head.kind == K_Q8_0 && c.V % 8 == 0 && d % 128 == 0 && !r.head_st) {
    void* v = nullptr;
    LAYA_CK(cudaMalloc(&v, (size_t)(d / 32) * c.V * 2));
    r.allocs.push_back(v);
    LAYA_CK(q8_scales_t(r.head, static_cast<half*>(v), c.V, big, 0, 0, r.stream));
    r.launches++;
    r.head_st = static_cast<const half*>(v);
  }
  return 0;
}

static Q8Weights q8_one(const QTensor& t, const half* st) {
  Q8Weights w{};
  w.q[0] = reinterpret_cast<const int8_t*>(t.q);
  w.rows[0] = t.rows;
  w.nseg = 1;
  w.st = st;
  return w;
}

Q8Weights q8_qkv(const Config& c, const Layer& L) {
  Q8Weights w{};
  const QTensor* t[3] = {&L.wq, &L.wk, &L.wv};
  for (int i = 0; i < 3; i++) {
    w.q[i] = reinterpret_cast<const int8_t*>(t[i]->q);
    w.rows[i] = t[i]->rows;
  }
  w.nseg = 3;
  w.st = L.sqkv_t;
  return w;
}

Q8Weights q8_gu(const Config& c, const Layer& L) {
  Q8Weights w{};
  w.q[0] = reinterpret_cast<const int8_t*>(L.wg.q);
  w.q[1] = reinterpret_cast<const int8_t*>(L.wu.q);
  w.rows[0] = w.rows[1] = c.ffn;
  w.nseg = 2;
  w.interleave = 1;
  w.st = L.sgu_t;
  return w;
}

Q8Weights q8_o(const Config& c, const Layer& L) { return q8_one(L.wo, L.so_t); }
Q8Weights q8_down(const Config& c, const Layer& L) { return q8_one(L.wd, L.sd_t); }
Q8Weights q8_head(const Replica& r) { return q8_one(r.head, r.head_st); }

int ensure_kv(Model& m, Replica& r, int pages) {
  if (pages <= r.kv_pages) return 0;
  const Config& c = m.cfg;
  int want = std::max(pages, r.kv_pages + r.kv_pages / 4);
  const size_t bytes = (size_t)c.L * want * c.KV * PAGE * c.hd * 2;
  r.kc.release();
  r.vc.release();
  if (int rc = r.kc.ensure(bytes)) return rc;
  if (int rc = r.vc.ensure(bytes)) return rc;
  // Attention kernels read whole pages and weight the unused slots of a
  // sequence's last page by zero: start from zeros so those slots hold no
  // Inf/NaN bit patterns (0 x Inf would poison the sum).
  LAYA_CK(cudaMemsetAsync(r.kc.p, 0, bytes, r.stream));
  LAYA_CK(cudaMemsetAsync(r.vc.p, 0, bytes, r.stream));
  r.kv_pages = want;
  return 0;
}

// ---------------------------------------------------------------- forward

// Prefill GEMMs launch with programmatic dependent launch (their first
// weight tiles come into L2 while the previous kernel drains) unless
// LAYA_GEMM_PDL=0.
static bool gemm_pdl() {
  static const bool on = [] {
    const char* e = std::getenv("LAYA_GEMM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

static int gemm(Replica& r, int cat, int epi, const half* A, int lda, const half* B, int ldb, GemmArgs a) {
  a.err = r.err;
  a.budget = kWaitBudget;
  ProfScope ps(r, cat);
  r.launches++;
  LAYA_CK(gemm_launch(epi, A, lda, B, ldb, a, r.num_sms, r.stream, gemm_pdl()));
  return 0;
}

static int gemm_q8(Replica& r, int cat, int epi, const half* A, int lda, const Q8Weights& w, GemmArgs a) {
  a.err = r.err;
  a.budget = kWaitBudget;
  ProfScope ps(r, cat);
  r.launches++;
  LAYA_CK(gemm_q8_launch(epi, A, lda, w, a, r.num_sms, r.stream, gemm_pdl()));
  return 0;
}

static int stage(Replica& r, int cat, const QTensor& t, half* out, int ldo, int grp, int gstride, int goff) {
  ProfScope ps(r, cat);
  r.launches++;
  LAYA_CK(dequant_f16(t, out, ldo, grp, gstride, goff, r.stream));
  return 0;
}

static bool poll_cancel(int (*canceled)(void*), void* user, std::mutex* mu) {
  if (!canceled) return false;
  if (mu) {
    std::lock_guard<std::mutex> lk(*mu);
    return canceled(user) != 0;
  }
  return canceled(user) != 0;
}

// Uploads host arrays through the pinned staging buffer (one sync first so a
// previous pass's copies out of the same buffer have finished).
static int upload_many(Replica& r, std::initializer_list<std::tuple<DevBuf*, const void*, size_t>> items) {
  size_t total = 0;
  for (auto& it : items) total += (std::get<2>(it) + 255) / 256 * 256;
  LAYA_CK(cudaStreamSynchronize(r.stream));
  if (int rc = r.pin.ensure(total)) return rc;
  size_t off = 0;
  for (auto& it : items) {
    DevBuf* b = std::get<0>(it);
    size_t n = std::get<2>(it);
    if (!n) continue;
    if (int rc = b->ensure(n)) return rc;
    std::memcpy(static_cast<char*>(r.pin.p) + off, std::get<1>(it), n);
    LAYA_CK(cudaMemcpyAsync(b->p, static_cast<char*>(r.pin.p) + off, n, cudaMemcpyHostToDevice, r.stream));
    r.h2d += (long long)n;
    off += (n + 255) / 256 * 256;
  }
  return 0;
}

int run_forward(Model& m, Replica& r, const PassPlan& p, const std::vector<int>& tables, int read_base,
                int (*canceled)(void*), void* user, std::mutex* cancel_mu) {
  const Config& c = m.cfg;
  const int M = (int)p.ids.size();
  if (!M) return 0;
  const int qd = c.H * c.hd, kd = c.KV * c.hd, d = c.d, ffn = c.ffn;
  cudaStream_t st = r.stream;
  int rc;
  if ((rc = upload_many(r, {{&r.ids, p.ids.data(), p.ids.size() * 4},
                            {&r.pos, p.pos.data(), p.pos.size() * 4},
                            {&r.slot, p.slot.data(), p.slot.size() * 4},
                            {&r.items, p.items.data(), p.items.size() * sizeof(AttnItem)},
                            {&r.tables, tables.data(), tables.size() * 4},
                            {&r.rows, p.read_rows.data(), p.read_rows.size() * 4}})))
    return rc;
  if ((rc = r.x.ensure((size_t)M * d * 4)) || (rc = r.h.ensure((size_t)M * d * 2)) ||
      (rc = r.qb.ensure((size_t)M * qd * 2)) || (rc = r.att.ensure((size_t)M * qd * 2)) ||
      (rc = r.act.ensure((size_t)M * ffn * 2)))
    return rc;
  // short passes over Q8_0 weights decode the quants inside the GEMMs
  const bool q8 = use_q8_gemm(m, r, M);
  if (q8 && (rc = ensure_q8_scales(m, r))) return rc;
  if (c.quantized && !q8 && (rc = ensure_f16_cache(m, r))) return rc;
  if (c.quantized && !q8 && !r.layers[0].rqkv16) {
    if ((rc = r.wqkv_s.ensure((size_t)(qd + 2 * kd) * d * 2)) || (rc = r.wo_s.ensure((size_t)d * qd * 2)) ||
        (rc = r.wgu_s.ensure((size_t)2 * ffn * d * 2)) || (rc = r.wd_s.ensure((size_t)d * ffn * 2)))
      return rc;
  }
  float* x = r.x.as<float>();
  half* h = r.h.as<half>();
  if (r.arm_start && (rc = timing_mark_start(r))) return rc;
  r.launches++;
  LAYA_CK(rows_f32(r.embd, r.ids.as<int>(), M, x, st));
  const float scale_log2 = (1.f / sqrtf((float)c.hd)) * 1.4426950408889634f;
  const size_t layer_elems = (size_t)r.kv_pages * c.KV * PAGE * c.hd;
  std::vector<cudaEvent_t> lev;
  const int big = 1 << 30;
  // Residual GEMMs with few output tiles (small M) split K; their partial sums
  // are merged, in split order, by the RMSNorm that next reads the residual.
  const char* ke = std::getenv("LAYA_KSPLIT");
  const bool ks_on = !(ke && ke[0] == '0');
  auto ksplit = [&](int N, int K) {
    return !ks_on ? 1 : q8 ? gemm_q8_ksplit(M, N, K, r.num_sms) : gemm_ksplit(M, N, K, r.num_sms);
  };
  const int ks_o = ksplit(d, qd);
  const int ks_d = ksplit(d, ffn);
  // the QKV GEMM splits K the same way when it has few tiles; its partial
  // planes (consumed by qkv_merge before the attention) share the buffer
  const int nqkv = qd + 2 * kd;
  const int ks_q = ksplit(nqkv, d);
  // one layer GEMM: on the Q8_0 blocks (q8) or on the F16 operand B16
  auto lgemm = [&](int cat, int epi, const half* A, int lda, const half* B16, const Q8Weights& w,
                   const GemmArgs& a) -> int {
    if (!q8) return gemm(r, cat, epi, A, lda, B16, lda, a);
    return gemm_q8(r, cat, epi, A, lda, w, a);
  };
  const size_t kpart_f = std::max((size_t)std::max(ks_o, ks_d) * M * d, (size_t)ks_q * M * nqkv);
  if (std::max(std::max(ks_o, ks_d), ks_q) > 1 && (rc = r.kpart.ensure(kpart_f * 4))) return rc;
  int pend = 0;  // K splits of x not yet merged (the gathered final norm merges without writing x back)
  auto norm = [&](const int* rows, int n, const float* w, half* o16, float* o32) -> cudaError_t {
    r.launches++;
    const int ns = pend;
    pend = 0;
    // launched early behind the previous kernel (it waits for that kernel's
    // output before reading), so its launch overlaps the GEMM's tail
    if (ns > 1)
      return rmsnorm_merge(x, rows, n, r.kpart.as<float>(), ns, (size_t)M * d, w, d, c.eps, o16, o32, st, gemm_pdl());
    return rmsnorm(x, rows, n, w, d, c.eps, o16, o32, st, gemm_pdl(), r.err);
  };
  for (int l = 0; l < c.L; l++) {
    const Layer& L = r.layers[l];
    if (canceled) {
      // keep at most two layers queued ahead of the device, then poll the
      // cancel callback between layers (src/models/openthai/model.rs:215-217)
      if (l >= 2) cudaEventSynchronize(lev[l - 2]);
      if (poll_cancel(canceled, user, cancel_mu)) {
        cudaStreamSynchronize(st);
        for (auto e : lev) cudaEventDestroy(e);
        return fail(LAYA_E_CANCELED, "request canceled");
      }
    }
    LAYA_CK(norm(nullptr, M, L.attn_norm, h, nullptr));
    const half* wqkv = L.wqkv16 ? L.wqkv16 : L.rqkv16;
    const Q8Weights w_qkv = q8 ? q8_qkv(c, L) : Q8Weights{};
    if (!wqkv && !q8) {
      half* s = r.wqkv_s.as<half>();
      if ((rc = stage(r, P_DEQUANT, L.wq, s, d, big, 0, 0)) || (rc = stage(r, P_DEQUANT, L.wk, s, d, big, 0, qd)) ||
          (rc = stage(r, P_DEQUANT, L.wv, s, d, big, 0, qd + kd)))
        return rc;
      wqkv = s;
    }
    GemmArgs a{};
    a.M = M;
    a.N = qd + 2 * kd;
    a.K = d;
    a.bias = L.bqkv;
    a.out = r.qb.p;
    a.ldo = qd;
    a.qd = qd;
    a.kd = kd;
    a.hd = c.hd;
    a.kvh = c.KV;
    a.pos = r.pos.as<int>();
    a.slot = r.slot.as<int>();
    a.rope = r.rope;
    a.kcache = r.kc.as<half>() + l * layer_elems;
    a.vcache = r.vc.as<half>() + l * layer_elems;
    a.page_size = PAGE;
    if (ks_q > 1) {
      // raw partial sums of each K split, then bias / RoPE / q rows / KV cache
      GemmArgs sp{};
      sp.M = M;
      sp.N = nqkv;
      sp.K = d;
      sp.ldo = nqkv;
      sp.ksplit = ks_q;
      sp.part = r.kpart.as<float>();
      if ((rc = lgemm(P_GEMM_QKV, EPI_RESID, h, d, wqkv, w_qkv, sp))) return rc;
      ProfScope ps(r, P_GEMM_QKV);
      r.launches++;
      LAYA_CK(qkv_merge(r.kpart.as<float>(), ks_q, (size_t)M * nqkv, M, L.bqkv, qd, kd, c.hd, c.KV, a.pos, a.slot,
                        r.rope, PAGE, r.qb.as<half>(), qd, a.kcache, a.vcache, st, gemm_pdl()));
    } else if ((rc = lgemm(P_GEMM_QKV, EPI_QKV, h, d, wqkv, w_qkv, a))) {
      return rc;
    }
    {
      AttnParams ap{};
      ap.q = r.qb.as<half>();
      ap.ldq = qd;
      ap.o = r.att.as<half>();
      ap.ldo = qd;
      ap.kc = a.kcache;
      ap.vc = a.vcache;
      ap.tables = r.tables.as<int>();
      ap.items = r.items.as<AttnItem>();
      ap.n_items = (int)p.items.size();
      ap.H = c.H;
      ap.KV = c.KV;
      ap.hd = c.hd;
      ap.scale_log2 = scale_log2;
      ap.q_rows = M;
      ap.kv_rows = r.kv_pages * c.KV * PAGE;
      ap.err = r.err;
      // the KV head's query heads share each unit, so its pages are loaded
      // and multiplied once for the group instead of once per head (4x fewer
      // page visits for question suffixes and option continuations)
      ap.pack = 1;
      ProfScope ps(r, P_ATTN);
      r.launches++;
      LAYA_CK(attention(ap, st));
    }
    const half* wo = L.wo16 ? L.wo16 : L.ro16;
    if (!wo && !q8) {
      if ((rc = stage(r, P_DEQUANT, L.wo, r.wo_s.as<half>(), qd, big, 0, 0))) return rc;
      wo = r.wo_s.as<half>();
    }
    GemmArgs b{};
    b.M = M;
    b.N = d;
    b.K = qd;
    b.resid = x;
    b.ldo = d;
    b.ksplit = ks_o;
    b.part = r.kpart.as<float>();
    if ((rc = lgemm(P_GEMM_O, EPI_RESID, r.att.as<half>(), qd, wo, q8 ? q8_o(c, L) : Q8Weights{}, b))) return rc;
    pend = ks_o;
    LAYA_CK(norm(nullptr, M, L.ffn_norm, h, nullptr));
    const half* wgu = L.wgu16 ? L.wgu16 : L.rgu16;
    if (!wgu && !q8) {
      half* s = r.wgu_s.as<half>();
      if ((rc = stage(r, P_DEQUANT, L.wg, s, d, 128, 256, 0)) || (rc = stage(r, P_DEQUANT, L.wu, s, d, 128, 256, 128)))
        return rc;
      wgu = s;
    }
    GemmArgs gu{};
    gu.M = M;
    gu.N = 2 * ffn;
    gu.K = d;
    gu.out = r.act.p;
    gu.ldo = ffn;
    if ((rc = lgemm(P_GEMM_GU, EPI_SWIGLU, h, d, wgu, q8 ? q8_gu(c, L) : Q8Weights{}, gu))) return rc;
    const half* wd = L.wd16 ? L.wd16 : L.rd16;
    if (!wd && !q8) {
      if ((rc = stage(r, P_DEQUANT, L.wd, r.wd_s.as<half>(), ffn, big, 0, 0))) return rc;
      wd = r.wd_s.as<half>();
    }
    GemmArgs dn{};
    dn.M = M;
    dn.N = d;
    dn.K = ffn;
    dn.resid = x;
    dn.ldo = d;
    dn.ksplit = ks_d;
    dn.part = r.kpart.as<float>();
    if ((rc = lgemm(P_GEMM_DOWN, EPI_RESID, r.act.as<half>(), ffn, wd, q8 ? q8_down(c, L) : Q8Weights{}, dn)))
      return rc;
    pend = ks_d;
    if (canceled) {
      cudaEvent_t e;
      LAYA_CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      LAYA_CK(cudaEventRecord(e, st));
      lev.push_back(e);
    }
  }
  for (auto e : lev) cudaEventDestroy(e);
  const int R = (int)p.read_rows.size();
  LAYA_CK(norm(r.rows.as<int>(), R, r.out_norm, r.hid16.as<half>() + (size_t)read_base * d,
               r.hid32.as<float>() + (size_t)read_base * d));
  return 0;
}

// ---------------------------------------------------------------- decide

int validate_batch(const Config& c, const laya_batch* b) {
  if (!b) return fail(LAYA_E_INVALID, "null batch");
  if (b->n_requests < 0) return fail(LAYA_E_INVALID, "negative request count");
  if (b->n_requests == 0) return 0;
  if (!b->ids || !b->offsets) return fail(LAYA_E_INVALID, "missing token ids");
  if (b->n_questions < 1 || !b->questions) return fail(LAYA_E_INVALID, "no questions");
  int max_extra = 0;
  for (int q = 0; q < b->n_questions; q++) {
    const laya_question& Q = b->questions[q];
    if (Q.kind < 0 || Q.kind > 2) return fail(LAYA_E_INVALID, "unknown question type");
    if (Q.n_options < 1 || Q.n_options > LAYA_MAX_OPTIONS) return fail(LAYA_E_INVALID, "question needs 1..16 options");
    if (Q.kind == LAYA_NOUL && Q.n_options != 2) return fail(LAYA_E_INVALID, "noul question needs exactly 2 options");
    if (Q.option_len < 1 || !Q.options) return fail(LAYA_E_INVALID, "invalid options");
    if (Q.suffix_len < 0 || (Q.suffix_len > 0 && !Q.suffix)) return fail(LAYA_E_INVALID, "invalid suffix");
    for (int i = 0; i < Q.n_options * Q.option_len; i++)
      if (Q.options[i] < 0 || Q.options[i] >= c.V) return fail(LAYA_E_INVALID, "option token id out of range");
    for (int i = 0; i < Q.suffix_len; i++)
      if (Q.suffix[i] < 0 || Q.suffix[i] >= c.V) return fail(LAYA_E_INVALID, "suffix token id out of range");
    max_extra = std::max(max_extra, Q.suffix_len + Q.option_len - 1);
  }
  if (b->offsets[0] != 0) return fail(LAYA_E_INVALID, "offsets[0] must be 0");
  for (int i = 0; i < b->n_requests; i++) {
    const int64_t len = b->offsets[i + 1] - b->offsets[i];
    if (len < 1) return fail(LAYA_E_INVALID, "empty token sequence");
    if (len + max_extra > c.ctx) return fail(LAYA_E_INVALID, "token sequence exceeds the context length");
    for (int64_t t = b->offsets[i]; t < b->offsets[i + 1]; t++)
      if (b->ids[t] < 0 || b->ids[t] >= c.V) return fail(LAYA_E_INVALID, "invalid token sequence");
  }
  return 0;
}

static float kind_temperature(const Config& c, int kind, int k) {
  const int bucket = k <= 2 ? 0 : k <= 5 ? 1 : k <= 10 ? 2 : 3;
  float t = c.has_bucket[kind][bucket] ? c.bucket[kind][bucket] : c.temperature[kind];
  return t > 1e-3f ? t : 1e-3f;
}

// Decision rules of src/models/laya/decision.rs:214-268 (softmax of
// tensor::softmax, src/tensor.rs:132-140; confidence :155-167).
static void apply_rules(const Config& c, int kind, int k, const float* logits, laya_answer* a) {
  const float t = kind_temperature(c, kind, k);
  float s[LAYA_MAX_OPTIONS], p[LAYA_MAX_OPTIONS];
  float mx = -INFINITY;
  for (int i = 0; i < k; i++) {
    s[i] = logits[i] / t;
    mx = fmaxf(mx, s[i]);
  }
  float sum = 0.f;
  for (int i = 0; i < k; i++) {
    p[i] = expf(s[i] - mx);
    sum += p[i];
  }
  for (int i = 0; i < k; i++) p[i] /= sum;
  std::memset(a, 0, sizeof(*a));
  a->kind = kind;
  a->n_options = k;
  a->choice = -1;
  if (kind == LAYA_CHOICE) {
    int best = 0;
    for (int i = 1; i < k; i++)
      if (p[i] > p[best]) best = i;
    a->choice = best;
  } else if (kind == LAYA_SCORE) {
    double sc = 0;
    for (int i = 0; i < k; i++) sc += (double)i * (double)p[i];
    a->score = (float)sc;
  } else {
    a->noul = p[1];
  }
  if (kind == LAYA_NOUL) {
    a->confidence = p[1] > 1.f - p[1] ? p[1] : 1.f - p[1];
  } else if (k < 2) {
    a->confidence = 1.f;
  } else {
    double e = 0;
    for (int i = 0; i < k; i++) {
      double x = std::max((double)p[i], 1e-12);
      e += x * std::log(x);
    }
    double conf = 1. - (-e) / std::log((double)k);
    a->confidence = (float)std::min(1.0, std::max(0.0, conf));
  }
  for (int i = 0; i < k; i++) {
    a->probabilities[i] = p[i];
    a->logits[i] = logits[i];
  }
}

static int wave_tokens() {
  const char* e = std::getenv("LAYA_WAVE_TOKENS");
  int v = e ? std::atoi(e) : 0;
  return v > 0 ? v : 65536;
}

int decide_shard(Model& m, Replica& r, const laya_batch& b, int r0, int r1, laya_answer* out,
                 int (*canceled)(void*), void* user, std::mutex* cancel_mu) {
  const Config& c = m.cfg;
  LAYA_CK(cudaSetDevice(r.device));
  const int nq = b.n_questions;
  bool any_full = false;
  for (int q = 0; q < nq; q++) any_full |= b.questions[q].option_len > 1;
  int rc;
  if ((rc = timing_begin_call(r))) return rc;
  if (any_full && (rc = ensure_head16(m, r))) return rc;
  LAYA_CK(cudaMemsetAsync(r.err, 0, 4, r.stream));
  const long budget = wave_tokens();
  int i = r0;
  while (i < r1) {
    long tok = 0;
    int j = i;
    while (j < r1 && (j == i || tok + (b.offsets[j + 1] - b.offsets[j]) <= budget)) {
      tok += b.offsets[j + 1] - b.offsets[j];
      j++;
    }
    const int nr = j - i;
    // ---- plan the wave
    PassPlan pre, br;
    std::vector<int> tables;
    std::vector<int2> cow;
    std::vector<char> read_lse_pre, read_lse_br;
    std::vector<int> cand_id, cand_read;  // cand_read: read index, branch reads offset later
    std::vector<char> cand_is_branch;
    struct Term {
      int cand, read;
      bool branch;
    };
    std::vector<std::vector<Term>> terms((size_t)nr * nq * LAYA_MAX_OPTIONS);
    std::vector<int> req_toff(nr), req_len(nr);
    int pages = 0;
    auto add_cand = [&](int read, bool branch, int id) {
      cand_id.push_back(id);
      cand_read.push_back(read);
      cand_is_branch.push_back(branch);
      return (int)cand_id.size() - 1;
    };
    for (int ri = 0; ri < nr; ri++) {
      const int64_t o0 = b.offsets[i + ri];
      const int len = (int)(b.offsets[i + ri + 1] - o0);
      const int toff = (int)tables.size();
      for (int pg = 0; pg < (len + PAGE - 1) / PAGE; pg++) tables.push_back(pages++);
      req_toff[ri] = toff;
      req_len[ri] = len;
      const int row0 = (int)pre.ids.size();
      for (int t = 0; t < len; t++) {
        pre.ids.push_back(b.ids[o0 + t]);
        pre.pos.push_back(t);
        pre.slot.push_back(tables[toff + t / PAGE] * PAGE + t % PAGE);
      }
      for (int t0 = 0; t0 < len; t0 += kAttnRows) pre.items.push_back({row0 + t0, std::min(kAttnRows, len - t0), t0, toff});
      for (int qi = 0; qi < nq; qi++) {
        const laya_question& Q = b.questions[qi];
        if (Q.suffix_len) continue;
        const int read = (int)pre.read_rows.size();
        pre.read_rows.push_back(row0 + len - 1);
        read_lse_pre.push_back(Q.option_len > 1);
        for (int o = 0; o < Q.n_options; o++) {
          const int ci = add_cand(read, false, Q.options[(size_t)o * Q.option_len]);
          terms[((size_t)ri * nq + qi) * LAYA_MAX_OPTIONS + o].push_back({ci, Q.option_len > 1 ? read : -1, false});
        }
      }
    }
    for (int ri = 0; ri < nr; ri++) {
      for (int qi = 0; qi < nq; qi++) {
        const laya_question& Q = b.questions[qi];
        if (Q.suffix_len == 0 && Q.option_len == 1) continue;
        const int S = Q.suffix_len, Lo = Q.option_len;
        const int nbranch = Lo == 1 ? 1 : Q.n_options;
        for (int bi = 0; bi < nbranch; bi++) {
          std::vector<int> tok(Q.suffix, Q.suffix + S);
          if (Lo > 1)
            for (int t = 0; t < Lo - 1; t++) tok.push_back(Q.options[(size_t)bi * Lo + t]);
          const int blen = (int)tok.size();
          if (!blen) continue;
          const int plen = req_len[ri], full = plen / PAGE, rem = plen % PAGE;
          const int toff = (int)tables.size();
          for (int pg = 0; pg < full; pg++) tables.push_back(tables[req_toff[ri] + pg]);
          if (rem) {
            const int np = pages++;
            cow.push_back(make_int2(tables[req_toff[ri] + full], np));
            tables.push_back(np);
          }
          const int need = (plen + blen + PAGE - 1) / PAGE;
          while ((int)tables.size() - toff < need) tables.push_back(pages++);
          const int row0 = (int)br.ids.size();
          for (int t = 0; t < blen; t++) {
            const int pos = plen + t;
            br.ids.push_back(tok[t]);
            br.pos.push_back(pos);
            br.slot.push_back(tables[toff + pos / PAGE] * PAGE + pos % PAGE);
          }
          for (int u0 = 0; u0 < blen; u0 += kAttnRows) br.items.push_back({row0 + u0, std::min(kAttnRows, blen - u0), plen + u0, toff});
          auto term = [&](int o) -> std::vector<Term>& {
            return terms[((size_t)ri * nq + qi) * LAYA_MAX_OPTIONS + o];
          };
          if (Lo == 1) {
            const int read = (int)br.read_rows.size();
            br.read_rows.push_back(row0 + blen - 1);
            read_lse_br.push_back(false);
            for (int o = 0; o < Q.n_options; o++) term(o).push_back({add_cand(read, true, Q.options[o]), -1, true});
          } else {
            const int o = bi;
            if (S > 0) {
              const int read = (int)br.read_rows.size();
              br.read_rows.push_back(row0 + S - 1);
              read_lse_br.push_back(true);
              term(o).push_back({add_cand(read, true, Q.options[(size_t)o * Lo]), read, true});
            }
            for (int t = 0; t < Lo - 1; t++) {
              const int read = (int)br.read_rows.size();
              br.read_rows.push_back(row0 + S + t);
              read_lse_br.push_back(true);
              term(o).push_back({add_cand(read, true, Q.options[(size_t)o * Lo + t + 1]), read, true});
            }
          }
        }
      }
    }
    // ---- run
    const int R1 = (int)pre.read_rows.size(), R = R1 + (int)br.read_rows.size();
    if ((rc = ensure_kv(m, r, pages))) return rc;
    if ((rc = r.hid32.ensure((size_t)std::max(R, 1) * c.d * 4)) || (rc = r.hid16.ensure((size_t)std::max(R, 1) * c.d * 2)))
      return rc;
    r.arm_start = true;
    if ((rc = run_forward(m, r, pre, tables, 0, canceled, user, cancel_mu))) return rc;
    if (!br.ids.empty()) {
      if (!cow.empty()) {
        if ((rc = upload_many(r, {{&r.cow, cow.data(), cow.size() * sizeof(int2)}}))) return rc;
        const size_t page_elems = (size_t)c.KV * PAGE * c.hd;
        r.launches++;
        LAYA_CK(kv_copy(r.kc.as<half>(), r.vc.as<half>(), r.cow.as<int2>(), (int)cow.size(), page_elems,
                        page_elems * r.kv_pages, c.L, r.stream));
      }
      if ((rc = run_forward(m, r, br, tables, R1, canceled, user, cancel_mu))) return rc;
    }
    // ---- heads
    const int Nc = (int)cand_id.size();
    std::vector<int> cread(Nc);
    for (int k = 0; k < Nc; k++) cread[k] = cand_read[k] + (cand_is_branch[k] ? R1 : 0);
    if ((rc = upload_many(r, {{&r.cand, cand_id.data(), (size_t)Nc * 4}, {&r.row_of, cread.data(), (size_t)Nc * 4}})))
      return rc;
    if ((rc = r.clog.ensure((size_t)std::max(Nc, 1) * 4))) return rc;
    r.launches++;
    LAYA_CK(head_restricted(r.head, r.hid32.as<float>(), r.cand.as<int>(), r.row_of.as<int>(), Nc, r.clog.as<float>(),
                            r.stream));
    bool need_lse = false;
    for (char v : read_lse_pre) need_lse |= v;
    for (char v : read_lse_br) need_lse |= v;
    if (need_lse) {
      const int chunk = std::max(128, (int)((256ull << 20) / ((size_t)c.V * 4)) / 128 * 128);
      if ((rc = r.flog.ensure((size_t)std::min(chunk, R) * c.V * 4)) || (rc = r.lse.ensure((size_t)R * 4))) return rc;
      for (int q0 = 0; q0 < R; q0 += chunk) {
        const int mr = std::min(chunk, R - q0);
        GemmArgs a{};
        a.M = mr;
        a.N = c.V;
        a.K = c.d;
        a.out = r.flog.p;
        a.ldo = c.V;
        if ((rc = gemm(r, P_GEMM_HEAD, EPI_F32, r.hid16.as<half>() + (size_t)q0 * c.d, c.d, r.head16, c.d, a)))
          return rc;
        r.launches++;
        LAYA_CK(lse_rows(r.flog.as<float>(), c.V, mr, r.lse.as<float>() + q0, r.stream));
      }
    }
    if ((rc = timing_mark_end(r))) return rc;
    std::vector<float> clog(Nc), lse(need_lse ? R : 0);
    LAYA_CK(cudaMemcpyAsync(clog.data(), r.clog.p, (size_t)Nc * 4, cudaMemcpyDeviceToHost, r.stream));
    if (need_lse) LAYA_CK(cudaMemcpyAsync(lse.data(), r.lse.p, (size_t)R * 4, cudaMemcpyDeviceToHost, r.stream));
    r.d2h += (long long)Nc * 4 + (need_lse ? (long long)R * 4 : 0) + 4;
    LAYA_CK(cudaStreamSynchronize(r.stream));
    unsigned err = 0;
    LAYA_CK(cudaMemcpy(&err, r.err, 4, cudaMemcpyDeviceToHost));
    if (err) return fail(LAYA_E_TIMEOUT, "a device-side wait ran out of its budget (code " + std::to_string(err) + ")");
    if (r.prof) prof_collect(r);
    // ---- answers
    for (int ri = 0; ri < nr; ri++)
      for (int qi = 0; qi < nq; qi++) {
        const laya_question& Q = b.questions[qi];
        float logit[LAYA_MAX_OPTIONS];
        for (int o = 0; o < Q.n_options; o++) {
          double s = 0;
          for (const Term& t : terms[((size_t)ri * nq + qi) * LAYA_MAX_OPTIONS + o]) {
            double v = clog[t.cand];
            if (t.read >= 0) v -= lse[t.read + (t.branch ? R1 : 0)];
            s += v;
          }
          logit[o] = (float)s;
          if (!std::isfinite(logit[o])) return fail(LAYA_E_NONFINITE, "non-finite model output");
        }
        apply_rules(c, Q.kind, Q.n_options, logit, &out[(size_t)(i + ri) * nq + qi]);
      }
    i = j;
  }
  return 0;
}

}  // namespace laya
