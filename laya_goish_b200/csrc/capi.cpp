// extern "C" entry points of laya_cuda.h.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "engine.h"
#include "gemm.h"
#include "laya_cuda.h"

using namespace laya;

namespace laya {
extern thread_local std::string g_err;
}

struct laya_model {
  Model m;
};

static int open_common(Gguf& g, const int* devices, int n_devices, laya_model** out) {
  if (!out) return fail(LAYA_E_INVALID, "null output handle");
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev < 1) return fail(LAYA_E_CUDA, "no CUDA device");
  std::vector<int> devs;
  if (!devices || n_devices <= 0)
    devs.push_back(0);
  else
    devs.assign(devices, devices + n_devices);
  for (int d : devs)
    if (d < 0 || d >= ndev) return fail(LAYA_E_INVALID, "invalid device index " + std::to_string(d));
  auto h = std::make_unique<laya_model>();
  std::string e = read_config(g, &h->m.cfg);
  if (!e.empty()) return fail(LAYA_E_FORMAT, e);
  h->m.reps.resize(devs.size());
  {
    // create the devices' contexts at once (a few hundred ms each)
    std::vector<int> uniq(devs);
    std::sort(uniq.begin(), uniq.end());
    uniq.erase(std::unique(uniq.begin(), uniq.end()), uniq.end());
    std::vector<std::thread> ts;
    for (int d : uniq)
      ts.emplace_back([d] {
        if (cudaSetDevice(d) == cudaSuccess) cudaFree(nullptr);
      });
    for (auto& t : ts) t.join();
  }
  // One replica from the file; the others copied device to device over
  // NVLink (LAYA_LOAD_PEER=0: every replica from the file).
  const char* pe = std::getenv("LAYA_LOAD_PEER");
  const bool peer = !(pe && pe[0] == '0');
  for (size_t i = 0; i < (peer ? 1 : devs.size()); i++) {
    if (int rc = load_replica(h->m, g, devs[i], h->m.reps[i])) {
      for (auto& r : h->m.reps) free_replica(r);
      return rc;
    }
  }
  if (peer && devs.size() > 1) {
    if (int rc = mirror_replicas(h->m, devs)) {
      for (auto& r : h->m.reps) free_replica(r);
      return rc;
    }
  }
  *out = h.release();
  return 0;
}

extern "C" {

const char* laya_last_error(void) { return g_err.c_str(); }

int laya_open(const char* path, const int* devices, int n_devices, laya_model** out) {
  if (!path) return fail(LAYA_E_INVALID, "null path");
  Gguf g;
  std::string e = g.open_file(path);
  if (!e.empty()) return fail(g.bytes() ? LAYA_E_FORMAT : LAYA_E_IO, e);
  return open_common(g, devices, n_devices, out);
}

int laya_open_memory(const uint8_t* gguf, size_t len, const int* devices, int n_devices, laya_model** out) {
  if (!gguf && len) return fail(LAYA_E_INVALID, "null GGUF image");
  Gguf g;
  static const uint8_t empty[1] = {0};
  std::string e = g.open_memory(gguf ? gguf : empty, len);
  if (!e.empty()) return fail(LAYA_E_FORMAT, e);
  return open_common(g, devices, n_devices, out);
}

int laya_layers(const laya_model* m) { return m ? m->m.cfg.L : fail(LAYA_E_INVALID, "null model"); }

int laya_info(const laya_model* m, laya_model_info* out) {
  if (!m || !out) return fail(LAYA_E_INVALID, "null argument");
  const Config& c = m->m.cfg;
  std::memset(out, 0, sizeof(*out));
  std::strncpy(out->architecture, c.arch.c_str(), sizeof(out->architecture) - 1);
  out->layers = c.L;
  out->d_model = c.d;
  out->heads = c.H;
  out->kv_heads = c.KV;
  out->head_dim = c.hd;
  out->ffn = c.ffn;
  out->vocab = c.V;
  out->context = c.ctx;
  out->weight_kind = c.wkind;
  out->n_devices = (int)m->m.reps.size();
  out->device_bytes = m->m.reps.empty() ? 0 : (int64_t)m->m.reps[0].weight_bytes;
  return 0;
}

int laya_validate(const laya_model* m, const laya_batch* b) {
  if (!m) return fail(LAYA_E_INVALID, "null model");
  return validate_batch(m->m.cfg, b);
}

int laya_decide_batch(laya_model* h, const laya_batch* b, laya_answer* out, int (*canceled)(void*), void* user) {
  if (!h) return fail(LAYA_E_INVALID, "null model");
  Model& m = h->m;
  std::lock_guard<std::mutex> lk(m.mu);
  if (int rc = validate_batch(m.cfg, b)) return rc;
  if (b->n_requests == 0) return 0;
  if (!out) return fail(LAYA_E_INVALID, "null answer buffer");
  const int nd = (int)m.reps.size();
  if (nd == 1 || b->n_requests == 1)
    return decide_shard(m, m.reps[0], *b, 0, b->n_requests, out, canceled, user, nullptr);
  // Shard contiguous request ranges across devices, balanced by prompt tokens;
  // one host thread per device; the batch fails as a whole on any error.
  std::vector<int> cut(nd + 1, b->n_requests);
  cut[0] = 0;
  const int64_t total = b->offsets[b->n_requests];
  int k = 1;
  for (int i = 0; i < b->n_requests && k < nd; i++)
    if (b->offsets[i + 1] * nd >= total * k) cut[k++] = i + 1;
  std::vector<int> rcs(nd, 0);
  std::vector<std::string> msgs(nd);
  std::mutex cancel_mu;
  std::vector<std::thread> th;
  for (int d = 0; d < nd; d++) {
    th.emplace_back([&, d] {
      if (cut[d] < cut[d + 1]) {
        rcs[d] = decide_shard(m, m.reps[d], *b, cut[d], cut[d + 1], out, canceled, user, &cancel_mu);
        if (rcs[d]) msgs[d] = g_err;
      }
    });
  }
  for (auto& t : th) t.join();
  for (int d = 0; d < nd; d++)
    if (rcs[d]) return fail(rcs[d], msgs[d]);
  return 0;
}

int laya_decode(laya_model* h, const int32_t* ids, const int64_t* offsets, int n_seqs, int steps, int32_t* out_tokens,
                float* stats) {
  if (!h || !ids || !offsets || !out_tokens) return fail(LAYA_E_INVALID, "null argument");
  Model& m = h->m;
  std::lock_guard<std::mutex> lk(m.mu);
  if (offsets[0] != 0) return fail(LAYA_E_INVALID, "offsets[0] must be 0");
  const int nd = std::min((int)m.reps.size(), std::max(n_seqs, 1));
  if (nd <= 1) return decode_run(m, m.reps[0], ids, offsets, n_seqs, steps, out_tokens, stats);
  std::vector<int> rcs(nd, 0);
  std::vector<std::string> msgs(nd);
  std::vector<std::vector<float>> st(nd, std::vector<float>(2, 0.f));
  std::vector<std::thread> th;
  for (int d = 0; d < nd; d++) {
    th.emplace_back([&, d] {
      const int s0 = (int)((int64_t)n_seqs * d / nd), s1 = (int)((int64_t)n_seqs * (d + 1) / nd);
      std::vector<int64_t> off(s1 - s0 + 1);
      for (int i = s0; i <= s1; i++) off[i - s0] = offsets[i] - offsets[s0];
      rcs[d] = decode_run(m, m.reps[d], ids + offsets[s0], off.data(), s1 - s0, steps, out_tokens + (size_t)s0 * steps,
                          st[d].data());
      if (rcs[d]) msgs[d] = g_err;
    });
  }
  for (auto& t : th) t.join();
  for (int d = 0; d < nd; d++)
    if (rcs[d]) return fail(rcs[d], msgs[d]);
  if (stats) {
    stats[0] = stats[1] = 0;
    for (auto& s : st) {
      stats[0] = std::max(stats[0], s[0]);
      stats[1] = std::max(stats[1], s[1]);
    }
  }
  return 0;
}

void laya_close(laya_model* h) {
  if (!h) return;
  for (auto& r : h->m.reps) free_replica(r);
  delete h;
}

int laya_forward(laya_model* h, const int32_t* ids, int n, const int32_t* read, int nread, float* out) {
  if (!h || !ids || !read || !out) return fail(LAYA_E_INVALID, "null argument");
  Model& m = h->m;
  std::lock_guard<std::mutex> lk(m.mu);
  const Config& c = m.cfg;
  if (n < 1 || n > c.ctx || nread < 1) return fail(LAYA_E_INVALID, "invalid token sequence");
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= c.V) return fail(LAYA_E_INVALID, "invalid token sequence");
  for (int i = 0; i < nread; i++)
    if (read[i] < 0 || read[i] >= n) return fail(LAYA_E_INVALID, "invalid read position");
  Replica& r = m.reps[0];
  if (cudaSetDevice(r.device) != cudaSuccess) return fail(LAYA_E_CUDA, "cudaSetDevice");
  PassPlan p;
  std::vector<int> tables;
  const int pages = (n + PAGE - 1) / PAGE;
  for (int i = 0; i < pages; i++) tables.push_back(i);
  for (int t = 0; t < n; t++) {
    p.ids.push_back(ids[t]);
    p.pos.push_back(t);
    p.slot.push_back(t);
  }
  for (int t0 = 0; t0 < n; t0 += kAttnRows) p.items.push_back({t0, std::min(kAttnRows, n - t0), t0, 0});
  p.read_rows.assign(read, read + nread);
  int rc;
  if ((rc = ensure_kv(m, r, pages)) || (rc = r.hid32.ensure((size_t)nread * c.d * 4)) ||
      (rc = r.hid16.ensure((size_t)nread * c.d * 2)))
    return rc;
  if (cudaMemsetAsync(r.err, 0, 4, r.stream) != cudaSuccess) return fail(LAYA_E_CUDA, "cudaMemsetAsync");
  if ((rc = run_forward(m, r, p, tables, 0, nullptr, nullptr, nullptr))) return rc;
  LAYA_CK(cudaMemcpyAsync(out, r.hid32.p, (size_t)nread * c.d * 4, cudaMemcpyDeviceToHost, r.stream));
  LAYA_CK(cudaStreamSynchronize(r.stream));
  unsigned err = 0;
  LAYA_CK(cudaMemcpy(&err, r.err, 4, cudaMemcpyDeviceToHost));
  if (err) return fail(LAYA_E_TIMEOUT, "a device-side wait ran out of its budget");
  if (r.prof) prof_collect(r);
  return 0;
}

int laya_tensor_f32(laya_model* h, const char* name, float* out, size_t max_elems) {
  if (!h || !name || !out) return fail(LAYA_E_INVALID, "null argument");
  Model& m = h->m;
  std::lock_guard<std::mutex> lk(m.mu);
  Replica& r = m.reps[0];
  auto it = r.named.find(name);
  if (it == r.named.end()) return fail(LAYA_E_INVALID, std::string("no device tensor ") + name);
  const QTensor& t = it->second;
  const size_t n = (size_t)t.rows * t.cols;
  if (n > max_elems) return fail(LAYA_E_INVALID, "output buffer too small");
  if (cudaSetDevice(r.device) != cudaSuccess) return fail(LAYA_E_CUDA, "cudaSetDevice");
  DevBuf tmp;
  if (int rc = tmp.ensure(n * 4)) return rc;
  cudaError_t e = rows_f32(t, nullptr, t.rows, tmp.as<float>(), r.stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, tmp.p, n * 4, cudaMemcpyDeviceToHost, r.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(r.stream);
  tmp.release();
  if (e != cudaSuccess) return cuda_fail(e, "laya_tensor_f32");
  return 0;
}

// Frees a call's temporary device buffers on every return path.
struct ReleaseOnExit {
  std::vector<DevBuf*> bufs;
  ~ReleaseOnExit() {
    for (DevBuf* b : bufs) b->release();
  }
};

int laya_wait_selftest(int device, long long budget_cycles) {
  if (budget_cycles < 1 || budget_cycles > 4000000000ll) return fail(LAYA_E_INVALID, "budget out of range");
  LAYA_CK(cudaSetDevice(device));
  DevBuf derr;
  ReleaseOnExit guard{{&derr}};
  if (int rc = derr.ensure(16)) return rc;
  cudaError_t e = cudaMemset(derr.p, 0, 16);
  if (e == cudaSuccess) e = wait_probe(derr.as<unsigned>(), budget_cycles, 0);
  unsigned err = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&err, derr.p, 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "laya_wait_selftest");
  if (err) return fail(LAYA_E_TIMEOUT, "a device-side wait ran out of its budget");
  return 0;
}

int laya_dequantize(int device, uint32_t kind, const uint8_t* blocks, size_t nbytes, float* out) {
  int block, size;
  if (!ggml_layout(kind, &block, &size)) return fail(LAYA_E_INVALID, "unsupported GGML tensor type");
  if (!blocks || !out) return fail(LAYA_E_INVALID, "null argument");
  const size_t nb = nbytes / (size_t)size;
  if (!nb) return 0;
  LAYA_CK(cudaSetDevice(device));
  DevBuf din, dout;
  ReleaseOnExit guard{{&din, &dout}};
  int rc;
  if ((rc = din.ensure(nb * size)) || (rc = dout.ensure(nb * block * 4))) return rc;
  cudaError_t e = cudaMemcpy(din.p, blocks, nb * size, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = dequant_raw((int)kind, din.as<uint8_t>(), nb, dout.as<float>(), 0);
  if (e == cudaSuccess) e = cudaMemcpy(out, dout.p, nb * block * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "laya_dequantize");
  return 0;
}

int laya_gated_delta(int device, const float* qkv, const float* a, const float* b, const float* dt,
                     const float* alog, int s, int nh, int hk, float* out) {
  if (!qkv || !a || !b || !dt || !alog || !out || s < 0 || nh < 1 || (hk != 64 && hk != 128))
    return fail(LAYA_E_INVALID, "invalid DeltaNet arguments (hk must be 64 or 128)");
  if (s == 0) return 0;
  LAYA_CK(cudaSetDevice(device));
  const size_t w = (size_t)nh * hk, nq = (size_t)s * 3 * w, nab = (size_t)s * nh, no = (size_t)s * w;
  DevBuf dq, da, db, dp, dkq, dout;
  ReleaseOnExit guard{{&dq, &da, &db, &dp, &dkq, &dout}};
  int rc;
  if ((rc = dq.ensure(nq * 4)) || (rc = da.ensure(nab * 4)) || (rc = db.ensure(nab * 4)) ||
      (rc = dp.ensure((size_t)2 * nh * 4)) || (rc = dkq.ensure(gated_delta_scratch(s, nh))) ||
      (rc = dout.ensure(no * 4)))
    return rc;
  float* dpar = dp.as<float>();
  cudaError_t e = cudaMemcpy(dq.p, qkv, nq * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(da.p, a, nab * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(db.p, b, nab * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dpar, dt, (size_t)nh * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dpar + nh, alog, (size_t)nh * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = gated_delta(dq.as<float>(), da.as<float>(), db.as<float>(), nh, dpar, dpar + nh, s, nh, hk, da.as<float>(),
                    db.as<float>(), dkq.as<float>(), dout.as<float>(), 0);
  if (e == cudaSuccess) e = cudaMemcpy(out, dout.p, no * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "laya_gated_delta");
  return 0;
}

int laya_gated_delta_mixer(int device, const float* raw, const float* z, const float* a, const float* b,
                           const float* conv, const float* dt, const float* alog, const float* normw, int s, int nh,
                           int hk, float* out) {
  if (!raw || !z || !a || !b || !conv || !dt || !alog || !normw || !out || s < 0 || nh < 1 || (hk != 64 && hk != 128))
    return fail(LAYA_E_INVALID, "invalid DeltaNet mixer arguments (hk must be 64 or 128)");
  if (s == 0) return 0;
  LAYA_CK(cudaSetDevice(device));
  const size_t w = (size_t)nh * hk, nr = (size_t)s * 3 * w, nz = (size_t)s * w, nab = (size_t)s * nh;
  DevBuf draw, dz, da, db, dconv, dpar, dsc, dout;
  ReleaseOnExit guard{{&draw, &dz, &da, &db, &dconv, &dpar, &dsc, &dout}};
  int rc;
  if ((rc = draw.ensure(nr * 4)) || (rc = dz.ensure(nz * 4)) || (rc = da.ensure(nab * 4)) ||
      (rc = db.ensure(nab * 4)) || (rc = dconv.ensure(3 * w * 4 * 4)) || (rc = dpar.ensure(((size_t)2 * nh + hk) * 4)) ||
      (rc = dsc.ensure(gated_delta_mixer_scratch(s, nh, hk))) || (rc = dout.ensure(nz * 4)))
    return rc;
  float* p = dpar.as<float>();
  cudaError_t e = cudaMemcpy(draw.p, raw, nr * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dz.p, z, nz * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(da.p, a, nab * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(db.p, b, nab * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dconv.p, conv, 3 * w * 4 * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(p, dt, (size_t)nh * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(p + nh, alog, (size_t)nh * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(p + 2 * nh, normw, (size_t)hk * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = gated_delta_mixer(draw.as<float>(), (int)(3 * w), dz.as<float>(), (int)w, da.as<float>(), db.as<float>(), nh,
                          dconv.as<float>(), p, p + nh, p + 2 * nh, s, nh, hk, dsc.as<float>(), dout.as<float>(),
                          nullptr, 0);
  if (e == cudaSuccess) e = cudaMemcpy(out, dout.p, nz * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "laya_gated_delta_mixer");
  return 0;
}

int laya_gated_attention(int device, const float* qgate, const float* k, const float* v, const float* qn,
                         const float* kn, int s, int H, int KV, int hd, int rot, float theta, float* out) {
  if (!qgate || !k || !v || !qn || !kn || !out || s < 0 || H < 1 || KV < 1 || H % KV ||
      (hd != 64 && hd != 128 && hd != 256) || rot < 0 || rot > hd || rot % 2)
    return fail(LAYA_E_INVALID, "invalid gated-attention arguments");
  if (s == 0) return 0;
  LAYA_CK(cudaSetDevice(device));
  const size_t nq = (size_t)s * H * 2 * hd, nk = (size_t)s * KV * hd, no = (size_t)s * H * hd;
  DevBuf dq, dk, dv, dn, dsc, dout, derr;
  ReleaseOnExit guard{{&dq, &dk, &dv, &dn, &dsc, &dout, &derr}};
  int rc;
  if ((rc = dq.ensure(nq * 4)) || (rc = dk.ensure(nk * 4)) || (rc = dv.ensure(nk * 4)) ||
      (rc = dn.ensure((size_t)2 * hd * 4)) || (rc = dsc.ensure(gated_attention_scratch(s, H, KV, hd))) ||
      (rc = dout.ensure(no * 2)) || (rc = derr.ensure(16)))
    return rc;
  float* dnw = dn.as<float>();
  cudaError_t e = cudaMemcpy(dq.p, qgate, nq * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dk.p, k, nk * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dv.p, v, nk * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dnw, qn, (size_t)hd * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dnw + hd, kn, (size_t)hd * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(derr.p, 0, 16);
  if (e == cudaSuccess)
    e = gated_attention(dq.as<float>(), 2 * H * hd, dk.as<float>(), dv.as<float>(), KV * hd, dnw, dnw + hd, s, H, KV,
                        hd, rot, theta, dsc.p, dout.as<half>(), derr.as<unsigned>(), 0);
  std::vector<uint16_t> o16(no);
  if (e == cudaSuccess) e = cudaMemcpy(o16.data(), dout.p, no * 2, cudaMemcpyDeviceToHost);
  unsigned err = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&err, derr.p, 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "laya_gated_attention");
  if (err) return fail(LAYA_E_TIMEOUT, "a device-side wait ran out of its budget");
  for (size_t i = 0; i < no; i++) out[i] = half_bits(o16[i]);
  return 0;
}

int laya_matrix_apply(int device, uint32_t kind, const uint8_t* w, int rows, int cols, const float* x, int m,
                      const float* bias, float* out) {
  int block, size;
  if (!ggml_layout(kind, &block, &size)) return fail(LAYA_E_INVALID, "unsupported GGML tensor type");
  if (!w || !x || !out || rows < 1 || cols < 1 || m < 0 || cols % block)
    return fail(LAYA_E_INVALID, "invalid matrix arguments");
  if (m == 0) return 0;
  LAYA_CK(cudaSetDevice(device));
  cudaDeviceProp prop;
  LAYA_CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return fail(LAYA_E_CUDA, "not an sm_100 GPU");
  const int ld = (cols + 7) / 8 * 8;
  const size_t wbytes = (size_t)rows * cols / block * size;
  DevBuf dw, dwf, dw16, dx, dx16, db, dy, derr;
  ReleaseOnExit guard{{&dw, &dwf, &dw16, &dx, &dx16, &db, &dy, &derr}};
  int rc;
  if ((rc = dw.ensure(wbytes)) || (rc = dwf.ensure((size_t)rows * cols * 4)) ||
      (rc = dw16.ensure((size_t)rows * ld * 2)) || (rc = dx.ensure((size_t)m * cols * 4)) ||
      (rc = dx16.ensure((size_t)m * ld * 2)) || (rc = db.ensure((size_t)rows * 4)) ||
      (rc = dy.ensure((size_t)m * rows * 4)) || (rc = derr.ensure(16)))
    return rc;
  cudaError_t e = cudaMemcpy(dw.p, w, wbytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dx.p, x, (size_t)m * cols * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && bias) e = cudaMemcpy(db.p, bias, (size_t)rows * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(derr.p, 0, 16);
  if (e == cudaSuccess) e = dequant_raw((int)kind, dw.as<uint8_t>(), wbytes / size, dwf.as<float>(), 0);
  if (e == cudaSuccess) e = f32_to_f16_pad(dwf.as<float>(), rows, cols, ld, dw16.as<half>(), 0);
  if (e == cudaSuccess) e = f32_to_f16_pad(dx.as<float>(), m, cols, ld, dx16.as<half>(), 0);
  if (e == cudaSuccess) {
    GemmArgs a{};
    a.M = m;
    a.N = rows;
    a.K = cols;
    a.bias = bias ? db.as<float>() : nullptr;
    a.out = dy.p;
    a.ldo = rows;
    a.err = derr.as<unsigned>();
    a.budget = 4000000000ll;
    e = gemm_launch(EPI_F32, dx16.as<half>(), ld, dw16.as<half>(), ld, a, prop.multiProcessorCount, 0);
  }
  if (e == cudaSuccess) e = cudaMemcpy(out, dy.p, (size_t)m * rows * 4, cudaMemcpyDeviceToHost);
  unsigned err = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&err, derr.p, 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "laya_matrix_apply");
  if (err) return fail(LAYA_E_TIMEOUT, "a device-side wait ran out of its budget");
  return 0;
}

int laya_last_timing(const laya_model* h, laya_timing* out) {
  if (!h || !out) return fail(LAYA_E_INVALID, "null argument");
  std::memset(out, 0, sizeof(*out));
  for (const auto& r : h->m.reps) {
    out->device_ms = std::max(out->device_ms, r.call_ms);
    out->launches += r.launches;
    out->h2d_bytes += r.h2d;
    out->d2h_bytes += r.d2h;
  }
  return 0;
}

int laya_profile_enable(laya_model* h, int enable) {
  if (!h) return fail(LAYA_E_INVALID, "null model");
  std::lock_guard<std::mutex> lk(h->m.mu);
  for (auto& r : h->m.reps) r.prof = enable != 0;
  return 0;
}

int laya_profile_read(laya_model* h, laya_profile_entry* out, int max) {
  if (!h) return fail(LAYA_E_INVALID, "null model");
  std::lock_guard<std::mutex> lk(h->m.mu);
  std::map<std::string, std::pair<long long, double>> acc;
  for (auto& r : h->m.reps) {
    for (auto& kv : r.prof_acc) {
      acc[kv.first].first += kv.second.first;
      acc[kv.first].second += kv.second.second;
    }
    r.prof_acc.clear();
  }
  int n = 0;
  for (auto& kv : acc) {
    if (out && n < max) {
      std::memset(&out[n], 0, sizeof(out[n]));
      std::strncpy(out[n].name, kv.first.c_str(), sizeof(out[n].name) - 1);
      out[n].launches = kv.second.first;
      out[n].total_ms = kv.second.second;
    }
    n++;
  }
  return n;
}

}  // extern "C"
