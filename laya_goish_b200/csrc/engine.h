// Host engine of the decision hot path: one immutable weight replica per
// GPU ("backends own immutable weights; request-local state must not escape
// a call", src/models/mod.rs:12), a batched prefill + shared-prefix branch
// forward, heads and the decision rules.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm.h"
#include "gguf.h"
#include "kernels.h"
#include "laya_cuda.h"

namespace laya {

constexpr int PAGE = 64;  // tokens per KV page (one attention key block)

int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define LAYA_CK(x)                                 \
  do {                                             \
    cudaError_t e_ = (x);                          \
    if (e_ != cudaSuccess) return cuda_fail(e_, #x); \
  } while (0)

struct Config {
  std::string arch;
  int L = 0, d = 0, H = 0, KV = 0, hd = 0, ffn = 0, V = 0, ctx = 0;
  float eps = 1e-5f, theta = 1e4f;
  bool bias = false;
  int wkind = 0;
  bool quantized = false;  // any layer matrix stored in a block-quantised type
  float temperature[3] = {1, 1, 1};
  bool has_bucket[3][4] = {};
  float bucket[3][4] = {};
};

// Grow-only device buffer.
struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
  int ensure(size_t bytes);
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
  void release();
};

struct HostBuf {
  void* p = nullptr;
  size_t cap = 0;
  int ensure(size_t bytes);
  void release();
};

struct Layer {
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
  QTensor wq{}, wk{}, wv{}, wo{}, wg{}, wu{}, wd{};
  const float* bqkv = nullptr;
  // F16 operands of the tcgen05 GEMMs, resident for F16 models; null for
  // quantised models, which decode into per-layer staging before each GEMM.
  const half* wqkv16 = nullptr;
  const half* wgu16 = nullptr;  // gate/up rows interleaved per 128
  const half* wo16 = nullptr;
  const half* wd16 = nullptr;
  // Quantised models: F16 images of the same four operands for the prefill
  // GEMMs, decoded once (ensure_f16_cache) instead of before every GEMM.
  const half* rqkv16 = nullptr;
  const half* rgu16 = nullptr;
  const half* ro16 = nullptr;
  const half* rd16 = nullptr;
  // Q8_0 models: the block scales of the same four operands transposed to
  // [K/32][N] in the operands' row order, for the GEMM that decodes the int8
  // quants in shared memory (gemm_q8_launch); built by ensure_q8_scales.
  const half* sqkv_t = nullptr;
  const half* sgu_t = nullptr;
  const half* so_t = nullptr;
  const half* sd_t = nullptr;
};

struct ProfEvent {
  int cat;
  cudaEvent_t a, b;
};

struct Replica {
  int device = 0, num_sms = 148;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  // (address, bytes) of every weight allocation made while loading, in
  // allocation order: another replica of the same model is these buffers
  // copied device to device, with its pointers relocated
  std::vector<std::pair<void*, size_t>> wmap;
  bool loading = false;
  size_t weight_bytes = 0;
  std::vector<Layer> layers;
  QTensor embd{}, head{};
  const float* out_norm = nullptr;
  const half* head16 = nullptr;  // F16 lm_head for full-vocabulary rows (lazy for quantised models)
  const half* head_st = nullptr;  // Q8_0 lm_head: block scales as [d/32][V] (ensure_q8_scales)
  // Packed streaming images of the decode GEMV operands (gemv3_pack), built
  // on the first small-batch decode: per layer qkv, o, gate/up, down, then
  // the head; null where the streaming GEMV does not apply.
  std::vector<const uint8_t*> gv_packed;
  const float2* rope = nullptr;  // [ctx][hd/2] (cos, sin)
  unsigned* err = nullptr;
  std::map<std::string, QTensor> named;
  // scratch
  DevBuf ids, pos, slot, x, h, qb, att, act, items, tables, rows, hid32, hid16, cand, row_of, clog, flog, lse, cow;
  DevBuf wqkv_s, wo_s, wgu_s, wd_s;  // F16 staging of one layer (quantised models)
  DevBuf kpart;                      // K-split partial sums of the residual GEMMs (small M)
  bool f16_cache_failed = false;     // no room for the F16 operand cache: stage per GEMM
  DevBuf kc, vc;
  int kv_pages = 0;
  HostBuf pin;
  // decode scratch
  DevBuf dx16, dlogits, dargmax, dpart;
  // timing of the current call
  bool arm_start = false;
  cudaEvent_t ev_start = nullptr, ev_end = nullptr;
  double call_ms = 0;
  long long launches = 0, h2d = 0, d2h = 0;
  // profiling
  bool prof = false;
  std::vector<ProfEvent> prof_events;
  std::vector<cudaEvent_t> event_pool;
  std::map<std::string, std::pair<long long, double>> prof_acc;
};

struct Model {
  Config cfg;
  std::vector<Replica> reps;
  std::mutex mu;  // calls on one model are serialised
};

// Token-level plan of one forward pass (prefill or branch).
struct PassPlan {
  std::vector<int> ids, pos, slot;
  std::vector<AttnItem> items;
  std::vector<int> read_rows;  // rows whose final-normed hidden is needed
};

std::string read_config(const Gguf& g, Config* c);
int load_replica(Model& m, const Gguf& g, int device, Replica& r);
// Copies loaded replicas to the other devices over NVLink: replicas[0] is
// loaded from the file, then every loaded replica copies itself to one
// unloaded device per round (1 -> 2 -> 4 -> 8 replicas).  Devices without
// peer access copy through the host (cudaMemcpyPeerAsync).
int mirror_replicas(Model& m, const std::vector<int>& devices);
void free_replica(Replica& r);
int ensure_kv(Model& m, Replica& r, int pages);
int run_forward(Model& m, Replica& r, const PassPlan& p, const std::vector<int>& tables, int read_base,
                int (*canceled)(void*), void* user, std::mutex* cancel_mu);
int ensure_head16(Model& m, Replica& r);
// Quantised models: decodes every layer's GEMM operands to resident F16 once
// (about 2 bytes per weight; skipped, and the per-GEMM staging kept, when the
// memory is not there or LAYA_F16_CACHE=0).
int ensure_f16_cache(Model& m, Replica& r);
// Whether a pass of M token rows runs its layer GEMMs on the Q8_0 blocks
// themselves (gemm_q8_launch): every layer matrix Q8_0, every GEMM's K and
// the q / k widths multiples of 128, and M at most LAYA_Q8_FUSED_MAX_M
// (default 256, where the weight bytes bound the pass); LAYA_Q8_FUSED=0
// turns it off.  The variables are read at every call.
bool use_q8_gemm(const Model& m, const Replica& r, int M);
// Builds the transposed block scales of every layer (and of a Q8_0 lm_head
// with V % 8 == 0) once: 1/16 byte per weight.
int ensure_q8_scales(Model& m, Replica& r);
// The four GEMM operands of layer L, and a Q8_0 lm_head, as Q8_0 blocks.
Q8Weights q8_qkv(const Config& c, const Layer& L);
Q8Weights q8_gu(const Config& c, const Layer& L);
Q8Weights q8_o(const Config& c, const Layer& L);
Q8Weights q8_down(const Config& c, const Layer& L);
Q8Weights q8_head(const Replica& r);
int decide_shard(Model& m, Replica& r, const laya_batch& b, int r0, int r1, laya_answer* out,
                 int (*canceled)(void*), void* user, std::mutex* cancel_mu);
int validate_batch(const Config& c, const laya_batch* b);
int decode_run(Model& m, Replica& r, const int32_t* ids, const int64_t* off, int n_seqs, int steps, int32_t* out,
               float* stats);

// profiling helpers
enum ProfCat { P_GEMM_QKV, P_GEMM_O, P_GEMM_GU, P_GEMM_DOWN, P_GEMM_HEAD, P_ATTN, P_DEQUANT, P_GEMV, P_ATTN_DEC, P_NCAT };
extern const char* kProfNames[P_NCAT];
void prof_begin(Replica& r, int cat, cudaEvent_t* a);
void prof_end(Replica& r, int cat, cudaEvent_t a);
void prof_collect(Replica& r);
int timing_begin_call(Replica& r);
int timing_mark_start(Replica& r);
int timing_mark_end(Replica& r);

}  // namespace laya
