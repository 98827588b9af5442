/*
 * CPU oracle for the Laya Goish decision hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference Rust CPU engine
 * (panudetjt/laya-goish), used solely as the parity checker for the CUDA
 * library and as the timed CPU baseline.  The product never links, loads or
 * calls it.  Each function cites the reference file:line it restates.
 *
 * Parity pins (see tests/test_oracle.py): the reference's own known-answer
 * tests (src/tensor.rs:196-218, src/models/laya/decision.rs:331-333), the
 * malformed-GGUF cases of validation/smoke.py:13 and
 * validation/test_registry.py:34-35, and golden dequantisation vectors
 * produced by gguf-py (tests/golden/make_golden.py).  The full decoder
 * forward has no reference-side golden output (the reference has no Llama/
 * Qwen2 decoder): that part is "parity unpinned" and is defined by this
 * restatement of the reference equations.
 */
#ifndef LAYA_ORACLE_H
#define LAYA_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/gguf.rs:226-246 */
float or_half(uint16_t x);
/* src/gguf.rs:81-93: returns 0 and fills block/size, or -1 for an unsupported kind */
int or_layout(uint32_t kind, int* block, int* size);
/* src/gguf.rs:250-336: out receives nbytes/size*block floats */
int or_decode(uint32_t kind, const uint8_t* b, size_t nbytes, float* out);

/* src/gguf.rs:95-180: validates a GGUF image; 0 on success, -1 with a message */
int or_gguf_check(const uint8_t* bytes, size_t n, char* err, size_t errlen);

/* src/tensor.rs:10-102: out[m][n] = x[m][k] . W[n][k]^T (+bias), AVX2/FMA, row split over threads */
void or_matrix_apply(const float* w, int rows, int cols, const float* x, int m,
                     const float* bias, int threads, float* out);
/* src/tensor.rs:132-140 */
void or_softmax(const float* x, int n, float* p);

/* OpenThai sequence mixers on one sequence x[s][d] -> out[s][d] (openthai.c):
 * gated full attention (Full::run, src/models/openthai/model.rs:243-299) and
 * the gated DeltaNet recurrence (Delta::run, model.rs:301-363).  Matrices are
 * row-major [out rows][in cols] F32.  Return 0, or < 0 on bad shapes. */
int or_ot_full(const float* x, int s, int d, int H, int KV, int hd, int rot, float theta, const float* wq,
               const float* wk, const float* wv, const float* wo, const float* qn, const float* kn, int threads,
               float* out);
int or_ot_full_core(const float* qgate, const float* k, const float* v, const float* qn, const float* kn, int s,
                    int H, int KV, int hd, int rot, float theta, float* out);
int or_ot_delta_core(const float* qkv, const float* a, const float* b, const float* dt, const float* alog, int s,
                     int nh, int hk, float* out);
int or_ot_delta_mid(const float* raw, const float* z, const float* a, const float* b, const float* conv,
                    const float* dt, const float* alog, const float* normw, int s, int nh, int hk, float* out);
int or_ot_delta(const float* x, int s, int d, int nh, int hk, const float* wqkv, const float* wz, const float* wa,
                const float* wb, const float* wo, const float* conv, const float* dt, const float* alog,
                const float* normw, int threads, float* out);
/* src/models/laya/decision.rs:155-167 */
float or_confidence(const float* p, int n);

typedef struct or_model or_model;

/* Loads a llama/qwen2 GGUF image and dequantises every matrix to F32, as the
 * reference does at load (src/models/openthai/model.rs:53-63, 96-191). */
or_model* or_model_load(const uint8_t* bytes, size_t n, int threads, char* err, size_t errlen);
void or_model_free(or_model* m);
int or_model_dim(const or_model* m, int what); /* 0 d, 1 layers, 2 vocab, 3 heads, 4 kv, 5 hd, 6 ffn */

/* Causal forward over ids[0..n), returning the final-normed hidden rows at
 * read positions (src/models/openthai/model.rs:192-241 with Llama
 * conventions).  out: nread*d floats.  0 on success. */
int or_forward(or_model* m, const int32_t* ids, int n, const int32_t* read, int nread, float* out);

/* The same forward with a K/V cache, so a shared prefix is computed once
 * and then extended (question suffixes, option continuations, greedy
 * decode).  or_cache_forward appends ids[0..n) at positions len..len+n-1 and
 * returns the final-normed hidden rows at read[] (indices into the n new
 * tokens); or_cache_truncate(c, n) drops every token from position n on.  The
 * rows are bit-identical to or_forward over the whole sequence. */
typedef struct or_cache or_cache;
or_cache* or_cache_new(const or_model* m, int capacity);
void or_cache_free(or_cache* c);
int or_cache_len(const or_cache* c);
int or_cache_truncate(or_cache* c, int n);
int or_cache_forward(or_model* m, or_cache* c, const int32_t* ids, int n, const int32_t* read, int nread, float* out);
/* Timing only: positions 0..n-1 cached with arbitrary values. */
int or_cache_fill_timing(or_cache* c, const or_model* m, int n);
/* Threads of the attention loop (default 1, as in the reference, whose
 * attention is single-threaded; more threads give the same bits). */
void or_model_attn_threads(or_model* m, int n);

/* Head logits for hidden rows: for each row, the logits of cand ids
 * (ncand > 0) or of the whole vocabulary (ncand == 0).  out: rows*(ncand or V). */
int or_head(or_model* m, const float* hidden, int rows, const int32_t* cand, int ncand, float* out);

/* One decide question for one request, restating src/models/laya/decision.rs:186-268
 * (one forward per question).  option_len == 1: restricted softmax over the
 * candidate logits.  option_len > 1: each option's score is the summed
 * full-vocabulary log-probability of its tokens.  Outputs: logits[k],
 * probs[k], choice/score/noul/confidence. */
typedef struct {
  int32_t kind, n_options, option_len, suffix_len;
  const int32_t* options;
  const int32_t* suffix;
} or_question;
typedef struct {
  int32_t kind, n_options, choice;
  float score, noul, confidence;
  float probabilities[16];
  float logits[16];
} or_answer;
int or_decide(or_model* m, const int32_t* ids, int n, const or_question* q, or_answer* out);

#ifdef __cplusplus
}
#endif
#endif
