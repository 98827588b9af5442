/*
 * laya_cuda.h — C ABI of the B200-native decision hot path of Laya Goish.
 *
 * The library owns all device memory; callers own every host buffer they
 * pass.  Only C types cross this boundary (no CUDA or torch types), so the
 * reference engine's Rust side can bind it with plain `extern "C"`
 * declarations.
 *
 * Status codes: 0 on success, a negative LAYA_E_* otherwise; the message of
 * the last failure on the calling thread is returned by laya_last_error().
 * These mirror the reference's Result<_, String> error classes, which its
 * server maps to 422 (invalid), 408 (canceled) and 500 (others)
 * (src/server.rs:263-318).
 */
#ifndef LAYA_CUDA_H
#define LAYA_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LAYA_OK 0
#define LAYA_E_INVALID (-1)     /* request or argument validation failed (422) */
#define LAYA_E_CANCELED (-2)    /* the cancel callback fired (408)             */
#define LAYA_E_CUDA (-3)        /* a CUDA call failed                          */
#define LAYA_E_TIMEOUT (-4)     /* a device-side wait ran out of its budget    */
#define LAYA_E_NONFINITE (-5)   /* non-finite model output                     */
#define LAYA_E_NOMEM (-6)       /* device or host allocation failed            */
#define LAYA_E_IO (-7)          /* the GGUF file could not be opened / mapped  */
#define LAYA_E_FORMAT (-8)      /* malformed or unsupported GGUF               */

#define LAYA_MAX_OPTIONS 16

/* Question kinds, in the reference's order ["choice", "score", "noul"]
 * (src/models/laya/decision.rs:196). */
#define LAYA_CHOICE 0
#define LAYA_SCORE 1
#define LAYA_NOUL 2

typedef struct laya_model laya_model;

/* One question, shared by every request of a batch (as the reference's
 * /v1/decide/batch shares `questions` across states, src/server.rs:235-258).
 * option_len == 1: options are single candidate tokens read at the end of
 *   prompt+suffix, decoded with the restricted softmax over the candidate
 *   logits (src/models/openthai/decision.rs:268-279).
 * option_len > 1: each option is a continuation scored by the sum of its
 *   tokens' full-vocabulary log-probabilities, then softmaxed over options. */
typedef struct laya_question {
  int32_t kind;
  int32_t n_options;       /* 1..16; LAYA_NOUL needs exactly 2 */
  int32_t option_len;      /* >= 1 */
  const int32_t* options;  /* n_options * option_len token ids */
  int32_t suffix_len;      /* tokens appended to each prompt before reading */
  const int32_t* suffix;
} laya_question;

typedef struct laya_batch {
  int32_t n_requests;
  const int32_t* ids;       /* all prompts, concatenated */
  const int64_t* offsets;   /* n_requests + 1, offsets[0] == 0 */
  int32_t n_questions;
  const laya_question* questions;
} laya_batch;

/* One answer per (request, question), request-major.  Fields follow the
 * reference's decision rules (src/models/laya/decision.rs:214-268):
 * choice = argmax with ties to the lowest index, score = sum_i i * p_i,
 * noul = p[1], confidence = max(p1, 1 - p1) for noul else 1 - H / ln k. */
typedef struct laya_answer {
  int32_t kind;
  int32_t n_options;
  int32_t choice;      /* LAYA_CHOICE: argmax index; -1 otherwise */
  float score;         /* LAYA_SCORE */
  float noul;          /* LAYA_NOUL */
  float confidence;
  float probabilities[LAYA_MAX_OPTIONS];
  float logits[LAYA_MAX_OPTIONS]; /* candidate logits, or summed continuation log-probs */
} laya_answer;

typedef struct laya_model_info {
  char architecture[32];   /* "llama" | "qwen2" */
  int32_t layers, d_model, heads, kv_heads, head_dim, ffn, vocab, context;
  int32_t weight_kind;     /* GGML type of blk.0.attn_q.weight */
  int32_t n_devices;
  int64_t device_bytes;    /* weight bytes resident per device */
} laya_model_info;

/* Opens a GGUF file (read-only mmap, as src/io.rs:56-97) and uploads one
 * immutable weight replica to each listed CUDA device.  Replaces
 * Gguf::open + models::load + Engine::new (src/gguf.rs:95-180,
 * src/models/mod.rs:65-70, src/engine.rs:16-39). */
int laya_open(const char* path, const int* devices, int n_devices, laya_model** out);
/* Same, from a GGUF image in host memory (needed only during the call). */
int laya_open_memory(const uint8_t* gguf, size_t len, const int* devices, int n_devices, laya_model** out);
/* Backend::layers (src/models/mod.rs:14). */
int laya_layers(const laya_model* m);
int laya_info(const laya_model* m, laya_model_info* out);
/* Backend::validate (src/models/mod.rs:15): checks a batch without running it. */
int laya_validate(const laya_model* m, const laya_batch* b);
/* Backend::decide (src/models/mod.rs:16-22), batched: the whole batch is
 * validated before any launch; requests are sharded across the model's
 * devices; answers come back in request order; one failure fails the batch.
 * `canceled` (may be NULL) is polled between layers (src/models/openthai/model.rs:215-217);
 * it may be called from several host threads and must be thread-safe. */
int laya_decide_batch(laya_model* m, const laya_batch* b, laya_answer* out, int (*canceled)(void*), void* user);
/* KV-cached greedy decode: each of n_seqs contexts is prefilled, then
 * `steps` tokens are generated by argmax over the full vocabulary.  There is
 * no reference counterpart (the reference has no KV cache or decode loop).
 * out_tokens: n_seqs * steps.  stats (may be NULL): [prefill_ms, decode_ms]. */
int laya_decode(laya_model* m, const int32_t* ids, const int64_t* offsets, int n_seqs, int steps,
                int32_t* out_tokens, float* stats);
void laya_close(laya_model* m);
/* Thread-local message of the last failure on this thread. */
const char* laya_last_error(void);

/* ---- kernel-level entry points, mirroring single reference functions ---- */

/* gguf::decode (src/gguf.rs:250-336) on device `device`: GGUF block bytes of
 * type `kind` -> nbytes / block_size * block_elems floats, bit-exact. */
int laya_dequantize(int device, uint32_t kind, const uint8_t* blocks, size_t nbytes, float* out);
/* Matrix::apply (src/tensor.rs:10-39): out[m][rows] = x[m][cols] . W^T (+bias),
 * where W is GGUF tensor bytes of type `kind` holding `rows` rows of `cols`
 * elements.  Computed on the tcgen05 GEMM with F16 operands (x and the
 * decoded W rounded to F16) and F32 accumulation.  bias may be NULL. */
int laya_matrix_apply(int device, uint32_t kind, const uint8_t* w, int rows, int cols, const float* x, int m,
                      const float* bias, float* out);
/* Model::forward (src/models/openthai/model.rs:192-241) on the model's
 * first device: final-normed hidden rows at `read` positions of one causal
 * sequence.  out: nread * d_model floats. */
int laya_forward(laya_model* m, const int32_t* ids, int n, const int32_t* read, int nread, float* out);
/* The gated DeltaNet recurrence of OpenThai's linear-attention layers
 * (Delta::run, src/models/openthai/model.rs:322-355) for one sequence of s
 * tokens on device `device`: qkv = s rows of [q | k | v] heads (3 * nh * hk
 * floats, after the causal convolution and SiLU), a and b = s rows of nh
 * gate projections, dt = dt_bias[nh], alog = A_log[nh]; out = s rows of
 * nh * hk floats, before the per-head output norm.  hk is 64 or 128 (the
 * reference uses 128).  Host buffers. */
int laya_gated_delta(int device, const float* qkv, const float* a, const float* b, const float* dt,
                     const float* alog, int s, int nh, int hk, float* out);
/* OpenThai's whole DeltaNet mixer after its projections (Delta::run,
 * src/models/openthai/model.rs:309-360) for one sequence: raw = s rows of
 * in_proj_qkv output (3 * nh * hk), z = s rows of in_proj_z (nh * hk), a / b
 * = s rows of nh, conv = the depthwise kernel [3 * nh * hk][4], dt, alog [nh],
 * normw [hk]; out = s rows of nh * hk: causal convolution + SiLU, the
 * recurrence, per-head RMSNorm and x SiLU(z), before out_proj.  Host buffers. */
int laya_gated_delta_mixer(int device, const float* raw, const float* z, const float* a, const float* b,
                           const float* conv, const float* dt, const float* alog, const float* normw, int s, int nh,
                           int hk, float* out);
/* The gated full attention of OpenThai's attention layers after their
 * projections (Full::run, src/models/openthai/model.rs:248-296) for one
 * sequence of s tokens: qgate = s rows of H heads x [query hd | gate hd],
 * k and v = s rows of KV x hd, qn / kn = the per-head q / k RMSNorm weights
 * (applied with offset 1, eps 1e-6); RoPE on the first `rot` dimensions of a
 * head with base theta (the reference: hd 256, rot 64, theta 1e7); out = s
 * rows of H x hd, sigmoid(gate) x attention, before o_proj.  hd 64, 128 or
 * 256; H a multiple of KV.  Host buffers.  Runs on the tcgen05 attention:
 * the normalised, rotated q and k and v are rounded to F16 (the tensor-core
 * operand type), scores and sums stay F32, the output is rounded to F16. */
int laya_gated_attention(int device, const float* qgate, const float* k, const float* v, const float* qn,
                         const float* kn, int s, int H, int KV, int hd, int rot, float theta, float* out);
/* OpenThai model on one GPU (Model::load / Model::forward,
 * src/models/openthai/model.rs:99-241).  The shape comes parsed from the
 * file's `openthai.config` by the host (its config checks, model.rs:99-135);
 * layer_full[l] is nonzero for a full-attention layer, zero for a DeltaNet
 * layer, and is read only during laya_openthai_open.  Weights are F32 or F16
 * tensors under the reference's names; the GEMMs run on F16 operands with F32
 * accumulation.  Constraints of the GPU forward: d a multiple of 32, ffn a
 * multiple of 128, head_dim 64/128/256, lin_dim 64/128. */
typedef struct laya_ot_config {
  int d, ffn, heads, kv_heads, head_dim, rot, lin_heads, lin_dim, vocab, slots, n_layers;
  float theta, eps;
  const uint8_t* layer_full;
} laya_ot_config;
typedef struct laya_ot_model laya_ot_model;
int laya_openthai_open(const char* path, int device, const laya_ot_config* cfg, laya_ot_model** out);
/* The same from a GGUF image in memory (the bytes of the reference's mapped
 * `Gguf`); the image is read during this call only. */
int laya_openthai_open_memory(const uint8_t* gguf, size_t len, int device, const laya_ot_config* cfg,
                              laya_ot_model** out);
/* Model::forward for one encoded pass: the slot logits (slot head + bias) at
 * the given positions -> out [npos][slots] (host buffers). */
int laya_openthai_forward(laya_ot_model* m, const int32_t* ids, int s, const int32_t* positions, int npos,
                          float* out);
/* Several passes in one forward (the permutation passes of a request,
 * src/models/openthai/decision.rs:258-262, which the reference runs one at a
 * time): nseq (1..256) sequences of lens[i] tokens concatenated in ids, each
 * causal on its own; positions index the concatenated rows -> out
 * [npos][slots].  Row-wise work (norms, projections, MLP, head) runs once
 * over all rows; each sequence's DeltaNet recurrence runs on its own stream,
 * so the sequences' recurrences overlap. */
int laya_openthai_forward_batch(laya_ot_model* m, const int32_t* ids, const int32_t* lens, int nseq,
                                const int32_t* positions, int npos, float* out);
void laya_openthai_close(laya_ot_model* m);
/* Decodes a weight tensor of the model from its device layout back to F32
 * (for parity checks of the upload transcoding).  out: element count floats. */
int laya_tensor_f32(laya_model* m, const char* name, float* out, size_t max_elems);

/* Allocation-free Matrix::apply.  No counterpart in the reference.
 * For callers that cannot allocate device memory — a host program whose own
 * pool already owns all of HBM, or a thread that must not stall on
 * cudaMalloc/cudaFree — this computes what laya_matrix_apply computes, but
 * w (GGUF bytes of type `kind`), x [m][cols] F32, bias [rows] F32 (may be
 * NULL) and out [m][rows] F32 are DEVICE pointers the caller owns, and the
 * F16 staging of the GEMM lives in a fixed array of LAYA_STATIC_SCRATCH_BYTES
 * inside the library, which every GPU on which the library's module is
 * loaded holds until the process exits.  Work runs on `stream` (a
 * cudaStream_t, NULL for the legacy default stream) on the current device;
 * the call returns after it finished.  Needing more than the limit — 256 B +
 * rows * ceil8(cols) * 2 + m * ceil8(cols) * 2 bytes, each part rounded up to
 * 256 (a 2048 x 2048 weight with m = 1024 fits) — is rejected with
 * LAYA_E_INVALID.  The first call on a device is its set-up: it looks up the
 * array's device address, and under CUDA's default lazy module loading that
 * is also when the module, and the 16 MiB array with it, is created on the
 * device.  So make the first call on each device early — before any stream
 * capture, and before the caller's own pool claims the device's memory (or
 * load modules eagerly, CUDA_MODULE_LOADING=EAGER).  A cudaDeviceReset in the
 * process invalidates the looked-up address: do not call this entry point
 * after one.  All calls on a device share the one array: calls that overlap
 * on the GPU (concurrent host threads or streams) race and must be
 * serialised by the caller.  It calls no cudaMalloc/cudaFree and no
 * allocating library. */
#define LAYA_STATIC_SCRATCH_BYTES (16u << 20)
int laya_matrix_apply_static(uint32_t kind, const uint8_t* w, int rows, int cols, const float* x, int m,
                             const float* bias, float* out, void* stream);

/* Failure-detection self-test; no counterpart in the reference.  Launches
 * one device-side wait that nothing completes, bounded by budget_cycles SM
 * clock cycles (1 .. 4e9) through the same helper as every pipeline wait of
 * the library, and returns what a real expiry returns: LAYA_E_TIMEOUT, with
 * the context still usable for the next call.  LAYA_OK would mean the wait
 * ended without its budget running out. */
int laya_wait_selftest(int device, long long budget_cycles);

/* ---- timing of the last laya_decide_batch / laya_decode call ---- */
typedef struct laya_timing {
  double device_ms;   /* CUDA-event time on the device stream(s), inputs already in HBM; max over devices */
  int64_t launches;   /* kernels launched by the library during the call (all devices) */
  int64_t h2d_bytes;  /* host-to-device bytes copied during the call */
  int64_t d2h_bytes;  /* device-to-host bytes copied during the call */
} laya_timing;
int laya_last_timing(const laya_model* m, laya_timing* out);

/* ---- profiling (CUDA events around each launch, per kernel class) ---- */
typedef struct laya_profile_entry {
  char name[32];
  int64_t launches;
  double total_ms;
} laya_profile_entry;
int laya_profile_enable(laya_model* m, int enable);
/* Copies up to `max` entries; returns the number of entries, or < 0. Resets the counters. */
int laya_profile_read(laya_model* m, laya_profile_entry* out, int max);

#ifdef __cplusplus
}
#endif
#endif
