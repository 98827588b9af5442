// Host interface of the memory-bound kernels and the attention (kernels.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "common.cuh"

namespace laya {

// One attention work unit: query rows [q_row, q_row + q_len) of one sequence
// at absolute positions pos0.., attending keys 0 .. pos0+q_len-1 through the
// page list tables[table_off ..] (one 64-token page per key block).
// Query rows per attention work item (one sequence's consecutive rows).
constexpr int kAttnRows = 128;

struct AttnItem {
  int q_row, q_len, pos0, table_off;  // q_len <= kAttnRows
};

struct AttnParams {
  const half* q;
  int ldq;
  half* o;
  int ldo;
  const half* kc;  // this layer's K pages [pages][KV][64][hd]
  const half* vc;
  const int* tables;
  const AttnItem* items;
  int n_items, H, KV, hd;
  float scale_log2;
  int q_rows;     // rows of q / o
  int kv_rows;    // rows of kc / vc: pages * KV * 64
  unsigned* err;  // device error word (bounded waits)
  // optional output gate (OpenThai): o *= sigmoid(gate[row * ldg + head * ghs + c])
  const float* gate;
  int ldg, ghs;
  // tcgen05 form: 1 = the H / KV query heads of a KV head share each unit
  // (K/V pages loaded and multiplied once per group), 0 = one head per unit
  // over up to 128 query rows
  int pack;
};

// tcgen05 attention (attn_tc.cu); cudaErrorNotSupported for head dims it
// does not cover.
cudaError_t attention_tc(const AttnParams& p, cudaStream_t st);

cudaError_t dequant_raw(int kind, const uint8_t* blocks, size_t nblocks, float* out, cudaStream_t st);
// One bounded wait that nothing completes (laya_wait_selftest).
cudaError_t wait_probe(unsigned* err, long long budget, cudaStream_t st);
cudaError_t dequant_f16(const QTensor& t, half* out, int ldo, int grp, int gstride, int goff, cudaStream_t st);
// pdl: launch with programmatic dependent launch allowed (decode graph).
cudaError_t rows_f32(const QTensor& t, const int* ids, int nrows, float* out, cudaStream_t st, bool pdl = false);
// err (may be null): device error word; with it, plain rows (rows null) take
// the bulk-copy kernel, whose bounded wait reports there.
cudaError_t rmsnorm(const float* x, const int* rows, int nrows, const float* w, int d, float eps, half* out16,
                    float* out32, cudaStream_t st, bool pdl = false, unsigned* err = nullptr);
// OpenThai's gated DeltaNet recurrence (deltanet.cu), one sequence: qkv
// [s][3 nh hk] after the convolution (q / k normalised in place); the gate
// projections of token i, head h at a / b[i * ldab + h]; decay / beta are
// written to dec / beta [s][nh] (they may alias a / b when ldab == nh);
// out [s][nh hk] before the output norm.
// kq: gated_delta_scratch(s, nh) bytes (the four-token groups' products).
size_t gated_delta_scratch(int s, int nh);
cudaError_t gated_delta(float* qkv, const float* a, const float* b, int ldab, const float* dt, const float* alog,
                        int s, int nh, int hk, float* dec, float* beta, float* kq, float* out, cudaStream_t st);
// The whole mixer after its projections: raw rows (stride ldraw) [3 nh hk],
// z rows (stride ldz) [nh hk], a / b as above; scratch holds
// gated_delta_mixer_scratch(s, nh, hk) bytes (16-byte aligned).  The result
// rows [s][nh hk] go to out (F32) or, when out16 is set, to out16 as F16
// (out is then the recurrence's scratch output).
size_t gated_delta_mixer_scratch(int s, int nh, int hk);
cudaError_t gated_delta_mixer(const float* raw, int ldraw, const float* z, int ldz, const float* a, const float* b,
                              int ldab, const float* conv, const float* dt, const float* alog, const float* normw,
                              int s, int nh, int hk, float* scratch, float* out, half* out16, cudaStream_t st);
// OpenThai gated attention after the projections (gated_attn.cu): rows of
// qgate [H][query hd | gate hd] (row stride ldqg), of k and v [KV][hd] (row
// stride ldkv), F32; q / k norm weights [hd] -> out16 [s][H * hd] F16 (the
// output projection's operand), on the tcgen05 attention.  scratch:
// gated_attention_scratch(...) bytes, 256-byte aligned.  hd 64/128/256.
size_t gated_attention_scratch(int s, int H, int KV, int hd);
cudaError_t gated_attention(const float* qgate, int ldqg, const float* k, const float* v, int ldkv, const float* qn,
                            const float* kn, int s, int H, int KV, int hd, int rot, float theta, void* scratch,
                            half* out16, unsigned* err, cudaStream_t st);
// rmsnorm of x + part[0] + ... + part[nsplit-1] (K-split partial sums of the
// GEMM that wrote x, planes split_stride floats apart); without a row gather
// (rows null) the merged rows are also written back to x.
cudaError_t rmsnorm_merge(float* x, const int* rows, int nrows, const float* part, int nsplit, size_t split_stride,
                          const float* w, int d, float eps, half* out16, float* out32, cudaStream_t st,
                          bool pdl = false);
// The QKV epilogue (bias, RoPE, q rows, paged K/V) of a QKV GEMM whose K
// was split: part holds nsplit planes [M][qd + 2 kd], split_stride floats apart.
cudaError_t qkv_merge(const float* part, int nsplit, size_t split_stride, int M, const float* bias, int qd, int kd,
                      int hd, int kvh, const int* pos, const int* slot, const float2* rope, int page_size, half* q,
                      int ldq, half* kc, half* vc, cudaStream_t st, bool pdl = false);
cudaError_t head_restricted(const QTensor& w, const float* hid, const int* cand, const int* row_of, int n, float* out,
                            cudaStream_t st);
cudaError_t lse_rows(const float* logits, int V, int n, float* out, cudaStream_t st);
cudaError_t f32_to_f16_pad(const float* x, int rows, int cols, int ld, half* y, cudaStream_t st);
cudaError_t kv_copy(half* kc, half* vc, const int2* pairs, int npairs, size_t page_elems, size_t layer_elems,
                    int layers, cudaStream_t st);
cudaError_t attention(const AttnParams& p, cudaStream_t st);

}  // namespace laya
