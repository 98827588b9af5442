// Host interface of the streaming decode GEMV (gemv.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace laya {

enum GemvMode : int {
  GV_PLAIN = 0,   // y[b][row] (+)= W[row] . x[b]
  GV_QKV = 1,     // q/k rows with RoPE, k/v appended to the paged cache, q -> F16
  GV_SWIGLU = 2,  // act[b][c] = silu(gate[c] . x[b]) * (up[c] . x[b]), F16
  GV_ARGMAX = 3,  // best[b] = max over rows of pack_logit(W[row] . x[b], row)
};

struct Gemv3Args {
  int mode;
  int nb;  // batch rows, 1..16
  int K;   // columns of every segment
  // PLAIN / ARGMAX: seg[0].  SWIGLU: gate seg[0] and up seg[1], or gate/up
  // rows interleaved per 128 in seg[0] (interleaved = 1).  QKV: q, k, v.
  QTensor seg[3];
  int interleaved;
  // Activations: F16 rows x[b * ldx + k] in global memory, or, when xres is
  // set, x = rmsnorm(xres[b * K + k]) * norm_w[k] built in shared memory.
  const half* x;
  int ldx;
  const float* xres;
  const float* norm_w;
  float eps;
  // PLAIN
  float* y;
  int ldy;
  int acc;
  // SWIGLU
  half* act;
  int ld_act;
  // ARGMAX
  unsigned long long* best;
  // QKV
  int qd, kd, hd, kvh;
  const float* bias;  // [qd + 2 kd] or null
  const int* pos;     // [nb]
  const int* slot;    // [nb]
  const float2* rope;  // [positions][hd / 2] (cos, sin)
  half* q;            // [nb][qd]
  half* kcache;
  half* vcache;       // [pages][kvh][page_size][hd]
  int page_size;
  // packed weight image of the segments (gemv3_pack), required by gemv3_launch
  const uint8_t* packed;
  // bounded waits
  unsigned* err;
  long long budget;
};

// Up to four GEMV phases run by one (cooperative) launch, in order, with a
// grid-wide barrier between consecutive phases: a phase may read what the
// previous phase wrote.  All phases share the batch rows and the block type.
struct GemvSeq {
  Gemv3Args ph[4];
  int tiles[4];
  int n;
  int kmax;        // largest K of the phases (activation staging)
  unsigned* gbar;  // grid barrier counter, zero at launch (n > 1)
};

// True when gemv3_launch handles these operands (Q8_0 or F16, K a multiple
// of 256, at most 16 batch rows, the staged activations fit).
bool gemv3_supported(const Gemv3Args& a);
// True when nb activation rows of up to kmax columns can be staged beside a
// ring of at least two stages.
bool gemv3_fits(int nb, int kmax);
// The segments' weights rearranged for streaming: per 16-row tile and per
// 1 KB of K, one contiguous stage image.  Depends only on mode, segments and
// K (not on the batch rows), so it is built once per model.
size_t gemv3_packed_bytes(const Gemv3Args& a);
cudaError_t gemv3_pack(const Gemv3Args& a, uint8_t* dst, cudaStream_t st);
cudaError_t gemv3_launch(const Gemv3Args& a, int num_sms, cudaStream_t st);
// Runs ph[0..n-1] as one launch; gbar must be zero when the launch starts.
cudaError_t gemv3_launch_seq(const Gemv3Args* ph, int n, unsigned* gbar, int num_sms, cudaStream_t st);

}  // namespace laya
