// Host interface of the tcgen05 prefill GEMM (gemm.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace laya {

// Epilogues fused into the GEMM.
enum Epi : int {
  EPI_F32 = 0,     // out F32 [M][ldo] = acc (+bias)
  EPI_F16 = 1,     // out F16 [M][ldo] = acc (+bias)
  EPI_RESID = 2,   // resid F32 [M][ldo] += acc            (tensor::add)
  EPI_SWIGLU = 3,  // out F16 [M][ldo] = silu(gate) * up   (gate/up rows interleaved per 128)
  EPI_QKV = 4,     // bias + RoPE; q -> out F16 [M][ldo]; k, v -> paged KV cache
};

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles;   // filled by gemm_launch
  int group;              // row bands per group of the CTA-pair tile walk (filled by gemm_launch)
  const float* bias;      // [N] or null
  void* out;
  int ldo;
  float* resid;
  // EPI_QKV
  int qd, kd, hd, kvh;
  const int* pos;         // [M] absolute token positions
  const int* slot;        // [M] KV slot = page * page_size + offset
  const float2* rope;     // [positions][hd/2] (cos, sin)
  half* kcache;
  half* vcache;           // [pages][kvh][page_size][hd]
  int page_size;
  unsigned* err;          // device error word; nonzero after a timed-out wait
  long long budget;       // wait budget in SM clock cycles
  // EPI_RESID split over K (gemm_ksplit): ksplit > 1 writes the partial sums
  // of split s to part[s][M][ldo] instead of adding into resid; the consumer
  // adds resid + part[0] + ... + part[ksplit-1] in that order.
  int ksplit;
  float* part;
};

// cuTensorMapEncodeTiled through the runtime's driver entry point: `rank`
// dimensions (innermost first), byte strides of dimensions 1..rank-1, box
// extents, a CUtensorMapDataType and a CUtensorMapSwizzle; element strides
// 1, zero fill out of bounds.  False when the driver rejects the map.
bool encode_tiled(CUtensorMap* m, int dtype, int rank, const void* base, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, int swizzle);

// A: [M][lda] F16 row-major activations, B: [N][ldb] F16 row-major weights
// (K contiguous).  lda, ldb multiples of 8; A, B 16-byte aligned.
// pdl: launch with programmatic dependent launch; the kernel then prefetches
// its first weight tiles into L2 while the previous kernel drains and waits
// for it (griddepcontrol.wait) before touching anything that kernel wrote.
cudaError_t gemm_launch(int epi, const half* A, int lda, const half* B, int ldb, GemmArgs a, int num_sms,
                        cudaStream_t st, bool pdl = false);
// K splits for an EPI_RESID GEMM of this shape: more than 1 when its 256 x 256
// output tiles would leave most CTA pairs idle.
int gemm_ksplit(int M, int N, int K, int num_sms);
// Row bands per group of the CTA-pair tile walk for a GEMM of n_tiles column tiles.
int gemm_pair_group(int n_tiles);

// Q8_0 weight operand of gemm_q8_launch, read from the resident blocks
// (int8 quants [rows][K] of each tensor) with no F16 copy: up to three
// tensors stacked along N (q | k | v), or two interleaved per 128 rows
// (gate / up, the row order of the fused SwiGLU epilogue).  `st` holds the
// blocks' F16 scales transposed to [K/32][N] in the operand's row order
// (q8_scales_t), so that one TMA box brings 4 blocks' scales of 128 rows.
struct Q8Weights {
  const int8_t* q[3];
  int rows[3];     // rows of each tensor; all but the last a multiple of 128
  int nseg;        // 1..3
  int interleave;  // 1: two tensors of equal rows alternating per 128 rows
  const half* st;  // [K/32][N]
};

// Y = X . W^T with W given as Q8_0 blocks, on the CTA-pair tcgen05 GEMM:
// TMA brings each 128 x 128 tile of int8 quants and its scales into shared
// memory, four converter warps write it as the swizzled F16 operand
// (d * q rounded once to F16, the value the F16 operand cache holds), and
// the tensor cores consume it; every weight byte is read from HBM once per
// 256-row band of X.  Same epilogues and K splits (EPI_RESID with
// a.ksplit > 1, see gemm_q8_ksplit) as gemm_launch; any M >= 1.
// Requires K % 128 == 0, lda % 8 == 0, N % 8 == 0, 16-byte aligned operands.
cudaError_t gemm_q8_launch(int epi, const half* A, int lda, const Q8Weights& w, GemmArgs a, int num_sms,
                           cudaStream_t st, bool pdl = false);
// K splits (in whole 128-column blocks) for an EPI_RESID gemm_q8_launch of
// this shape: more than 1 when its output tiles would leave most CTA pairs idle.
int gemm_q8_ksplit(int M, int N, int K, int num_sms);
// dst[(k/32) * ldst + orow(n)] = scale of block k/32 of row n of Q8_0 tensor
// t, with orow(n) = (n / grp) * gstride + goff + n % grp (the row placement
// of dequant_f16).
cudaError_t q8_scales_t(const QTensor& t, half* dst, int ldst, int grp, int gstride, int goff, cudaStream_t st);

}  // namespace laya
