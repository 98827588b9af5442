// Host interface of the tcgen05 prefill GEMM (gemm.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>

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
// output tiles would leave most CTA pairs idle (M > 128 only).
int gemm_ksplit(int M, int N, int K, int num_sms);

}  // namespace laya
