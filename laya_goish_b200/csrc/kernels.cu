// Memory-bound kernels of the decision hot path and the paged causal GQA
// attention.  Each cites the reference function it replaces.
#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cstdlib>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"
#include "mma.cuh"
#include "ptx.cuh"
#include "launch.h"

namespace laya {

// ---------------------------------------------------------------- dequant

// gguf::decode (src/gguf.rs:250-336) on the original GGUF block bytes:
// one thread per block (per element for F32/F16), decode_raw_block's
// arithmetic, written as F32.
__global__ void dequant_raw_kernel(int kind, const uint8_t* __restrict__ b, size_t nblocks, float* __restrict__ out) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  decode_raw_block(kind, b, i, F32Sink{out});
}

// A device-side wait that nothing completes: one thread waits on a fresh
// mbarrier (one expected arrival, none ever made) with the same bounded
// helper as every pipeline wait of the library, records the expiry in the
// error word when the budget runs out, and returns; the other threads leave
// at once.  Nothing is in flight when it ends, so the context stays usable.
__global__ void wait_probe_kernel(unsigned* err, long long budget) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  mbar_fence_init();
  if (!mbar_wait(&bar, 0, budget)) atomicOr(err, 1u << 20);
}

cudaError_t wait_probe(unsigned* err, long long budget, cudaStream_t st) {
  wait_probe_kernel<<<1, 32, 0, st>>>(err, budget);
  return cudaGetLastError();
}

cudaError_t dequant_raw(int kind, const uint8_t* blocks, size_t nblocks, float* out, cudaStream_t st) {
  if (!nblocks) return cudaSuccess;
  dequant_raw_kernel<<<(unsigned)((nblocks + 255) / 256), 256, 0, st>>>(kind, blocks, nblocks, out);
  return cudaGetLastError();
}

// Decodes a weight from its HBM layout into an F16 matrix row block used as
// the tcgen05 B operand.  Output row of source row n:
// (n / grp) * gstride + goff + (n % grp), so q/k/v rows can be stacked and
// gate/up rows interleaved per 128 rows for the fused SwiGLU epilogue.
__global__ void dequant_f16_kernel(QTensor t, half* __restrict__ out, int ldo, int grp, int gstride, int goff) {
  const int groups = t.cols / 32;
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)t.rows * groups) return;
  const int n = (int)(i / groups), g = (int)(i % groups);
  float v[32];
  dq32(t, n, g * 32, v);
  const size_t orow = (size_t)(n / grp) * gstride + goff + (n % grp);
  uint4* dst = reinterpret_cast<uint4*>(out + orow * ldo + g * 32);
#pragma unroll
  for (int c = 0; c < 4; c++) {
    half2 h[4];
#pragma unroll
    for (int j = 0; j < 4; j++) h[j] = __floats2half2_rn(v[8 * c + 2 * j], v[8 * c + 2 * j + 1]);
    dst[c] = *reinterpret_cast<uint4*>(h);
  }
}

cudaError_t dequant_f16(const QTensor& t, half* out, int ldo, int grp, int gstride, int goff, cudaStream_t st) {
  size_t n = (size_t)t.rows * (t.cols / 32);
  if (!n) return cudaSuccess;
  dequant_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(t, out, ldo, grp, gstride, goff);
  return cudaGetLastError();
}

// Decodes whole rows to F32 (row list optional): the embedding lookup of
// src/models/openthai/model.rs:205-213 and the tensor read-back used by the
// parity tests.
__global__ void rows_f32_kernel(QTensor t, const int* __restrict__ ids, int nrows, float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int groups = t.cols / 32;
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)nrows * groups) return;
  const int r = (int)(i / groups), g = (int)(i % groups);
  const int n = ids ? ids[r] : r;
  float v[32];
  dq32(t, n, g * 32, v);
  float4* dst = reinterpret_cast<float4*>(out + (size_t)r * t.cols + g * 32);
#pragma unroll
  for (int c = 0; c < 8; c++) dst[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

cudaError_t rows_f32(const QTensor& t, const int* ids, int nrows, float* out, cudaStream_t st, bool pdl) {
  size_t n = (size_t)nrows * (t.cols / 32);
  if (!n) return cudaSuccess;
  return launch_k(rows_f32_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, pdl, t, ids, nrows, out);
}

// ---------------------------------------------------------------- RMSNorm

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < (int)(blockDim.x / 32) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

// rms (src/models/openthai/model.rs:84-94), offset 0, eps from the GGUF:
// y = x / sqrt(mean(x^2) + eps) * w.  One block per output row; optional
// source-row gather (answer-position gather, model.rs:232-235).
// part (nsplit planes of split_stride floats, may be null): K-split partial
// sums of the GEMM that produced x; they are added first, in plane order.
// Without a row gather the merged rows are also written back to x; with one
// they are not (a gather may name a row more than once, and the residual is
// not read again after the gathered final norm).
__device__ __forceinline__ float4 merged_row4(const float* x, const float* part, int nsplit, size_t split_stride,
                                              size_t off) {
  float4 v = *reinterpret_cast<const float4*>(x + off);
  // unrolled so several planes' loads are in flight; the adds keep split order
#pragma unroll 4
  for (int s = 0; s < nsplit; s++) {
    const float4 p = *reinterpret_cast<const float4*>(part + s * split_stride + off);
    v.x += p.x;
    v.y += p.y;
    v.z += p.z;
    v.w += p.w;
  }
  return v;
}

__device__ __forceinline__ void rms_out(float4 v, float scale, const float* w, int i, size_t obase, half* out16,
                                        float* out32) {
  const float4 g = *reinterpret_cast<const float4*>(w + i);
  const float y0 = v.x * scale * g.x, y1 = v.y * scale * g.y, y2 = v.z * scale * g.z, y3 = v.w * scale * g.w;
  if (out16) {
    half2 a = __floats2half2_rn(y0, y1), b = __floats2half2_rn(y2, y3);
    uint2 u = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    *reinterpret_cast<uint2*>(out16 + obase + i) = u;
  }
  if (out32) *reinterpret_cast<float4*>(out32 + obase + i) = make_float4(y0, y1, y2, y3);
}

// One CTA per row.  Rows of up to RN_HELD x 4 x blockDim elements (4096 at
// 256 threads) stay in registers between the sum of squares and the output
// pass, so x is read once (6 B per element moved with an F16 output).
constexpr int RN_HELD = 4;

__global__ void rmsnorm_kernel(float* __restrict__ x, const int* __restrict__ rows, const float* __restrict__ w,
                               int d, float eps, half* __restrict__ out16, float* __restrict__ out32,
                               const float* __restrict__ part, int nsplit, size_t split_stride) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const size_t roff = (size_t)(rows ? rows[r] : r) * d, obase = (size_t)r * d;
  const bool write_back = nsplit && !rows;
  const int step = blockDim.x * 4, held_end = RN_HELD * step;
  float4 v[RN_HELD];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < RN_HELD; u++) {
    const int i = threadIdx.x * 4 + u * step;
    if (i < d) {
      v[u] = merged_row4(x, part, nsplit, split_stride, roff + i);
      if (write_back) *reinterpret_cast<float4*>(x + roff + i) = v[u];
      ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
    }
  }
  for (int i = threadIdx.x * 4 + held_end; i < d; i += step) {  // rows wider than the register tile
    const float4 t = merged_row4(x, part, nsplit, split_stride, roff + i);
    if (write_back) *reinterpret_cast<float4*>(x + roff + i) = t;
    ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
  }
  ss = block_sum(ss, red);
  const float scale = 1.f / sqrtf(ss / (float)d + eps);
#pragma unroll
  for (int u = 0; u < RN_HELD; u++) {
    const int i = threadIdx.x * 4 + u * step;
    if (i < d) rms_out(v[u], scale, w, i, obase, out16, out32);
  }
  for (int i = threadIdx.x * 4 + held_end; i < d; i += step) {
    // the same thread wrote these elements back above, or re-merges them
    const float4 t = merged_row4(x, part, write_back ? 0 : nsplit, split_stride, roff + i);
    rms_out(t, scale, w, i, obase, out16, out32);
  }
}

// Plain rows (no gather, no K-split partials): one 128-thread CTA per row
// fetches the whole F32 row with one bulk copy into shared memory, so up to
// 16 rows per SM are in flight (the register-held kernel keeps 8 CTAs of 256
// threads per SM, too few bytes in flight to reach HBM speed).
constexpr int RNB_THREADS = 128;
__global__ void __launch_bounds__(RNB_THREADS) rmsnorm_bulk_kernel(const float* __restrict__ x,
                                                                   const float* __restrict__ w, int d, float eps,
                                                                   half* __restrict__ out16, float* __restrict__ out32,
                                                                   unsigned* err) {
  extern __shared__ float4 rnb_row[];
  __shared__ uint64_t bar;
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    mbar_expect_tx(&bar, (uint32_t)d * 4);
    bulk_g2s(rnb_row, x + (size_t)r * d, (uint32_t)d * 4, &bar);
  }
  __syncthreads();
  if (!mbar_wait(&bar, 0, 2000000000ll)) {
    if (threadIdx.x == 0) atomicOr(err, 1u << 20);
    mbar_wait(&bar, 0, 2000000000ll);  // give the copy in flight a second bounded wait before leaving
    return;
  }
  // The sum of squares in exactly the order of rmsnorm_kernel's 256 threads
  // (thread t sums float4 columns t, t + 256, ...; warps reduce by xor
  // shuffles, then warp 0 over the 8 warp sums), so both kernels give the
  // same bits: this thread plays threads t and t + 128 of that layout.
  float sa = 0.f, sb = 0.f;
  for (int i = threadIdx.x; i < d / 4; i += 256) {
    const float4 v = rnb_row[i];
    sa += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int i = threadIdx.x + 128; i < d / 4; i += 256) {
    const float4 v = rnb_row[i];
    sb += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
    sb += __shfl_xor_sync(0xffffffffu, sb, o);
  }
  const int wq = threadIdx.x / 32, lq = threadIdx.x % 32;
  if (lq == 0) {
    red[wq] = sa;
    red[wq + 4] = sb;
  }
  __syncthreads();
  if (wq == 0) {
    float t = lq < 8 ? red[lq] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lq == 0) red[0] = t;
  }
  __syncthreads();
  const float ss = red[0];
  const float scale = 1.f / sqrtf(ss / (float)d + eps);
  for (int i = threadIdx.x; i < d / 4; i += RNB_THREADS) rms_out(rnb_row[i], scale, w, 4 * i, (size_t)r * d, out16, out32);
}

cudaError_t rmsnorm(const float* x, const int* rows, int nrows, const float* w, int d, float eps, half* out16,
                    float* out32, cudaStream_t st, bool pdl, unsigned* err) {
  if (!nrows) return cudaSuccess;
  if (!rows && err && d % 4 == 0 && d <= 12288 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    static std::atomic<bool> configured[64];  // per device; any host thread may launch
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
      cudaError_t e = cudaFuncSetAttribute(rmsnorm_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 48 * 1024);
      if (e != cudaSuccess) return e;
      configured[dev & 63] = true;
    }
    return launch_k(rmsnorm_bulk_kernel, dim3(nrows), dim3(RNB_THREADS), (size_t)d * 4, st, pdl, x, w, d, eps, out16,
                    out32, err);
  }
  return launch_k(rmsnorm_kernel, dim3(nrows), dim3(256), 0, st, pdl, const_cast<float*>(x), rows, w, d, eps, out16,
                  out32, (const float*)nullptr, 0, (size_t)0);
}

// The QKV epilogue of a QKV GEMM split over K (few output tiles): x =
// part[0] + ... + part[nsplit-1] (planes split_stride floats apart, rows of
// n = qd + 2 kd) + bias, then rotate-half RoPE on the q and k heads
// (src/tensor.rs:158-171, the (cos, sin) table of the fused epilogue), q ->
// F16 rows q[m * ldq + c], k / v -> the paged KV cache at slot[m].  One CTA
// per token row; a thread takes four (j, j + hd/2) pairs of a q / k head or
// four v columns, as 16-byte loads from every plane.
__device__ __forceinline__ float4 qkv_sum4(const float* row, int nsplit, size_t split_stride, const float* bias,
                                           int c) {
  float4 x = *reinterpret_cast<const float4*>(row + c);
#pragma unroll 4
  for (int s2 = 1; s2 < nsplit; s2++) {
    const float4 y = *reinterpret_cast<const float4*>(row + (size_t)s2 * split_stride + c);
    x.x += y.x;
    x.y += y.y;
    x.z += y.z;
    x.w += y.w;
  }
  if (bias) {
    const float4 b = *reinterpret_cast<const float4*>(bias + c);
    x.x += b.x;
    x.y += b.y;
    x.z += b.z;
    x.w += b.w;
  }
  return x;
}

__global__ void qkv_merge_kernel(const float* __restrict__ part, int nsplit, size_t split_stride,
                                 const float* __restrict__ bias, int qd, int kd, int hd, int kvh,
                                 const int* __restrict__ pos, const int* __restrict__ slot,
                                 const float2* __restrict__ rope, int page_size, half* __restrict__ q, int ldq,
                                 half* __restrict__ kc, half* __restrict__ vc) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x, n = qd + 2 * kd, half_hd = hd / 2;
  const float* row = part + (size_t)m * n;
  const int p = pos[m], sl = slot[m];
  const int page = sl / page_size, off = sl % page_size;
  const int nrot = (qd + kd) / 8, nv = kd / 4;  // four-pair groups of q / k, four-column groups of v
  // grid.y CTAs share a row, so many rows' loads are in flight at once
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < nrot + nv; i += gridDim.y * blockDim.x) {
    if (i < nrot) {
      const bool isq = i < qd / 8;
      const int j = 4 * (isq ? i : i - qd / 8);  // first of four pairs
      const int head = j / half_hd, jj = j % half_hd;
      const int c0 = (isq ? 0 : qd) + head * hd + jj, c1 = c0 + half_hd;
      const float4 a = qkv_sum4(row, nsplit, split_stride, bias, c0);
      const float4 b = qkv_sum4(row, nsplit, split_stride, bias, c1);
      const float4* cs4 = reinterpret_cast<const float4*>(rope + (size_t)p * half_hd + jj);
      const float4 t0 = cs4[0], t1 = cs4[1];  // (cos, sin) of pairs jj .. jj + 3
      const float xa[4] = {a.x, a.y, a.z, a.w}, xb[4] = {b.x, b.y, b.z, b.w};
      const float co[4] = {t0.x, t0.z, t1.x, t1.z}, si[4] = {t0.y, t0.w, t1.y, t1.w};
      __align__(8) half y0[4], y1[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        y0[e] = __float2half_rn(xa[e] * co[e] - xb[e] * si[e]);
        y1[e] = __float2half_rn(xb[e] * co[e] + xa[e] * si[e]);
      }
      half* dst = isq ? q + (size_t)m * ldq + c0 - jj
                      : kc + (((size_t)page * kvh + head) * page_size + off) * hd;
      *reinterpret_cast<uint2*>(dst + jj) = *reinterpret_cast<const uint2*>(y0);
      *reinterpret_cast<uint2*>(dst + jj + half_hd) = *reinterpret_cast<const uint2*>(y1);
    } else {
      const int j = 4 * (i - nrot), c = qd + kd + j;
      const int head = j / hd, jj = j % hd;
      const float4 v = qkv_sum4(row, nsplit, split_stride, bias, c);
      __align__(8) half y[4] = {__float2half_rn(v.x), __float2half_rn(v.y), __float2half_rn(v.z),
                                __float2half_rn(v.w)};
      *reinterpret_cast<uint2*>(vc + (((size_t)page * kvh + head) * page_size + off) * hd + jj) =
          *reinterpret_cast<const uint2*>(y);
    }
  }
}

cudaError_t qkv_merge(const float* part, int nsplit, size_t split_stride, int M, const float* bias, int qd, int kd,
                      int hd, int kvh, const int* pos, const int* slot, const float2* rope, int page_size, half* q,
                      int ldq, half* kc, half* vc, cudaStream_t st, bool pdl) {
  if (M <= 0) return cudaSuccess;
  // 16-byte loads of the planes and 8-byte stores: rows, bias and the
  // (cos, sin) table in four-column steps
  if (hd % 8 || qd % 8 || kd % 8 || (split_stride % 4) || (ldq % 4) ||
      (reinterpret_cast<uintptr_t>(part) & 15) || (reinterpret_cast<uintptr_t>(bias) & 15) ||
      (reinterpret_cast<uintptr_t>(rope) & 15))
    return cudaErrorInvalidValue;
  const int groups = (qd + kd) / 8 + kd / 4;  // work items of one row
  return launch_k(qkv_merge_kernel, dim3(M, (groups + 63) / 64), dim3(64), 0, st, pdl, part, nsplit, split_stride,
                  bias, qd, kd, hd, kvh,
                  pos, slot, rope, page_size, q, ldq, kc, vc);
}

cudaError_t rmsnorm_merge(float* x, const int* rows, int nrows, const float* part, int nsplit, size_t split_stride,
                          const float* w, int d, float eps, half* out16, float* out32, cudaStream_t st, bool pdl) {
  if (!nrows) return cudaSuccess;
  // one float4 of the row per thread (up to 1024 threads): every plane's
  // load of a column is in flight at once across the row
  const int threads = std::min(1024, std::max(128, (d / 4 + 31) / 32 * 32));
  return launch_k(rmsnorm_kernel, dim3(nrows), dim3(threads), 0, st, pdl, x, rows, w, d, eps, out16, out32, part,
                  part ? nsplit : 0, split_stride);
}

// ---------------------------------------------------------------- heads

// Restricted head: logits of the candidate rows of the untied lm_head only
// (slot head of src/models/openthai/model.rs:236-240 restricted to the
// candidate ids, read as in src/models/openthai/decision.rs:268-279).
// One warp per (row, candidate); F32 hidden, weights decoded on the fly.
__global__ void head_restricted_kernel(QTensor w, const float* __restrict__ hid, const int* __restrict__ cand,
                                       const int* __restrict__ row_of, int n, float* __restrict__ out) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (gw >= n) return;
  const int id = cand[gw];
  const float* h = hid + (size_t)row_of[gw] * w.cols;
  float acc = 0.f;
  for (int g = lane; g < w.cols / 32; g += 32) {
    float v[32];
    dq32(w, id, g * 32, v);
    const float4* hp = reinterpret_cast<const float4*>(h + g * 32);
#pragma unroll
    for (int c = 0; c < 8; c++) {
      float4 x = hp[c];
      acc += v[4 * c] * x.x + v[4 * c + 1] * x.y + v[4 * c + 2] * x.z + v[4 * c + 3] * x.w;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
  if (lane == 0) out[gw] = acc;
}

cudaError_t head_restricted(const QTensor& w, const float* hid, const int* cand, const int* row_of, int n, float* out,
                            cudaStream_t st) {
  if (!n) return cudaSuccess;
  head_restricted_kernel<<<(n * 32 + 255) / 256, 256, 0, st>>>(w, hid, cand, row_of, n, out);
  return cudaGetLastError();
}

// Full-vocabulary log-sum-exp per row, for multi-token options scored by
// summed log-probabilities: lse = max + log(sum(exp(x - max))).
__global__ void lse_kernel(const float* __restrict__ logits, int V, float* __restrict__ out) {
  __shared__ float red[32];
  const int i = blockIdx.x;
  const float* x = logits + (size_t)i * V;
  float mx = -FLT_MAX;
  for (int c = threadIdx.x; c < V; c += blockDim.x) mx = fmaxf(mx, x[c]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -FLT_MAX;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float s = 0.f;
  for (int c = threadIdx.x; c < V; c += blockDim.x) s += expf(x[c] - mx);
  s = block_sum(s, red);
  if (threadIdx.x == 0) out[i] = mx + logf(s);
}

cudaError_t lse_rows(const float* logits, int V, int n, float* out, cudaStream_t st) {
  if (!n) return cudaSuccess;
  lse_kernel<<<n, 512, 0, st>>>(logits, V, out);
  return cudaGetLastError();
}

// F32 [rows][cols] -> F16 [rows][ld], zero padding columns cols..ld-1.
__global__ void f32_to_f16_pad_kernel(const float* __restrict__ x, int rows, int cols, int ld, half* __restrict__ y) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * ld) return;
  const int r = (int)(i / ld), c = (int)(i % ld);
  y[i] = __float2half_rn(c < cols ? x[(size_t)r * cols + c] : 0.f);
}

cudaError_t f32_to_f16_pad(const float* x, int rows, int cols, int ld, half* y, cudaStream_t st) {
  size_t n = (size_t)rows * ld;
  if (!n) return cudaSuccess;
  f32_to_f16_pad_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, rows, cols, ld, y);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- KV pages

// Copy-on-write of partially filled shared-prefix pages: each pair copies
// one page (K and V, every layer) so a branch can append after it.
__global__ void kv_copy_kernel(half* kc, half* vc, const int2* __restrict__ pairs, size_t page_elems,
                               size_t layer_elems, int layers) {
  const int2 p = pairs[blockIdx.y];
  const size_t n16 = page_elems / 8;
  for (int l = 0; l < layers; l++) {
    const uint4* ks = reinterpret_cast<const uint4*>(kc + l * layer_elems + (size_t)p.x * page_elems);
    const uint4* vs = reinterpret_cast<const uint4*>(vc + l * layer_elems + (size_t)p.x * page_elems);
    uint4* kd = reinterpret_cast<uint4*>(kc + l * layer_elems + (size_t)p.y * page_elems);
    uint4* vd = reinterpret_cast<uint4*>(vc + l * layer_elems + (size_t)p.y * page_elems);
    for (size_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
      kd[i] = ks[i];
      vd[i] = vs[i];
    }
  }
}

cudaError_t kv_copy(half* kc, half* vc, const int2* pairs, int npairs, size_t page_elems, size_t layer_elems,
                    int layers, cudaStream_t st) {
  if (!npairs) return cudaSuccess;
  kv_copy_kernel<<<dim3(8, npairs), 256, 0, st>>>(kc, vc, pairs, page_elems, layer_elems, layers);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- attention

// Causal GQA attention over the paged KV cache (src/models/openthai/model.rs:276-294:
// softmax(q.k * scale) over keys j <= i, then .v, with kv head = h / (H/KV)).
// One CTA = 64 query rows of one sequence x one query head; 4 warps of 16
// rows; flash-style online softmax over 64-key blocks (one page each),
// double-buffered cp.async loads, XOR-swizzled shared memory.
template <int HD>
__global__ void __launch_bounds__(128) attn_kernel(const half* __restrict__ q, int ldq, half* __restrict__ o, int ldo,
                                                   const half* __restrict__ kc, const half* __restrict__ vc,
                                                   const int* __restrict__ tables, const AttnItem* __restrict__ items,
                                                   int H, int KV, float scale_log2) {
  constexpr int BQ = 64, BKV = 64, CH = HD / 8;
  extern __shared__ uint4 smem_attn[];
  half* sQ = reinterpret_cast<half*>(smem_attn);
  half* sK = sQ + BQ * HD;
  half* sV = sK + 2 * BKV * HD;
  // an item holds up to kAttnRows rows; this CTA takes the 64-row half blockIdx.z
  AttnItem it = items[blockIdx.x];
  it.q_row += 64 * blockIdx.z;
  it.pos0 += 64 * blockIdx.z;
  it.q_len -= 64 * blockIdx.z;
  if (it.q_len <= 0) return;
  if (it.q_len > 64) it.q_len = 64;
  const int h = blockIdx.y, kvh = h / (H / KV);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_keys = it.pos0 + it.q_len;
  const int n_blocks = (n_keys + BKV - 1) / BKV;
  auto sw = [](int r, int c) { return r * HD + ((c ^ (r & 7)) << 3); };

  for (int i = threadIdx.x; i < BQ * CH; i += 128) {
    const int r = i / CH, c = i % CH;
    if (r < it.q_len)
      cp_async16(sQ + sw(r, c), q + (size_t)(it.q_row + r) * ldq + h * HD + c * 8);
    else
      *reinterpret_cast<uint4*>(sQ + sw(r, c)) = make_uint4(0, 0, 0, 0);
  }
  auto load_kv = [&](int kb, int buf) {
    const int page = tables[it.table_off + kb];
    const size_t base = ((size_t)page * KV + kvh) * BKV * HD;
    const int valid = min(BKV, n_keys - kb * BKV);
    half* dk = sK + buf * BKV * HD;
    half* dv = sV + buf * BKV * HD;
    for (int i = threadIdx.x; i < BKV * CH; i += 128) {
      const int r = i / CH, c = i % CH;
      if (r < valid) {
        cp_async16(dk + sw(r, c), kc + base + r * HD + c * 8);
        cp_async16(dv + sw(r, c), vc + base + r * HD + c * 8);
      } else {
        *reinterpret_cast<uint4*>(dk + sw(r, c)) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dv + sw(r, c)) = make_uint4(0, 0, 0, 0);
      }
    }
  };
  load_kv(0, 0);
  cp_commit();

  const int g = lane / 4, t = lane % 4;
  const int row0 = warp * 16 + g;
  const int pos_a = it.pos0 + row0, pos_b = pos_a + 8;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float acc[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  uint32_t qf[HD / 16][4];

  for (int kb = 0; kb < n_blocks; kb++) {
    if (kb + 1 < n_blocks) {
      load_kv(kb + 1, (kb + 1) & 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; kk++) ldsm_x4(qf[kk], sQ + sw(warp * 16 + (lane % 16), kk * 2 + lane / 16));
    }
    const half* bK = sK + (kb & 1) * BKV * HD;
    const half* bV = sV + (kb & 1) * BKV * HD;
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; kk++) {
#pragma unroll
      for (int nj = 0; nj < 8; nj += 2) {
        uint32_t b[4];
        const int mat = lane / 8;
        ldsm_x4(b, bK + sw(nj * 8 + (lane % 8) + (mat / 2) * 8, kk * 2 + (mat % 2)));
        mma16816(s[nj], qf[kk], b[0], b[1]);
        mma16816(s[nj + 1], qf[kk], b[2], b[3]);
      }
    }
    // Scores stay unscaled until the exponent (the scale is positive, so
    // the running maximum is the same).  Only blocks that reach past the
    // CTA's first query position or past the last key need the causal mask.
    if (kb * BKV + BKV - 1 > it.pos0 || kb * BKV + BKV > n_keys) {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int key = kb * BKV + j * 8 + 2 * t;
#pragma unroll
        for (int e = 0; e < 2; e++) {
          if (key + e > pos_a || key + e >= n_keys) s[j][e] = -INFINITY;
          if (key + e > pos_b || key + e >= n_keys) s[j][2 + e] = -INFINITY;
        }
      }
    }
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      mx_a = fmaxf(mx_a, fmaxf(s[j][0], s[j][1]));
      mx_b = fmaxf(mx_b, fmaxf(s[j][2], s[j][3]));
    }
#pragma unroll
    for (int o2 = 1; o2 <= 2; o2 <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffff, mx_a, o2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffff, mx_b, o2));
    }
    // Block 0 always holds key 0 <= every query position, so the maxima are
    // finite from the first block on.
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float ca = exp2f((m_a - mn_a) * scale_log2), cb = exp2f((m_b - mn_b) * scale_log2);
    m_a = mn_a;
    m_b = mn_b;
    const float oa = -mn_a * scale_log2, ob = -mn_b * scale_log2;
    float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      s[j][0] = exp2f(fmaf(s[j][0], scale_log2, oa));
      s[j][1] = exp2f(fmaf(s[j][1], scale_log2, oa));
      s[j][2] = exp2f(fmaf(s[j][2], scale_log2, ob));
      s[j][3] = exp2f(fmaf(s[j][3], scale_log2, ob));
      sum_a += s[j][0] + s[j][1];
      sum_b += s[j][2] + s[j][3];
    }
#pragma unroll
    for (int o2 = 1; o2 <= 2; o2 <<= 1) {
      sum_a += __shfl_xor_sync(0xffffffff, sum_a, o2);
      sum_b += __shfl_xor_sync(0xffffffff, sum_b, o2);
    }
    l_a = l_a * ca + sum_a;
    l_b = l_b * cb + sum_b;
#pragma unroll
    for (int i = 0; i < HD / 8; i++) {
      acc[i][0] *= ca;
      acc[i][1] *= ca;
      acc[i][2] *= cb;
      acc[i][3] *= cb;
    }
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      uint32_t pa[4] = {pack_h2(s[2 * kk][0], s[2 * kk][1]), pack_h2(s[2 * kk][2], s[2 * kk][3]),
                        pack_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack_h2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int nd = 0; nd < HD / 8; nd += 2) {
        uint32_t b[4];
        const int mat = lane / 8;
        ldsm_x4_t(b, bV + sw(kk * 16 + (lane % 8) + (mat % 2) * 8, nd + mat / 2));
        mma16816(acc[nd], pa, b[0], b[1]);
        mma16816(acc[nd + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  const float ia = 1.f / l_a, ib = 1.f / l_b;
  if (row0 < it.q_len) {
    half* dst = o + (size_t)(it.q_row + row0) * ldo + h * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; i++)
      *reinterpret_cast<uint32_t*>(dst + i * 8 + 2 * t) = pack_h2(acc[i][0] * ia, acc[i][1] * ia);
  }
  if (row0 + 8 < it.q_len) {
    half* dst = o + (size_t)(it.q_row + row0 + 8) * ldo + h * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; i++)
      *reinterpret_cast<uint32_t*>(dst + i * 8 + 2 * t) = pack_h2(acc[i][2] * ib, acc[i][3] * ib);
  }
}

template <int HD>
static cudaError_t attn_launch(const AttnParams& p, cudaStream_t st) {
  const int smem = 5 * 64 * HD * 2;
  static std::atomic<bool> configured[64];  // per device; any host thread may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  attn_kernel<HD><<<dim3(p.n_items, p.H, kAttnRows / 64), 128, smem, st>>>(p.q, p.ldq, p.o, p.ldo, p.kc, p.vc,
                                                                            p.tables, p.items, p.H, p.KV,
                                                                            p.scale_log2);
  return cudaGetLastError();
}

static bool attn_tc_enabled() {
  const char* e = std::getenv("LAYA_ATTN_TC");
  return !(e && e[0] == '0');
}

cudaError_t attention(const AttnParams& p, cudaStream_t st) {
  if (!p.n_items) return cudaSuccess;
  if (attn_tc_enabled()) {
    const cudaError_t e = attention_tc(p, st);
    if (e != cudaErrorNotSupported) return e;
  }
  if (p.hd == 64) return attn_launch<64>(p, st);
  if (p.hd == 128) return attn_launch<128>(p, st);
  return cudaErrorInvalidValue;
}

}  // namespace laya
