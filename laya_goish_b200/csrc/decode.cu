// KV-cached greedy decode (no reference counterpart: the reference has no
// KV cache and no decode loop, src/models/laya/decision.rs:302).
//
// Each step appends one token per sequence.  Small batches run the linear
// layers as bandwidth-bound GEMVs that stream the quantised weights once with
// 128-bit loads (four 32-element groups in flight per lane), decode them in
// registers and fuse SwiGLU and the residual add; larger batches reuse the
// tcgen05 GEMM.  Attention stages each 64-token K/V page in shared memory and
// splits the key axis across CTAs so a single sequence still covers the GPU.
// All per-step inputs live at fixed device addresses, advanced by a
// one-thread-block kernel, so the whole step is captured once as a CUDA
// graph and replayed for every generated token.
#include <atomic>
#include <algorithm>
#include <cfloat>
#include <chrono>
#include <cstdlib>
#include <cstring>

#include "engine.h"
#include "gemm.h"
#include "gemv.h"
#include "launch.h"
#include "mma.cuh"
#include "ptx.cuh"

namespace laya {

// ---------------------------------------------------------------- GEMV

struct GemvSeg {
  QTensor w;
  float* y;  // y[b * ldy + row]
  int ldy;
  int acc;   // add into y (fused residual) instead of storing
};

// Up to three matrices share one launch (q, k, v); in SwiGLU mode a warp
// computes the gate row and the up row of one FFN column and writes
// silu(gate) * up as F16 (src/models/openthai/model.rs:225-230).
struct GemvPlan {
  GemvSeg seg[3];
  int nseg;
  int rows;  // warps' rows: sum of segment rows, or ffn in SwiGLU mode
  const half* x;
  int ldx;
  int swiglu;  // 0 off, 1 gate = seg[0] and up = seg[1], 2 interleaved gate/up rows in seg[0]
  half* act;
  int ld_act;
  unsigned long long* best;  // greedy mode: per batch row, max of pack_logit(value, row)
  // Fused RMSNorm input (src/models/openthai/model.rs:84-94): when xres is
  // set, x = rmsnorm(xres[b], norm_w, eps) is built per block in shared
  // memory (F16) instead of being read from a separate normalised buffer.
  const float* xres;
  const float* norm_w;
  float eps;
};


// Raw 16-byte slots of the next groups of one row, loaded ahead of their use
// so many loads are in flight.  A Q8_0 group (32 int8 + scale) takes 2
// slots, an F16 group 4; lane l holds groups l, l+32, ...
template <int NV>
struct RowRaw {
  static_assert(NV >= 4 && NV % 4 == 0, "a batch must hold at least one F16 group (4 slots)");
  uint4 v[NV];
  uint32_t sc[NV / 2];
};

// Groups held per batch: always >= 1 because NV >= 4.
__device__ __forceinline__ int groups_per_batch(int kind, int nv) { return kind == K_Q8_0 ? nv / 2 : nv / 4; }

template <int NV>
__device__ __forceinline__ void row_load(const QTensor& w, int n, int g0, int groups, RowRaw<NV>& r) {
  if (w.kind == K_Q8_0) {
    const uint4* qp = reinterpret_cast<const uint4*>(w.q + (size_t)n * w.cols);
    const uint16_t* sp = w.s + (size_t)n * groups;
#pragma unroll
    for (int u = 0; u < NV / 2; u++) {
      const int g = g0 + 32 * u;
      if (g < groups) {
        r.v[2 * u] = __ldg(qp + 2 * g);
        r.v[2 * u + 1] = __ldg(qp + 2 * g + 1);
        r.sc[u] = __ldg(sp + g);
      }
    }
  } else if (w.kind == K_F16) {
    const uint4* qp = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w.q) + (size_t)n * w.cols);
#pragma unroll
    for (int u = 0; u < NV / 4; u++) {
      const int g = g0 + 32 * u;
      if (g < groups)
#pragma unroll
        for (int c = 0; c < 4; c++) r.v[4 * u + c] = __ldg(qp + 4 * g + c);
    }
  }
}

// int8 byte j of w (as stored, two's complement) to float without I2F:
// bytes are biased by 128 and placed in the mantissa of 2^23, and the exact
// difference with 2^23 + 128 recovers q (integers below 2^24 are exact).
__device__ __forceinline__ float q8_to_f(uint32_t wbiased, int j) {
  return __uint_as_float(__byte_perm(wbiased, 0x4B000000u, 0x7540u + j)) - 8388736.f;
}

// Activation access: F32 rows staged in shared memory (fast path), or F16
// rows in global memory.
struct XSrc {
  const float* xs;  // [B][K] F32 in shared memory, or null
  const half* xg;   // [B][ldx] F16 in global memory
  int ld;
};

// Staged rows keep each 32-element group in 36 floats: lanes own different
// groups, and the 144-byte stride puts consecutive lanes 4 banks apart.
__device__ __forceinline__ int xs_index(int k) { return (k >> 5) * 36 + (k & 31); }

template <int B, bool XS>
__device__ __forceinline__ void load_x8(const XSrc& x, int b, int k, float (&v)[8]) {
  if (XS) {
    const float* base = x.xs + (size_t)b * x.ld + xs_index(k);
    const float4 a = *reinterpret_cast<const float4*>(base);
    const float4 c = *reinterpret_cast<const float4*>(base + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(x.xg + (size_t)b * x.ld + k);
    const half2* h = reinterpret_cast<const half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float2 f = __half22float2(h[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  }
}

template <int B, int NV, bool XS>
__device__ __forceinline__ void row_use(const QTensor& w, const RowRaw<NV>& r, int g0, int groups, const XSrc& x,
                                        float (&acc)[B]) {
  if (w.kind == K_Q8_0) {
#pragma unroll
    for (int u = 0; u < NV / 2; u++) {
      const int g = g0 + 32 * u;
      if (g >= groups) break;
      const float d = half_bits(r.sc[u]);
      const uint32_t wd[8] = {r.v[2 * u].x ^ 0x80808080u,     r.v[2 * u].y ^ 0x80808080u,
                              r.v[2 * u].z ^ 0x80808080u,     r.v[2 * u].w ^ 0x80808080u,
                              r.v[2 * u + 1].x ^ 0x80808080u, r.v[2 * u + 1].y ^ 0x80808080u,
                              r.v[2 * u + 1].z ^ 0x80808080u, r.v[2 * u + 1].w ^ 0x80808080u};
      float part[B];
#pragma unroll
      for (int b = 0; b < B; b++) part[b] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float wf[8];
#pragma unroll
        for (int j = 0; j < 8; j++) wf[j] = q8_to_f(wd[2 * c + j / 4], j % 4);
#pragma unroll
        for (int b = 0; b < B; b++) {
          float xv[8];
          load_x8<B, XS>(x, b, g * 32 + c * 8, xv);
#pragma unroll
          for (int j = 0; j < 8; j++) part[b] = fmaf(wf[j], xv[j], part[b]);
        }
      }
#pragma unroll
      for (int b = 0; b < B; b++) acc[b] = fmaf(d, part[b], acc[b]);
    }
  } else {
#pragma unroll
    for (int u = 0; u < NV / 4; u++) {
      const int g = g0 + 32 * u;
      if (g >= groups) break;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float wf[8];
        const half2* h = reinterpret_cast<const half2*>(&r.v[4 * u + c]);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(h[e]);
          wf[2 * e] = f.x;
          wf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int b = 0; b < B; b++) {
          float xv[8];
          load_x8<B, XS>(x, b, g * 32 + c * 8, xv);
#pragma unroll
          for (int j = 0; j < 8; j++) acc[b] = fmaf(wf[j], xv[j], acc[b]);
        }
      }
    }
  }
}

// Dot products of one row with the B activation rows: the first batch of
// groups is already in `raw` (loaded before pdl_wait); block types without
// a prefetch path decode through dq32.
template <int B, int NV, bool FAST, bool XS>
__device__ __forceinline__ void row_dot(const QTensor& w, int n, const XSrc& x, int lane, RowRaw<NV>& raw,
                                        bool first_loaded, float (&acc)[B]) {
  const int groups = w.cols / 32;
  if (FAST || w.kind == K_Q8_0 || w.kind == K_F16) {
    const int gpb = groups_per_batch(w.kind, NV);
    const int step = 32 * (gpb > 0 ? gpb : 1);
    for (int g0 = lane; g0 < groups; g0 += step) {
      if (g0 != lane || !first_loaded) row_load<NV>(w, n, g0, groups, raw);
      row_use<B, NV, XS>(w, raw, g0, groups, x, acc);
    }
  } else {
    for (int g = lane; g < groups; g += 32) {
      float wf[32];
      dq32(w, n, g * 32, wf);
#pragma unroll
      for (int c = 0; c < 4; c++)
#pragma unroll
        for (int b = 0; b < B; b++) {
          float xv[8];
          load_x8<B, XS>(x, b, g * 32 + c * 8, xv);
#pragma unroll
          for (int j = 0; j < 8; j++) acc[b] = fmaf(wf[c * 8 + j], xv[j], acc[b]);
        }
    }
  }
}

template <int B>
__device__ __forceinline__ void warp_sum(float (&acc)[B]) {
#pragma unroll
  for (int b = 0; b < B; b++) {
    float v = acc[b];
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
    acc[b] = v;
  }
}

// Builds the block's F32 activation rows in shared memory, once per block:
// either x = rmsnorm(xres[b], norm_w, eps) from the F32 residual stream
// (src/models/openthai/model.rs:84-94), or the F16 rows of p.x widened.
template <int B>
__device__ __forceinline__ void stage_x(const GemvPlan& p, int K, float* xs) {
  __shared__ float red[8][B];
  __shared__ float scale[B];
  const int tid = threadIdx.x, lane = tid % 32, wb = tid / 32;
  if (p.xres) {
    float ss[B];
#pragma unroll
    for (int b = 0; b < B; b++) ss[b] = 0.f;
    for (int k = tid * 4; k < K; k += blockDim.x * 4)
#pragma unroll
      for (int b = 0; b < B; b++) {
        const float4 v = *reinterpret_cast<const float4*>(p.xres + (size_t)b * K + k);
        ss[b] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
#pragma unroll
    for (int b = 0; b < B; b++) {
      float v = ss[b];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
      if (lane == 0) red[wb][b] = v;
    }
    __syncthreads();
    if (tid < B) {
      float t = 0.f;
      for (int i = 0; i < (int)(blockDim.x / 32); i++) t += red[i][tid];
      scale[tid] = 1.f / sqrtf(t / (float)K + p.eps);
    }
    __syncthreads();
    for (int k = tid * 4; k < K; k += blockDim.x * 4) {
      const float4 g = *reinterpret_cast<const float4*>(p.norm_w + k);
#pragma unroll
      for (int b = 0; b < B; b++) {
        const float4 v = *reinterpret_cast<const float4*>(p.xres + (size_t)b * K + k);
        const float sc = scale[b];
        *reinterpret_cast<float4*>(xs + (size_t)b * (K / 32 * 36) + xs_index(k)) =
            make_float4(v.x * sc * g.x, v.y * sc * g.y, v.z * sc * g.z, v.w * sc * g.w);
      }
    }
  } else {
    for (int k = tid * 8; k < K; k += blockDim.x * 8)
#pragma unroll
      for (int b = 0; b < B; b++) {
        const uint4 u = *reinterpret_cast<const uint4*>(p.x + (size_t)b * p.ldx + k);
        const half2* h = reinterpret_cast<const half2*>(&u);
        float4 lo, hi;
        float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]), f2 = __half22float2(h[2]),
               f3 = __half22float2(h[3]);
        lo = make_float4(f0.x, f0.y, f1.x, f1.y);
        hi = make_float4(f2.x, f2.y, f3.x, f3.y);
        *reinterpret_cast<float4*>(xs + (size_t)b * (K / 32 * 36) + xs_index(k)) = lo;
        *reinterpret_cast<float4*>(xs + (size_t)b * (K / 32 * 36) + xs_index(k + 4)) = hi;
      }
  }
  __syncthreads();
}

constexpr size_t kGemvSmem = 96 * 1024;  // largest F32 activation stage per block

// Persistent warps: warp w handles output rows w, w + W, ... two at a time
// (or the gate and up rows of one FFN column in SwiGLU mode), so each lane
// keeps several 16-byte weight loads in flight and the grid (sized to fill
// the SMs) streams continuously.  The first weight loads are issued before
// pdl_wait(): weights never depend on the previous kernel, so their latency
// overlaps that kernel's tail.  In greedy mode (p.best) the rows are logits:
// the block keeps the running (logit, row) maximum and merges it with one
// atomicMax per batch row.
template <int B, bool FAST, bool XS>
__global__ void __launch_bounds__(256, (B <= 2 ? 3 : B <= 8 ? 2 : 1)) gemv2_kernel(const GemvPlan p) {
  constexpr int NV = 4;  // slots per row batch: Q8_0 2 groups, F16 1 group
  extern __shared__ uint4 gemv_smem[];
  const int lane = threadIdx.x % 32;
  const int W = gridDim.x * (blockDim.x / 32);
  const int w0 = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int K = p.seg[0].w.cols;
  // activations: XS = staged as F32 rows in shared memory (they fit), else F16 from global
  constexpr bool staged = XS;
  XSrc x{staged ? reinterpret_cast<const float*>(gemv_smem) : nullptr, p.x, staged ? K / 32 * 36 : p.ldx};
  if (p.swiglu) {
    const QTensor& wg = p.seg[0].w;
    const QTensor& wu = p.swiglu == 2 ? p.seg[0].w : p.seg[1].w;
    RowRaw<NV> rg, ru;
    auto rows_of = [&](int r, int& ng, int& nu) {
      ng = p.swiglu == 2 ? (r / 128) * 256 + r % 128 : r;
      nu = p.swiglu == 2 ? ng + 128 : r;
    };
    if (w0 < p.rows) {
      int ng, nu;
      rows_of(w0, ng, nu);
      row_load<NV>(wg, ng, lane, wg.cols / 32, rg);
      row_load<NV>(wu, nu, lane, wu.cols / 32, ru);
    }
    pdl_wait();
    pdl_trigger();
    if (staged) stage_x<B>(p, K, reinterpret_cast<float*>(gemv_smem));
    for (int r = w0; r < p.rows; r += W) {
      int ng, nu;
      rows_of(r, ng, nu);
      float g[B], u[B];
#pragma unroll
      for (int b = 0; b < B; b++) g[b] = u[b] = 0.f;
      if (r != w0) {
        row_load<NV>(wg, ng, lane, wg.cols / 32, rg);
        row_load<NV>(wu, nu, lane, wu.cols / 32, ru);
      }
      row_dot<B, NV, FAST, XS>(wg, ng, x, lane, rg, true, g);
      row_dot<B, NV, FAST, XS>(wu, nu, x, lane, ru, true, u);
      warp_sum<B>(g);
      warp_sum<B>(u);
      if (lane < B) {
        float gv = 0.f, uv = 0.f;
#pragma unroll
        for (int b = 0; b < B; b++)
          if (b == lane) {
            gv = g[b];
            uv = u[b];
          }
        p.act[(size_t)lane * p.ld_act + r] = __float2half_rn(gv / (1.f + __expf(-gv)) * uv);
      }
    }
    return;
  }
  auto locate = [&](int r, int& s, int& n) {
    s = 0;
    n = r;
    if (p.nseg > 1 && n >= p.seg[0].w.rows) {
      n -= p.seg[0].w.rows;
      s = 1;
      if (p.nseg > 2 && n >= p.seg[1].w.rows) {
        n -= p.seg[1].w.rows;
        s = 2;
      }
    }
  };
  auto mat = [&](int s) -> const QTensor& { return s == 0 ? p.seg[0].w : s == 1 ? p.seg[1].w : p.seg[2].w; };
  RowRaw<NV> ra, rb;
  {
    int s, n;
    if (w0 < p.rows) {
      locate(w0, s, n);
      row_load<NV>(mat(s), n, lane, mat(s).cols / 32, ra);
    }
    if (w0 + W < p.rows) {
      locate(w0 + W, s, n);
      row_load<NV>(mat(s), n, lane, mat(s).cols / 32, rb);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (staged) stage_x<B>(p, K, reinterpret_cast<float*>(gemv_smem));
  unsigned long long best[B];
#pragma unroll
  for (int b = 0; b < B; b++) best[b] = 0ull;
  auto finish = [&](int r, int s, int n, float (&acc)[B]) {
    warp_sum<B>(acc);
    if (p.best) {
#pragma unroll
      for (int b = 0; b < B; b++) {
        const unsigned long long k = pack_logit(acc[b], r);
        best[b] = k > best[b] ? k : best[b];
      }
    } else if (lane < B) {
      float v = 0.f;
#pragma unroll
      for (int b = 0; b < B; b++)
        if (b == lane) v = acc[b];
      float* y = s == 0 ? p.seg[0].y : s == 1 ? p.seg[1].y : p.seg[2].y;
      const int ldy = s == 0 ? p.seg[0].ldy : s == 1 ? p.seg[1].ldy : p.seg[2].ldy;
      const int accf = s == 0 ? p.seg[0].acc : s == 1 ? p.seg[1].acc : p.seg[2].acc;
      float* dst = y + (size_t)lane * ldy + n;
      *dst = accf ? *dst + v : v;
    }
  };
  for (int r = w0; r < p.rows; r += 2 * W) {
    const int r2 = r + W;
    int sa, na, sb = 0, nb2 = 0;
    locate(r, sa, na);
    if (r2 < p.rows) locate(r2, sb, nb2);
    if (r != w0) {  // both rows' first batches are issued before either is used
      row_load<NV>(mat(sa), na, lane, mat(sa).cols / 32, ra);
      if (r2 < p.rows) row_load<NV>(mat(sb), nb2, lane, mat(sb).cols / 32, rb);
    }
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; b++) acc[b] = 0.f;
    row_dot<B, NV, FAST, XS>(mat(sa), na, x, lane, ra, true, acc);
    finish(r, sa, na, acc);
    if (r2 < p.rows) {
#pragma unroll
      for (int b = 0; b < B; b++) acc[b] = 0.f;
      row_dot<B, NV, FAST, XS>(mat(sb), nb2, x, lane, rb, true, acc);
      finish(r2, sb, nb2, acc);
    }
  }
  if (p.best) {
    __shared__ unsigned long long blk[8][B];
    const int wb = threadIdx.x / 32;
    if (lane == 0)
#pragma unroll
      for (int b = 0; b < B; b++) blk[wb][b] = best[b];
    __syncthreads();
    if (threadIdx.x < B) {
      unsigned long long k = 0ull;
      for (int i = 0; i < (int)(blockDim.x / 32); i++) k = blk[i][threadIdx.x] > k ? blk[i][threadIdx.x] : k;
      atomicMax(p.best + threadIdx.x, k);
    }
  }
}

template <int B, bool FAST, bool XS>
static cudaError_t gemv2_bx(const GemvPlan& p, dim3 grid, size_t smem, cudaStream_t st) {
  static std::atomic<bool> configured[64];  // per device; any host thread may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemv2_kernel<B, FAST, XS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvSmem);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  return launch_k(gemv2_kernel<B, FAST, XS>, grid, dim3(256), smem, st, true, p);
}

template <int B, bool FAST>
static cudaError_t gemv2_b(const GemvPlan& p, dim3 grid, size_t smem, cudaStream_t st) {
  return smem ? gemv2_bx<B, FAST, true>(p, grid, smem, st) : gemv2_bx<B, FAST, false>(p, grid, smem, st);
}

template <bool FAST>
static cudaError_t gemv2_k(const GemvPlan& p, int nb, int num_sms, cudaStream_t st) {
  // enough warps to fill every SM at the kernel's occupancy, at most one per row
  const int per_sm = nb <= 2 ? 3 : nb <= 8 ? 2 : 1;
  const int blocks = std::min((p.rows + 7) / 8, num_sms * per_sm);
  const dim3 grid((unsigned)std::max(blocks, 1));
  const size_t need = (size_t)nb * (p.seg[0].w.cols / 32 * 36) * 4;
  if (p.xres && need > kGemvSmem) return cudaErrorInvalidValue;
  const size_t smem = need <= kGemvSmem ? need : 0;
  switch (nb) {
    case 1: return gemv2_b<1, FAST>(p, grid, smem, st);
    case 2: return gemv2_b<2, FAST>(p, grid, smem, st);
    case 4: return gemv2_b<4, FAST>(p, grid, smem, st);
    case 8: return gemv2_b<8, FAST>(p, grid, smem, st);
    case 16: return gemv2_b<16, FAST>(p, grid, smem, st);
  }
  return cudaErrorInvalidValue;
}

static cudaError_t gemv2(const GemvPlan& p, int nb, int num_sms, cudaStream_t st) {
  bool fast = true;
  for (int i = 0; i < (p.nseg > 0 ? p.nseg : 1); i++)
    fast &= p.seg[i].w.kind == K_Q8_0 || p.seg[i].w.kind == K_F16;
  return fast ? gemv2_k<true>(p, nb, num_sms, st) : gemv2_k<false>(p, nb, num_sms, st);
}

// ---------------------------------------------------------------- small kernels

// qkv F32 [B][qd+2kd] (+bias) -> rotate-half RoPE on q and k, q -> F16
// [B][qd], k and v appended to the paged cache at slot[b].
__global__ void rope_append_kernel(const float* __restrict__ qkv, const float* __restrict__ bias, int qd, int kd,
                                   int hd, int kvh, const int* __restrict__ pos, const int* __restrict__ slot,
                                   const float2* __restrict__ rope, half* __restrict__ q, half* __restrict__ kc,
                                   half* __restrict__ vc) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int n = qd + 2 * kd, half_hd = hd / 2;
  const float* row = qkv + (size_t)b * n;
  const int p = pos[b], s = slot[b];
  const int page = s / PAGE, off = s % PAGE;
  for (int i = threadIdx.x; i < qd / 2 + kd / 2 + kd; i += blockDim.x) {
    if (i < qd / 2 + kd / 2) {
      const bool isq = i < qd / 2;
      const int j = isq ? i : i - qd / 2;
      const int head = j / half_hd, jj = j % half_hd;
      const int c0 = (isq ? 0 : qd) + head * hd + jj, c1 = c0 + half_hd;
      float x0 = row[c0], x1 = row[c1];
      if (bias) {
        x0 += bias[c0];
        x1 += bias[c1];
      }
      const float2 cs = rope[(size_t)p * half_hd + jj];
      const float y0 = x0 * cs.x - x1 * cs.y, y1 = x1 * cs.x + x0 * cs.y;
      if (isq) {
        q[(size_t)b * qd + c0] = __float2half_rn(y0);
        q[(size_t)b * qd + c1] = __float2half_rn(y1);
      } else {
        half* dst = kc + (((size_t)page * kvh + head) * PAGE + off) * hd;
        dst[jj] = __float2half_rn(y0);
        dst[jj + half_hd] = __float2half_rn(y1);
      }
    } else {
      const int j = i - qd / 2 - kd / 2, c = qd + kd + j;
      float v = row[c];
      if (bias) v += bias[c];
      const int head = j / hd, jj = j % hd;
      vc[(((size_t)page * kvh + head) * PAGE + off) * hd + jj] = __float2half_rn(v);
    }
  }
}

// Greedy token from full-vocabulary logits (large batches, where the head
// runs on the tensor-core GEMM): best[b] = max over ids of pack_logit.
__global__ void argmax_best_kernel(const float* __restrict__ logits, int V, unsigned long long* __restrict__ best) {
  __shared__ unsigned long long sk[32];
  pdl_wait();
  pdl_trigger();
  const float* x = logits + (size_t)blockIdx.x * V;
  unsigned long long k = 0ull;
  for (int c = threadIdx.x; c < V; c += blockDim.x) {
    const unsigned long long kc = pack_logit(x[c], c);
    k = kc > k ? kc : k;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long ok = __shfl_xor_sync(0xffffffff, k, o);
    k = ok > k ? ok : k;
  }
  if (threadIdx.x % 32 == 0) sk[threadIdx.x / 32] = k;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)blockDim.x / 32; w++) k = sk[w] > k ? sk[w] : k;
    best[blockIdx.x] = k;
  }
}

struct DecSeq {
  int table_off, n_keys;
};

// Start of decode step s = ++counter: the greedy token of the previous step
// (or of the prefill) is taken from best[], recorded in toks[s-1] and fed to
// this step, best[] is cleared for this step's head, and the step's
// position, KV slot and key count move to fixed device addresses.
__global__ void advance_kernel(int* counter, unsigned long long* __restrict__ best, int* __restrict__ toks,
                               const int* __restrict__ pos_all, const int* __restrict__ slot_all,
                               const DecSeq* __restrict__ seq_all, int nb, int* __restrict__ cur_tok,
                               int* __restrict__ cur_pos, int* __restrict__ cur_slot, DecSeq* __restrict__ cur_seq,
                               unsigned* __restrict__ gbar, int n_gbar) {
  __shared__ int s;
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) s = *counter + 1;
  for (int i = threadIdx.x; i < n_gbar; i += blockDim.x) gbar[i] = 0u;  // this step's grid barriers
  __syncthreads();
  for (int i = threadIdx.x; i < nb; i += blockDim.x) {
    const int tok = unpack_row(best[i]);
    toks[(size_t)(s - 1) * nb + i] = tok;
    cur_tok[i] = tok;
    best[i] = 0ull;
    cur_pos[i] = pos_all[(size_t)s * nb + i];
    cur_slot[i] = slot_all[(size_t)s * nb + i];
    cur_seq[i] = seq_all[(size_t)s * nb + i];
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = s;
}

// Records the last step's greedy tokens.
__global__ void finalize_kernel(const unsigned long long* __restrict__ best, int* __restrict__ toks, int row, int nb) {
  for (int i = threadIdx.x; i < nb; i += blockDim.x) toks[(size_t)row * nb + i] = unpack_row(best[i]);
}

// ---------------------------------------------------------------- decode attention

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

// One CTA (4 warps) per (sequence, kv head, split of whole pages).  Each
// 64-token K/V page is staged in shared memory with cp.async (double
// buffered; K rows padded to 16-byte-aligned, bank-conflict-free strides);
// all threads score the G query heads of the GQA group against the page,
// then each warp updates the online softmax and P.V of its heads.  Writes
// the split's (max, sum, unnormalised output) for attn_combine_kernel.
template <int HD, int G>
__global__ void __launch_bounds__(128) attn_dec2_kernel(const half* __restrict__ q, const half* __restrict__ kc,
                                                        const half* __restrict__ vc, const int* __restrict__ tables,
                                                        const DecSeq* __restrict__ seqs, int KV, float scale_log2,
                                                        int split_pages, int splits, float* __restrict__ part) {
  constexpr int KP = HD + 8, DPL = HD / 32, HPW = (G + 3) / 4;
  extern __shared__ uint4 dsm[];
  half* sK = reinterpret_cast<half*>(dsm);                 // [2][64][KP]
  half* sV = sK + 2 * 64 * KP;                             // [2][64][HD]
  float* sQ = reinterpret_cast<float*>(sV + 2 * 64 * HD);  // [G][HD]
  float* sP = sQ + G * HD;                                 // [G][64]
  const int b = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
  const int H = KV * G;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  pdl_wait();
  pdl_trigger();
  const DecSeq s = seqs[b];
  const int n_pages = (s.n_keys + PAGE - 1) / PAGE;
  const int p0 = sp * split_pages, p1 = min(n_pages, p0 + split_pages);
  for (int i = tid; i < G * HD; i += 128) sQ[i] = __half2float(q[((size_t)b * H + kvh * G) * HD + i]);
  float m[HPW], l[HPW], acc[HPW][DPL];
#pragma unroll
  for (int hh = 0; hh < HPW; hh++) {
    m[hh] = -INFINITY;
    l[hh] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; d++) acc[hh][d] = 0.f;
  }
  auto load = [&](int p, int buf) {
    const int page = tables[s.table_off + p];
    const half* kp = kc + ((size_t)page * KV + kvh) * PAGE * HD;
    const half* vp = vc + ((size_t)page * KV + kvh) * PAGE * HD;
    for (int i = tid; i < PAGE * HD / 8; i += 128) {
      const int r = i / (HD / 8), c = i % (HD / 8);
      cp16(sK + (size_t)buf * 64 * KP + r * KP + c * 8, kp + r * HD + c * 8);
      cp16(sV + (size_t)buf * 64 * HD + r * HD + c * 8, vp + r * HD + c * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (p0 < p1) load(p0, 0);
  for (int p = p0; p < p1; p++) {
    const int buf = (p - p0) & 1;
    if (p + 1 < p1) {
      load(p + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const half* bK = sK + (size_t)buf * 64 * KP;
    const half* bV = sV + (size_t)buf * 64 * HD;
    for (int i = tid; i < G * 64; i += 128) {
      const int g = i / 64, j = i % 64;
      const half* kr = bK + j * KP;
      const float* qg = sQ + g * HD;
      float dot = 0.f;
#pragma unroll
      for (int c = 0; c < HD; c += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(kr + c);
        const half2* h = reinterpret_cast<const half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(h[e]);
          dot = fmaf(qg[c + 2 * e], f.x, dot);
          dot = fmaf(qg[c + 2 * e + 1], f.y, dot);
        }
      }
      sP[g * 64 + j] = (p * PAGE + j) < s.n_keys ? dot * scale_log2 : -INFINITY;
    }
    __syncthreads();
#pragma unroll
    for (int hh = 0; hh < HPW; hh++) {
      const int g = warp + 4 * hh;
      if (g >= G) break;
      const float s0 = sP[g * 64 + lane], s1 = sP[g * 64 + 32 + lane];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
      const float mn = fmaxf(m[hh], mx);
      const float corr = mn == -INFINITY ? 1.f : exp2f(m[hh] - mn);
      const float e0 = s0 == -INFINITY ? 0.f : exp2f(s0 - mn);
      const float e1 = s1 == -INFINITY ? 0.f : exp2f(s1 - mn);
      float sum = e0 + e1;
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffff, sum, o);
      l[hh] = l[hh] * corr + sum;
      m[hh] = mn;
#pragma unroll
      for (int d = 0; d < DPL; d++) acc[hh][d] *= corr;
#pragma unroll 16
      for (int j = 0; j < 64; j++) {
        const float pj = __shfl_sync(0xffffffff, j < 32 ? e0 : e1, j & 31);
        const half* vr = bV + j * HD + lane * DPL;
        if constexpr (DPL == 2) {
          const float2 f = __half22float2(*reinterpret_cast<const half2*>(vr));
          acc[hh][0] = fmaf(pj, f.x, acc[hh][0]);
          acc[hh][1] = fmaf(pj, f.y, acc[hh][1]);
        } else {
          const uint2 u = *reinterpret_cast<const uint2*>(vr);
          const half2* h2 = reinterpret_cast<const half2*>(&u);
          const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
          acc[hh][0] = fmaf(pj, f0.x, acc[hh][0]);
          acc[hh][1] = fmaf(pj, f0.y, acc[hh][1]);
          acc[hh][2] = fmaf(pj, f1.x, acc[hh][2]);
          acc[hh][3] = fmaf(pj, f1.y, acc[hh][3]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int hh = 0; hh < HPW; hh++) {
    const int g = warp + 4 * hh;
    if (g >= G) break;
    float* dst = part + (((size_t)b * H + kvh * G + g) * splits + sp) * (HD + 2);
    if (lane == 0) {
      dst[0] = m[hh];
      dst[1] = l[hh];
    }
#pragma unroll
    for (int d = 0; d < DPL; d++) dst[2 + lane * DPL + d] = acc[hh][d];
  }
}

// Decode attention for a GQA group of G <= 8 query heads over whole 64-token
// pages, one CTA per (sequence, kv head, split of pages).  A producer warp
// streams each page's K and V blocks into a shared-memory ring with 2-D
// tensor-map loads (64 rows x 128 B boxes, 128-byte swizzle); consumer warp
// w takes pages w, w+4, ... of the split, each with its own online softmax
// (src/models/openthai/model.rs:276-294), and the group's heads are the rows
// of mma.sync m16n8k16 tiles (S = Q.K^T, then P.V).  The four warps' states
// are merged in shared memory and written as one split partial in the form
// attn_combine_kernel reads (max in log2 units, sum, unnormalised output).
__device__ __forceinline__ int kv_off(int r, int c) {  // byte offset of 16-byte chunk c of page row r
  return (c >> 3) * 8192 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

template <int HD>
struct Dec3 {
  static constexpr int NW = 4;                    // consumer warps
  static constexpr int S = HD == 64 ? 8 : 4;      // ring stages (pages)
  static constexpr int PAGE_BYTES = 64 * HD * 2;  // K or V of one page
  static constexpr int STAGE = 2 * PAGE_BYTES;
  static constexpr int SMEM = S * STAGE + 2 * S * 8 + NW * 8 * (HD + 2) * 4 + 1024;
  // cluster form: the leader also holds every split's partial [CLS][8][HD + 2]
  // and the merge weights [8][CLS + 1]
  static constexpr int CLS = 8;  // most CTAs (key splits) per cluster
  static constexpr int SMEM_CL = SMEM + CLS * 8 * (HD + 2) * 4 + 8 * (CLS + 1) * 4;
};

// CL: the key splits (2..CLS) of one (sequence, kv head) form a cluster; each
// CTA stores its split partial into the leader's shared memory (DSMEM), and
// after one cluster barrier the leader merges them and writes the heads'
// F16 output rows, so no separate merge launch is needed.
template <int HD, int G, bool CL>
__global__ void __launch_bounds__(160, 1)
    attn_dec3_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                     const half* __restrict__ q, const int* __restrict__ tables, const DecSeq* __restrict__ seqs,
                     int KV, float scale_log2, int split_pages, int splits, float* __restrict__ part,
                     half* __restrict__ out, unsigned* err, long long budget) {
  using C = Dec3<HD>;
  extern __shared__ uint8_t d3_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(d3_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::S * C::STAGE);
  uint64_t* empty = full + C::S;
  float* comb = reinterpret_cast<float*>(empty + C::S);  // [NW][8][HD + 2]
  const int b = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
  const int H = KV * G;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::S; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  // CL: every CTA of the cluster must be running before any stores into the
  // leader's shared memory; this arrival is waited on just before them.
  if constexpr (CL) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  // The sequence table (written by the step's first kernel), the page table
  // and every K/V page except the one that holds this step's new key row
  // (written by the kernel just before this one) were written two or more
  // kernels back, which had completed before the previous kernel passed its
  // own griddepcontrol.wait and let this one start: the first pages' loads
  // are issued before waiting on the previous kernel.
  const DecSeq s = seqs[b];
  const int n_pages = (s.n_keys + PAGE - 1) / PAGE;
  const int p0 = sp * split_pages, p1 = min(n_pages, p0 + split_pages);
  const int np = max(0, p1 - p0);
  const int g = lane >> 2, t = lane & 3;
  auto load_page = [&](int i) {
    const int st = i % C::S;
    if (!mbar_wait(&empty[st], ((i / C::S) & 1) ^ 1, budget)) atomicOr(err, 1024u);
    const int row = (tables[s.table_off + p0 + i] * KV + kvh) * PAGE;
    uint8_t* dst = sm + st * C::STAGE;
    mbar_expect_tx(&full[st], C::STAGE);
#pragma unroll
    for (int hb = 0; hb < HD / 64; hb++) {
      tma_load_2d(dst + hb * 8192, &tk, &full[st], hb * 64, row);
      tma_load_2d(dst + C::PAGE_BYTES + hb * 8192, &tv, &full[st], hb * 64, row);
    }
  };
  // split-local index of the page holding the new row (np when it is not in this split)
  const int last = min(np, (s.n_keys - 1) / PAGE - p0);
  const int pre = max(0, min(min(np, C::S), last));
  if (warp == C::NW && lane == 0)
    for (int i = 0; i < pre; i++) load_page(i);
  pdl_wait();  // q and the new K/V row were written by the previous kernel
  pdl_trigger();
  if (warp == C::NW) {
    if (lane == 0)
      for (int i = pre; i < np; i++) load_page(i);
  } else {
    // Q of head g of the group as the A fragment (rows g + 8 are zero)
    uint32_t qa[HD / 16][4];
    const half* qg = q + ((size_t)b * H + kvh * G + (g < G ? g : 0)) * HD;
#pragma unroll
    for (int kk = 0; kk < HD / 16; kk++) {
      qa[kk][0] = g < G ? *reinterpret_cast<const uint32_t*>(qg + kk * 16 + 2 * t) : 0u;
      qa[kk][1] = 0u;
      qa[kk][2] = g < G ? *reinterpret_cast<const uint32_t*>(qg + kk * 16 + 8 + 2 * t) : 0u;
      qa[kk][3] = 0u;
    }
    float m = -INFINITY, l = 0.f;  // m in raw score units
    float acc[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    for (int i = warp; i < np; i += C::NW) {
      const int st = i % C::S;
      if (!mbar_wait(&full[st], (i / C::S) & 1, budget) && lane == 0) atomicOr(err, 2048u);
      const uint8_t* sK = sm + st * C::STAGE;
      const uint8_t* sV = sK + C::PAGE_BYTES;
      float sc[8][4];
#pragma unroll
      for (int j = 0; j < 8; j++) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < HD / 16; kk++) {
#pragma unroll
        for (int nj = 0; nj < 8; nj += 2) {
          uint32_t bf[4];
          const int mat = lane / 8;
          ldsm_x4(bf, sK + kv_off(nj * 8 + (lane % 8) + (mat / 2) * 8, kk * 2 + (mat % 2)));
          mma16816(sc[nj], qa[kk], bf[0], bf[1]);
          mma16816(sc[nj + 1], qa[kk], bf[2], bf[3]);
        }
      }
      const int key0 = (p0 + i) * PAGE;
      if (key0 + PAGE > s.n_keys) {
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
          for (int e = 0; e < 2; e++)
            if (key0 + j * 8 + 2 * t + e >= s.n_keys) sc[j][e] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; j++) mx = fmaxf(mx, fmaxf(sc[j][0], sc[j][1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      // every page of the split holds at least one key, so mn is finite
      const float mn = fmaxf(m, mx);
      const float corr = exp2f((m - mn) * scale_log2), off = -mn * scale_log2;
      m = mn;
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        sc[j][0] = exp2f(fmaf(sc[j][0], scale_log2, off));
        sc[j][1] = exp2f(fmaf(sc[j][1], scale_log2, off));
        sum += sc[j][0] + sc[j][1];
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      l = l * corr + sum;
#pragma unroll
      for (int d = 0; d < HD / 8; d++) {
        acc[d][0] *= corr;
        acc[d][1] *= corr;
      }
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const uint32_t pa[4] = {pack_h2(sc[2 * kk][0], sc[2 * kk][1]), 0u, pack_h2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]),
                                0u};
#pragma unroll
        for (int nd = 0; nd < HD / 8; nd += 2) {
          uint32_t bf[4];
          const int mat = lane / 8;
          ldsm_x4_t(bf, sV + kv_off(kk * 16 + (lane % 8) + (mat % 2) * 8, nd + mat / 2));
          mma16816(acc[nd], pa, bf[0], bf[1]);
          mma16816(acc[nd + 1], pa, bf[2], bf[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (g < G) {
      float* cw = comb + (warp * 8 + g) * (HD + 2);
      if (t == 0) {
        cw[0] = m == -INFINITY ? -INFINITY : m * scale_log2;
        cw[1] = l;
      }
#pragma unroll
      for (int d = 0; d < HD / 8; d++) {
        cw[2 + d * 8 + 2 * t] = acc[d][0];
        cw[2 + d * 8 + 2 * t + 1] = acc[d][1];
      }
    }
  }
  __syncthreads();
  // merge the consumer warps: one split partial per head of the group
  float* cp = comb + C::NW * 8 * (HD + 2);  // CL: the leader's [CLS][G][HD + 2]
  if constexpr (CL) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  for (int idx = threadIdx.x; idx < G * (HD + 2); idx += blockDim.x) {
    const int gg = idx / (HD + 2), c = idx % (HD + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < C::NW; w++) M = fmaxf(M, comb[(w * 8 + gg) * (HD + 2)]);
    float v = c == 0 ? M : 0.f;
    if (c > 0 && M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < C::NW; w++) {
        const float mw = comb[(w * 8 + gg) * (HD + 2)];
        if (mw != -INFINITY) v += exp2f(mw - M) * comb[(w * 8 + gg) * (HD + 2) + c];
      }
    }
    if constexpr (CL) {
      const uint32_t dst = cluster_addr(cp + ((size_t)sp * G + gg) * (HD + 2) + c, 0);
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(v) : "memory");
    } else {
      part[(((size_t)b * H + kvh * G + gg) * splits + sp) * (HD + 2) + c] = v;
    }
  }
  if constexpr (CL) {
    // o = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s over the cluster's splits
    cluster_sync();
    if (sp != 0) return;
    float* wts = cp + C::CLS * G * (HD + 2);  // [G][CLS + 1]: split weights, then 1 / l
    if (threadIdx.x < G) {
      const int gg = threadIdx.x;
      float M = -INFINITY;
      for (int s2 = 0; s2 < splits; s2++) M = fmaxf(M, cp[(s2 * G + gg) * (HD + 2)]);
      float l = 0.f;
      for (int s2 = 0; s2 < splits; s2++) {
        const float ms = cp[(s2 * G + gg) * (HD + 2)];
        const float wgt = ms == -INFINITY ? 0.f : exp2f(ms - M);
        wts[gg * (C::CLS + 1) + s2] = wgt;
        l += wgt * cp[(s2 * G + gg) * (HD + 2) + 1];
      }
      wts[gg * (C::CLS + 1) + C::CLS] = 1.f / l;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
      const int gg = idx / HD, d = idx % HD;
      float v = 0.f;
      for (int s2 = 0; s2 < splits; s2++) v += wts[gg * (C::CLS + 1) + s2] * cp[(s2 * G + gg) * (HD + 2) + 2 + d];
      out[((size_t)b * H + kvh * G + gg) * HD + d] = __float2half_rn(v * wts[gg * (C::CLS + 1) + C::CLS]);
    }
  }
}

// Merges the key splits: o = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s.
// The split weights are computed once into shared memory; then the threads
// (dims x split subsets) sum independent, coalesced loads.
__global__ void attn_combine_kernel(const float* __restrict__ part, int H, int HD, int splits, half* __restrict__ o) {
  extern __shared__ float cs[];  // [splits] weights, then [blockDim] partial sums
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, h = blockIdx.y;
  const float* p = part + ((size_t)b * H + h) * splits * (HD + 2);
  float mx = -INFINITY;
  for (int s = threadIdx.x; s < splits; s += blockDim.x) mx = fmaxf(mx, p[(size_t)s * (HD + 2)]);
#pragma unroll
  for (int o2 = 16; o2; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o2));
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int w = 1; w < (int)blockDim.x / 32; w++) m = fmaxf(m, red[w]);
    red[0] = m;
  }
  __syncthreads();
  const float M = red[0];
  __syncthreads();
  float l = 0.f;
  for (int s = threadIdx.x; s < splits; s += blockDim.x) {
    const float ms = p[(size_t)s * (HD + 2)];
    const float wgt = ms == -INFINITY ? 0.f : exp2f(ms - M);
    cs[s] = wgt;
    l += wgt * p[(size_t)s * (HD + 2) + 1];
  }
#pragma unroll
  for (int o2 = 16; o2; o2 >>= 1) l += __shfl_xor_sync(0xffffffff, l, o2);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = l;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; w++) t += red[w];
    red[0] = t;
  }
  __syncthreads();
  const float inv = 1.f / red[0];
  const int ways = blockDim.x / HD;  // threads per dimension
  const int dd = threadIdx.x % HD, part_i = threadIdx.x / HD;
  float acc = 0.f;
  if (part_i < ways) {
#pragma unroll 8
    for (int s = part_i; s < splits; s += ways) acc += cs[s] * p[(size_t)s * (HD + 2) + 2 + dd];
  }
  float* ps = cs + splits;
  ps[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x < HD) {
    float t = 0.f;
    for (int i = 0; i < ways; i++) t += ps[i * HD + threadIdx.x];
    o[((size_t)b * H + h) * HD + threadIdx.x] = __float2half_rn(t * inv);
  }
}

// ---------------------------------------------------------------- host

struct AttnShape {
  int splits, split_pages;    // attn_dec2_kernel
  int splits3, split_pages3;  // attn_dec3_kernel: one CTA per SM, so at most one wave of CTAs
  bool cluster;               // attn_dec3_kernel with its splits as one cluster
  int splits_cl, split_pages_cl;
};

static bool dec3_cluster_enabled() {
  const char* e = std::getenv("LAYA_DEC_CLUSTER");
  return !(e && e[0] == '0');
}

static AttnShape attn_shape(const Replica& r, const Config& c, int nb, int max_keys) {
  const int pages = (max_keys + PAGE - 1) / PAGE;
  int splits = std::max(1, (4 * r.num_sms + nb * c.KV - 1) / (nb * c.KV));
  splits = std::min(splits, pages);
  const int split_pages = (pages + splits - 1) / splits;
  int s3 = std::max(1, std::min(r.num_sms / (nb * c.KV), (pages + 1) / 2));
  const int sp3 = (pages + s3 - 1) / s3;
  // clusters of a power of two of splits (2..CLS) within one wave of CTAs;
  // trailing splits may hold no page (their partial has weight 0)
  constexpr int CLS = Dec3<64>::CLS;
  const int n3 = (pages + sp3 - 1) / sp3;
  int cls = CLS;
  while (cls > 1 && (nb * c.KV * cls > r.num_sms || cls > pages)) cls /= 2;
  const int spcl = (pages + cls - 1) / cls;
  const bool cl = dec3_cluster_enabled() && cls >= 2;
  return {(pages + split_pages - 1) / split_pages, split_pages, n3, sp3, cl, cl ? cls : 0, spcl};
}

static bool seq_enabled() {
  const char* e = std::getenv("LAYA_DECODE_SEQ");
  return !(e && e[0] == '0');
}

static bool dec3_enabled() {
  const char* e = std::getenv("LAYA_DEC_ATTN3");
  return !(e && e[0] == '0');
}

template <int HD, int G>
static cudaError_t launch_dec3(dim3 grid, cudaStream_t st, const CUtensorMap& tk, const CUtensorMap& tv,
                               const half* q, const int* tables, const DecSeq* seqs, int KV, float sl2,
                               int split_pages, int splits, float* part, half* out, bool cl, unsigned* err) {
  static std::atomic<bool> configured[64];  // per device; any host thread may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e =
        cudaFuncSetAttribute(attn_dec3_kernel<HD, G, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, Dec3<HD>::SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_dec3_kernel<HD, G, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Dec3<HD>::SMEM_CL);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  if (!cl)
    return launch_k(attn_dec3_kernel<HD, G, false>, grid, dim3(160), (size_t)Dec3<HD>::SMEM, st, true, tk, tv, q,
                    tables, seqs, KV, sl2, split_pages, splits, part, out, err, 4000000000ll);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(160);
  cfg.dynamicSmemBytes = Dec3<HD>::SMEM_CL;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = splits;  // one cluster per (sequence, kv head)
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, attn_dec3_kernel<HD, G, true>, tk, tv, q, tables, seqs, KV, sl2, split_pages,
                            splits, part, out, err, 4000000000ll);
}

template <int HD, int G>
static cudaError_t launch_dec2(dim3 grid, cudaStream_t st, const half* q, const half* kc, const half* vc,
                               const int* tables, const DecSeq* seqs, int KV, float sl2, int split_pages, int splits,
                               float* part) {
  const int smem = (2 * 64 * (HD + 8) + 2 * 64 * HD) * 2 + (G * HD + G * 64) * 4;
  static std::atomic<bool> configured[64];  // per device; any host thread may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(attn_dec2_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  return launch_k(attn_dec2_kernel<HD, G>, grid, dim3(128), smem, st, true, q, kc, vc, tables, seqs, KV, sl2,
                  split_pages, splits, part);
}

static int decode_attention(Model& m, Replica& r, int nb, const half* q, const half* kc, const half* vc,
                            const DecSeq* seqs, const AttnShape& sh, half* out) {
  const Config& c = m.cfg;
  const float sl2 = (1.f / sqrtf((float)c.hd)) * 1.4426950408889634f;
  const int G = c.H / c.KV;
  cudaEvent_t a;
  prof_begin(r, P_ATTN_DEC, &a);
  r.launches += 2;
  cudaError_t e = cudaErrorNotSupported;
  const int* tb = r.tables.as<int>();
  float* part = r.dpart.as<float>();
  int splits = sh.splits;
  bool cl = false;
  if (dec3_enabled() && G <= 8 && (c.hd == 64 || c.hd == 128)) {
    // K and V of this layer as [pages * kv_heads * 64 rows][hd] F16, 64 x 64 boxes
    CUtensorMap tk, tv;
    const uint64_t dims[2] = {(uint64_t)c.hd, (uint64_t)r.kv_pages * c.KV * PAGE}, strides[1] = {(uint64_t)c.hd * 2};
    const uint32_t box[2] = {64, 64};
    if (!encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, vc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(LAYA_E_CUDA, "KV tensor map");
    // Few (sequence, kv head) pairs: eight key splits per pair as one
    // cluster that merges its partials itself (no merge launch).
    cl = sh.cluster;
    const int sp3 = cl ? sh.split_pages_cl : sh.split_pages3;
    splits = cl ? sh.splits_cl : sh.splits3;
    const dim3 g3(nb, c.KV, splits);
#define LAYA_DEC3(HDV, GV)                                                                                    \
  if (c.hd == HDV && G == GV)                                                                                 \
    e = launch_dec3<HDV, GV>(g3, r.stream, tk, tv, q, tb, seqs, c.KV, sl2, sp3, splits, part, out, cl, r.err);
    LAYA_DEC3(64, 1)
    LAYA_DEC3(64, 2)
    LAYA_DEC3(64, 4)
    LAYA_DEC3(64, 8)
    LAYA_DEC3(128, 1)
    LAYA_DEC3(128, 2)
    LAYA_DEC3(128, 4)
    LAYA_DEC3(128, 7)
    LAYA_DEC3(128, 8)
#undef LAYA_DEC3
    if (e == cudaErrorNotSupported) {  // the split-merge form below
      cl = false;
      splits = sh.splits;
    }
  }
  const dim3 grid(nb, c.KV, sh.splits);
#define LAYA_DEC2(HDV, GV)                                                                                         \
  if (e == cudaErrorNotSupported && c.hd == HDV && G == GV)                                                       \
    e = launch_dec2<HDV, GV>(grid, r.stream, q, kc, vc, tb, seqs, c.KV, sl2, sh.split_pages, sh.splits, part);
  LAYA_DEC2(64, 1)
  LAYA_DEC2(64, 2)
  LAYA_DEC2(64, 4)
  LAYA_DEC2(64, 8)
  LAYA_DEC2(128, 1)
  LAYA_DEC2(128, 2)
  LAYA_DEC2(128, 4)
  LAYA_DEC2(128, 7)
  LAYA_DEC2(128, 8)
#undef LAYA_DEC2
  if (e == cudaErrorNotSupported) return fail(LAYA_E_INVALID, "unsupported head grouping for decode");
  if (e != cudaSuccess) return cuda_fail(e, "attn_dec2_kernel");
  if (cl) {
    r.launches--;
  } else {
    const int cthreads = 256;
    LAYA_CK(launch_k(attn_combine_kernel, dim3(nb, c.H), dim3(cthreads), (size_t)(splits + cthreads) * 4, r.stream,
                     true, (const float*)part, c.H, c.hd, splits, out));
  }
  prof_end(r, P_ATTN_DEC, a);
  return 0;
}

static int run_gemv(Replica& r, const GemvPlan& p, int nb) {
  cudaEvent_t a;
  prof_begin(r, P_GEMV, &a);
  r.launches++;
  LAYA_CK(gemv2(p, nb, r.num_sms, r.stream));
  prof_end(r, P_GEMV, a);
  return 0;
}

static Gemv3Args gv3_base(Replica& r, int mode, int nb, int K) {
  Gemv3Args a{};
  a.mode = mode;
  a.nb = nb;
  a.K = K;
  a.err = r.err;
  a.budget = 4000000000ll;
  return a;
}

static int run_gemv3(Replica& r, const Gemv3Args& a) {
  cudaEvent_t ev;
  prof_begin(r, P_GEMV, &ev);
  r.launches++;
  LAYA_CK(gemv3_launch(a, r.num_sms, r.stream));
  prof_end(r, P_GEMV, ev);
  return 0;
}

// Weight-side arguments of the four GEMV launches of layer l (i = 0 qkv,
// 1 attention output, 2 gate/up, 3 down) and of the head (l = L).
static Gemv3Args gv3_weights(const Model& m, const Replica& r, int l, int i) {
  const Config& c = m.cfg;
  Gemv3Args a{};
  a.nb = 1;
  if (l == c.L) {
    a.mode = GV_ARGMAX;
    a.K = c.d;
    a.seg[0] = r.head;
    return a;
  }
  const Layer& L = r.layers[l];
  switch (i) {
    case 0:
      a.mode = GV_QKV;
      a.K = c.d;
      a.seg[0] = L.wq;
      a.seg[1] = L.wk;
      a.seg[2] = L.wv;
      a.qd = c.H * c.hd;
      a.kd = c.KV * c.hd;
      a.hd = c.hd;
      a.kvh = c.KV;
      break;
    case 1:
      a.mode = GV_PLAIN;
      a.K = c.H * c.hd;
      a.seg[0] = L.wo;
      break;
    case 2:
      a.mode = GV_SWIGLU;
      a.K = c.d;
      a.seg[0] = L.wg;
      a.seg[1] = L.wu;
      a.interleaved = L.wgu16 != nullptr;
      break;
    default:
      a.mode = GV_PLAIN;
      a.K = c.ffn;
      a.seg[0] = L.wd;
  }
  return a;
}

// Builds the packed streaming images once per replica (device memory held
// until close).  A layer whose operands do not all pack keeps the
// warp-per-row GEMV.
static int ensure_gv_packed(const Model& m, Replica& r) {
  const Config& c = m.cfg;
  if ((int)r.gv_packed.size() == 4 * c.L + 1) return 0;
  std::vector<const uint8_t*> out(4 * c.L + 1, nullptr);
  for (int l = 0; l <= c.L; l++) {
    const int nops = l == c.L ? 1 : 4;
    std::vector<size_t> bytes(nops);
    bool ok = true;
    for (int i = 0; i < nops; i++) {
      bytes[i] = gemv3_packed_bytes(gv3_weights(m, r, l, i));
      ok &= bytes[i] > 0;
    }
    if (!ok) continue;
    for (int i = 0; i < nops; i++) {
      void* p = nullptr;
      LAYA_CK(cudaMalloc(&p, bytes[i]));
      r.allocs.push_back(p);
      LAYA_CK(gemv3_pack(gv3_weights(m, r, l, i), static_cast<uint8_t*>(p), r.stream));
      out[4 * l + i] = static_cast<const uint8_t*>(p);
    }
  }
  LAYA_CK(cudaStreamSynchronize(r.stream));
  r.gv_packed = out;
  return 0;
}

static bool gemv3_enabled() {
  const char* e = std::getenv("LAYA_GEMV3");
  return !(e && e[0] == '0');
}

static GemvPlan plan1(const QTensor& w, const half* x, int ldx, float* y, int ldy, int acc) {
  GemvPlan p{};
  p.seg[0] = {w, y, ldy, acc};
  p.nseg = 1;
  p.rows = w.rows;
  p.x = x;
  p.ldx = ldx;
  return p;
}

// Batches above this size run the linear layers on the tcgen05 GEMM.
static constexpr int kGemvMaxBatch = 16;

static int pad_batch(int nb);

// Whether a decode batch of nb sequences runs its linear layers as GEMVs:
// at most kGemvMaxBatch rows, and, with the streaming GEMV, only when its
// staged activation rows (the widest K of the layer) fit beside its ring;
// otherwise the tcgen05 GEMM takes them (e.g. 16 rows of the 8192-wide
// down projection would need 262 KB of shared memory).
static bool gemv_batch(const Config& c, int nb) {
  if (nb > kGemvMaxBatch) return false;
  if (!gemv3_enabled()) return true;
  return gemv3_fits(pad_batch(nb), std::max(c.d, std::max(c.ffn, c.H * c.hd)));
}

static int pad_batch(int nb) { return nb <= 1 ? 1 : nb <= 2 ? 2 : nb <= 4 ? 4 : nb <= 8 ? 8 : 16; }

// Fixed device addresses of the per-step inputs.
struct StepIO {
  int* counter;
  unsigned long long* best;  // [nb] packed (logit, id) maxima of the current step
  int* toks;  // [steps][nb] greedy tokens
  const int *pos_all, *slot_all;
  const DecSeq* seq_all;
  int *cur_tok, *cur_pos, *cur_slot;
  DecSeq* cur_seq;
  unsigned* gbar;  // [layers] grid barrier counters of the multi-phase GEMV launches
  int n_gbar;
};

// One decode step for nb sequences; every pointer it uses is fixed, so the
// launch sequence can be captured once and replayed.
static int decode_step(Model& m, Replica& r, int nb, const StepIO& io, const AttnShape& sh) {
  const Config& c = m.cfg;
  const int qd = c.H * c.hd, kd = c.KV * c.hd, d = c.d, ffn = c.ffn;
  cudaStream_t st = r.stream;
  const bool small = gemv_batch(c, nb);
  const int nbp = small ? pad_batch(nb) : nb;  // GEMV batch (padded rows are zero)
  // Batches past the GEMV run the layer GEMMs on the Q8_0 blocks where the
  // model allows (scales and split planes were prepared by decode_run), else
  // on the F16 operands: the residual and QKV GEMMs split K when their output
  // tiles are few, and the next RMSNorm / qkv_merge adds the partial planes
  // in split order.
  const bool q8 = !small && use_q8_gemm(m, r, nb) && r.layers.back().sqkv_t;
  auto dsplit = [&](int N, int K) {
    return small ? 1 : q8 ? gemm_q8_ksplit(nb, N, K, r.num_sms) : gemm_ksplit(nb, N, K, r.num_sms);
  };
  const int ks_q = dsplit(qd + 2 * kd, d);
  const int ks_o = dsplit(d, qd);
  const int ks_d = dsplit(d, ffn);
  int pend = 0;  // K splits of x not yet merged
  int rc;
  r.launches++;
  LAYA_CK(launch_k(advance_kernel, dim3(1), dim3(256), 0, st, true, io.counter, io.best, io.toks, io.pos_all,
                   io.slot_all, io.seq_all, nb, io.cur_tok, io.cur_pos, io.cur_slot, io.cur_seq, io.gbar,
                   io.n_gbar));
  float* x = r.x.as<float>();
  r.launches++;
  LAYA_CK(rows_f32(r.embd, io.cur_tok, nb, x, st, true));
  half* h = r.h.as<half>();
  float* f = r.dlogits.as<float>();  // F32 scratch for GEMV outputs
  const size_t layer_elems = (size_t)r.kv_pages * c.KV * PAGE * c.hd;
  const int big = 1 << 30;
  auto gemm_d = [&](int cat, int epi, const half* A, int lda, const half* B, int ldb, GemmArgs a) -> int {
    a.err = r.err;
    a.budget = 4000000000ll;
    cudaEvent_t ev;
    prof_begin(r, cat, &ev);
    r.launches++;
    LAYA_CK(gemm_launch(epi, A, lda, B, ldb, a, r.num_sms, st));
    prof_end(r, cat, ev);
    return 0;
  };
  auto gemm_q8d = [&](int cat, int epi, const half* A, int lda, const Q8Weights& w, GemmArgs a) -> int {
    a.err = r.err;
    a.budget = 4000000000ll;
    cudaEvent_t ev;
    prof_begin(r, cat, &ev);
    r.launches++;
    LAYA_CK(gemm_q8_launch(epi, A, lda, w, a, r.num_sms, st));
    prof_end(r, cat, ev);
    return 0;
  };
  // RMSNorm of the residual rows into h, adding pending K-split planes first
  auto dnorm = [&](const float* w) -> int {
    r.launches++;
    const int ns = pend;
    pend = 0;
    if (ns > 1)
      LAYA_CK(rmsnorm_merge(x, nullptr, nb, r.kpart.as<float>(), ns, (size_t)nb * d, w, d, c.eps, h, nullptr, st));
    else
      LAYA_CK(rmsnorm(x, nullptr, nb, w, d, c.eps, h, nullptr, st));
    return 0;
  };
  auto stage = [&](const QTensor& t, half* out, int ldo, int grp, int gstride, int goff) -> int {
    r.launches++;
    LAYA_CK(dequant_f16(t, out, ldo, grp, gstride, goff, st));
    return 0;
  };
  const bool packed_all = (int)r.gv_packed.size() == 4 * c.L + 1;
  // The four streaming-GEMV operands of layer l: g[0] qkv, g[1] attention
  // output, g[2] gate/up, g[3] down.  Returns whether all of them run on it.
  auto layer_args = [&](int l, Gemv3Args* g) -> bool {
    const Layer& L = r.layers[l];
    half* kcl = r.kc.as<half>() + l * layer_elems;
    half* vcl = r.vc.as<half>() + l * layer_elems;
    Gemv3Args& gq = g[0];
    gq = gv3_base(r, GV_QKV, nb, d);
    gq.seg[0] = L.wq;
    gq.seg[1] = L.wk;
    gq.seg[2] = L.wv;
    gq.xres = x;  // RMSNorm fused (src/models/openthai/model.rs:84-94)
    gq.norm_w = L.attn_norm;
    gq.eps = c.eps;
    gq.qd = qd;
    gq.kd = kd;
    gq.hd = c.hd;
    gq.kvh = c.KV;
    gq.bias = L.bqkv;
    gq.pos = io.cur_pos;
    gq.slot = io.cur_slot;
    gq.rope = r.rope;
    gq.q = r.qb.as<half>();
    gq.kcache = kcl;
    gq.vcache = vcl;
    gq.page_size = PAGE;
    Gemv3Args& go = g[1];
    go = gv3_base(r, GV_PLAIN, nb, qd);
    go.seg[0] = L.wo;
    go.x = r.att.as<half>();
    go.ldx = qd;
    go.y = x;  // residual add (tensor::add, src/tensor.rs:123-128)
    go.ldy = d;
    go.acc = 1;
    Gemv3Args& gg = g[2];
    gg = gv3_base(r, GV_SWIGLU, nb, d);
    gg.seg[0] = L.wg;
    gg.seg[1] = L.wu;
    gg.interleaved = L.wgu16 != nullptr;
    gg.xres = x;
    gg.norm_w = L.ffn_norm;
    gg.eps = c.eps;
    gg.act = r.act.as<half>();
    gg.ld_act = ffn;
    Gemv3Args& gd = g[3];
    gd = gv3_base(r, GV_PLAIN, nb, ffn);
    gd.seg[0] = L.wd;
    gd.x = r.act.as<half>();
    gd.ldx = ffn;
    gd.y = x;
    gd.ldy = d;
    gd.acc = 1;
    if (!(small && gemv3_enabled() && packed_all)) return false;
    for (int i = 0; i < 4; i++) {
      g[i].packed = r.gv_packed[4 * l + i];
      if (!g[i].packed || !gemv3_supported(g[i])) return false;
    }
    return true;
  };
  Gemv3Args gh = gv3_base(r, GV_ARGMAX, nb, d);
  gh.seg[0] = r.head;
  gh.xres = x;
  gh.norm_w = r.out_norm;
  gh.eps = c.eps;
  gh.best = io.best;
  gh.packed = packed_all ? r.gv_packed[4 * c.L] : nullptr;
  const bool head3 = small && gemv3_enabled() && gh.packed && gemv3_supported(gh);
  // Whole-model chaining: after layer l's attention, one cooperative launch
  // runs attention output, gate/up, down and the next layer's qkv (the head
  // after the last layer), so the weights stream without a launch gap.
  std::vector<Gemv3Args> ga(4 * c.L);
  bool seq = head3 && seq_enabled() && io.gbar && io.n_gbar >= c.L;
  for (int l = 0; seq && l < c.L; l++) {
    seq = layer_args(l, &ga[4 * l]);
    for (int i = 0; seq && i < 4; i++) seq = ga[4 * l + i].seg[0].kind == gh.seg[0].kind;
  }
  for (int l = 0; l < c.L; l++) {
    const Layer& L = r.layers[l];
    half* kcl = r.kc.as<half>() + l * layer_elems;
    half* vcl = r.vc.as<half>() + l * layer_elems;
    Gemv3Args g4[4];
    const bool v3 = layer_args(l, g4);
    Gemv3Args &gq = g4[0], &go = g4[1], &gg = g4[2], &gd = g4[3];
    if (!small && (rc = dnorm(L.attn_norm))) return rc;
    if (seq) {
      if (l == 0 && (rc = run_gemv3(r, gq))) return rc;  // later layers' qkv ran in the previous chain
    } else if (small && v3) {
      if ((rc = run_gemv3(r, gq))) return rc;
    } else if (small) {
      GemvPlan p{};
      if (L.wqkv16) {
        QTensor fused = L.wq;
        fused.rows = qd + 2 * kd;
        p = plan1(fused, h, d, f, qd + 2 * kd, 0);
      } else {
        p.seg[0] = {L.wq, f, qd + 2 * kd, 0};
        p.seg[1] = {L.wk, f + qd, qd + 2 * kd, 0};
        p.seg[2] = {L.wv, f + qd + kd, qd + 2 * kd, 0};
        p.nseg = 3;
        p.rows = qd + 2 * kd;
      }
      p.xres = x;  // RMSNorm fused into the GEMV (padded batch rows of x are zero)
      p.norm_w = L.attn_norm;
      p.eps = c.eps;
      if ((rc = run_gemv(r, p, nbp))) return rc;
      r.launches++;
      LAYA_CK(launch_k(rope_append_kernel, dim3(nb), dim3(256), 0, st, true, (const float*)f, L.bqkv, qd, kd, c.hd,
                       c.KV, (const int*)io.cur_pos, (const int*)io.cur_slot, r.rope, r.qb.as<half>(), kcl, vcl));
    } else if (q8) {
      if (ks_q > 1) {
        GemmArgs sp{};
        sp.M = nb;
        sp.N = qd + 2 * kd;
        sp.K = d;
        sp.ldo = qd + 2 * kd;
        sp.ksplit = ks_q;
        sp.part = r.kpart.as<float>();
        if ((rc = gemm_q8d(P_GEMM_QKV, EPI_RESID, h, d, q8_qkv(c, L), sp))) return rc;
        r.launches++;
        LAYA_CK(qkv_merge(r.kpart.as<float>(), ks_q, (size_t)nb * (qd + 2 * kd), nb, L.bqkv, qd, kd, c.hd, c.KV,
                          io.cur_pos, io.cur_slot, r.rope, PAGE, r.qb.as<half>(), qd, kcl, vcl, st));
      } else {
        GemmArgs a{};
        a.M = nb;
        a.N = qd + 2 * kd;
        a.K = d;
        a.bias = L.bqkv;
        a.out = r.qb.p;
        a.ldo = qd;
        a.qd = qd;
        a.kd = kd;
        a.hd = c.hd;
        a.kvh = c.KV;
        a.pos = io.cur_pos;
        a.slot = io.cur_slot;
        a.rope = r.rope;
        a.kcache = kcl;
        a.vcache = vcl;
        a.page_size = PAGE;
        if ((rc = gemm_q8d(P_GEMM_QKV, EPI_QKV, h, d, q8_qkv(c, L), a))) return rc;
      }
    } else {
      const half* wqkv = L.wqkv16 ? L.wqkv16 : L.rqkv16;
      if (!wqkv) {
        half* s = r.wqkv_s.as<half>();
        if ((rc = stage(L.wq, s, d, big, 0, 0)) || (rc = stage(L.wk, s, d, big, 0, qd)) ||
            (rc = stage(L.wv, s, d, big, 0, qd + kd)))
          return rc;
        wqkv = s;
      }
      GemmArgs a{};
      a.M = nb;
      a.N = qd + 2 * kd;
      a.K = d;
      a.bias = L.bqkv;
      a.out = r.qb.p;
      a.ldo = qd;
      a.qd = qd;
      a.kd = kd;
      a.hd = c.hd;
      a.kvh = c.KV;
      a.pos = io.cur_pos;
      a.slot = io.cur_slot;
      a.rope = r.rope;
      a.kcache = kcl;
      a.vcache = vcl;
      a.page_size = PAGE;
      if (ks_q > 1) {
        GemmArgs sp{};
        sp.M = nb;
        sp.N = qd + 2 * kd;
        sp.K = d;
        sp.ldo = qd + 2 * kd;
        sp.ksplit = ks_q;
        sp.part = r.kpart.as<float>();
        if ((rc = gemm_d(P_GEMM_QKV, EPI_RESID, h, d, wqkv, d, sp))) return rc;
        r.launches++;
        LAYA_CK(qkv_merge(r.kpart.as<float>(), ks_q, (size_t)nb * (qd + 2 * kd), nb, L.bqkv, qd, kd, c.hd, c.KV,
                          io.cur_pos, io.cur_slot, r.rope, PAGE, r.qb.as<half>(), qd, kcl, vcl, st));
      } else if ((rc = gemm_d(P_GEMM_QKV, EPI_QKV, h, d, wqkv, d, a))) {
        return rc;
      }
    }
    if ((rc = decode_attention(m, r, nb, r.qb.as<half>(), kcl, vcl, io.cur_seq, sh, r.att.as<half>()))) return rc;
    if (seq) {
      const Gemv3Args ph[4] = {go, gg, gd, l + 1 < c.L ? ga[4 * (l + 1)] : gh};
      cudaEvent_t ev;
      prof_begin(r, P_GEMV, &ev);
      r.launches++;
      LAYA_CK(gemv3_launch_seq(ph, 4, io.gbar + l, r.num_sms, st));
      prof_end(r, P_GEMV, ev);
      continue;
    }
    if (small && v3) {
      if ((rc = run_gemv3(r, go))) return rc;
    } else if (small) {
      if ((rc = run_gemv(r, plan1(L.wo, r.att.as<half>(), qd, x, d, 1), nbp))) return rc;
    } else if (q8) {
      GemmArgs b{};
      b.M = nb;
      b.N = d;
      b.K = qd;
      b.resid = x;
      b.ldo = d;
      b.ksplit = ks_o;
      b.part = r.kpart.as<float>();
      if ((rc = gemm_q8d(P_GEMM_O, EPI_RESID, r.att.as<half>(), qd, q8_o(c, L), b))) return rc;
      pend = ks_o;
    } else {
      const half* wo = L.wo16 ? L.wo16 : L.ro16;
      if (!wo) {
        if ((rc = stage(L.wo, r.wo_s.as<half>(), qd, big, 0, 0))) return rc;
        wo = r.wo_s.as<half>();
      }
      GemmArgs b{};
      b.M = nb;
      b.N = d;
      b.K = qd;
      b.resid = x;
      b.ldo = d;
      b.ksplit = ks_o;
      b.part = r.kpart.as<float>();
      if ((rc = gemm_d(P_GEMM_O, EPI_RESID, r.att.as<half>(), qd, wo, qd, b))) return rc;
      pend = ks_o;
    }
    if (!small && (rc = dnorm(L.ffn_norm))) return rc;
    if (small && v3) {
      if ((rc = run_gemv3(r, gg))) return rc;
      if ((rc = run_gemv3(r, gd))) return rc;
    } else if (small) {
      GemvPlan p{};
      p.xres = x;
      p.norm_w = L.ffn_norm;
      p.eps = c.eps;
      p.rows = ffn;
      p.act = r.act.as<half>();
      p.ld_act = ffn;
      if (L.wgu16) {
        p.seg[0] = {L.wg, nullptr, 0, 0};  // interleaved gate/up operand
        p.nseg = 1;
        p.swiglu = 2;
      } else {
        p.seg[0] = {L.wg, nullptr, 0, 0};
        p.seg[1] = {L.wu, nullptr, 0, 0};
        p.nseg = 2;
        p.swiglu = 1;
      }
      if ((rc = run_gemv(r, p, nbp))) return rc;
      if ((rc = run_gemv(r, plan1(L.wd, r.act.as<half>(), ffn, x, d, 1), nbp))) return rc;
    } else if (q8) {
      GemmArgs gu{};
      gu.M = nb;
      gu.N = 2 * ffn;
      gu.K = d;
      gu.out = r.act.p;
      gu.ldo = ffn;
      if ((rc = gemm_q8d(P_GEMM_GU, EPI_SWIGLU, h, d, q8_gu(c, L), gu))) return rc;
      GemmArgs dn{};
      dn.M = nb;
      dn.N = d;
      dn.K = ffn;
      dn.resid = x;
      dn.ldo = d;
      dn.ksplit = ks_d;
      dn.part = r.kpart.as<float>();
      if ((rc = gemm_q8d(P_GEMM_DOWN, EPI_RESID, r.act.as<half>(), ffn, q8_down(c, L), dn))) return rc;
      pend = ks_d;
    } else {
      const half* wgu = L.wgu16 ? L.wgu16 : L.rgu16;
      if (!wgu) {
        half* s = r.wgu_s.as<half>();
        if ((rc = stage(L.wg, s, d, 128, 256, 0)) || (rc = stage(L.wu, s, d, 128, 256, 128))) return rc;
        wgu = s;
      }
      GemmArgs gu{};
      gu.M = nb;
      gu.N = 2 * ffn;
      gu.K = d;
      gu.out = r.act.p;
      gu.ldo = ffn;
      if ((rc = gemm_d(P_GEMM_GU, EPI_SWIGLU, h, d, wgu, d, gu))) return rc;
      const half* wd = L.wd16 ? L.wd16 : L.rd16;
      if (!wd) {
        if ((rc = stage(L.wd, r.wd_s.as<half>(), ffn, big, 0, 0))) return rc;
        wd = r.wd_s.as<half>();
      }
      GemmArgs dn{};
      dn.M = nb;
      dn.N = d;
      dn.K = ffn;
      dn.resid = x;
      dn.ldo = d;
      dn.ksplit = ks_d;
      dn.part = r.kpart.as<float>();
      if ((rc = gemm_d(P_GEMM_DOWN, EPI_RESID, r.act.as<half>(), ffn, wd, ffn, dn))) return rc;
      pend = ks_d;
    }
  }
  // final norm + full-vocabulary logits + greedy argmax
  if (!small && (rc = dnorm(r.out_norm))) return rc;
  float* logits = r.dlogits.as<float>();
  if (seq) {
    // the head ran at the end of the last layer's chain
  } else if (head3) {
    // head GEMV with the final RMSNorm and the greedy argmax fused
    if ((rc = run_gemv3(r, gh))) return rc;
  } else if (small) {
    // head GEMV with the final RMSNorm and the greedy argmax fused
    GemvPlan hp = plan1(r.head, nullptr, d, nullptr, 0, 0);
    hp.xres = x;
    hp.norm_w = r.out_norm;
    hp.eps = c.eps;
    hp.best = io.best;
    if ((rc = run_gemv(r, hp, nbp))) return rc;
  } else {
    GemmArgs a{};
    a.M = nb;
    a.N = c.V;
    a.K = d;
    a.out = logits;
    a.ldo = c.V;
    if (q8 && r.head_st) {
      if ((rc = gemm_q8d(P_GEMM_HEAD, EPI_F32, h, d, q8_head(r), a))) return rc;
    } else if ((rc = gemm_d(P_GEMM_HEAD, EPI_F32, h, d, r.head16, d, a))) {
      return rc;
    }
    r.launches++;
    LAYA_CK(launch_k(argmax_best_kernel, dim3(nb), dim3(256), 0, st, false, (const float*)logits, c.V, io.best));
  }
  return 0;
}

static bool graphs_enabled() {
  const char* e = std::getenv("LAYA_DECODE_GRAPH");
  return !(e && e[0] == '0');
}

int decode_run(Model& m, Replica& r, const int32_t* ids, const int64_t* off, int n_seqs, int steps, int32_t* out,
               float* stats) {
  const Config& c = m.cfg;
  LAYA_CK(cudaSetDevice(r.device));
  if (n_seqs < 1 || steps < 1) return fail(LAYA_E_INVALID, "decode needs at least one sequence and one step");
  for (int i = 0; i < n_seqs; i++) {
    const int64_t len = off[i + 1] - off[i];
    if (len < 1 || len + steps > c.ctx) return fail(LAYA_E_INVALID, "decode sequence exceeds the context length");
    for (int64_t t = off[i]; t < off[i + 1]; t++)
      if (ids[t] < 0 || ids[t] >= c.V) return fail(LAYA_E_INVALID, "invalid token sequence");
  }
  int rc;
  if ((rc = timing_begin_call(r))) return rc;
  const bool small = gemv_batch(c, n_seqs);
  // batched steps on the Q8_0 blocks: their transposed scales exist before
  // the step is captured into a graph
  const bool q8 = !small && use_q8_gemm(m, r, n_seqs);
  if (q8 && (rc = ensure_q8_scales(m, r))) return rc;
  if (!small && !(q8 && r.head_st) && (rc = ensure_head16(m, r))) return rc;
  if (small && gemv3_enabled() && (rc = ensure_gv_packed(m, r))) return rc;
  // pages: context + generated tokens per sequence
  std::vector<int> tables, toff(n_seqs), clen(n_seqs);
  int pages = 0, max_keys = 0;
  PassPlan pre;
  for (int i = 0; i < n_seqs; i++) {
    const int len = (int)(off[i + 1] - off[i]);
    clen[i] = len;
    toff[i] = (int)tables.size();
    for (int p = 0; p < (len + steps + PAGE - 1) / PAGE; p++) tables.push_back(pages++);
    const int row0 = (int)pre.ids.size();
    for (int t = 0; t < len; t++) {
      pre.ids.push_back(ids[off[i] + t]);
      pre.pos.push_back(t);
      pre.slot.push_back(tables[toff[i] + t / PAGE] * PAGE + t % PAGE);
    }
    for (int t0 = 0; t0 < len; t0 += kAttnRows) pre.items.push_back({row0 + t0, std::min(kAttnRows, len - t0), t0, toff[i]});
    pre.read_rows.push_back(row0 + len - 1);
    max_keys = std::max(max_keys, len + steps);
  }
  if ((rc = ensure_kv(m, r, pages))) return rc;
  LAYA_CK(cudaMemsetAsync(r.err, 0, 4, r.stream));
  const int R = n_seqs;
  if ((rc = r.hid32.ensure((size_t)R * c.d * 4)) || (rc = r.hid16.ensure((size_t)R * c.d * 2))) return rc;
  const int qd = c.H * c.hd, kd = c.KV * c.hd;
  const int nbp = small ? pad_batch(n_seqs) : n_seqs;
  // per-step inputs for all steps, uploaded once
  const size_t nmeta = (size_t)steps * n_seqs;
  std::vector<int> pos_all(nmeta, 0), slot_all(nmeta, 0);
  std::vector<DecSeq> seq_all(nmeta, DecSeq{0, 0});
  for (int s = 1; s < steps; s++)
    for (int i = 0; i < n_seqs; i++) {
      const int p = clen[i] + s - 1;
      pos_all[(size_t)s * n_seqs + i] = p;
      slot_all[(size_t)s * n_seqs + i] = tables[toff[i] + p / PAGE] * PAGE + p % PAGE;
      seq_all[(size_t)s * n_seqs + i] = {toff[i], p + 1};
    }
  auto t0 = std::chrono::steady_clock::now();
  // prefill the contexts, then the first greedy token from the last position
  if ((rc = run_forward(m, r, pre, tables, 0, nullptr, nullptr, nullptr))) return rc;
  if ((rc = r.dlogits.ensure(std::max((size_t)nbp * c.V, (size_t)nbp * std::max(qd + 2 * kd, 2 * c.ffn)) * 4)))
    return rc;
  // device state: [counter | best | toks | pos_all | slot_all | seq_all | cur_tok | cur_pos | cur_slot | cur_seq]
  const size_t best_bytes = ((size_t)n_seqs * 8 + 255) / 256 * 256;
  const size_t meta_bytes = 256 + best_bytes + nmeta * 4 * 3 + nmeta * sizeof(DecSeq) +
                            (size_t)n_seqs * (12 + sizeof(DecSeq)) + 256 + (size_t)c.L * 4 + 256;
  if ((rc = r.dargmax.ensure(meta_bytes))) return rc;
  char* base = static_cast<char*>(r.dargmax.p);
  StepIO io;
  io.counter = reinterpret_cast<int*>(base);
  io.best = reinterpret_cast<unsigned long long*>(base + 256);
  io.toks = reinterpret_cast<int*>(base + 256 + best_bytes);
  int* dpos = io.toks + nmeta;
  int* dslot = dpos + nmeta;
  DecSeq* dseq = reinterpret_cast<DecSeq*>(dslot + nmeta);
  io.pos_all = dpos;
  io.slot_all = dslot;
  io.seq_all = dseq;
  io.cur_tok = reinterpret_cast<int*>(dseq + nmeta);
  io.cur_pos = io.cur_tok + n_seqs;
  io.cur_slot = io.cur_pos + n_seqs;
  io.cur_seq = reinterpret_cast<DecSeq*>(io.cur_slot + n_seqs);
  io.gbar = reinterpret_cast<unsigned*>(reinterpret_cast<uintptr_t>(io.cur_seq + n_seqs + 63) & ~uintptr_t(255));
  io.n_gbar = c.L;
  LAYA_CK(cudaMemsetAsync(io.best, 0, best_bytes, r.stream));
  Gemv3Args gh0 = gv3_base(r, GV_ARGMAX, R, c.d);
  gh0.seg[0] = r.head;
  gh0.x = r.hid16.as<half>();  // final-normed F16 hidden rows of the prefill
  gh0.ldx = c.d;
  gh0.best = io.best;
  gh0.packed = (int)r.gv_packed.size() == 4 * c.L + 1 ? r.gv_packed[4 * c.L] : nullptr;
  if (small && gemv3_enabled() && gh0.packed && gemv3_supported(gh0)) {
    if ((rc = run_gemv3(r, gh0))) return rc;
  } else if (small) {
    // GEMV operands want F16 hidden rows, zero-padded to the GEMV batch
    if ((rc = r.dx16.ensure((size_t)nbp * c.d * 2))) return rc;
    LAYA_CK(cudaMemsetAsync(r.dx16.p, 0, (size_t)nbp * c.d * 2, r.stream));
    LAYA_CK(cudaMemcpyAsync(r.dx16.p, r.hid16.p, (size_t)R * c.d * 2, cudaMemcpyDeviceToDevice, r.stream));
    GemvPlan hp = plan1(r.head, r.dx16.as<half>(), c.d, nullptr, 0, 0);
    hp.best = io.best;
    if ((rc = run_gemv(r, hp, nbp))) return rc;
  } else {
    GemmArgs a{};
    a.M = R;
    a.N = c.V;
    a.K = c.d;
    a.out = r.dlogits.p;
    a.ldo = c.V;
    a.err = r.err;
    a.budget = 4000000000ll;
    r.launches++;
    if (q8 && r.head_st)
      LAYA_CK(gemm_q8_launch(EPI_F32, r.hid16.as<half>(), c.d, q8_head(r), a, r.num_sms, r.stream));
    else
      LAYA_CK(gemm_launch(EPI_F32, r.hid16.as<half>(), c.d, r.head16, c.d, a, r.num_sms, r.stream));
    r.launches++;
    argmax_best_kernel<<<R, 256, 0, r.stream>>>(r.dlogits.as<float>(), c.V, io.best);
    LAYA_CK(cudaGetLastError());
  }
  // decode buffers sized for the padded batch; padded rows stay zero
  if ((rc = r.x.ensure((size_t)nbp * c.d * 4)) || (rc = r.h.ensure((size_t)nbp * c.d * 2)) ||
      (rc = r.qb.ensure((size_t)nbp * qd * 2)) || (rc = r.att.ensure((size_t)nbp * qd * 2)) ||
      (rc = r.act.ensure((size_t)nbp * c.ffn * 2)))
    return rc;
  if (!small) {
    // K-split partial planes of the step's GEMMs (allocated before any capture)
    auto ks = [&](int N, int K) {
      return q8 ? gemm_q8_ksplit(n_seqs, N, K, r.num_sms) : gemm_ksplit(n_seqs, N, K, r.num_sms);
    };
    const int sq = ks(qd + 2 * kd, c.d);
    const int so = std::max(ks(c.d, qd), ks(c.d, c.ffn));
    const size_t f = std::max((size_t)sq * n_seqs * (qd + 2 * kd), (size_t)so * n_seqs * c.d);
    if (std::max(sq, so) > 1 && (rc = r.kpart.ensure(f * 4))) return rc;
  }
  const AttnShape sh = attn_shape(r, c, n_seqs, max_keys);
  if ((rc = r.dpart.ensure((size_t)n_seqs * c.H * sh.splits * (c.hd + 2) * 4)) ||
      (rc = r.tables.ensure(tables.size() * 4)))
    return rc;
  LAYA_CK(cudaMemsetAsync(r.x.p, 0, (size_t)nbp * c.d * 4, r.stream));  // padded rows stay zero
  LAYA_CK(cudaMemsetAsync(r.h.p, 0, (size_t)nbp * c.d * 2, r.stream));
  LAYA_CK(cudaMemsetAsync(r.att.p, 0, (size_t)nbp * qd * 2, r.stream));
  LAYA_CK(cudaMemsetAsync(r.act.p, 0, (size_t)nbp * c.ffn * 2, r.stream));
  LAYA_CK(cudaMemsetAsync(io.counter, 0, 4, r.stream));
  LAYA_CK(cudaMemcpyAsync(r.tables.p, tables.data(), tables.size() * 4, cudaMemcpyHostToDevice, r.stream));
  LAYA_CK(cudaMemcpyAsync(dpos, pos_all.data(), nmeta * 4, cudaMemcpyHostToDevice, r.stream));
  LAYA_CK(cudaMemcpyAsync(dslot, slot_all.data(), nmeta * 4, cudaMemcpyHostToDevice, r.stream));
  LAYA_CK(cudaMemcpyAsync(dseq, seq_all.data(), nmeta * sizeof(DecSeq), cudaMemcpyHostToDevice, r.stream));
  LAYA_CK(cudaStreamSynchronize(r.stream));
  r.h2d += (long long)(tables.size() * 4 + nmeta * (8 + sizeof(DecSeq)));
  if (r.prof) {
    // keep the prefill's kernels apart from the per-step breakdown
    prof_collect(r);
    std::map<std::string, std::pair<long long, double>> pre_acc;
    for (auto& kv : r.prof_acc) pre_acc["prefill:" + kv.first] = kv.second;
    r.prof_acc.swap(pre_acc);
  }
  auto t1 = std::chrono::steady_clock::now();
  if ((rc = timing_mark_start(r))) return rc;
  // step 1 runs directly (it also configures kernels and collects the per-kernel
  // profile); the remaining steps replay a captured graph of the same launches
  if (steps > 1 && (rc = decode_step(m, r, n_seqs, io, sh))) return rc;
  if (steps > 2) {
    if (graphs_enabled()) {
      const bool prof = r.prof;
      r.prof = false;
      cudaGraph_t graph = nullptr;
      cudaGraphExec_t exec = nullptr;
      const long long launches0 = r.launches;
      LAYA_CK(cudaStreamBeginCapture(r.stream, cudaStreamCaptureModeThreadLocal));
      rc = decode_step(m, r, n_seqs, io, sh);
      cudaError_t e = cudaStreamEndCapture(r.stream, &graph);
      r.prof = prof;
      const long long per_step = r.launches - launches0;
      if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
      }
      if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
      e = cudaGraphInstantiate(&exec, graph, 0);
      if (e == cudaSuccess)
        for (int s = 2; s < steps && e == cudaSuccess; s++) e = cudaGraphLaunch(exec, r.stream);
      r.launches += per_step * (steps - 3);
      if (e == cudaSuccess) e = cudaStreamSynchronize(r.stream);
      if (exec) cudaGraphExecDestroy(exec);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess) return cuda_fail(e, "decode graph");
    } else {
      for (int s = 2; s < steps && !rc; s++) rc = decode_step(m, r, n_seqs, io, sh);
      if (rc) return rc;
    }
  }
  r.launches++;
  finalize_kernel<<<1, 256, 0, r.stream>>>(io.best, io.toks, steps - 1, n_seqs);
  LAYA_CK(cudaGetLastError());
  if ((rc = timing_mark_end(r))) return rc;
  auto t2 = std::chrono::steady_clock::now();
  std::vector<int> tk(nmeta);
  LAYA_CK(cudaMemcpy(tk.data(), io.toks, nmeta * 4, cudaMemcpyDeviceToHost));
  r.d2h += (long long)nmeta * 4;
  for (int s = 0; s < steps; s++)
    for (int i = 0; i < n_seqs; i++) out[(size_t)i * steps + s] = tk[(size_t)s * n_seqs + i];
  unsigned err = 0;
  LAYA_CK(cudaMemcpy(&err, r.err, 4, cudaMemcpyDeviceToHost));
  if (err) return fail(LAYA_E_TIMEOUT, "a device-side wait ran out of its budget");
  if (r.prof) prof_collect(r);
  if (stats) {
    stats[0] = std::chrono::duration<float, std::milli>(t1 - t0).count();
    stats[1] = std::chrono::duration<float, std::milli>(t2 - t1).count();
  }
  return 0;
}

}  // namespace laya
