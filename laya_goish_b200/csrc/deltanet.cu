// Gated DeltaNet recurrence of the OpenThai linear-attention layers
// (Delta::run, src/models/openthai/model.rs:322-355), one sequence:
//
//   q, k = L2-normalised (q also / sqrt(hk)); decay = exp(-exp(A_log) *
//   softplus(a + dt_bias)); beta = sigmoid(b)
//   S = decay * S;  delta = beta * (v - k^T S);  S += k delta^T;  o = q^T S
//
// with a per-head state S [key hk][value hk] starting at zero.
//
// Two kernels.  delta_prep_kernel does the per-token work that does not
// depend on S in parallel over (token, head): the two L2 norms (in place in
// qkv) and decay / beta (in place in a / b).  delta_scan_kernel then runs
// the token-sequential part.  The value columns of S are independent of one
// another (delta and o of column c read only column c), so a head's columns
// are split over HK / 16 CTAs; inside a CTA eight lanes share one column,
// each holding HK / 8 of its keys in registers, and a token's two key sums
// are 3-step shuffle trees over those lanes.  Tokens are staged in chunks of
// 16 in shared memory, double-buffered: the next chunk's loads are issued
// into registers before the current chunk is processed.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace delta {
constexpr int T = 16;   // tokens per staged chunk
constexpr int CPB = 16; // value columns per CTA
constexpr int G = 8;    // lanes per column (key groups)
constexpr int THREADS = CPB * G;
}  // namespace delta

// a / b: the gate projections of token i, head h at a[i * ldab + h] and
// b[i * ldab + h]; decay / beta go to dec / beta [s][nh] (may alias a / b
// when ldab == nh).
template <int HK>
__global__ void __launch_bounds__(256) delta_prep_kernel(float* __restrict__ qkv, const float* a, const float* b,
                                                         int ldab, const float* __restrict__ dt,
                                                         const float* __restrict__ alog, int s, int nh, float* dec,
                                                         float* beta) {
  constexpr int PL = HK / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (gw >= s * nh) return;
  const int i = gw / nh, h = gw % nh, w = nh * HK;
  float* q = qkv + (size_t)i * 3 * w + h * HK;
  float* k = q + w;
  float qv[PL], kv[PL], q2 = 0.f, k2 = 0.f;
#pragma unroll
  for (int u = 0; u < PL; u++) {
    qv[u] = q[lane + 32 * u];
    kv[u] = k[lane + 32 * u];
    q2 += qv[u] * qv[u];
    k2 += kv[u] * kv[u];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    q2 += __shfl_xor_sync(0xffffffffu, q2, o);
    k2 += __shfl_xor_sync(0xffffffffu, k2, o);
  }
  const float qs = 1.f / sqrtf(q2 + 1e-6f) / sqrtf((float)HK);
  const float ks = 1.f / sqrtf(k2 + 1e-6f);
#pragma unroll
  for (int u = 0; u < PL; u++) {
    q[lane + 32 * u] = qv[u] * qs;
    k[lane + 32 * u] = kv[u] * ks;
  }
  if (lane == 0) {
    const size_t e = (size_t)i * nh + h, src = (size_t)i * ldab + h;
    const float x = a[src] + dt[h];
    const float bv = b[src];
    const float sp = x > 20.f ? x : log1pf(expf(x));
    dec[e] = expf(-expf(alog[h]) * sp);
    beta[e] = 1.f / (1.f + expf(-bv));
  }
}

// Thread (column cl = tid / 8, group g = tid % 8) of CTA (head, column block)
// holds S[j][c] for its keys j = 32 m + 4 g + r (m < HK / 32, r < 4), so a
// group's float4 reads of a staged key row are eight consecutive 16-byte
// words (no bank conflicts).
template <int HK>
__global__ void __launch_bounds__(delta::THREADS) delta_scan_kernel(const float* __restrict__ qkv,
                                                                   const float* __restrict__ dec,
                                                                   const float* __restrict__ beta, int s, int nh,
                                                                   float* __restrict__ out) {
  using namespace delta;
  constexpr int M = HK / 32;            // float4 words of keys per thread
  constexpr int QW = T * HK / 4;        // float4 words of one staged q (or k) chunk
  constexpr int QPT = QW / THREADS;     // ... per thread
  static_assert(QW % THREADS == 0, "chunk words must divide over the block");
  constexpr int VW = T * CPB / 4;       // float4 words of the staged v chunk
  static_assert(VW <= THREADS, "v chunk must fit one word per thread");
  __shared__ __align__(16) float Qs[2][T][HK];
  __shared__ __align__(16) float Ks[2][T][HK];
  __shared__ __align__(16) float Vs[2][T][CPB];
  __shared__ float Ds[2][T], Bs[2][T];
  __shared__ float Op[T][CPB][G + 1];  // the chunk's per-lane output partials (padded row)
  const int tid = threadIdx.x, g = tid % G, cl = tid / G;
  const int h = blockIdx.x, c0 = blockIdx.y * CPB, w = nh * HK;
  const size_t C = (size_t)3 * w;
  float S[4 * M];
#pragma unroll
  for (int j = 0; j < 4 * M; j++) S[j] = 0.f;

  float4 rq[QPT], rk[QPT], rv = make_float4(0.f, 0.f, 0.f, 0.f);
  float rd = 0.f;
  auto fetch = [&](int i0) {
#pragma unroll
    for (int u = 0; u < QPT; u++) {
      const int idx = tid + u * THREADS, t = idx / (HK / 4), x = idx % (HK / 4), i = i0 + t;
      const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
      const float* row = qkv + (size_t)i * C + h * HK + 4 * x;
      rq[u] = i < s ? *reinterpret_cast<const float4*>(row) : zero;
      rk[u] = i < s ? *reinterpret_cast<const float4*>(row + w) : zero;
    }
    if (tid < VW) {
      const int t = tid / (CPB / 4), x = tid % (CPB / 4), i = i0 + t;
      rv = i < s ? *reinterpret_cast<const float4*>(qkv + (size_t)i * C + 2 * w + h * HK + c0 + 4 * x)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (tid < 2 * T) {
      const int t = tid % T, i = i0 + t;
      rd = i < s ? (tid < T ? dec : beta)[(size_t)i * nh + h] : 0.f;
    }
  };
  auto stage = [&](int buf) {
#pragma unroll
    for (int u = 0; u < QPT; u++) {
      const int idx = tid + u * THREADS, t = idx / (HK / 4), x = idx % (HK / 4);
      reinterpret_cast<float4*>(&Qs[buf][t][0])[x] = rq[u];
      reinterpret_cast<float4*>(&Ks[buf][t][0])[x] = rk[u];
    }
    if (tid < VW) reinterpret_cast<float4*>(&Vs[buf][tid / (CPB / 4)][0])[tid % (CPB / 4)] = rv;
    if (tid < T) Ds[buf][tid] = rd;
    else if (tid < 2 * T) Bs[buf][tid - T] = rd;
  };

  const int nch = (s + T - 1) / T;
  fetch(0);
  stage(0);
  __syncthreads();
  for (int ch = 0; ch < nch; ch++) {
    const int buf = ch & 1, i0 = ch * T;
    if (ch + 1 < nch) fetch(i0 + T);
    const int tn = min(T, s - i0);
    // Per token the critical path is decay, the key sum k . S (four partial
    // sums, then the 3-step shuffle tree over the column's lanes), delta and
    // the rank-1 update; the output q . S of the token is this lane's
    // partial only, parked in shared memory and reduced once per chunk.
    for (int t = 0; t < tn; t++) {
      const float dcy = Ds[buf][t], bt = Bs[buf][t], v = Vs[buf][t][cl];
      float kk[4 * M];
#pragma unroll
      for (int m = 0; m < M; m++) {
        const float4 k4 = reinterpret_cast<const float4*>(&Ks[buf][t][0])[8 * m + g];
        kk[4 * m] = k4.x, kk[4 * m + 1] = k4.y, kk[4 * m + 2] = k4.z, kk[4 * m + 3] = k4.w;
      }
      float dp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 4 * M; j++) {
        S[j] *= dcy;
        dp[j & 3] += S[j] * kk[j];
      }
      float dsum = (dp[0] + dp[1]) + (dp[2] + dp[3]);
#pragma unroll
      for (int o = 1; o < G; o <<= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
      const float delta = (v - dsum) * bt;
      float op[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int m = 0; m < M; m++) {
        const float4 q4 = reinterpret_cast<const float4*>(&Qs[buf][t][0])[8 * m + g];
        S[4 * m] += kk[4 * m] * delta;
        S[4 * m + 1] += kk[4 * m + 1] * delta;
        S[4 * m + 2] += kk[4 * m + 2] * delta;
        S[4 * m + 3] += kk[4 * m + 3] * delta;
        op[0] += S[4 * m] * q4.x;
        op[1] += S[4 * m + 1] * q4.y;
        op[2] += S[4 * m + 2] * q4.z;
        op[3] += S[4 * m + 3] * q4.w;
      }
      Op[t][cl][g] = (op[0] + op[1]) + (op[2] + op[3]);
    }
    __syncthreads();
    // the chunk's outputs: thread (token, column) sums its 8 lane partials
    for (int e = tid; e < tn * CPB; e += THREADS) {
      const int t = e / CPB, c = e % CPB;
      float o = 0.f;
#pragma unroll
      for (int j = 0; j < G; j++) o += Op[t][c][j];
      out[(size_t)(i0 + t) * w + h * HK + c0 + c] = o;
    }
    if (ch + 1 < nch) stage(buf ^ 1);
    __syncthreads();
  }
}

// Causal depthwise convolution of width 4 over the token axis, then SiLU
// (model.rs:309-320): out[i][c] = silu(sum_j raw[i + j - 3][c] conv[c][j]),
// terms before token 0 left out, summed in j order.
__global__ void conv_silu_kernel(const float* __restrict__ raw, int ldraw, const float* __restrict__ conv, int s,
                                 int C, float* __restrict__ out) {
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (size_t)s * C) return;
  const int i = (int)(e / C), c = (int)(e % C);
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++)
    if (i + j >= 3) acc += raw[(size_t)(i + j - 3) * ldraw + c] * conv[(size_t)c * 4 + j];
  out[e] = acc / (1.f + expf(-acc));
}

// Per-head RMSNorm (weight offset 0, eps 1e-6) of the recurrence output,
// then x SiLU(z) (model.rs:356-360); one warp per (token, head) row.
template <int HK>
__global__ void norm_gate_kernel(float* __restrict__ o, const float* __restrict__ z, int ldz, int nh,
                                 const float* __restrict__ w, int rows) {
  constexpr int PL = HK / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (gw >= rows) return;
  float* r = o + (size_t)gw * HK;
  const float* zr = z + (size_t)(gw / nh) * ldz + (size_t)(gw % nh) * HK;
  float v[PL], ss = 0.f;
#pragma unroll
  for (int u = 0; u < PL; u++) {
    v[u] = r[lane + 32 * u];
    ss += v[u] * v[u];
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float scale = 1.f / sqrtf(ss / (float)HK + 1e-6f);
#pragma unroll
  for (int u = 0; u < PL; u++) {
    const float zz = zr[lane + 32 * u];
    r[lane + 32 * u] = v[u] * scale * w[lane + 32 * u] * (zz / (1.f + expf(-zz)));
  }
}

cudaError_t gated_delta_mixer(const float* raw, int ldraw, const float* z, int ldz, const float* a, const float* b,
                              int ldab, const float* conv, const float* dt, const float* alog, const float* normw,
                              int s, int nh, int hk, float* scratch, float* out, cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (nh < 1 || (hk != 64 && hk != 128)) return cudaErrorInvalidValue;
  const size_t C = (size_t)3 * nh * hk, n = (size_t)s * C;
  float* qkv = scratch;
  float* dec = scratch + n;
  float* beta = dec + (size_t)s * nh;
  conv_silu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(raw, ldraw, conv, s, (int)C, qkv);
  cudaError_t e = gated_delta(qkv, a, b, ldab, dt, alog, s, nh, hk, dec, beta, out, st);
  if (e != cudaSuccess) return e;
  const int rows = s * nh;
  if (hk == 128)
    norm_gate_kernel<128><<<(rows + 7) / 8, 256, 0, st>>>(out, z, ldz, nh, normw, rows);
  else
    norm_gate_kernel<64><<<(rows + 7) / 8, 256, 0, st>>>(out, z, ldz, nh, normw, rows);
  return cudaGetLastError();
}

size_t gated_delta_mixer_scratch(int s, int nh, int hk) { return (size_t)s * (3 * nh * hk + 2 * nh) * 4; }

cudaError_t gated_delta(float* qkv, const float* a, const float* b, int ldab, const float* dt, const float* alog,
                        int s, int nh, int hk, float* dec, float* beta, float* out, cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (nh < 1 || (hk != 64 && hk != 128)) return cudaErrorInvalidValue;
  const unsigned prep_blocks = (unsigned)(((size_t)s * nh + 7) / 8);
  const dim3 grid(nh, hk / delta::CPB);
  if (hk == 128) {
    delta_prep_kernel<128><<<prep_blocks, 256, 0, st>>>(qkv, a, b, ldab, dt, alog, s, nh, dec, beta);
    delta_scan_kernel<128><<<grid, delta::THREADS, 0, st>>>(qkv, dec, beta, s, nh, out);
  } else {
    delta_prep_kernel<64><<<prep_blocks, 256, 0, st>>>(qkv, a, b, ldab, dt, alog, s, nh, dec, beta);
    delta_scan_kernel<64><<<grid, delta::THREADS, 0, st>>>(qkv, dec, beta, s, nh, out);
  }
  return cudaGetLastError();
}

}  // namespace laya
