// Gated DeltaNet recurrence of the OpenThai linear-attention layers
// (Delta::run, src/models/openthai/model.rs:322-355), one sequence:
//
//   q, k = L2-normalised (q also / sqrt(hk)); decay = exp(-exp(A_log) *
//   softplus(a + dt_bias)); beta = sigmoid(b)
//   S = decay * S;  delta = beta * (v - k^T S);  S += k delta^T;  o = q^T S
//
// with a per-head state S [key hk][value hk] starting at zero.
//
// Two kernels.  delta_prep_kernel does the work that does not depend on S
// in parallel over (group of four tokens, head): the two L2 norms (in place
// in qkv), decay / beta, and the group's key-key products k_m . k_i (i < m)
// and query-key products q_m . k_i (i <= m).  delta_scan_kernel then runs
// the sequential part four
// tokens at a time: with S0 the state before the group and a_m the decays,
//   r_m = k_m . S0,  p_m = q_m . S0                 (eight independent sums)
//   delta_m = beta_m (v_m - A_m r_m - sum_{i<m} a_{i+1..m} (k_m . k_i) delta_i)
//   o_m = A_m p_m + sum_{i<=m} a_{i+1..m} (q_m . k_i) delta_i
//   S  <- A_3 S0 + sum_i a_{i+1..3} k_i delta_i^T
// (A_m = a_0 ... a_m, a_{i+1..m} the product of the decays after token i), the
// token recurrence reassociated, so the four key sums share one pass of
// shuffle trees.  The value columns of S are independent of one
// another (delta and o of column c read only column c), so a head's columns
// are split over HK / 16 CTAs; inside a CTA eight lanes share one column,
// each holding HK / 8 of its keys in registers, and a token's two key sums
// are 3-step shuffle trees over those lanes.  Tokens are staged in chunks of
// 16 in shared memory, double-buffered: the next chunk's loads are issued
// into registers before the current chunk is processed.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "launch.h"

#define LAYA_DN_CK(x)                     \
  do {                                    \
    const cudaError_t e_ = (x);           \
    if (e_ != cudaSuccess) return e_;     \
  } while (0)

namespace laya {

namespace delta {
constexpr int T = 16;   // tokens per staged chunk
constexpr int CPB = 16; // value columns per CTA
constexpr int G = 8;    // lanes per column (key groups)
constexpr int THREADS = CPB * G;
}  // namespace delta

// Two F32 lanes in one 64-bit register pair (low word first) and the packed
// F32x2 arithmetic of sm_100 (each lane an ordinary IEEE fma / mul, so the
// results equal the scalar forms bit for bit, at one instruction per pair).
using f32x2 = unsigned long long;
__device__ __forceinline__ f32x2 pk2(float a, float b) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpk2(f32x2 v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// One warp per (group of four tokens, head), the per-token work that does
// not depend on the state: the two L2 norms of q and k (written back in
// place), decay and beta (a / b: the gate projections of token i, head h at
// a[i * ldab + h] and b[i * ldab + h]; decay / beta go to dec / beta [s][nh],
// which may alias a / b when ldab == nh), then from the normalised rows the
// group's 6 key-key and 10 query-key products, stored as
// kq[(quad * nh + h) * 16 + ...]: k1k0, k2k0, k2k1, k3k0, k3k1, k3k2, then
// q0k0, q1k0, q1k1, q2k0, q2k1, q2k2, q3k0, q3k1, q3k2, q3k3 (tokens past s
// count as zero).
template <int HK>
__global__ void __launch_bounds__(256) delta_prep_kernel(float* __restrict__ qkv, const float* a, const float* b,
                                                         int ldab, const float* __restrict__ dt,
                                                         const float* __restrict__ alog, int s, int nh, float* dec,
                                                         float* beta, float* __restrict__ kq) {
  pdl_wait();
  pdl_trigger();
  constexpr int PL = HK / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  const int nq = (s + 3) / 4;
  if (gw >= nq * nh) return;
  const int qd = gw / nh, h = gw % nh, w = nh * HK;
  float qv[4][PL], kv[4][PL];
#pragma unroll
  for (int m = 0; m < 4; m++) {
    const int i = 4 * qd + m;
    float* q = qkv + (size_t)i * 3 * w + h * HK;
    float* k = q + w;
    float q2 = 0.f, k2 = 0.f;
#pragma unroll
    for (int u = 0; u < PL; u++) {
      qv[m][u] = i < s ? q[lane + 32 * u] : 0.f;
      kv[m][u] = i < s ? k[lane + 32 * u] : 0.f;
      q2 += qv[m][u] * qv[m][u];
      k2 += kv[m][u] * kv[m][u];
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
      qv[m][u] *= qs;
      kv[m][u] *= ks;
      if (i < s) {
        q[lane + 32 * u] = qv[m][u];
        k[lane + 32 * u] = kv[m][u];
      }
    }
  }
  if (lane < 4 && 4 * qd + lane < s) {
    const int i = 4 * qd + lane;
    const size_t e = (size_t)i * nh + h, src = (size_t)i * ldab + h;
    const float x = a[src] + dt[h];
    const float bv = b[src];
    const float sp = x > 20.f ? x : log1pf(expf(x));
    dec[e] = expf(-expf(alog[h]) * sp);
    beta[e] = 1.f / (1.f + expf(-bv));
  }
  float d[16];
  int n = 0;
  for (int m = 1; m < 4; m++)
    for (int i = 0; i < m; i++) {
      float x = 0.f;
#pragma unroll
      for (int u = 0; u < PL; u++) x += kv[m][u] * kv[i][u];
      d[n++] = x;
    }
  for (int m = 0; m < 4; m++)
    for (int i = 0; i <= m; i++) {
      float x = 0.f;
#pragma unroll
      for (int u = 0; u < PL; u++) x += qv[m][u] * kv[i][u];
      d[n++] = x;
    }
#pragma unroll
  for (int e = 0; e < 16; e++)
#pragma unroll
    for (int o = 16; o; o >>= 1) d[e] += __shfl_xor_sync(0xffffffffu, d[e], o);
  if (lane < 16) {
    float v = d[0];
#pragma unroll
    for (int e = 1; e < 16; e++) v = lane == e ? d[e] : v;
    kq[(size_t)gw * 16 + lane] = v;
  }
}

// Thread (column cl = tid / 8, group g = tid % 8) of CTA (head, column block)
// holds S[j][c] for its keys j = 32 m + 4 g + r (m < HK / 32, r < 4), so a
// group's float4 reads of a staged key row are eight consecutive 16-byte
// words (no bank conflicts).
template <int HK>
__global__ void __launch_bounds__(delta::THREADS) delta_scan_kernel(const float* __restrict__ qkv,
                                                                   const float* __restrict__ dec,
                                                                   const float* __restrict__ beta,
                                                                   const float* __restrict__ kq, int s, int nh,
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
  __shared__ float KQ[2][T / 4][16];   // the chunk's groups' key-key / query-key products
  __shared__ float Op[T][CPB][G + 1];  // the chunk's per-lane output partials (padded row)
  const int tid = threadIdx.x, g = tid % G, cl = tid / G;
  const int h = blockIdx.x, c0 = blockIdx.y * CPB, w = nh * HK;
  const size_t C = (size_t)3 * w;
  // S[j][c] of this thread's keys as pairs: S2[2 mm + e] = keys 4 (G mm + g) + 2 e, + 1
  f32x2 S2[2 * M];
#pragma unroll
  for (int j = 0; j < 2 * M; j++) S2[j] = pk2(0.f, 0.f);
  float4 rq[QPT], rk[QPT], rv = make_float4(0.f, 0.f, 0.f, 0.f);
  float rd = 0.f, rkq = 0.f;
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
    if (tid >= 64 && tid < 64 + 4 * T) {
      const int e = tid - 64, qd = i0 / 4 + e / 16;
      rkq = qd < (s + 3) / 4 ? kq[((size_t)qd * nh + h) * 16 + e % 16] : 0.f;
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
    if (tid >= 64 && tid < 64 + 4 * T) KQ[buf][(tid - 64) / 16][(tid - 64) % 16] = rkq;
  };

  const int nch = (s + T - 1) / T;
  fetch(0);
  stage(0);
  __syncthreads();
  for (int ch = 0; ch < nch; ch++) {
    const int buf = ch & 1, i0 = ch * T;
    if (ch + 1 < nch) fetch(i0 + T);
    const int tn = min(T, s - i0);
    // Four tokens at a time: the eight sums k_m . S0 and q_m . S0 over this
    // lane's keys, the key sums reduced over the column's lanes together,
    // then the per-column solve for delta_0..3 (every lane of the column
    // computes the same values) and one state update for the group.
    for (int t = 0; t < tn; t += 4) {
      const float* kqg = KQ[buf][t / 4];
      float r[4], pp[4];
#pragma unroll
      for (int m = 0; m < 4; m++) {
        // running partials (rr[0], rr[1]) and (rr[2], rr[3]) as two pairs
        f32x2 rr[2] = {pk2(0.f, 0.f), pk2(0.f, 0.f)}, qq[2] = {pk2(0.f, 0.f), pk2(0.f, 0.f)};
#pragma unroll
        for (int mm = 0; mm < M; mm++) {
          const ulonglong2 k4 = reinterpret_cast<const ulonglong2*>(&Ks[buf][t + m][0])[G * mm + g];
          const ulonglong2 q4 = reinterpret_cast<const ulonglong2*>(&Qs[buf][t + m][0])[G * mm + g];
          rr[0] = fma2(S2[2 * mm], k4.x, rr[0]);
          rr[1] = fma2(S2[2 * mm + 1], k4.y, rr[1]);
          qq[0] = fma2(S2[2 * mm], q4.x, qq[0]);
          qq[1] = fma2(S2[2 * mm + 1], q4.y, qq[1]);
        }
        float a0, a1, a2, a3;
        unpk2(rr[0], a0, a1);
        unpk2(rr[1], a2, a3);
        r[m] = (a0 + a1) + (a2 + a3);
        unpk2(qq[0], a0, a1);
        unpk2(qq[1], a2, a3);
        pp[m] = (a0 + a1) + (a2 + a3);
      }
#pragma unroll
      for (int o = 1; o < G; o <<= 1)
#pragma unroll
        for (int m = 0; m < 4; m++) r[m] += __shfl_xor_sync(0xffffffffu, r[m], o);
      float a[4], bt[4], v[4];
#pragma unroll
      for (int m = 0; m < 4; m++) {
        a[m] = Ds[buf][t + m];
        bt[m] = Bs[buf][t + m];
        v[m] = Vs[buf][t + m][cl];
      }
      // A_m = a_0 .. a_m; x_mi = a_{i+1} .. a_m (products of later decays)
      const float A0 = a[0], A1 = A0 * a[1], A2 = A1 * a[2], A3 = A2 * a[3];
      const float x10 = a[1], x21 = a[2], x20 = a[2] * a[1], x32 = a[3], x31 = a[3] * a[2], x30 = x31 * a[1];
      const float d0 = bt[0] * (v[0] - A0 * r[0]);
      const float d1 = bt[1] * (v[1] - (A1 * r[1] + x10 * kqg[0] * d0));
      const float d2 = bt[2] * (v[2] - (A2 * r[2] + x20 * kqg[1] * d0 + x21 * kqg[2] * d1));
      const float d3 = bt[3] * (v[3] - (A3 * r[3] + x30 * kqg[3] * d0 + x31 * kqg[4] * d1 + x32 * kqg[5] * d2));
      // outputs: this lane's share of A_m p_m, plus (lane 0) the delta terms
      const bool l0 = g == 0;
      Op[t][cl][g] = A0 * pp[0] + (l0 ? kqg[6] * d0 : 0.f);
      Op[t + 1][cl][g] = A1 * pp[1] + (l0 ? x10 * kqg[7] * d0 + kqg[8] * d1 : 0.f);
      Op[t + 2][cl][g] = A2 * pp[2] + (l0 ? x20 * kqg[9] * d0 + x21 * kqg[10] * d1 + kqg[11] * d2 : 0.f);
      Op[t + 3][cl][g] =
          A3 * pp[3] + (l0 ? x30 * kqg[12] * d0 + x31 * kqg[13] * d1 + x32 * kqg[14] * d2 + kqg[15] * d3 : 0.f);
      // S <- A_3 S0 + x30 k0 d0 + x31 k1 d1 + x32 k2 d2 + k3 d3
      const f32x2 A3p = pk2(A3, A3), w0p = pk2(x30 * d0, x30 * d0), w1p = pk2(x31 * d1, x31 * d1),
                  w2p = pk2(x32 * d2, x32 * d2), d3p = pk2(d3, d3);
#pragma unroll
      for (int mm = 0; mm < M; mm++) {
        const ulonglong2 k0 = reinterpret_cast<const ulonglong2*>(&Ks[buf][t][0])[G * mm + g];
        const ulonglong2 k1 = reinterpret_cast<const ulonglong2*>(&Ks[buf][t + 1][0])[G * mm + g];
        const ulonglong2 k2 = reinterpret_cast<const ulonglong2*>(&Ks[buf][t + 2][0])[G * mm + g];
        const ulonglong2 k3 = reinterpret_cast<const ulonglong2*>(&Ks[buf][t + 3][0])[G * mm + g];
        S2[2 * mm] = fma2(k3.x, d3p, fma2(k2.x, w2p, fma2(k1.x, w1p, fma2(k0.x, w0p, mul2(A3p, S2[2 * mm])))));
        S2[2 * mm + 1] =
            fma2(k3.y, d3p, fma2(k2.y, w2p, fma2(k1.y, w1p, fma2(k0.y, w0p, mul2(A3p, S2[2 * mm + 1])))));
      }
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
  pdl_wait();
  pdl_trigger();
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (size_t)s * C) return;
  const int i = (int)(e / C), c = (int)(e % C);
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++)
    if (i + j >= 3) acc += raw[(size_t)(i + j - 3) * ldraw + c] * conv[(size_t)c * 4 + j];
  out[e] = acc / (1.f + expf(-acc));
}

// The same on four channels x eight consecutive tokens per thread with
// 16-byte loads and stores (raw and out 16-byte aligned, ldraw and C
// multiples of 4): the eleven input rows of the window are loaded once,
// the four taps of each channel are one float4.  grid.y = token block.
__global__ void conv_silu4_kernel(const float* __restrict__ raw, int ldraw, const float* __restrict__ conv, int s,
                                  int C, float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  constexpr int TT = 8;  // tokens per thread
  const int c = 4 * (blockIdx.x * blockDim.x + threadIdx.x), i0 = blockIdx.y * TT;
  if (c >= C) return;
  float4 w[4];
#pragma unroll
  for (int u = 0; u < 4; u++) w[u] = __ldg(reinterpret_cast<const float4*>(conv + (size_t)(c + u) * 4));
  float4 x[TT + 3];
#pragma unroll
  for (int r = 0; r < TT + 3; r++) {
    const int i = i0 + r - 3;
    x[r] = (i >= 0 && i < s) ? __ldg(reinterpret_cast<const float4*>(raw + (size_t)i * ldraw + c))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int t = 0; t < TT; t++) {
    const int i = i0 + t;
    if (i >= s) break;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (i + j < 3) continue;  // terms before token 0 are left out
      const float4 xv = x[t + j];
      const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float wj = j == 0 ? w[u].x : j == 1 ? w[u].y : j == 2 ? w[u].z : w[u].w;
        acc[u] += xs[u] * wj;
      }
    }
    float4 r;
    r.x = acc[0] / (1.f + expf(-acc[0]));
    r.y = acc[1] / (1.f + expf(-acc[1]));
    r.z = acc[2] / (1.f + expf(-acc[2]));
    r.w = acc[3] / (1.f + expf(-acc[3]));
    *reinterpret_cast<float4*>(out + (size_t)i * C + c) = r;
  }
}

// Per-head RMSNorm (weight offset 0, eps 1e-6) of the recurrence output,
// then x SiLU(z) (model.rs:356-360); one warp per (token, head) row, each
// lane HK / 32 consecutive elements as one vector load of o and of z (rows
// 16-byte aligned, ldz a multiple of 4).  The result goes to o (F32, in
// place) or, when out16 is set, to out16 as F16 rows [s][nh HK] (the output
// projection's operand) with o left as it was.
template <int HK>
__global__ void norm_gate_kernel(float* __restrict__ o, const float* __restrict__ z, int ldz, int nh,
                                 const float* __restrict__ w, int rows, half* __restrict__ out16) {
  pdl_wait();
  pdl_trigger();
  constexpr int PL = HK / 32;  // consecutive elements per lane (4 or 2), one vector load each
  using VecF = typename std::conditional<PL == 4, float4, float2>::type;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (gw >= rows) return;
  float* r = o + (size_t)gw * HK + lane * PL;
  const float* zr = z + (size_t)(gw / nh) * ldz + (size_t)(gw % nh) * HK + lane * PL;
  float v[PL], zz[PL], wv[PL];
  {
    const VecF a = *reinterpret_cast<const VecF*>(r);
    const VecF b = *reinterpret_cast<const VecF*>(zr);
    const float* pa = reinterpret_cast<const float*>(&a);
    const float* pb = reinterpret_cast<const float*>(&b);
#pragma unroll
    for (int u = 0; u < PL; u++) {
      v[u] = pa[u];
      zz[u] = pb[u];
      wv[u] = __ldg(w + lane * PL + u);  // the norm weights need no alignment
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < PL; u++) ss += v[u] * v[u];
#pragma unroll
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float scale = 1.f / sqrtf(ss / (float)HK + 1e-6f);
  float y[PL];
#pragma unroll
  for (int u = 0; u < PL; u++) y[u] = v[u] * scale * wv[u] * (zz[u] / (1.f + expf(-zz[u])));
  if (out16) {
    __align__(8) half hv[PL];
#pragma unroll
    for (int u = 0; u < PL; u++) hv[u] = __float2half_rn(y[u]);
    half* dst = out16 + (size_t)gw * HK + lane * PL;
    if constexpr (PL == 4)
      *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(hv);
    else
      *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(hv);
  } else {
    VecF t;
    float* pt = reinterpret_cast<float*>(&t);
#pragma unroll
    for (int u = 0; u < PL; u++) pt[u] = y[u];
    *reinterpret_cast<VecF*>(r) = t;
  }
}

cudaError_t gated_delta_mixer(const float* raw, int ldraw, const float* z, int ldz, const float* a, const float* b,
                              int ldab, const float* conv, const float* dt, const float* alog, const float* normw,
                              int s, int nh, int hk, float* scratch, float* out, half* out16, cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (nh < 1 || (hk != 64 && hk != 128)) return cudaErrorInvalidValue;
  // vector loads of the recurrence output and of z in the output norm
  if ((ldz % 4) || (reinterpret_cast<uintptr_t>(z) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(out16) & 15))
    return cudaErrorInvalidValue;
  const size_t C = (size_t)3 * nh * hk, n = (size_t)s * C;
  // programmatic dependent launch on a created stream (each kernel waits for
  // its predecessor's output before reading); plain launches on stream 0
  const bool pdl = st != nullptr;
  float* qkv = scratch;
  float* dec = scratch + n;
  float* beta = dec + (size_t)s * nh;
  float* kq = beta + (size_t)s * nh;
  if (ldraw % 4 == 0 && (reinterpret_cast<uintptr_t>(raw) & 15) == 0 && (reinterpret_cast<uintptr_t>(qkv) & 15) == 0 &&
      (s + 7) / 8 <= 65535)
    LAYA_DN_CK(launch_k(conv_silu4_kernel, dim3((unsigned)((C / 4 + 127) / 128), (unsigned)((s + 7) / 8)), dim3(128),
                        0, st, pdl, raw, ldraw, conv, s, (int)C, qkv));
  else
    LAYA_DN_CK(launch_k(conv_silu_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, pdl, raw, ldraw, conv, s,
                        (int)C, qkv));
  cudaError_t e = gated_delta(qkv, a, b, ldab, dt, alog, s, nh, hk, dec, beta, kq, out, st);
  if (e != cudaSuccess) return e;
  const int rows = s * nh;
  if (hk == 128)
    LAYA_DN_CK(launch_k(norm_gate_kernel<128>, dim3((rows + 7) / 8), dim3(256), 0, st, pdl, out, z, ldz, nh, normw, rows,
                        out16));
  else
    LAYA_DN_CK(launch_k(norm_gate_kernel<64>, dim3((rows + 7) / 8), dim3(256), 0, st, pdl, out, z, ldz, nh, normw, rows,
                        out16));
  return cudaGetLastError();
}

size_t gated_delta_mixer_scratch(int s, int nh, int hk) {
  return (size_t)s * (3 * nh * hk + 2 * nh) * 4 + gated_delta_scratch(s, nh);
}

size_t gated_delta_scratch(int s, int nh) { return (size_t)((s + 3) / 4) * nh * 16 * 4; }

cudaError_t gated_delta(float* qkv, const float* a, const float* b, int ldab, const float* dt, const float* alog,
                        int s, int nh, int hk, float* dec, float* beta, float* kq, float* out, cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (nh < 1 || (hk != 64 && hk != 128) || !kq) return cudaErrorInvalidValue;
  const bool pdl = st != nullptr;
  const unsigned prep_blocks = (unsigned)(((size_t)((s + 3) / 4) * nh + 7) / 8);
  const dim3 grid(nh, hk / delta::CPB);
  if (hk == 128) {
    // The scan launches only once the prep is done (no programmatic early
    // launch): launched early, its 128 CTAs were placed wherever the prep
    // left room, several to an SM, and the latency-bound scan took twice as
    // long.
    LAYA_DN_CK(launch_k(delta_prep_kernel<128>, dim3(prep_blocks), dim3(256), 0, st, pdl, qkv, a, b, ldab, dt, alog, s, nh,
                        dec, beta, kq));
    LAYA_DN_CK(launch_k(delta_scan_kernel<128>, grid, dim3(delta::THREADS), 0, st, false, (const float*)qkv,
                        (const float*)dec, (const float*)beta, (const float*)kq, s, nh, out));
  } else {
    LAYA_DN_CK(launch_k(delta_prep_kernel<64>, dim3(prep_blocks), dim3(256), 0, st, pdl, qkv, a, b, ldab, dt, alog, s, nh,
                        dec, beta, kq));
    LAYA_DN_CK(launch_k(delta_scan_kernel<64>, grid, dim3(delta::THREADS), 0, st, false, (const float*)qkv,
                        (const float*)dec, (const float*)beta, (const float*)kq, s, nh, out));
  }
  return cudaGetLastError();
}

}  // namespace laya
