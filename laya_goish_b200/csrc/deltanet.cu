// Gated DeltaNet recurrence of the OpenThai linear-attention layers
// (Delta::run, src/models/openthai/model.rs:322-355), one sequence:
//
//   q, k = L2-normalised (q also / sqrt(hk)); decay = exp(-exp(A_log) *
//   softplus(a + dt_bias)); beta = sigmoid(b)
//   S = decay * S;  delta = beta * (v - k^T S);  S += k delta^T;  o = q^T S
//
// with a per-head state S [key hk][value hk] starting at zero.
//
// Chunked form (chunks of C = 64 tokens, per head; g_t = the running sum of
// log decays inside the chunk, gamma_t = exp(g_t)): with S0 the state at the
// chunk start,
//   S_t   = gamma_t S0 + sum_{i<=t} (gamma_t / gamma_i) k_i delta_i^T
//   Delta = U0 - W S0,   W = T diag(beta gamma) K,  U0 = T diag(beta) V,
//           T = (I + A)^-1, A_ti = beta_t (gamma_t / gamma_i) k_t . k_i (i < t)
//   O     = (Gamma Q) S0 + Pm Delta,   Pm_ti = (gamma_t / gamma_i) q_t . k_i (i <= t)
//   S_C   = gamma_C S0 + Kd^T Delta,   Kd_i = (gamma_C / gamma_i) k_i
// which is the token recurrence above, reassociated (every ratio
// gamma_t / gamma_i <= 1 is formed from the log sums, so nothing overflows).
//
// Three kernels.  delta_prep_kernel does the per-token work in parallel over
// (token, head): the two L2 norms (in place in qkv), the log decay and beta.
// delta_chunk_kernel builds every chunk's W, U0, Gamma Q, Kd and Pm in
// parallel over (chunk, head), with T from a forward substitution.
// delta_state_kernel then walks the chunks in order for one head and a block
// of 16 value columns (the columns of S are independent), the state held in
// registers, key-group partial sums reduced through shared memory.
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace delta {
constexpr int C = 64;        // tokens per chunk
constexpr int CB = 16;       // value columns per state CTA
constexpr int KG = 16;       // key groups per state CTA (thread = key group x column)
constexpr int THREADS = 256;
}  // namespace delta

// a / b: the gate projections of token i, head h at a[i * ldab + h] and
// b[i * ldab + h]; the log decay -exp(A_log) softplus(a + dt) and beta go to
// ldec / beta [s][nh] (may alias a / b when ldab == nh).
template <int HK>
__global__ void __launch_bounds__(256) delta_prep_kernel(float* __restrict__ qkv, const float* a, const float* b,
                                                         int ldab, const float* __restrict__ dt,
                                                         const float* __restrict__ alog, int s, int nh, float* ldec,
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
    ldec[e] = -expf(alog[h]) * sp;
    beta[e] = 1.f / (1.f + expf(-bv));
  }
}

// One (chunk, head): stage the chunk's normalised q and k, v, beta and log
// decay (rows past s are zero, so padded tokens add nothing), then
//   g   = running sums of the log decays,
//   KK  = K K^T and QK = Q K^T as 4 x 4 register tiles per thread,
//   A   (strictly lower) and Pm (lower, diagonal included) from them,
//   T   = (I + A)^-1 by forward substitution, one column per thread,
//   W   = T diag(beta gamma) K and U0 = T diag(beta) V (4 x 8 tiles),
// and write W, U0, Gamma Q, Kd [C][HK], Pm [C][C] and gamma_C.
// Shared rows are padded to HK + 1 floats (no bank conflicts on columns).
template <int HK>
__global__ void __launch_bounds__(delta::THREADS) delta_chunk_kernel(const float* __restrict__ qkv,
                                                                    const float* __restrict__ ldec,
                                                                    const float* __restrict__ beta, int s, int nh,
                                                                    float* __restrict__ wout, float* __restrict__ uout,
                                                                    float* __restrict__ qgout, float* __restrict__ kdout,
                                                                    float* __restrict__ pmout, float* __restrict__ gcout) {
  using namespace delta;
  constexpr int LD = HK + 1, LDC = C + 1;
  extern __shared__ float dsm[];
  float* Ks = dsm;                // [C][LD]
  float* Qs = Ks + C * LD;        // [C][LD]
  float* Vs = Qs + C * LD;        // [C][LD]
  float* As = Vs + C * LD;        // [C][LDC]  A
  float* Ts = As + C * LDC;       // [C][LDC]  T
  float* gs = Ts + C * LDC;       // [C]
  float* bs = gs + C;             // [C]
  const int ch = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int w = nh * HK, t0 = ch * C;
  const size_t slot = (size_t)ch * nh + h;
  for (int e = tid; e < C * HK; e += THREADS) {
    const int t = e / HK, j = e % HK, i = t0 + t;
    const bool live = i < s;
    const float* row = qkv + (size_t)i * 3 * w + h * HK + j;
    Qs[t * LD + j] = live ? row[0] : 0.f;
    Ks[t * LD + j] = live ? row[w] : 0.f;
    Vs[t * LD + j] = live ? row[2 * w] : 0.f;
  }
  if (tid < C) {
    const int i = t0 + tid;
    gs[tid] = i < s ? ldec[(size_t)i * nh + h] : 0.f;
    bs[tid] = i < s ? beta[(size_t)i * nh + h] : 0.f;
  }
  __syncthreads();
  if (tid == 0)
    for (int t = 1; t < C; t++) gs[t] += gs[t - 1];  // in token order
  __syncthreads();
  {
    // KK and QK: thread (rt, ri) owns rows t = 4 rt .. 4 rt + 3, columns i = 4 ri .. 4 ri + 3
    const int rt = tid / 16, ri = tid % 16;
    float kk[4][4] = {}, qk[4][4] = {};
    for (int j = 0; j < HK; j++) {
      float kt[4], qt[4], ki[4];
#pragma unroll
      for (int r = 0; r < 4; r++) {
        kt[r] = Ks[(4 * rt + r) * LD + j];
        qt[r] = Qs[(4 * rt + r) * LD + j];
        ki[r] = Ks[(4 * ri + r) * LD + j];
      }
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          kk[r][c] = fmaf(kt[r], ki[c], kk[r][c]);
          qk[r][c] = fmaf(qt[r], ki[c], qk[r][c]);
        }
    }
    float* pm = pmout + slot * C * C;
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const int t = 4 * rt + r, i = 4 * ri + c;
        const float ratio = i <= t ? expf(gs[t] - gs[i]) : 0.f;
        As[t * LDC + i] = i < t ? bs[t] * ratio * kk[r][c] : 0.f;
        pm[t * C + i] = ratio * qk[r][c];
      }
  }
  __syncthreads();
  // T = (I + A)^-1, lower triangular with a unit diagonal: row t is
  // e_t - sum_{i<t} A[t][i] T[i][:]; thread c keeps column c
  if (tid < C) {
    const int c = tid;
    for (int t = 0; t < C; t++) {
      float v = t == c ? 1.f : 0.f;
      for (int i = c; i < t; i++) v = fmaf(-As[t * LDC + i], Ts[i * LDC + c], v);
      Ts[t * LDC + c] = t >= c ? v : 0.f;
    }
  }
  __syncthreads();
  {
    // W and U0: thread (rt, rj) owns rows t = 4 rt .. + 3, columns j = rj, rj + 16, ... (HK / 16 of them)
    constexpr int NJ = HK / 16;
    const int rt = tid / 16, rj = tid % 16;
    float wa[4][NJ] = {}, ua[4][NJ] = {};
    for (int i = 0; i <= 4 * rt + 3; i++) {
      const float sb = bs[i], sg = bs[i] * expf(gs[i]);
      float tt[4];
#pragma unroll
      for (int r = 0; r < 4; r++) tt[r] = Ts[(4 * rt + r) * LDC + i];
#pragma unroll
      for (int q = 0; q < NJ; q++) {
        const float kv = Ks[i * LD + rj + 16 * q] * sg, vv = Vs[i * LD + rj + 16 * q] * sb;
#pragma unroll
        for (int r = 0; r < 4; r++) {
          wa[r][q] = fmaf(tt[r], kv, wa[r][q]);
          ua[r][q] = fmaf(tt[r], vv, ua[r][q]);
        }
      }
    }
    const float gC = gs[C - 1];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int t = 4 * rt + r;
      const float eg = expf(gs[t]), ed = expf(gC - gs[t]);
#pragma unroll
      for (int q = 0; q < NJ; q++) {
        const int j = rj + 16 * q;
        const size_t o = (slot * C + t) * HK + j;
        wout[o] = wa[r][q];
        uout[o] = ua[r][q];
        qgout[o] = eg * Qs[t * LD + j];
        kdout[o] = ed * Ks[t * LD + j];
      }
    }
    if (tid == 0) gcout[slot] = expf(gC);
  }
}

// One head, value columns c0 .. c0 + 15: the chunks in order.  Thread (kg,
// c) holds S[j][c] for its HK / 16 keys j = kg * HK / 16 + r in registers.
// Per chunk: Delta = U0 - W S0 and the Gamma Q S0 part of O as key-group
// partials reduced in shared memory, O += Pm Delta, S = gamma_C S0 + Kd^T
// Delta.
template <int HK>
__global__ void __launch_bounds__(delta::THREADS) delta_state_kernel(const float* __restrict__ wk,
                                                                    const float* __restrict__ uk,
                                                                    const float* __restrict__ qgk,
                                                                    const float* __restrict__ kdk,
                                                                    const float* __restrict__ pmk,
                                                                    const float* __restrict__ gck, int s, int nh,
                                                                    float* __restrict__ out) {
  using namespace delta;
  constexpr int NK = HK / KG;  // keys per thread
  extern __shared__ float ssm[];
  float* R1 = ssm;                  // [KG][C][CB] partials of W S0
  float* R2 = R1 + KG * C * CB;     // [KG][C][CB] partials of Gamma Q S0
  float* Dl = R2 + KG * C * CB;     // [C][CB] Delta
  const int h = blockIdx.x, c0 = blockIdx.y * CB, tid = threadIdx.x;
  const int kg = tid / CB, c = tid % CB, w = nh * HK;
  const int nch = (s + C - 1) / C;
  float S[NK];
#pragma unroll
  for (int r = 0; r < NK; r++) S[r] = 0.f;
  for (int ch = 0; ch < nch; ch++) {
    const size_t slot = (size_t)ch * nh + h;
    const float* W = wk + slot * C * HK;
    const float* QG = qgk + slot * C * HK;
    const float* KD = kdk + slot * C * HK;
    const float* PM = pmk + slot * C * C;
    const float* U0 = uk + slot * C * HK;
    for (int t = 0; t < C; t++) {
      float p1 = 0.f, p2 = 0.f;
#pragma unroll
      for (int r = 0; r < NK; r++) {
        const int j = kg * NK + r;
        p1 = fmaf(__ldg(W + t * HK + j), S[r], p1);
        p2 = fmaf(__ldg(QG + t * HK + j), S[r], p2);
      }
      R1[(kg * C + t) * CB + c] = p1;
      R2[(kg * C + t) * CB + c] = p2;
    }
    __syncthreads();
    for (int e = tid; e < C * CB; e += THREADS) {
      const int t = e / CB, cc = e % CB;
      float a = 0.f, q = 0.f;
#pragma unroll
      for (int g = 0; g < KG; g++) {
        a += R1[(g * C + t) * CB + cc];
        q += R2[(g * C + t) * CB + cc];
      }
      Dl[t * CB + cc] = __ldg(U0 + t * HK + c0 + cc) - a;
      R2[t * CB + cc] = q;  // group 0's slot of R2 now holds the full Gamma Q S0 sum
    }
    __syncthreads();
    for (int e = tid; e < C * CB; e += THREADS) {
      const int t = e / CB, cc = e % CB;
      float o = R2[t * CB + cc];
      for (int i = 0; i <= t; i++) o = fmaf(__ldg(PM + t * C + i), Dl[i * CB + cc], o);
      const int tok = ch * C + t;
      if (tok < s) out[(size_t)tok * w + h * HK + c0 + cc] = o;
    }
    const float gC = __ldg(gck + slot);
    float acc[NK];
#pragma unroll
    for (int r = 0; r < NK; r++) acc[r] = gC * S[r];
    for (int i = 0; i < C; i++) {
      const float d = Dl[i * CB + c];
#pragma unroll
      for (int r = 0; r < NK; r++) acc[r] = fmaf(__ldg(KD + i * HK + kg * NK + r), d, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < NK; r++) S[r] = acc[r];
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
  float* ldec = scratch + n;
  float* beta = ldec + (size_t)s * nh;
  float* chunks = beta + ((size_t)s * nh + 63) / 64 * 64;
  conv_silu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(raw, ldraw, conv, s, (int)C, qkv);
  cudaError_t e = gated_delta(qkv, a, b, ldab, dt, alog, s, nh, hk, ldec, beta, chunks, out, st);
  if (e != cudaSuccess) return e;
  const int rows = s * nh;
  if (hk == 128)
    norm_gate_kernel<128><<<(rows + 7) / 8, 256, 0, st>>>(out, z, ldz, nh, normw, rows);
  else
    norm_gate_kernel<64><<<(rows + 7) / 8, 256, 0, st>>>(out, z, ldz, nh, normw, rows);
  return cudaGetLastError();
}

size_t gated_delta_mixer_scratch(int s, int nh, int hk) {
  return ((size_t)s * (3 * nh * hk + nh) + ((size_t)s * nh + 63) / 64 * 64) * 4 + gated_delta_scratch(s, nh, hk);
}

size_t gated_delta_scratch(int s, int nh, int hk) {
  const size_t slots = (size_t)((s + delta::C - 1) / delta::C) * nh;
  return (slots * (4 * delta::C * hk + delta::C * delta::C + 1) + 64) * 4;
}

template <int HK>
static cudaError_t gated_delta_go(float* qkv, const float* a, const float* b, int ldab, const float* dt,
                                  const float* alog, int s, int nh, float* ldec, float* beta, float* chunks,
                                  float* out, cudaStream_t st) {
  using namespace delta;
  const unsigned prep_blocks = (unsigned)(((size_t)s * nh + 7) / 8);
  delta_prep_kernel<HK><<<prep_blocks, 256, 0, st>>>(qkv, a, b, ldab, dt, alog, s, nh, ldec, beta);
  const int nch = (s + C - 1) / C;
  const size_t slots = (size_t)nch * nh, mat = (size_t)C * HK;
  float* W = chunks;
  float* U = W + slots * mat;
  float* QG = U + slots * mat;
  float* KD = QG + slots * mat;
  float* PM = KD + slots * mat;
  float* GC = PM + slots * C * C;
  constexpr int smem1 = (3 * C * (HK + 1) + 2 * C * (C + 1) + 2 * C) * 4;
  constexpr int smem2 = (2 * KG * C * CB + C * CB) * 4;
  static std::atomic<bool> configured[64];  // per device; any host thread may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(delta_chunk_kernel<HK>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(delta_state_kernel<HK>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  delta_chunk_kernel<HK><<<dim3(nch, nh), THREADS, smem1, st>>>(qkv, ldec, beta, s, nh, W, U, QG, KD, PM, GC);
  delta_state_kernel<HK><<<dim3(nh, HK / CB), THREADS, smem2, st>>>(W, U, QG, KD, PM, GC, s, nh, out);
  return cudaGetLastError();
}

cudaError_t gated_delta(float* qkv, const float* a, const float* b, int ldab, const float* dt, const float* alog,
                        int s, int nh, int hk, float* ldec, float* beta, float* chunks, float* out, cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (nh < 1 || (hk != 64 && hk != 128) || !chunks) return cudaErrorInvalidValue;
  if (hk == 128) return gated_delta_go<128>(qkv, a, b, ldab, dt, alog, s, nh, ldec, beta, chunks, out, st);
  return gated_delta_go<64>(qkv, a, b, ldab, dt, alog, s, nh, ldec, beta, chunks, out, st);
}

}  // namespace laya
