// Gated DeltaNet recurrence of the OpenThai linear-attention layers
// (Delta::run, src/models/openthai/model.rs:322-355), one sequence:
//
//   q, k = L2-normalised (q also / sqrt(hk)); decay = exp(-exp(A_log) *
//   softplus(a + dt_bias)); beta = sigmoid(b)
//   S = decay * S;  delta = beta * (v - k^T S);  S += k delta^T;  o = q^T S
//
// with a per-head state S [key hk][value hk] starting at zero.  One CTA per
// head, one thread per value column: the thread keeps its column of S in
// registers (hk floats), so a token costs two passes over the column plus
// two block reductions (|q|^2, |k|^2).  Tokens are sequential; a chunked
// (WY-form) scan that runs the token blocks on the tensor cores is the
// faster form for long prompts.
#include "common.cuh"
#include "kernels.h"

namespace laya {

template <int HK>
__global__ void __launch_bounds__(HK) gated_delta_kernel(const float* __restrict__ qkv, const float* __restrict__ a,
                                                         const float* __restrict__ b, const float* __restrict__ dt,
                                                         const float* __restrict__ alog, int s, int nh,
                                                         float* __restrict__ out) {
  constexpr int NW = HK / 32;
  __shared__ float kk[HK], qq[HK];
  __shared__ float red[2][NW];
  const int h = blockIdx.x, c = threadIdx.x, lane = c & 31, warp = c >> 5;
  const int w = nh * HK, C = 3 * w;
  float S[HK];  // S[j] = state[j][c]
#pragma unroll
  for (int j = 0; j < HK; j++) S[j] = 0.f;
  const float ea = expf(alog[h]), dth = dt[h];
  for (int i = 0; i < s; i++) {
    const float* row = qkv + (size_t)i * C;
    const float q = row[h * HK + c], k = row[w + h * HK + c], v = row[2 * w + h * HK + c];
    float q2 = q * q, k2 = k * k;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      q2 += __shfl_xor_sync(0xffffffffu, q2, o);
      k2 += __shfl_xor_sync(0xffffffffu, k2, o);
    }
    if (lane == 0) {
      red[0][warp] = q2;
      red[1][warp] = k2;
    }
    __syncthreads();
    float qsum = 0.f, ksum = 0.f;
#pragma unroll
    for (int u = 0; u < NW; u++) {
      qsum += red[0][u];
      ksum += red[1][u];
    }
    const float qs = 1.f / sqrtf(qsum + 1e-6f) / sqrtf((float)HK);
    const float ks = 1.f / sqrtf(ksum + 1e-6f);
    const float x = a[(size_t)i * nh + h] + dth;
    const float sp = x > 20.f ? x : log1pf(expf(x));
    const float decay = expf(-ea * sp);
    const float beta = 1.f / (1.f + expf(-b[(size_t)i * nh + h]));
    kk[c] = k * ks;
    qq[c] = q * qs;
    __syncthreads();
    float delta = 0.f;
#pragma unroll
    for (int j = 0; j < HK; j++) {
      S[j] *= decay;
      delta += S[j] * kk[j];
    }
    delta = (v - delta) * beta;
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < HK; j++) {
      S[j] += kk[j] * delta;
      o += S[j] * qq[j];
    }
    out[(size_t)i * w + h * HK + c] = o;
    __syncthreads();  // kk, qq and red are rewritten by the next token
  }
}

// Causal depthwise convolution of width 4 over the token axis, then SiLU
// (model.rs:309-320): out[i][c] = silu(sum_j raw[i + j - 3][c] conv[c][j]),
// terms before token 0 left out, summed in j order.
__global__ void conv_silu_kernel(const float* __restrict__ raw, const float* __restrict__ conv, int s, int C,
                                 float* __restrict__ out) {
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (size_t)s * C) return;
  const int i = (int)(e / C), c = (int)(e % C);
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++)
    if (i + j >= 3) acc += raw[(size_t)(i + j - 3) * C + c] * conv[(size_t)c * 4 + j];
  out[e] = acc / (1.f + expf(-acc));
}

// Per-head RMSNorm (weight offset 0, eps 1e-6) of the recurrence output,
// then x SiLU(z) (model.rs:356-360); one warp per (token, head) row.
template <int HK>
__global__ void norm_gate_kernel(float* __restrict__ o, const float* __restrict__ z, const float* __restrict__ w,
                                 int rows) {
  constexpr int PL = HK / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (gw >= rows) return;
  float* r = o + (size_t)gw * HK;
  const float* zr = z + (size_t)gw * HK;
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

cudaError_t gated_delta_mixer(const float* raw, const float* z, const float* a, const float* b, const float* conv,
                              const float* dt, const float* alog, const float* normw, int s, int nh, int hk,
                              float* qkv_scratch, float* out, cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (nh < 1 || (hk != 64 && hk != 128)) return cudaErrorInvalidValue;
  const size_t C = (size_t)3 * nh * hk, n = (size_t)s * C;
  conv_silu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(raw, conv, s, (int)C, qkv_scratch);
  cudaError_t e = gated_delta(qkv_scratch, a, b, dt, alog, s, nh, hk, out, st);
  if (e != cudaSuccess) return e;
  const int rows = s * nh;
  if (hk == 128)
    norm_gate_kernel<128><<<(rows + 7) / 8, 256, 0, st>>>(out, z, normw, rows);
  else
    norm_gate_kernel<64><<<(rows + 7) / 8, 256, 0, st>>>(out, z, normw, rows);
  return cudaGetLastError();
}

cudaError_t gated_delta(const float* qkv, const float* a, const float* b, const float* dt, const float* alog, int s,
                        int nh, int hk, float* out, cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (nh < 1) return cudaErrorInvalidValue;
  if (hk == 128)
    gated_delta_kernel<128><<<nh, 128, 0, st>>>(qkv, a, b, dt, alog, s, nh, out);
  else if (hk == 64)
    gated_delta_kernel<64><<<nh, 64, 0, st>>>(qkv, a, b, dt, alog, s, nh, out);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace laya
