// Gated full attention of the OpenThai layers (Full::run,
// src/models/openthai/model.rs:248-296) after the projections, one
// sequence:
//   q / k: per-head RMSNorm with weight offset 1 (eps 1e-6), then rotate-half
//          RoPE on the first `rot` dimensions (pairs j, j + rot/2, angle
//          pos / theta^(2j/rot));
//   out[i, h] = sigmoid(gate[i, h]) * softmax_j<=i(q_i . k_j / sqrt(hd)) v_j,
//          GQA: query head h reads KV head h / (H / KV).
// Two kernels: gattn_prep_kernel normalises and rotates every query and key
// head once (one warp per head row); gattn_kernel runs one CTA of 8 warps
// per (token, query head), each warp an online softmax over every 8th key
// with the row's hd/32 dimensions per lane, merged in shared memory.  A
// first, correct form on CUDA cores; the head-dim-256 tcgen05 version is the
// fast one.
#include "common.cuh"
#include "kernels.h"

namespace laya {

// One warp per (token, head) row of q (heads 0..H-1, read from qgate) or k
// (heads H..H+KV-1): RMSNorm (offset 1) and the partial rotation, written to
// qr [s][H][hd] / kr [s][KV][hd].
template <int HD>
__global__ void gattn_prep_kernel(const float* __restrict__ qgate, const float* __restrict__ k,
                                  const float* __restrict__ qn, const float* __restrict__ kn, int s, int H, int KV,
                                  int rot, float theta, float* __restrict__ qr, float* __restrict__ kr) {
  constexpr int PL = HD / 32;  // dimensions per lane: lane l holds l, l + 32, ...
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  const int rows = s * (H + KV);
  if (gw >= rows) return;
  const int i = gw / (H + KV), hh = gw % (H + KV);
  const bool isq = hh < H;
  const float* src = isq ? qgate + ((size_t)i * H + hh) * 2 * HD : k + ((size_t)i * KV + (hh - H)) * HD;
  const float* wn = isq ? qn : kn;
  float* dst = isq ? qr + ((size_t)i * H + hh) * HD : kr + ((size_t)i * KV + (hh - H)) * HD;
  float v[PL];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < PL; u++) {
    v[u] = src[lane + 32 * u];
    ss += v[u] * v[u];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float scale = 1.f / sqrtf(ss / (float)HD + 1e-6f);
#pragma unroll
  for (int u = 0; u < PL; u++) v[u] = v[u] * scale * (1.f + wn[lane + 32 * u]);
  // rotation: write the normalised row, then each lane rotates its pairs
#pragma unroll
  for (int u = 0; u < PL; u++) dst[lane + 32 * u] = v[u];
  __syncwarp();
  const int half = rot / 2;
  for (int j = lane; j < half; j += 32) {
    const float angle = (float)i / powf(theta, (float)(2 * j) / (float)rot);
    const float co = cosf(angle), si = sinf(angle);
    const float a = dst[j], b = dst[j + half];
    dst[j] = a * co - b * si;
    dst[j + half] = b * co + a * si;
  }
}

template <int HD>
__global__ void __launch_bounds__(256) gattn_kernel(const float* __restrict__ qr, const float* __restrict__ kr,
                                                    const float* __restrict__ v, const float* __restrict__ qgate,
                                                    int s, int H, int KV, float* __restrict__ out) {
  constexpr int PL = HD / 32, NW = 8;
  __shared__ float wm[NW], wl[NW];
  __shared__ float wacc[NW][HD];
  const int i = blockIdx.x / H, h = blockIdx.x % H;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kh = h / (H / KV);
  const float root = sqrtf((float)HD);
  float q[PL];
#pragma unroll
  for (int u = 0; u < PL; u++) q[u] = qr[((size_t)i * H + h) * HD + lane + 32 * u];
  float m = -INFINITY, l = 0.f, acc[PL];
#pragma unroll
  for (int u = 0; u < PL; u++) acc[u] = 0.f;
  for (int j = warp; j <= i; j += NW) {
    const float* kj = kr + ((size_t)j * KV + kh) * HD;
    const float* vj = v + ((size_t)j * KV + kh) * HD;
    float dot = 0.f;
#pragma unroll
    for (int u = 0; u < PL; u++) dot += q[u] * kj[lane + 32 * u];
#pragma unroll
    for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float sc = dot / root;
    const float mn = fmaxf(m, sc);
    const float corr = expf(m - mn), p = expf(sc - mn);  // corr = 0 on the first key (m = -inf)
    l = l * corr + p;
#pragma unroll
    for (int u = 0; u < PL; u++) acc[u] = acc[u] * corr + p * vj[lane + 32 * u];
    m = mn;
  }
  if (lane == 0) {
    wm[warp] = m;
    wl[warp] = l;
  }
#pragma unroll
  for (int u = 0; u < PL; u++) wacc[warp][lane + 32 * u] = acc[u];
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w]);
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < NW; w++)
    if (wm[w] != -INFINITY) L += expf(wm[w] - M) * wl[w];
  for (int c = threadIdx.x; c < HD; c += blockDim.x) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < NW; w++)
      if (wm[w] != -INFINITY) o += expf(wm[w] - M) * wacc[w][c];
    const float g = qgate[((size_t)i * H + h) * 2 * HD + HD + c];
    out[((size_t)i * H + h) * HD + c] = o / L * (1.f / (1.f + expf(-g)));
  }
}

template <int HD>
static cudaError_t gattn_go(const float* qgate, const float* k, const float* v, const float* qn, const float* kn,
                            int s, int H, int KV, int rot, float theta, float* qr, float* kr, float* out,
                            cudaStream_t st) {
  const int rows = s * (H + KV);
  gattn_prep_kernel<HD><<<(rows + 7) / 8, 256, 0, st>>>(qgate, k, qn, kn, s, H, KV, rot, theta, qr, kr);
  gattn_kernel<HD><<<s * H, 256, 0, st>>>(qr, kr, v, qgate, s, H, KV, out);
  return cudaGetLastError();
}

cudaError_t gated_attention(const float* qgate, const float* k, const float* v, const float* qn, const float* kn,
                            int s, int H, int KV, int hd, int rot, float theta, float* scratch, float* out,
                            cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (H < 1 || KV < 1 || H % KV || rot < 0 || rot > hd || rot % 2) return cudaErrorInvalidValue;
  float* qr = scratch;
  float* kr = scratch + (size_t)s * H * hd;
  if (hd == 256) return gattn_go<256>(qgate, k, v, qn, kn, s, H, KV, rot, theta, qr, kr, out, st);
  if (hd == 128) return gattn_go<128>(qgate, k, v, qn, kn, s, H, KV, rot, theta, qr, kr, out, st);
  if (hd == 64) return gattn_go<64>(qgate, k, v, qn, kn, s, H, KV, rot, theta, qr, kr, out, st);
  return cudaErrorInvalidValue;
}

}  // namespace laya
