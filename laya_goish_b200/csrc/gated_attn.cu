// Gated full attention of the OpenThai layers (Full::run,
// src/models/openthai/model.rs:248-296) after the projections, one
// sequence:
//   q / k: per-head RMSNorm with weight offset 1 (eps 1e-6), then rotate-half
//          RoPE on the first `rot` dimensions (pairs j, j + rot/2, angle
//          pos / theta^(2j/rot));
//   out[i, h] = sigmoid(gate[i, h]) * softmax_j<=i(q_i . k_j / sqrt(hd)) v_j,
//          GQA: query head h reads KV head h / (H / KV).
// gattn_prep_kernel normalises and rotates every query and key head once
// (one warp per head row) and writes the F16 operands of the tensor-core
// attention: Q as [s][H * hd] rows, K and V as 64-token pages
// [pages][KV][64][hd] (the paged layout of the decoder's KV cache, one
// sequence, page p = tokens 64p .. 64p + 63, rows past the sequence zero),
// plus the attention's work list.  The causal attention itself is the
// tcgen05 kernel of attn_tc.cu (S and O in TMEM; head dim 256 keeps one Q
// buffer and one O accumulator), which applies the sigmoid gate in its
// epilogue and writes F16 rows, the operand of the output projection.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "launch.h"

namespace laya {

namespace {

constexpr int kUnitRows = 128;  // query rows per attention work item
constexpr int kPage = 64;

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

struct GaLayout {
  size_t q16, k16, v16, items, tables, total;
};

GaLayout ga_layout(int s, int H, int KV, int hd) {
  const size_t pages = ((size_t)s + kPage - 1) / kPage, units = ((size_t)s + kUnitRows - 1) / kUnitRows;
  GaLayout L;
  L.q16 = 0;
  L.k16 = L.q16 + align256((size_t)s * H * hd * 2);
  L.v16 = L.k16 + align256(pages * kPage * KV * hd * 2);
  L.items = L.v16 + align256(pages * kPage * KV * hd * 2);
  L.tables = L.items + align256(units * sizeof(AttnItem));
  L.total = L.tables + align256(pages * 4);
  return L;
}

}  // namespace

// One warp per (token, head) row of q (heads 0..H-1, read from qgate), of k
// (heads H..H+KV-1) or of v (heads H+KV..H+2KV-1), for tokens 0 .. pages*64-1
// (rows past s are zero).  q and k: RMSNorm (offset 1) and the partial
// rotation in F32 in the warp's shared row, then rounded to F16.
template <int HD>
__global__ void __launch_bounds__(256) gattn_prep_kernel(const float* __restrict__ qgate, int ldqg,
                                                         const float* __restrict__ k, const float* __restrict__ v,
                                                         int ldkv, const float* __restrict__ qn,
                                                         const float* __restrict__ kn, int s, int H, int KV, int rot,
                                                         float theta, half* __restrict__ q16, half* __restrict__ k16,
                                                         half* __restrict__ v16, AttnItem* __restrict__ items,
                                                         int* __restrict__ tables) {
  constexpr int PL = HD / 32;  // dimensions per lane: lane l holds l, l + 32, ...
  __shared__ float rowbuf[8][HD];
  pdl_wait();  // the projections were written by the previous kernel
  pdl_trigger();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32, wib = threadIdx.x / 32;
  const int pages = (s + kPage - 1) / kPage;
  // the work list: item u = query rows 128u .. of the one sequence, all pages in order
  const int gt = blockIdx.x * blockDim.x + threadIdx.x;
  if (gt < (s + kUnitRows - 1) / kUnitRows) items[gt] = {gt * kUnitRows, min(kUnitRows, s - gt * kUnitRows), gt * kUnitRows, 0};
  if (gt < pages) tables[gt] = gt;
  const int per = H + 2 * KV;
  if (gw >= pages * kPage * per) return;
  const int i = gw / per, hh = gw % per;
  const int pg = i / kPage, r = i % kPage;
  if (hh >= H + KV) {  // v row
    const int kh = hh - H - KV;
    half* dst = v16 + (((size_t)pg * KV + kh) * kPage + r) * HD;
#pragma unroll
    for (int u = 0; u < PL; u++)
      dst[lane + 32 * u] = __float2half_rn(i < s ? v[(size_t)i * ldkv + (size_t)kh * HD + lane + 32 * u] : 0.f);
    return;
  }
  const bool isq = hh < H;
  half* dst = isq ? q16 + ((size_t)i * H + hh) * HD : k16 + (((size_t)pg * KV + (hh - H)) * kPage + r) * HD;
  if (i >= s) {
    if (!isq)
#pragma unroll
      for (int u = 0; u < PL; u++) dst[lane + 32 * u] = __float2half_rn(0.f);
    return;
  }
  const float* src = isq ? qgate + (size_t)i * ldqg + (size_t)hh * 2 * HD : k + (size_t)i * ldkv + (size_t)(hh - H) * HD;
  const float* wn = isq ? qn : kn;
  float* row = rowbuf[wib];
  float x[PL];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < PL; u++) {
    x[u] = src[lane + 32 * u];
    ss += x[u] * x[u];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float scale = 1.f / sqrtf(ss / (float)HD + 1e-6f);
#pragma unroll
  for (int u = 0; u < PL; u++) row[lane + 32 * u] = x[u] * scale * (1.f + wn[lane + 32 * u]);
  __syncwarp();
  // rotate-half on the first rot dimensions (pairs j, j + rot/2)
  const int half_rot = rot / 2;
  for (int j = lane; j < half_rot; j += 32) {
    const float angle = (float)i / powf(theta, (float)(2 * j) / (float)rot);
    const float co = cosf(angle), si = sinf(angle);
    const float a = row[j], b = row[j + half_rot];
    row[j] = a * co - b * si;
    row[j + half_rot] = b * co + a * si;
  }
  __syncwarp();
#pragma unroll
  for (int u = 0; u < PL; u++) dst[lane + 32 * u] = __float2half_rn(row[lane + 32 * u]);
}

size_t gated_attention_scratch(int s, int H, int KV, int hd) { return s > 0 ? ga_layout(s, H, KV, hd).total : 0; }

cudaError_t gated_attention(const float* qgate, int ldqg, const float* k, const float* v, int ldkv, const float* qn,
                            const float* kn, int s, int H, int KV, int hd, int rot, float theta, void* scratch,
                            half* out16, unsigned* err, cudaStream_t st) {
  if (s <= 0) return cudaSuccess;
  if (H < 1 || KV < 1 || H % KV || rot < 0 || rot > hd || rot % 2 || !err || ldqg < 2 * H * hd || ldkv < KV * hd)
    return cudaErrorInvalidValue;
  if ((hd != 64 && hd != 128 && hd != 256) || (reinterpret_cast<uintptr_t>(scratch) & 255)) return cudaErrorInvalidValue;
  const GaLayout L = ga_layout(s, H, KV, hd);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  half* q16 = reinterpret_cast<half*>(base + L.q16);
  half* k16 = reinterpret_cast<half*>(base + L.k16);
  half* v16 = reinterpret_cast<half*>(base + L.v16);
  AttnItem* items = reinterpret_cast<AttnItem*>(base + L.items);
  int* tables = reinterpret_cast<int*>(base + L.tables);
  const int pages = (s + kPage - 1) / kPage;
  const size_t rows = (size_t)pages * kPage * (H + 2 * KV);
  const unsigned blocks = (unsigned)std::max<size_t>((rows + 7) / 8, ((size_t)pages + 255) / 256);
  cudaError_t e = cudaSuccess;
#define LAYA_GA_PREP(HDV)                                                                                   \
  e = launch_k(gattn_prep_kernel<HDV>, dim3(blocks), dim3(256), 0, st, st != nullptr, qgate, ldqg, k, v, ldkv, qn, kn, \
               s, H, KV, rot, theta, q16, k16, v16, items, tables)
  if (hd == 256)
    LAYA_GA_PREP(256);
  else if (hd == 128)
    LAYA_GA_PREP(128);
  else
    LAYA_GA_PREP(64);
#undef LAYA_GA_PREP
  if (e != cudaSuccess) return e;
  AttnParams p{};
  p.q = q16;
  p.ldq = H * hd;
  p.o = out16;
  p.ldo = H * hd;
  p.kc = k16;
  p.vc = v16;
  p.tables = tables;
  p.items = items;
  p.n_items = (s + kUnitRows - 1) / kUnitRows;
  p.H = H;
  p.KV = KV;
  p.hd = hd;
  p.scale_log2 = (1.f / sqrtf((float)hd)) * 1.4426950408889634f;
  p.q_rows = s;
  p.kv_rows = pages * KV * kPage;
  p.err = err;
  p.gate = qgate + hd;  // the gate half of each head's [query hd | gate hd]
  p.ldg = ldqg;
  p.ghs = 2 * hd;
  p.pack = 1;  // the query heads of a KV head share each unit
  return attention_tc(p, st);
}

}  // namespace laya
