// KV-cached greedy decode (no reference counterpart: the reference has no
// KV cache and no decode loop, src/models/laya/decision.rs:302).
//
// Each step appends one token per sequence.  Small batches run the linear
// layers as bandwidth-bound GEMVs that read the quantised weights once with
// 128-bit loads and decode them in registers; larger batches reuse the
// tcgen05 GEMM path.  Attention over the paged cache is split along the
// key axis so that even a single sequence spreads over all SMs.
#include <cfloat>
#include <algorithm>
#include <chrono>
#include <cstring>

#include "engine.h"
#include "gemm.h"

namespace laya {

// ---------------------------------------------------------------- GEMV

// y[b][n] (+)= sum_k x[b][k] * W[n][k] for B <= 16 rows of F16 x.
// One warp per ROWS output rows; lanes stride over 32-element groups of K,
// decoding the weights once per group (dq32) and reusing them for all B.
template <int B, int ROWS>
__global__ void __launch_bounds__(256) gemv_kernel(QTensor w, const half* __restrict__ x, int ldx,
                                                   float* __restrict__ y, int ldy, int accumulate) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  const int n0 = warp * ROWS;
  if (n0 >= w.rows) return;
  const int groups = w.cols / 32;
  float acc[ROWS][B];
#pragma unroll
  for (int r = 0; r < ROWS; r++)
#pragma unroll
    for (int b = 0; b < B; b++) acc[r][b] = 0.f;
  for (int g = lane; g < groups; g += 32) {
    float wv[ROWS][32];
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
      if (n0 + r < w.rows) dq32(w, n0 + r, g * 32, wv[r]);
      else {
#pragma unroll
        for (int i = 0; i < 32; i++) wv[r][i] = 0.f;
      }
    }
#pragma unroll
    for (int b = 0; b < B; b++) {
      const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)b * ldx + g * 32);
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint4 u = __ldg(xp + c);
        const half2* hp = reinterpret_cast<const half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          float2 f = __half22float2(hp[e]);
#pragma unroll
          for (int r = 0; r < ROWS; r++) {
            acc[r][b] = fmaf(wv[r][c * 8 + 2 * e], f.x, acc[r][b]);
            acc[r][b] = fmaf(wv[r][c * 8 + 2 * e + 1], f.y, acc[r][b]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS; r++)
#pragma unroll
    for (int b = 0; b < B; b++) {
      float v = acc[r][b];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
      acc[r][b] = v;
    }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
      if (n0 + r >= w.rows) break;
#pragma unroll
      for (int b = 0; b < B; b++) {
        float* dst = y + (size_t)b * ldy + n0 + r;
        *dst = accumulate ? *dst + acc[r][b] : acc[r][b];
      }
    }
  }
}

template <int B>
static cudaError_t gemv_b(const QTensor& w, const half* x, int ldx, float* y, int ldy, int acc, cudaStream_t st) {
  constexpr int ROWS = B >= 16 ? 1 : 2;
  const int warps = (w.rows + ROWS - 1) / ROWS;
  gemv_kernel<B, ROWS><<<(warps * 32 + 255) / 256, 256, 0, st>>>(w, x, ldx, y, ldy, acc);
  return cudaGetLastError();
}

cudaError_t gemv(const QTensor& w, const half* x, int ldx, int nb, float* y, int ldy, int acc, cudaStream_t st) {
  switch (nb) {
    case 1: return gemv_b<1>(w, x, ldx, y, ldy, acc, st);
    case 2: return gemv_b<2>(w, x, ldx, y, ldy, acc, st);
    case 4: return gemv_b<4>(w, x, ldx, y, ldy, acc, st);
    case 8: return gemv_b<8>(w, x, ldx, y, ldy, acc, st);
    case 16: return gemv_b<16>(w, x, ldx, y, ldy, acc, st);
  }
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- small kernels

// qkv F32 [B][qd+2kd] (+bias) -> rotate-half RoPE on q and k, q -> F16
// [B][qd], k and v appended to the paged cache at slot[b].
__global__ void rope_append_kernel(const float* __restrict__ qkv, const float* __restrict__ bias, int qd, int kd,
                                   int hd, int kvh, const int* __restrict__ pos, const int* __restrict__ slot,
                                   const float2* __restrict__ rope, half* __restrict__ q, half* __restrict__ kc,
                                   half* __restrict__ vc) {
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

// act[b][f] = silu(gate) * up (src/models/openthai/model.rs:225-230); gate/up
// either interleaved per 128 columns in one [B][2*ffn] buffer or separate.
__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, int ffn, int interleaved,
                              half* __restrict__ act) {
  const int b = blockIdx.y;
  for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < ffn; f += gridDim.x * blockDim.x) {
    float gv, uv;
    if (interleaved) {
      const size_t base = (size_t)b * 2 * ffn + (size_t)(f / 128) * 256 + f % 128;
      gv = g[base];
      uv = g[base + 128];
    } else {
      gv = g[(size_t)b * ffn + f];
      uv = u[(size_t)b * ffn + f];
    }
    act[(size_t)b * ffn + f] = __float2half_rn(gv / (1.f + __expf(-gv)) * uv);
  }
}

// Greedy token: argmax over the vocabulary, ties to the lowest id.
__global__ void argmax_kernel(const float* __restrict__ logits, int V, int* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const float* x = logits + (size_t)blockIdx.x * V;
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < V; c += blockDim.x) {
    const float v = x[c];
    if (v > best || (v == best && c < bi)) {
      best = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffff, best, o);
    const int oi = __shfl_xor_sync(0xffffffff, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (threadIdx.x % 32 == 0) {
    sv[threadIdx.x / 32] = best;
    si[threadIdx.x / 32] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)blockDim.x / 32; w++)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    out[blockIdx.x] = bi;
  }
}

__global__ void f32_to_f16_kernel(const float* __restrict__ x, size_t n, half* __restrict__ y) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

// ---------------------------------------------------------------- decode attention

struct DecSeq {
  int table_off, n_keys;
};

// One CTA per (sequence, kv head, key split); one warp per query head of the
// GQA group.  Lanes own keys for the scores and head-dim slices for P.V.
// Writes the split's (max, sum, unnormalised output) for the combine step.
template <int HD>
__global__ void attn_decode_kernel(const half* __restrict__ q, const half* __restrict__ kc, const half* __restrict__ vc,
                                   const int* __restrict__ tables, const DecSeq* __restrict__ seqs, int H, int KV,
                                   float scale_log2, int split_len, int splits, float* __restrict__ part) {
  const int b = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
  const int G = H / KV;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (warp >= G) return;
  const int h = kvh * G + warp;
  const DecSeq s = seqs[b];
  const int k0 = sp * split_len, k1 = min(s.n_keys, k0 + split_len);
  constexpr int DPL = HD / 32;  // head dims per lane
  float qv[HD];
  const half* qp = q + ((size_t)b * H + h) * HD;
#pragma unroll
  for (int i = 0; i < HD; i += 8) {
    uint4 u = *reinterpret_cast<const uint4*>(qp + i);
    const half2* hp = reinterpret_cast<const half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; e++) {
      float2 f = __half22float2(hp[e]);
      qv[i + 2 * e] = f.x;
      qv[i + 2 * e + 1] = f.y;
    }
  }
  float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; i++) acc[i] = 0.f;
  for (int j0 = k0; j0 < k1; j0 += 32) {
    const int j = j0 + lane;
    float sc = -INFINITY;
    if (j < k1) {
      const int page = tables[s.table_off + j / PAGE];
      const half* kp = kc + (((size_t)page * KV + kvh) * PAGE + j % PAGE) * HD;
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < HD; i += 8) {
        uint4 u = __ldg(reinterpret_cast<const uint4*>(kp + i));
        const half2* hp = reinterpret_cast<const half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          float2 f = __half22float2(hp[e]);
          dot = fmaf(qv[i + 2 * e], f.x, dot);
          dot = fmaf(qv[i + 2 * e + 1], f.y, dot);
        }
      }
      sc = dot * scale_log2;
    }
    float mx = sc;
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
    const float mn = fmaxf(m, mx);
    const float corr = exp2f(m - mn);
    const float p = j < k1 ? exp2f(sc - mn) : 0.f;
    float ps = p;
#pragma unroll
    for (int o = 16; o; o >>= 1) ps += __shfl_xor_sync(0xffffffff, ps, o);
    l = l * corr + ps;
    m = mn;
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[i] *= corr;
    const int cnt = min(32, k1 - j0);
    for (int jj = 0; jj < cnt; jj++) {
      const float pj = __shfl_sync(0xffffffff, p, jj);
      const int key = j0 + jj;
      const int page = tables[s.table_off + key / PAGE];
      const half* vp = vc + (((size_t)page * KV + kvh) * PAGE + key % PAGE) * HD + lane * DPL;
      if constexpr (DPL == 2) {
        const float2 f = __half22float2(*reinterpret_cast<const half2*>(vp));
        acc[0] = fmaf(pj, f.x, acc[0]);
        acc[1] = fmaf(pj, f.y, acc[1]);
      } else {
        const uint2 u = *reinterpret_cast<const uint2*>(vp);
        const half2* hp = reinterpret_cast<const half2*>(&u);
        const float2 f0 = __half22float2(hp[0]), f1 = __half22float2(hp[1]);
        acc[0] = fmaf(pj, f0.x, acc[0]);
        acc[1] = fmaf(pj, f0.y, acc[1]);
        acc[2] = fmaf(pj, f1.x, acc[2]);
        acc[3] = fmaf(pj, f1.y, acc[3]);
      }
    }
  }
  float* dst = part + (((size_t)b * H + h) * splits + sp) * (HD + 2);
  if (lane == 0) {
    dst[0] = m;
    dst[1] = l;
  }
#pragma unroll
  for (int i = 0; i < DPL; i++) dst[2 + lane * DPL + i] = acc[i];
}

// Merges the key splits: o = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s.
__global__ void attn_combine_kernel(const float* __restrict__ part, int H, int HD, int splits, half* __restrict__ o) {
  const int b = blockIdx.x, h = blockIdx.y;
  const float* p = part + ((size_t)b * H + h) * splits * (HD + 2);
  float M = -INFINITY;
  for (int s = 0; s < splits; s++) M = fmaxf(M, p[s * (HD + 2)]);
  float L = 0.f;
  for (int s = 0; s < splits; s++) {
    const float ms = p[s * (HD + 2)];
    if (ms != -INFINITY) L += exp2f(ms - M) * p[s * (HD + 2) + 1];
  }
  for (int dd = threadIdx.x; dd < HD; dd += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; s++) {
      const float ms = p[s * (HD + 2)];
      if (ms != -INFINITY) acc += exp2f(ms - M) * p[s * (HD + 2) + 2 + dd];
    }
    o[((size_t)b * H + h) * HD + dd] = __float2half_rn(acc / L);
  }
}

// ---------------------------------------------------------------- host

static int decode_attention(Model& m, Replica& r, int nb, const half* q, const half* kc, const half* vc,
                            const DecSeq* seqs, int max_keys, half* out) {
  const Config& c = m.cfg;
  int splits = std::max(1, (2 * r.num_sms * 4 + nb * c.KV - 1) / (nb * c.KV));
  const int max_splits = (max_keys + PAGE - 1) / PAGE;
  splits = std::min(splits, max_splits);
  int split_len = (max_keys + splits - 1) / splits;
  split_len = (split_len + 31) / 32 * 32;
  splits = (max_keys + split_len - 1) / split_len;
  const size_t part_elems = (size_t)nb * c.H * splits * (c.hd + 2);
  if (int rc = r.dpart.ensure(part_elems * 4)) return rc;
  const float scale_log2 = (1.f / sqrtf((float)c.hd)) * 1.4426950408889634f;
  const int G = c.H / c.KV;
  dim3 grid(nb, c.KV, splits);
  {
    cudaEvent_t a;
    prof_begin(r, P_ATTN_DEC, &a);
    r.launches += 2;
    if (c.hd == 64)
      attn_decode_kernel<64><<<grid, 32 * G, 0, r.stream>>>(q, kc, vc, r.tables.as<int>(), seqs, c.H,
                                                          c.KV, scale_log2, split_len, splits, r.dpart.as<float>());
    else
      attn_decode_kernel<128><<<grid, 32 * G, 0, r.stream>>>(q, kc, vc, r.tables.as<int>(), seqs, c.H,
                                                           c.KV, scale_log2, split_len, splits, r.dpart.as<float>());
    LAYA_CK(cudaGetLastError());
    attn_combine_kernel<<<dim3(nb, c.H), 128, 0, r.stream>>>(r.dpart.as<float>(), c.H, c.hd, splits, out);
    LAYA_CK(cudaGetLastError());
    prof_end(r, P_ATTN_DEC, a);
  }
  return 0;
}

static int run_gemv(Replica& r, const QTensor& w, const half* x, int ldx, int nb, float* y, int ldy, int acc) {
  cudaEvent_t a;
  prof_begin(r, P_GEMV, &a);
  r.launches++;
  LAYA_CK(gemv(w, x, ldx, nb, y, ldy, acc, r.stream));
  prof_end(r, P_GEMV, a);
  return 0;
}

// Batches above this size run the linear layers on the tcgen05 GEMM.
static constexpr int kGemvMaxBatch = 16;

static int pad_batch(int nb) { return nb <= 1 ? 1 : nb <= 2 ? 2 : nb <= 4 ? 4 : nb <= 8 ? 8 : 16; }

// One decode step for nb sequences: tokens tok_in, positions pos, KV slots
// slot; writes the greedy tokens to tok_out.  Everything stays on the device,
// so consecutive steps run back to back.
static int decode_step(Model& m, Replica& r, int nb, const int* tok_in, const int* pos, const int* slot,
                       const DecSeq* seqs, int max_keys, int* tok_out) {
  const Config& c = m.cfg;
  const int qd = c.H * c.hd, kd = c.KV * c.hd, d = c.d, ffn = c.ffn;
  cudaStream_t st = r.stream;
  const bool small = nb <= kGemvMaxBatch;
  const int nbp = small ? pad_batch(nb) : nb;  // GEMV batch (padded rows are zero)
  int rc;
  float* x = r.x.as<float>();
  r.launches++;
  LAYA_CK(rows_f32(r.embd, tok_in, nb, x, st));
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
  auto stage = [&](const QTensor& t, half* out, int ldo, int grp, int gstride, int goff) -> int {
    r.launches++;
    LAYA_CK(dequant_f16(t, out, ldo, grp, gstride, goff, st));
    return 0;
  };
  for (int l = 0; l < c.L; l++) {
    const Layer& L = r.layers[l];
    half* kcl = r.kc.as<half>() + l * layer_elems;
    half* vcl = r.vc.as<half>() + l * layer_elems;
    r.launches++;
    LAYA_CK(rmsnorm(x, nullptr, nb, L.attn_norm, d, c.eps, h, nullptr, st));
    if (small) {
      if (L.wqkv16) {
        QTensor fused = L.wq;
        fused.rows = qd + 2 * kd;
        if ((rc = run_gemv(r, fused, h, d, nbp, f, qd + 2 * kd, 0))) return rc;
      } else {
        if ((rc = run_gemv(r, L.wq, h, d, nbp, f, qd + 2 * kd, 0)) ||
            (rc = run_gemv(r, L.wk, h, d, nbp, f + qd, qd + 2 * kd, 0)) ||
            (rc = run_gemv(r, L.wv, h, d, nbp, f + qd + kd, qd + 2 * kd, 0)))
          return rc;
      }
      r.launches++;
      rope_append_kernel<<<nb, 256, 0, st>>>(f, L.bqkv, qd, kd, c.hd, c.KV, pos, slot, r.rope, r.qb.as<half>(), kcl,
                                             vcl);
      LAYA_CK(cudaGetLastError());
    } else {
      const half* wqkv = L.wqkv16;
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
      a.pos = pos;
      a.slot = slot;
      a.rope = r.rope;
      a.kcache = kcl;
      a.vcache = vcl;
      a.page_size = PAGE;
      if ((rc = gemm_d(P_GEMM_QKV, EPI_QKV, h, d, wqkv, d, a))) return rc;
    }
    if ((rc = decode_attention(m, r, nb, r.qb.as<half>(), kcl, vcl, seqs, max_keys, r.att.as<half>()))) return rc;
    if (small) {
      if ((rc = run_gemv(r, L.wo, r.att.as<half>(), qd, nbp, x, d, 1))) return rc;
    } else {
      const half* wo = L.wo16;
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
      if ((rc = gemm_d(P_GEMM_O, EPI_RESID, r.att.as<half>(), qd, wo, qd, b))) return rc;
    }
    r.launches++;
    LAYA_CK(rmsnorm(x, nullptr, nb, L.ffn_norm, d, c.eps, h, nullptr, st));
    if (small) {
      r.launches++;
      if (L.wgu16) {
        if ((rc = run_gemv(r, L.wg, h, d, nbp, f, 2 * ffn, 0))) return rc;
        swiglu_kernel<<<dim3((ffn + 255) / 256, nb), 256, 0, st>>>(f, nullptr, ffn, 1, r.act.as<half>());
      } else {
        if ((rc = run_gemv(r, L.wg, h, d, nbp, f, ffn, 0)) ||
            (rc = run_gemv(r, L.wu, h, d, nbp, f + (size_t)nbp * ffn, ffn, 0)))
          return rc;
        swiglu_kernel<<<dim3((ffn + 255) / 256, nb), 256, 0, st>>>(f, f + (size_t)nbp * ffn, ffn, 0,
                                                                   r.act.as<half>());
      }
      LAYA_CK(cudaGetLastError());
      if ((rc = run_gemv(r, L.wd, r.act.as<half>(), ffn, nbp, x, d, 1))) return rc;
    } else {
      const half* wgu = L.wgu16;
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
      const half* wd = L.wd16;
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
      if ((rc = gemm_d(P_GEMM_DOWN, EPI_RESID, r.act.as<half>(), ffn, wd, ffn, dn))) return rc;
    }
  }
  // final norm + full-vocabulary logits + greedy argmax
  r.launches++;
  LAYA_CK(rmsnorm(x, nullptr, nb, r.out_norm, d, c.eps, h, nullptr, st));
  float* logits = r.dlogits.as<float>();
  if (small) {
    if ((rc = run_gemv(r, r.head, h, d, nbp, logits, c.V, 0))) return rc;
  } else {
    GemmArgs a{};
    a.M = nb;
    a.N = c.V;
    a.K = d;
    a.out = logits;
    a.ldo = c.V;
    if ((rc = gemm_d(P_GEMM_HEAD, EPI_F32, h, d, r.head16, d, a))) return rc;
  }
  r.launches++;
  argmax_kernel<<<nb, 256, 0, st>>>(logits, c.V, tok_out);
  LAYA_CK(cudaGetLastError());
  return 0;
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
  const bool small = n_seqs <= kGemvMaxBatch;
  if (!small && (rc = ensure_head16(m, r))) return rc;
  // pages: context + generated tokens per sequence
  std::vector<int> tables, toff(n_seqs), clen(n_seqs);
  int pages = 0;
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
    for (int t0 = 0; t0 < len; t0 += 64) pre.items.push_back({row0 + t0, std::min(64, len - t0), t0, toff[i]});
    pre.read_rows.push_back(row0 + len - 1);
  }
  if ((rc = ensure_kv(m, r, pages))) return rc;
  LAYA_CK(cudaMemsetAsync(r.err, 0, 4, r.stream));
  const int R = n_seqs;
  if ((rc = r.hid32.ensure((size_t)R * c.d * 4)) || (rc = r.hid16.ensure((size_t)R * c.d * 2))) return rc;
  const int qd = c.H * c.hd, kd = c.KV * c.hd;
  const int nbp = small ? pad_batch(n_seqs) : n_seqs;
  // per-step metadata for all steps, uploaded once: positions, slots, key counts
  std::vector<int> pos_all((size_t)steps * n_seqs), slot_all((size_t)steps * n_seqs);
  std::vector<DecSeq> seq_all((size_t)steps * n_seqs);
  std::vector<int> step_keys(steps, 0);
  for (int s = 1; s < steps; s++)
    for (int i = 0; i < n_seqs; i++) {
      const int p = clen[i] + s - 1;
      pos_all[(size_t)s * n_seqs + i] = p;
      slot_all[(size_t)s * n_seqs + i] = tables[toff[i] + p / PAGE] * PAGE + p % PAGE;
      seq_all[(size_t)s * n_seqs + i] = {toff[i], p + 1};
      step_keys[s] = std::max(step_keys[s], p + 1);
    }
  auto t0 = std::chrono::steady_clock::now();
  // prefill the contexts, then the first greedy token from the last position
  if ((rc = run_forward(m, r, pre, tables, 0, nullptr, nullptr, nullptr))) return rc;
  if ((rc = r.dlogits.ensure(std::max((size_t)nbp * c.V, (size_t)nbp * std::max(qd + 2 * kd, 2 * c.ffn)) * 4)) ||
      (rc = r.dargmax.ensure((size_t)steps * n_seqs * 4)))
    return rc;
  if (small) {
    // GEMV operands want F16 hidden rows, zero-padded to the GEMV batch
    if ((rc = r.dx16.ensure((size_t)nbp * c.d * 2))) return rc;
    LAYA_CK(cudaMemsetAsync(r.dx16.p, 0, (size_t)nbp * c.d * 2, r.stream));
    LAYA_CK(cudaMemcpyAsync(r.dx16.p, r.hid16.p, (size_t)R * c.d * 2, cudaMemcpyDeviceToDevice, r.stream));
    if ((rc = run_gemv(r, r.head, r.dx16.as<half>(), c.d, nbp, r.dlogits.as<float>(), c.V, 0))) return rc;
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
    LAYA_CK(gemm_launch(EPI_F32, r.hid16.as<half>(), c.d, r.head16, c.d, a, r.num_sms, r.stream));
  }
  int* toks = r.dargmax.as<int>();  // [steps][n_seqs] greedy tokens
  r.launches++;
  argmax_kernel<<<R, 256, 0, r.stream>>>(r.dlogits.as<float>(), c.V, toks);
  LAYA_CK(cudaGetLastError());
  // decode buffers sized for the padded batch; padded rows stay zero
  if ((rc = r.x.ensure((size_t)nbp * c.d * 4)) || (rc = r.h.ensure((size_t)nbp * c.d * 2)) ||
      (rc = r.qb.ensure((size_t)nbp * qd * 2)) || (rc = r.att.ensure((size_t)nbp * qd * 2)) ||
      (rc = r.act.ensure((size_t)nbp * c.ffn * 2)))
    return rc;
  LAYA_CK(cudaMemsetAsync(r.h.p, 0, (size_t)nbp * c.d * 2, r.stream));
  LAYA_CK(cudaMemsetAsync(r.att.p, 0, (size_t)nbp * qd * 2, r.stream));
  LAYA_CK(cudaMemsetAsync(r.act.p, 0, (size_t)nbp * c.ffn * 2, r.stream));
  DevBuf dmeta;
  const size_t nmeta = (size_t)steps * n_seqs;
  if ((rc = dmeta.ensure(nmeta * (8 + sizeof(DecSeq))))) return rc;
  int* dpos = dmeta.as<int>();
  int* dslot = dpos + nmeta;
  DecSeq* dseq = reinterpret_cast<DecSeq*>(dslot + nmeta);
  if ((rc = r.tables.ensure(tables.size() * 4))) {
    dmeta.release();
    return rc;
  }
  cudaError_t e = cudaMemcpyAsync(r.tables.p, tables.data(), tables.size() * 4, cudaMemcpyHostToDevice, r.stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dpos, pos_all.data(), nmeta * 4, cudaMemcpyHostToDevice, r.stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dslot, slot_all.data(), nmeta * 4, cudaMemcpyHostToDevice, r.stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dseq, seq_all.data(), nmeta * sizeof(DecSeq), cudaMemcpyHostToDevice, r.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(r.stream);
  r.h2d += (long long)(tables.size() * 4 + nmeta * (8 + sizeof(DecSeq)));
  if (e != cudaSuccess) {
    dmeta.release();
    return cuda_fail(e, "decode metadata upload");
  }
  auto t1 = std::chrono::steady_clock::now();
  if ((rc = timing_mark_start(r))) {
    dmeta.release();
    return rc;
  }
  for (int s = 1; s < steps && !rc; s++) {
    const size_t o = (size_t)s * n_seqs;
    rc = decode_step(m, r, n_seqs, toks + o - n_seqs, dpos + o, dslot + o, dseq + o, step_keys[s], toks + o);
  }
  if (!rc) rc = timing_mark_end(r);
  auto t2 = std::chrono::steady_clock::now();
  if (!rc) {
    std::vector<int> tk(nmeta);
    e = cudaMemcpy(tk.data(), toks, nmeta * 4, cudaMemcpyDeviceToHost);
    r.d2h += (long long)nmeta * 4;
    if (e != cudaSuccess) rc = cuda_fail(e, "decode token read-back");
    for (int s = 0; s < steps && !rc; s++)
      for (int i = 0; i < n_seqs; i++) out[(size_t)i * steps + s] = tk[(size_t)s * n_seqs + i];
  }
  dmeta.release();
  if (rc) return rc;
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
