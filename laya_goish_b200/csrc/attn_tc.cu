// Causal GQA prefill attention on the 5th-generation tensor cores
// (src/models/openthai/model.rs:276-294: softmax(q.k * scale) over keys
// j <= i, then .v, with kv head = h / (H/KV)), flash-style over the paged
// KV cache.
//
// Work unit = up to 128 query rows of one sequence x one query head; a
// persistent CTA (192 threads) runs a strided list of units:
//   warp 0     : TMA producer: the Q tile once, then each 64-key page's K and
//                V blocks into a ring (64 x 128 B boxes, 128-byte swizzle)
//   warp 1     : allocates TMEM; one thread issues S_j = Q.K_j^T (M 128,
//                N 64) into one of two TMEM score buffers, then
//                O += P_{j-1}.V_{j-1} (M 128, N hd) into the TMEM output, V
//                read in place as an MN-major operand
//   warps 2..5 : softmax, thread = query row = TMEM lane: scores from TMEM,
//                causal mask on boundary pages, exponentials against a
//                running reference maximum, P (F16) into shared memory as
//                the next MMA's A operand.  O in TMEM is rescaled only when
//                a row's maximum grows by more than 2^8 over the reference,
//                so P stays <= 256 and the rescale is rare; l is kept with
//                the same reference.
// tcgen05.commit of S_j covers every earlier MMA of the thread, so when a
// softmax warp sees S_j, P.V of page j-2 has finished: its P buffer may be
// rewritten, and o_done is in phase j-1 or later, so its parity identifies
// page j-1 unambiguously; the final read of O waits on its own barrier.
#include <atomic>
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"
#include "launch.h"
#include "mma.cuh"
#include "ptx.cuh"

namespace laya {

template <int HD>
struct Atc {
  // K pages are released as soon as their S MMA is done, V pages only after
  // their P.V MMA, so the K ring is the deeper one.  Head dim 256 (OpenThai's
  // gated attention) keeps one Q buffer and one O accumulator so that its
  // 64 KB Q tile and 32 KB pages fit: the next unit's P.V then waits for the
  // previous unit's O to be read.
  static constexpr int NQ = HD == 256 ? 1 : 2;     // Q buffers
  static constexpr int NO = HD == 256 ? 1 : 2;     // O accumulators in TMEM
  static constexpr int NK = HD == 256 ? 2 : 3;
  static constexpr int NV = HD == 128 ? 3 : 2;
  static constexpr int Q_BYTES = 128 * HD * 2;     // [HD/64 blocks][128 rows][128 B]
  static constexpr int KV_BYTES = 64 * HD * 2;     // K or V page: [HD/64 blocks][64 rows][128 B]
  static constexpr int P_BYTES = 128 * 64 * 2;     // [128 rows][64 keys] F16
  static constexpr int OFF_K = NQ * Q_BYTES;
  static constexpr int OFF_V = OFF_K + NK * KV_BYTES;
  static constexpr int OFF_P = OFF_V + NV * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int TMEM_COLS = HD == 64 ? 256 : 512;  // S buffers at 0, 64; O buffers at 128 (+ HD)
  static constexpr int O_COL = 128;
  static constexpr int CTAS_PER_SM = HD == 64 ? 2 : 1;
  static_assert(O_COL + NO * HD <= TMEM_COLS, "TMEM columns");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// 2^x with the SFU's approximate exponent (PTX ex2.approx.ftz: relative
// error ~2^-22, far below the F16 rounding of P); 2^-inf = 0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// K-major operand descriptor of k-step kk (16 elements) of a tile stored as
// 64-element (128-byte) column blocks `block_bytes` apart.
__device__ __forceinline__ uint64_t kdesc(const uint8_t* base, int kk, int block_bytes) {
  return sw128_desc(smem_u32(base + (kk >> 2) * block_bytes + (kk & 3) * 32));
}

struct AtcUnit {
  int q_row, rows, pos0, table_off;  // query tokens q_row .. q_row + rows - 1 at positions pos0 ..
  int hg, n_keys, nblk;              // head group: query heads hg * gp .. hg * gp + gp - 1
};

// Rows of the 128-row tile per query head when gp heads share a unit: the
// packed form puts the gp = H / KV heads of one KV head in one tile (row =
// g * RT + t), so each K/V page is loaded and multiplied once for the group;
// gp = 1 is one head per unit over 128 tokens.  A multiple of 8 (whole
// swizzle atoms).
__host__ __device__ __forceinline__ int atc_rt(int gp) { return (128 / gp) & ~7; }

// Unit u = (item, block sb of RT tokens, head group hg of NHG).  Items hold
// up to 128 tokens, so an item has ceil(128 / RT) blocks; a block past the
// item's tokens is an empty unit (rows <= 0) that every role skips.
__device__ __forceinline__ AtcUnit atc_unit(const AttnItem* items, int u, int SB, int NHG, int RT) {
  AtcUnit w;
  const AttnItem it = items[u / (SB * NHG)];
  const int rem = u % (SB * NHG), t0 = (rem / NHG) * RT;
  w.hg = rem % NHG;
  w.rows = min(RT, it.q_len - t0);
  w.q_row = it.q_row + t0;
  w.pos0 = it.pos0 + t0;
  w.table_off = it.table_off;
  w.n_keys = w.pos0 + max(w.rows, 0);
  w.nblk = (w.n_keys + 63) / 64;
  return w;
}

// Persistent: CTA c takes work units u = c, c + gridDim.x, ... (see
// atc_unit; CTAs running together share K/V pages in L2).  All
// ring, buffer and barrier indices run over the CTA's global page count g
// and unit count k, so the producer fetches the next unit's Q and pages
// while the current unit is still being computed.
template <int HD>
__global__ void __launch_bounds__(192, Atc<HD>::CTAS_PER_SM)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, half* __restrict__ o, int ldo,
                   const int* __restrict__ tables, const AttnItem* __restrict__ items, int n_units, int H, int KV,
                   int gp,
                   float scale_log2, const float* __restrict__ gate, int ldg, int ghs, unsigned* err,
                   long long budget) {
  using C = Atc<HD>;
  extern __shared__ uint8_t at_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(at_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm;
  uint8_t* sK = sm + C::OFF_K;
  uint8_t* sV = sm + C::OFF_V;
  uint8_t* sP = sm + C::OFF_P;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);  // [2] Q of unit k in buffer k % NQ
  uint64_t* q_empty = q_full + 2;                                   // [2] the unit's last S MMA is done
  uint64_t* k_full = q_empty + 2;                                   // [NK] K of page g in stage g % NK
  uint64_t* k_empty = k_full + C::NK;                               // [NK] its S MMA is done
  uint64_t* v_full = k_empty + C::NK;                               // [NV] V of page g in stage g % NV
  uint64_t* v_empty = v_full + C::NV;                               // [NV] its P.V MMA is done
  uint64_t* s_full = v_empty + C::NV;                               // [2] S of page g in buffer g & 1
  uint64_t* s_empty = s_full + 2;                                   // [2] 4 softmax warps read it
  uint64_t* p_full = s_empty + 2;                                   // [2] P of page g written (4 warps)
  uint64_t* o_done = p_full + 2;                                    // one phase per P.V page
  uint64_t* o_full = o_done + 1;                                    // [2] O of unit k (buffer k % NO) complete
  uint64_t* o_empty = o_full + 2;                                   // [2] O of unit k read (4 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // G heads per unit (gp), NHG head groups, GQ query heads per KV head
  const int G = gp, NHG = H / gp, GQ = H / KV, RT = atc_rt(G), SB = (128 + RT - 1) / RT;
  // Q rows G * RT .. 127 are never loaded (G not a power of two): zero, so
  // their scores stay finite; they are never written out.
  for (int i = threadIdx.x; i < C::NQ * (HD / 64) * (128 - G * RT) * 8; i += blockDim.x) {
    const int per = (128 - G * RT) * 8, blk = i / per, e = i % per;
    reinterpret_cast<uint4*>(sQ + blk * 16384 + G * RT * 128)[e] = make_uint4(0u, 0u, 0u, 0u);
  }
  fence_async_smem();
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; b++) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&o_full[b], 1);
      mbar_init(&o_empty[b], 4);
    }
    for (int i = 0; i < C::NK; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < C::NV; i++) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(o_done, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  // Launched early behind the previous kernel: everything above is set-up;
  // every global read below waits for that kernel's output.
  pdl_wait();
  pdl_trigger();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      for (int u = blockIdx.x, k = 0; u < n_units; u += gridDim.x) {
        const AtcUnit w = atc_unit(items, u, SB, NHG, RT);
        if (w.rows <= 0) continue;
        const int qb = k % C::NQ;
        if (!mbar_wait(&q_empty[qb], ((k / C::NQ) & 1) ^ 1, budget)) atomicOr(err, 1u << 12);
        mbar_expect_tx(&q_full[qb], (uint32_t)(G * RT * 128 * (HD / 64)));
        // head g of the group: RT token rows into tile rows g * RT ..
#pragma unroll
        for (int hb = 0; hb < HD / 64; hb++)
          for (int gg = 0; gg < G; gg++)
            tma_load_2d(sQ + qb * C::Q_BYTES + hb * 16384 + gg * RT * 128, &tq, &q_full[qb],
                        (w.hg * G + gg) * HD + hb * 64, w.q_row);
        k++;
        for (int j = 0; j < w.nblk; j++, g++) {
          const int row = (tables[w.table_off + j] * KV + w.hg * G / GQ) * 64;
          const int ks = g % C::NK, vs = g % C::NV;
          if (!mbar_wait(&k_empty[ks], ((g / C::NK) & 1) ^ 1, budget)) atomicOr(err, 1u << 12);
          mbar_expect_tx(&k_full[ks], C::KV_BYTES);
#pragma unroll
          for (int hb = 0; hb < HD / 64; hb++)
            tma_load_2d(sK + ks * C::KV_BYTES + hb * 8192, &tk, &k_full[ks], hb * 64, row);
          if (!mbar_wait(&v_empty[vs], ((g / C::NV) & 1) ^ 1, budget)) atomicOr(err, 1u << 12);
          mbar_expect_tx(&v_full[vs], C::KV_BYTES);
#pragma unroll
          for (int hb = 0; hb < HD / 64; hb++)
            tma_load_2d(sV + vs * C::KV_BYTES + hb * 8192, &tv, &v_full[vs], hb * 64, row);
        }
      }
      // Drain: the last use of every stage is released (its MMA finished)
      // before the CTA may exit, so no MMA completion arrives afterwards.
      for (int x = g - 1; x >= 0 && x >= g - C::NK; x--)
        if (!mbar_wait(&k_empty[x % C::NK], (x / C::NK) & 1, budget)) atomicOr(err, 1u << 20);
      for (int x = g - 1; x >= 0 && x >= g - C::NV; x--)
        if (!mbar_wait(&v_empty[x % C::NV], (x / C::NV) & 1, budget)) atomicOr(err, 1u << 20);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idS = idesc_f16_f32(128, 64);
      const uint32_t idO = idesc_f16_f32(128, HD) | (1u << 16);  // B (V) MN-major
      // P.V of page pg (stage pst) into O buffer pob; first / last page of its unit
      int pg = -1, pob = 0, pk = 0;
      bool pfirst = false, plast = false;
      auto issue_pv = [&]() {
        const int pb = pg & 1;
        if (pfirst && !mbar_wait(&o_empty[pob], ((pk / C::NO) & 1) ^ 1, budget)) atomicOr(err, 1u << 16);
        const int vs = pg % C::NV;
        if (!mbar_wait(&p_full[pb], (pg >> 1) & 1, budget)) atomicOr(err, 1u << 16);
        if (!mbar_wait(&v_full[vs], (pg / C::NV) & 1, budget)) atomicOr(err, 1u << 16);
        tc_fence_after();
        const uint8_t* v = sV + vs * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          umma_f16(tbase + C::O_COL + pob * HD, sw128_desc(smem_u32(sP + pb * C::P_BYTES + kk * 32)),
                   sw128_mn_desc(smem_u32(v + kk * 2048), 8192, 1024), idO, (!pfirst || kk > 0) ? 1u : 0u);
        umma_commit(&v_empty[vs]);
        umma_commit(o_done);
        if (plast) umma_commit(&o_full[pob]);
      };
      int g = 0;
      for (int u = blockIdx.x, k = -1; u < n_units; u += gridDim.x) {
        const AtcUnit w = atc_unit(items, u, SB, NHG, RT);
        if (w.rows <= 0) continue;
        k++;
        const int qb = k % C::NQ;
        if (!mbar_wait(&q_full[qb], (k / C::NQ) & 1, budget)) atomicOr(err, 1u << 13);
        for (int j = 0; j < w.nblk; j++, g++) {
          const int ks = g % C::NK, sb = g & 1;
          if (!mbar_wait(&k_full[ks], (g / C::NK) & 1, budget)) atomicOr(err, 1u << 14);
          if (!mbar_wait(&s_empty[sb], ((g >> 1) & 1) ^ 1, budget)) atomicOr(err, 1u << 15);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 16; kk++)
            umma_f16(tbase + sb * 64, kdesc(sQ + qb * C::Q_BYTES, kk, 16384), kdesc(sK + ks * C::KV_BYTES, kk, 8192),
                     idS, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[sb]);
          umma_commit(&k_empty[ks]);
          if (j == w.nblk - 1) umma_commit(&q_empty[qb]);
          if (pg >= 0) issue_pv();
          pg = g;
          pob = k % C::NO;
          pk = k;
          pfirst = j == 0;
          plast = j == w.nblk - 1;
        }
      }
      if (pg >= 0) issue_pv();
    }
  } else {
    // softmax: thread = query row r = TMEM lane r
    const int quarter = warp % 4, r = quarter * 32 + lane;
    const uint32_t tl = tbase + ((uint32_t)(quarter * 32) << 16);
    int g = 0;
    const int rg = r / RT, rt = r % RT;  // this row's head in the group and token in the block
    for (int u = blockIdx.x, k = -1; u < n_units; u += gridDim.x) {
      const AtcUnit w = atc_unit(items, u, SB, NHG, RT);
      if (w.rows <= 0) continue;
      k++;
      const int ob = k % C::NO;
      const int pos = w.pos0 + rt;
      float mref = -INFINITY, l = 0.f;  // reference maximum in log2 units
      for (int j = 0; j < w.nblk; j++, g++) {
        const int sb = g & 1;
        if (!mbar_wait(&s_full[sb], (g >> 1) & 1, budget) && lane == 0) atomicOr(err, 1u << 17);
        tc_fence_after();
        uint32_t v0[32], v1[32];
        __syncwarp();
        tmem_ld32(tl + sb * 64, v0);
        tmem_ld32(tl + sb * 64 + 32, v1);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[sb]);
        float s[64];
#pragma unroll
        for (int c = 0; c < 32; c++) {
          s[c] = __uint_as_float(v0[c]);
          s[32 + c] = __uint_as_float(v1[c]);
        }
        const int key0 = j * 64;
        if (key0 + 63 > w.pos0 || key0 + 64 > w.n_keys) {
          // keys key0 + c with c > lim are masked (causal, and past the last key)
          const int lim = min(pos, w.n_keys - 1) - key0;
#pragma unroll
          for (int c = 0; c < 64; c++) s[c] = c > lim ? -INFINITY : s[c];
        }
        float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int c = 4; c < 64; c++) m4[c & 3] = fmaxf(m4[c & 3], s[c]);
        // raw scores; the scale is positive, so the maximum commutes with it
        const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale_log2;
        // Page 0 holds key 0 <= every position, so mref is finite from j = 0
        // on.  A row moves its reference when its maximum exceeds it by more
        // than 8 (P stays <= 2^8); the warp rescales its rows of O together,
        // because TMEM loads and stores are warp-wide.
        const float nref = mx > mref + 8.f ? mx : mref;
        const float corr = ex2(mref - nref);  // 1 when unchanged; unused at j = 0
        if (j > 0 && __any_sync(0xffffffffu, nref != mref)) {
          // O holds P.V of this unit's pages < j once page g-1's MMA is done
          if (!mbar_wait(o_done, (g - 1) & 1, budget) && lane == 0) atomicOr(err, 1u << 18);
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < HD / 32; c++) {
            uint32_t v[32];
            __syncwarp();
            tmem_ld32(tl + C::O_COL + ob * HD + c * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
            tmem_st32(tl + C::O_COL + ob * HD + c * 32, v);
          }
          tmem_st_wait();
          l *= corr;
        }
        mref = nref;
        // Packed F32x2 FMA / add (one instruction per two scores, the same
        // IEEE results as two fmaf / two adds); the sums keep the order of
        // four running partials l[c % 4].
        unsigned long long sc2, nm2, acc2[2];
        asm("mov.b64 %0, {%1, %1};" : "=l"(sc2) : "f"(scale_log2));
        asm("mov.b64 %0, {%1, %1};" : "=l"(nm2) : "f"(-mref));
        asm("mov.b64 %0, {%1, %1};" : "=l"(acc2[0]) : "f"(0.f));
        acc2[1] = acc2[0];
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          unsigned long long x2, e2, p2;
          asm("mov.b64 %0, {%1, %2};" : "=l"(x2) : "f"(s[c]), "f"(s[c + 1]));
          asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(e2) : "l"(x2), "l"(sc2), "l"(nm2));
          float e0, e1;
          asm("mov.b64 {%0, %1}, %2;" : "=f"(e0), "=f"(e1) : "l"(e2));
          s[c] = ex2(e0);
          s[c + 1] = ex2(e1);
          asm("mov.b64 %0, {%1, %2};" : "=l"(p2) : "f"(s[c]), "f"(s[c + 1]));
          asm("add.rn.f32x2 %0, %1, %2;" : "=l"(acc2[(c >> 1) & 1]) : "l"(acc2[(c >> 1) & 1]), "l"(p2));
        }
        float l4[4];
        asm("mov.b64 {%0, %1}, %2;" : "=f"(l4[0]), "=f"(l4[1]) : "l"(acc2[0]));
        asm("mov.b64 {%0, %1}, %2;" : "=f"(l4[2]), "=f"(l4[3]) : "l"(acc2[1]));
        l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
        // P row r: [128 rows][64 keys] F16, 16-byte unit u of row r at u ^ (r % 8)
        uint8_t* prow = sP + sb * C::P_BYTES + r * 128;
#pragma unroll
        for (int u8 = 0; u8 < 8; u8++) {
          uint4 pw;
          pw.x = pack_h2(s[8 * u8], s[8 * u8 + 1]);
          pw.y = pack_h2(s[8 * u8 + 2], s[8 * u8 + 3]);
          pw.z = pack_h2(s[8 * u8 + 4], s[8 * u8 + 5]);
          pw.w = pack_h2(s[8 * u8 + 6], s[8 * u8 + 7]);
          *reinterpret_cast<uint4*>(prow + ((u8 ^ (r & 7)) << 4)) = pw;
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
      }
      // O of this unit
      if (!mbar_wait(&o_full[ob], (k / C::NO) & 1, budget) && lane == 0) atomicOr(err, 1u << 19);
      tc_fence_after();
      const float inv = 1.f / l;
#pragma unroll
      for (int c = 0; c < HD / 32; c++) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(tl + C::O_COL + ob * HD + c * 32, v);
        tmem_ld_wait();
        if (rg < G && rt < w.rows) {
          const int h = w.hg * G + rg;
          half* dst = o + (size_t)(w.q_row + rt) * ldo + h * HD + c * 32;
          if (gate) {
            // OpenThai's output gate: o * sigmoid(gate) (src/models/openthai/model.rs:293-295);
            // the row's 32 gate values as eight 16-byte loads (rows are 16-byte aligned)
            const float4* gr = reinterpret_cast<const float4*>(gate + (size_t)(w.q_row + rt) * ldg + h * ghs + c * 32);
#pragma unroll
            for (int i4 = 0; i4 < 8; i4++) {
              const float4 gv = __ldg(gr + i4);
              const float gg[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
              for (int e = 0; e < 4; e++)
                v[4 * i4 + e] = __float_as_uint(__uint_as_float(v[4 * i4 + e]) * inv * (1.f / (1.f + expf(-gg[e]))));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = __float_as_uint(__uint_as_float(v[i]) * inv);
          }
#pragma unroll
          for (int u4 = 0; u4 < 4; u4++) {
            uint4 ow;
            ow.x = pack_h2(__uint_as_float(v[8 * u4]), __uint_as_float(v[8 * u4 + 1]));
            ow.y = pack_h2(__uint_as_float(v[8 * u4 + 2]), __uint_as_float(v[8 * u4 + 3]));
            ow.z = pack_h2(__uint_as_float(v[8 * u4 + 4]), __uint_as_float(v[8 * u4 + 5]));
            ow.w = pack_h2(__uint_as_float(v[8 * u4 + 6]), __uint_as_float(v[8 * u4 + 7]));
            reinterpret_cast<uint4*>(dst)[u4] = ow;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[ob]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// LAYA_ATTN_PACK=0 / 1 overrides the caller's choice of packed units.
static int attn_pack_forced() {
  static const int forced = [] {
    const char* e = std::getenv("LAYA_ATTN_PACK");
    return e ? std::atoi(e) : -1;
  }();
  return forced;
}

template <int HD>
static cudaError_t attn_tc_go(const AttnParams& p, const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tv, cudaStream_t st) {
  static std::atomic<bool> configured[64];  // per device; any host thread may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, Atc<HD>::SMEM);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  static std::atomic<int> sms[64];
  if (!sms[dev & 63]) {
    int n = 0;
    cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sms[dev & 63] = n;
  }
  const int gp = (attn_pack_forced() >= 0 ? attn_pack_forced() : p.pack) ? p.H / p.KV : 1;
  const int RT = atc_rt(gp), units = p.n_items * ((128 + RT - 1) / RT) * (p.H / gp);
  const int grid = std::min(units, Atc<HD>::CTAS_PER_SM * sms[dev & 63]);
  // programmatic dependent launch: the CTAs set up their barriers and TMEM
  // while the previous kernel drains
  return launch_k(attn_tc_kernel<HD>, dim3(grid), dim3(192), (size_t)Atc<HD>::SMEM, st, true, tq, tk, tv, p.o, p.ldo,
                  p.tables, p.items, units, p.H, p.KV, gp, p.scale_log2, p.gate, p.ldg, p.ghs, p.err, 100000000ll);
}

cudaError_t attention_tc(const AttnParams& p, cudaStream_t st) {
  if (!p.n_items) return cudaSuccess;
  if ((p.hd != 64 && p.hd != 128 && p.hd != 256) || !p.err || p.q_rows <= 0 || p.kv_rows <= 0 || (p.ldq % 8))
    return cudaErrorNotSupported;
  if (p.gate && ((reinterpret_cast<uintptr_t>(p.gate) & 15) || (p.ldg % 4) || (p.ghs % 4))) return cudaErrorInvalidValue;
  CUtensorMap tq, tk, tv;
  const uint64_t qdims[2] = {(uint64_t)p.ldq, (uint64_t)p.q_rows}, qstr[1] = {(uint64_t)p.ldq * 2};
  if (p.H % p.KV || p.H / p.KV > 16) return cudaErrorNotSupported;
  const int gp = (attn_pack_forced() >= 0 ? attn_pack_forced() : p.pack) ? p.H / p.KV : 1;
  const uint32_t qbox[2] = {64, (uint32_t)atc_rt(gp)};  // one head's block of query rows
  const uint64_t kdims[2] = {(uint64_t)p.hd, (uint64_t)p.kv_rows}, kstr[1] = {(uint64_t)p.hd * 2};
  const uint32_t kbox[2] = {64, 64};
  if (!encode_tiled(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.q, qdims, qstr, qbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.kc, kdims, kstr, kbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.vc, kdims, kstr, kbox, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (p.hd == 64) return attn_tc_go<64>(p, tq, tk, tv, st);
  if (p.hd == 128) return attn_tc_go<128>(p, tq, tk, tv, st);
  return attn_tc_go<256>(p, tq, tk, tv, st);
}

}  // namespace laya
