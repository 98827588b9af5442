// Causal GQA prefill attention on the 5th-generation tensor cores
// (src/models/openthai/model.rs:276-294: softmax(q.k * scale) over keys
// j <= i, then .v, with kv head = h / (H/KV)), flash-style over the paged
// KV cache.
//
// One CTA = up to 128 query rows of one sequence x one query head,
// 192 threads:
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
#include <cuda.h>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"
#include "mma.cuh"
#include "ptx.cuh"

namespace laya {

template <int HD>
struct Atc {
  static constexpr int NS = HD == 64 ? 3 : 3;      // K/V ring stages (pages)
  static constexpr int Q_BYTES = 128 * HD * 2;     // [HD/64 blocks][128 rows][128 B]
  static constexpr int KV_BYTES = 64 * HD * 2;     // K or V page: [HD/64 blocks][64 rows][128 B]
  static constexpr int STAGE = 2 * KV_BYTES;
  static constexpr int P_BYTES = 128 * 64 * 2;     // [128 rows][64 keys] F16
  static constexpr int OFF_KV = Q_BYTES;
  static constexpr int OFF_P = OFF_KV + NS * STAGE;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int TMEM_COLS = 256;            // S buffers at 0 and 64, O at 128
  static constexpr int O_COL = 128;
};

// K-major operand descriptor of k-step kk (16 elements) of a tile stored as
// 64-element (128-byte) column blocks `block_bytes` apart.
__device__ __forceinline__ uint64_t kdesc(const uint8_t* base, int kk, int block_bytes) {
  return sw128_desc(smem_u32(base + (kk >> 2) * block_bytes + (kk & 3) * 32));
}

template <int HD>
__global__ void __launch_bounds__(192, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, half* __restrict__ o, int ldo,
                   const int* __restrict__ tables, const AttnItem* __restrict__ items, int H, int KV,
                   float scale_log2, unsigned* err, long long budget) {
  using C = Atc<HD>;
  extern __shared__ uint8_t at_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(at_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm;
  uint8_t* sKV = sm + C::OFF_KV;
  uint8_t* sP = sm + C::OFF_P;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + C::NS;
  uint64_t* s_full = kv_empty + C::NS;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 2;   // one phase per P.V page
  uint64_t* o_final = o_done + 1;  // the last P.V
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);

  const AttnItem it = items[blockIdx.x];
  const int h = blockIdx.y, kvh = h / (H / KV);
  const int n_keys = it.pos0 + it.q_len;
  const int nblk = (n_keys + 63) / 64;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::NS; s++) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&p_full[b], 4);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int hb = 0; hb < HD / 64; hb++) tma_load_2d(sQ + hb * 16384, &tq, q_full, h * HD + hb * 64, it.q_row);
      for (int j = 0; j < nblk; j++) {
        const int st = j % C::NS;
        if (!mbar_wait(&kv_empty[st], ((j / C::NS) & 1) ^ 1, budget)) atomicOr(err, 1u << 12);
        const int row = (tables[it.table_off + j] * KV + kvh) * 64;
        uint8_t* dst = sKV + st * C::STAGE;
        mbar_expect_tx(&kv_full[st], C::STAGE);
#pragma unroll
        for (int hb = 0; hb < HD / 64; hb++) {
          tma_load_2d(dst + hb * 8192, &tk, &kv_full[st], hb * 64, row);
          tma_load_2d(dst + C::KV_BYTES + hb * 8192, &tv, &kv_full[st], hb * 64, row);
        }
      }
      // Drain: the last use of every stage is released (its P.V finished)
      // before the CTA may exit, so no MMA completion arrives afterwards.
      for (int j = nblk - 1; j >= 0 && j >= nblk - C::NS; j--)
        if (!mbar_wait(&kv_empty[j % C::NS], (j / C::NS) & 1, budget)) atomicOr(err, 1u << 20);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idS = idesc_f16_f32(128, 64);
      const uint32_t idO = idesc_f16_f32(128, HD) | (1u << 16);  // B (V) MN-major
      if (!mbar_wait(q_full, 0, budget)) atomicOr(err, 1u << 13);
      tc_fence_after();
      for (int j = 0; j <= nblk; j++) {
        if (j < nblk) {
          const int st = j % C::NS, sb = j & 1;
          if (!mbar_wait(&kv_full[st], (j / C::NS) & 1, budget)) atomicOr(err, 1u << 14);
          if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1, budget)) atomicOr(err, 1u << 15);
          tc_fence_after();
          const uint8_t* sK = sKV + st * C::STAGE;
#pragma unroll
          for (int kk = 0; kk < HD / 16; kk++)
            umma_f16(tbase + sb * 64, kdesc(sQ, kk, 16384), kdesc(sK, kk, 8192), idS, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[sb]);
        }
        if (j >= 1) {
          const int jj = j - 1, st = jj % C::NS, pb = jj & 1;
          if (!mbar_wait(&p_full[pb], (jj >> 1) & 1, budget)) atomicOr(err, 1u << 16);
          tc_fence_after();
          const uint8_t* sV = sKV + st * C::STAGE + C::KV_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            umma_f16(tbase + C::O_COL, sw128_desc(smem_u32(sP + pb * C::P_BYTES + kk * 32)),
                     sw128_mn_desc(smem_u32(sV + kk * 2048), 8192, 1024), idO, (jj > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&kv_empty[st]);
          umma_commit(o_done);
          if (jj == nblk - 1) umma_commit(o_final);
        }
      }
    }
  } else {
    // softmax: thread = query row r = TMEM lane r
    const int quarter = warp % 4, r = quarter * 32 + lane;
    const int pos = it.pos0 + r;
    const uint32_t tl = tbase + ((uint32_t)(quarter * 32) << 16);
    float mref = -INFINITY, l = 0.f;  // reference maximum in log2 units
    for (int j = 0; j < nblk; j++) {
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, budget) && lane == 0) atomicOr(err, 1u << 17);
      tc_fence_after();
      float s[64];
      {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(tl + sb * 64, v);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; c++) s[c] = __uint_as_float(v[c]) * scale_log2;
        tmem_ld32(tl + sb * 64 + 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; c++) s[32 + c] = __uint_as_float(v[c]) * scale_log2;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      const int key0 = j * 64;
      if (key0 + 63 > it.pos0 || key0 + 64 > n_keys) {
#pragma unroll
        for (int c = 0; c < 64; c++)
          if (key0 + c > pos || key0 + c >= n_keys) s[c] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; c++) mx = fmaxf(mx, s[c]);
      // Page 0 holds key 0 <= every position, so mref is finite from j = 0 on.
      // A row moves its reference when its maximum exceeds it by more than 8
      // (P stays <= 2^8); the warp rescales its rows of O together, because
      // TMEM loads and stores are warp-wide.
      const float nref = mx > mref + 8.f ? mx : mref;
      const float corr = exp2f(mref - nref);  // 1 when unchanged; unused at j = 0
      if (j > 0 && __any_sync(0xffffffffu, nref != mref)) {
        // O holds P.V of pages < j once page j-1's MMA is done
        if (!mbar_wait(o_done, (j - 1) & 1, budget) && lane == 0) atomicOr(err, 1u << 18);
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD / 32; c++) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32(tl + C::O_COL + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
          tmem_st32(tl + C::O_COL + c * 32, v);
        }
        tmem_st_wait();
        l *= corr;
      }
      mref = nref;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 64; c++) {
        s[c] = exp2f(s[c] - mref);
        sum += s[c];
      }
      l += sum;
      // P row r: [128 rows][64 keys] F16, 16-byte unit u of row r at u ^ (r % 8)
      uint8_t* prow = sP + sb * C::P_BYTES + r * 128;
#pragma unroll
      for (int u = 0; u < 8; u++) {
        uint4 w;
        w.x = pack_h2(s[8 * u], s[8 * u + 1]);
        w.y = pack_h2(s[8 * u + 2], s[8 * u + 3]);
        w.z = pack_h2(s[8 * u + 4], s[8 * u + 5]);
        w.w = pack_h2(s[8 * u + 6], s[8 * u + 7]);
        *reinterpret_cast<uint4*>(prow + ((u ^ (r & 7)) << 4)) = w;
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    // (o_done's parity cannot tell page nblk-1 from nblk-3 here: at this
    // point only the P.V of page nblk-3 is known to be done)
    if (!mbar_wait(o_final, 0, budget) && lane == 0) atomicOr(err, 1u << 19);
    tc_fence_after();
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < HD / 32; c++) {
      uint32_t v[32];
      __syncwarp();
      tmem_ld32(tl + C::O_COL + c * 32, v);
      tmem_ld_wait();
      if (r < it.q_len) {
        half* dst = o + (size_t)(it.q_row + r) * ldo + h * HD + c * 32;
#pragma unroll
        for (int u = 0; u < 4; u++) {
          uint4 w;
          w.x = pack_h2(__uint_as_float(v[8 * u]) * inv, __uint_as_float(v[8 * u + 1]) * inv);
          w.y = pack_h2(__uint_as_float(v[8 * u + 2]) * inv, __uint_as_float(v[8 * u + 3]) * inv);
          w.z = pack_h2(__uint_as_float(v[8 * u + 4]) * inv, __uint_as_float(v[8 * u + 5]) * inv);
          w.w = pack_h2(__uint_as_float(v[8 * u + 6]) * inv, __uint_as_float(v[8 * u + 7]) * inv);
          reinterpret_cast<uint4*>(dst)[u] = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

template <int HD>
static cudaError_t attn_tc_go(const AttnParams& p, const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tv, cudaStream_t st) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, Atc<HD>::SMEM);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  attn_tc_kernel<HD><<<dim3(p.n_items, p.H), 192, Atc<HD>::SMEM, st>>>(
      tq, tk, tv, p.o, p.ldo, p.tables, p.items, p.H, p.KV, p.scale_log2, p.err, 100000000ll);
  return cudaGetLastError();
}

cudaError_t attention_tc(const AttnParams& p, cudaStream_t st) {
  if (!p.n_items) return cudaSuccess;
  if ((p.hd != 64 && p.hd != 128) || !p.err || p.q_rows <= 0 || p.kv_rows <= 0 || (p.ldq % 8)) return cudaErrorNotSupported;
  CUtensorMap tq, tk, tv;
  const uint64_t qdims[2] = {(uint64_t)p.ldq, (uint64_t)p.q_rows}, qstr[1] = {(uint64_t)p.ldq * 2};
  const uint32_t qbox[2] = {64, 128};
  const uint64_t kdims[2] = {(uint64_t)p.hd, (uint64_t)p.kv_rows}, kstr[1] = {(uint64_t)p.hd * 2};
  const uint32_t kbox[2] = {64, 64};
  if (!encode_tiled(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.q, qdims, qstr, qbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.kc, kdims, kstr, kbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.vc, kdims, kstr, kbox, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (p.hd == 64) return attn_tc_go<64>(p, tq, tk, tv, st);
  return attn_tc_go<128>(p, tq, tk, tv, st);
}

}  // namespace laya
