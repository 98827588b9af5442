// Prefill GEMM with Q8_0 weights decoded inside the kernel's shared-memory
// staging (tcgen05 + TMEM, CTA pairs).
//
//   Y[M x N] = X[M x K] . W[N x K]^T,  W as Q8_0 blocks: W[n][k] = d[n][k/32] * q[n][k]
//
// The contract is the reference's Matrix::apply (src/tensor.rs:10-102) over a
// matrix that the reference decodes to F32 at load (src/gguf.rs:250-260,
// src/models/openthai/model.rs:61).  Here the quants stay in HBM as int8 and
// are decoded per tile on the way to the tensor cores, so a pass reads 1.06
// bytes per weight (int8 + one F16 scale per 32) instead of the 2 bytes of
// the resident F16 operand cache; at the small M of short prompts, branch
// passes and batched decode steps those bytes are the bound.
//
// Per CTA of a pair (tile 256 x 256; this CTA owns 128 rows of X and 128
// rows of W):
//   warp 0      weight stream: per 128-column K block one int8 box (128 rows
//               x 128 B, 128-byte swizzle) and one scale box (4 blocks x 128
//               rows) into a raw stage, up to Q8_RS stages ahead
//   warp 10     X stream: per 64-column K block the X box (pair form, counted
//               on the leader's barrier), up to Q8_XS stages ahead
//   warp 1      TMEM allocation; on the leader one thread issues
//               tcgen05.mma.cta_group::2 per operand stage
//   warps 6..9  converters: thread t decodes the first 64 columns of row t of
//               each raw stage into row t of an operand stage's W half in the
//               UMMA 128-byte swizzle (16-byte unit j of row r at
//               (j ^ r % 8) * 16) and arrives on the leader's barrier of that
//               stage
//   warps 2..5  the second 64 columns the same way while the unit's MMAs run,
//               then the epilogue (the F16 GEMM's: bias, residual TMA
//               reduce-add or K-split planes, SwiGLU, QKV + RoPE + paged KV)
// Barriers:
//   xfull[s]   leader only; 1 arrival (leader's expect_tx) + both CTAs' X bytes
//   bfull[s]   leader only; 8 converter-warp arrivals (4 per CTA)
//   x/bempty   each CTA; the leader's MMA commits to both CTAs
//   rfull[r]   each CTA; its producer's expect_tx + the raw boxes' bytes
//   rempty[r]  each CTA; 8 converter-warp arrivals (4 per half)
//   tfull/tempty as in the F16 pair kernel
// Every TMA load reads this GPU's own memory into the issuing CTA's own
// shared memory.  Every wait is bounded and a timeout sets a bit of a.err.
#include <atomic>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "gemm_epi.cuh"

namespace laya {

// Shared memory: three rings.  The raw ring holds the HBM weight stream in
// flight (a CTA streams its weight rows only as fast as it keeps boxes
// outstanding); the X ring runs ahead of the MMAs by its own depth, since X
// comes from L2 at about a microsecond per round trip; the converted W ring
// lets the converters work two stages ahead of the MMAs, so that the barrier
// hand-offs between them (commit -> converters -> leader) overlap the MMAs.
constexpr int Q8_XS = 3;               // X stages, 64 K columns each
constexpr int Q8_FS = 4;               // converted W stages, 64 K columns each
constexpr int Q8_RS = 4;               // raw stages, 128 K columns each
constexpr int Q8_THREADS = 352;
constexpr int Q8_PA = 128 * BK * 2;    // this CTA's 128 X rows of a stage
constexpr int Q8_PB = 128 * BK * 2;    // this CTA's 128 W rows of a stage, as F16
constexpr int Q8_RAW = 128 * 128;      // 128 rows x 128 int8 quants
constexpr int Q8_SCL = 4 * 128 * 2;    // [4 blocks][128 rows] F16 scales
constexpr int Q8_OFF_B = Q8_XS * Q8_PA;
constexpr int Q8_OFF_RAW = Q8_OFF_B + Q8_FS * Q8_PB;
constexpr int Q8_OFF_SCL = Q8_OFF_RAW + Q8_RS * Q8_RAW;
constexpr int Q8_OFF_STG = (Q8_OFF_SCL + Q8_RS * Q8_SCL + 1023) / 1024 * 1024;
constexpr int Q8_OFF_BAR = Q8_OFF_STG + 4 * 2 * 4096;
constexpr int Q8_SMEM = Q8_OFF_BAR + 256 + 1024;
static_assert(Q8_SMEM <= 227 * 1024, "Q8_0 pair GEMM shared memory");
static_assert((Q8_OFF_B | Q8_OFF_RAW | Q8_OFF_STG) % 1024 == 0, "swizzled stages must be 1024-byte aligned");
static_assert(Q8_FS % 2 == 0, "a raw stage fills two consecutive operand stages of one phase");
static_assert(2 * (Q8_XS + Q8_FS + Q8_RS + 4) * 8 + 4 <= 256, "Q8_0 pair GEMM barriers");

// Row layout of the W operand across its tensors (see Q8Weights).
struct Q8Seg {
  int start[3];
  int nseg;
  int interleave;
};

// Tensor index and its first row for the 128 W rows starting at operand row R0.
__device__ __forceinline__ void q8_rows(const Q8Seg& s, int R0, int& mi, int& lr) {
  if (s.interleave) {
    mi = (R0 >> 7) & 1;
    lr = (R0 >> 8) << 7;
    return;
  }
  mi = 0;
  lr = R0;
  for (int i = 1; i < s.nseg; i++)
    if (R0 >= s.start[i]) {
      mi = i;
      lr = R0 - s.start[i];
    }
}

// 16 int8 quants (one 16-byte unit) times the block scale d, as 16 F16.
// Each byte, biased by 128, becomes the low byte of 1024 + (q + 128) in
// F16; subtracting 1152 gives q exactly, and one F16 multiply by d rounds
// the exact product d * q once (the value of rounding the F32 product
// d * q, which is exact, to F16).
__device__ __forceinline__ void q8_decode16(uint4 v, __half2 d, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t e0 = __byte_perm(w[i], 0x64646464u, 0x4140);  // quants 4i, 4i+1
    const uint32_t e1 = __byte_perm(w[i], 0x64646464u, 0x4342);  // quants 4i+2, 4i+3
    __half2 h0 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&e0), bias), d);
    __half2 h1 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&e1), bias), d);
    o[2 * i] = *reinterpret_cast<uint32_t*>(&h0);
    o[2 * i + 1] = *reinterpret_cast<uint32_t*>(&h1);
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

// Advances a ring position and flips its phase bit on wrap-around.
template <int N>
__device__ __forceinline__ void ring_next(int& s, uint32_t& ph) {
  if (++s == N) {
    s = 0;
    ph ^= 1;
  }
}

// Decodes, for the raw stages of K blocks k0..k1-1 of one work unit, the
// 64-column half `half` of weight row t into operand stage fs + half (each
// raw stage fills operand stages fs and fs + 1, which share a phase), then
// arrives on the leader's barrier of that stage and releases the raw stage.
// Four warps per CTA take each half.  False after a timed-out wait (the
// lanes agree on the outcome of every wait, so a timeout never splits a warp).
__device__ __forceinline__ bool q8_convert_unit(int k0, int k1, int t, int half, int lane, const uint8_t* sRaw,
                                                const uint8_t* sScl, uint8_t* sB, uint64_t* rfull, uint64_t* rempty,
                                                uint64_t* bfull, uint64_t* bempty, int& fs, uint32_t& fph, int& rs,
                                                uint32_t& rph, long long budget, unsigned* err) {
  const int sw = t & 7;
  for (int kq = k0; kq < k1; kq++) {
    const int os = fs + half;
    if (!__all_sync(0xffffffffu, mbar_wait(&rfull[rs], rph, budget)) ||
        !__all_sync(0xffffffffu, mbar_poll_cluster(&bempty[os], fph ^ 1, budget))) {
      if (lane == 0) atomicOr(err, 32u);
      return false;
    }
    const uint8_t* raw = sRaw + rs * Q8_RAW + t * 128;
    const __half* scl = reinterpret_cast<const __half*>(sScl + rs * Q8_SCL);
    // four independent 16-quant units per thread: loads first, then the
    // decodes, so their latencies overlap
    uint4 v[4];
#pragma unroll
    for (int c = 0; c < 4; c++) v[c] = *reinterpret_cast<const uint4*>(raw + (((4 * half + c) ^ sw) << 4));
    const __half2 d0 = __half2half2(scl[(2 * half) * 128 + t]), d1 = __half2half2(scl[(2 * half + 1) * 128 + t]);
    uint8_t* dst = sB + os * Q8_PB + t * 128;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      uint4 lo, hi;
      q8_decode16(v[c], c < 2 ? d0 : d1, lo, hi);
      *reinterpret_cast<uint4*>(dst + (((2 * c) ^ sw) << 4)) = lo;
      *reinterpret_cast<uint4*>(dst + (((2 * c + 1) ^ sw) << 4)) = hi;
    }
    fence_async_smem();  // the tensor cores read what this thread wrote
    __syncwarp();
    if (lane == 0) {
      mbar_arrive_peer(cluster_addr(&bfull[os], 0));
      mbar_arrive(&rempty[rs]);
    }
    ring_next<Q8_FS>(fs, fph);
    ring_next<Q8_FS>(fs, fph);
    ring_next<Q8_RS>(rs, rph);
  }
  return true;
}

template <int EPI, int HD>
__global__ void __launch_bounds__(Q8_THREADS, 1)
    gemm_q8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ0,
                        const __grid_constant__ CUtensorMap tmQ1, const __grid_constant__ CUtensorMap tmQ2,
                        const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmR,
                        const GemmArgs a, const Q8Seg seg) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Q8_OFF_B;
  uint8_t* sRaw = smem + Q8_OFF_RAW;
  uint8_t* sScl = smem + Q8_OFF_SCL;
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + Q8_OFF_BAR);
  uint64_t* xempty = xfull + Q8_XS;
  uint64_t* bfull = xempty + Q8_XS;
  uint64_t* bempty = bfull + Q8_FS;
  uint64_t* rfull = bempty + Q8_FS;
  uint64_t* rempty = rfull + Q8_RS;
  uint64_t* tfull = rempty + Q8_RS;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Q8_XS; s++) {
      mbar_init(&xfull[s], 1);  // leader: its expect_tx of both CTAs' X boxes
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < Q8_FS; s++) {
      mbar_init(&bfull[s], 8);  // leader: 4 converter warps of each CTA
      mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < Q8_RS; s++) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 8);  // 4 converter warps per half
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmQ0);
    tma_prefetch_desc(&tmS);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles = a.m_tiles * a.n_tiles;
  const int kqn = a.K / 128;  // 128-column K blocks
  const int nsplit = (EPI == EPI_RESID && a.ksplit > 1) ? a.ksplit : 1;
  const int kqs = (kqn + nsplit - 1) / nsplit;
  const int total = tiles * nsplit;
  const long long budget = a.budget;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (warp == 0) {
    if (elect_one()) {
      // Weight stream: the quants never depend on the previous kernel, so
      // this thread starts at once (no griddepcontrol.wait) and keeps up to
      // Q8_RS raw boxes in flight ahead of the converters.
      int rs = 0;
      uint32_t rph = 0;
      int rissued[Q8_RS];
      for (int s = 0; s < Q8_RS; s++) rissued[s] = -1;
      bool ok = true;
      for (int unit = cluster; unit < total && ok; unit += nclusters) {
        const int tile = unit % tiles, sp = unit / tiles;
        int mt, nt, mi, lr;
        pair_tile(a, tile, mt, nt);
        const int R0 = nt * 256 + (int)rank * 128;
        q8_rows(seg, R0, mi, lr);
        const CUtensorMap* tq = mi == 0 ? &tmQ0 : mi == 1 ? &tmQ1 : &tmQ2;
        const int k1 = min(kqn, (sp + 1) * kqs);
        for (int kq = sp * kqs; kq < k1; kq++) {
          if (!mbar_wait(&rempty[rs], rph ^ 1, budget)) {
            atomicOr(a.err, 1u);
            ok = false;
            break;
          }
          rissued[rs] = (int)rph;
          mbar_expect_tx(&rfull[rs], Q8_RAW + Q8_SCL);
          tma_load_2d(sRaw + rs * Q8_RAW, tq, &rfull[rs], kq * 128, lr);
          tma_load_2d(sScl + rs * Q8_SCL, &tmS, &rfull[rs], R0, kq * 4);
          ring_next<Q8_RS>(rs, rph);
        }
      }
      // no raw box is still in flight when the CTA exits
      for (int s = 0; s < Q8_RS; s++)
        if (rissued[s] >= 0 && !mbar_wait(&rfull[s], (uint32_t)rissued[s], budget)) atomicOr(a.err, 16u);
    }
  } else if (warp == 10) {
    if (elect_one()) {
      // X stream (the previous kernel's output): one box per 64 K columns,
      // counted on the leader's barrier, up to Q8_XS stages ahead of the MMAs.
      pdl_wait();
      pdl_trigger();
      int xs = 0;
      uint32_t xph = 0;
      bool ok = true;
      for (int unit = cluster; unit < total && ok; unit += nclusters) {
        const int tile = unit % tiles, sp = unit / tiles;
        int mt, nt;
        pair_tile(a, tile, mt, nt);
        const int k1 = min(kqn, (sp + 1) * kqs);
        for (int kb = 2 * sp * kqs; kb < 2 * k1; kb++) {
          if (!mbar_wait(&xempty[xs], xph ^ 1, budget)) {
            atomicOr(a.err, 1u);
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&xfull[xs], 2 * Q8_PA);
          tma_load_2d_pair(sA + xs * Q8_PA, &tmA, cluster_addr(&xfull[xs], 0), kb * 64, mt * 256 + (int)rank * 128);
          ring_next<Q8_XS>(xs, xph);
        }
      }
      // Drain: every X stage's last fill is consumed before this CTA may exit
      // (no MMA still reads its shared memory, no commit arrives after exit).
      for (int i = 0; i < Q8_XS; i++) {
        if (!mbar_wait(&xempty[xs], xph ^ 1, budget)) atomicOr(a.err, 16u);
        ring_next<Q8_XS>(xs, xph);
      }
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      const uint32_t idesc = idesc_f16_f32(256, BN);
      int xs = 0, fs = 0, acc = 0;
      uint32_t xph = 0, fph = 0, acc_phase = 0;
      bool ok = true;
      for (int unit = cluster; unit < total && ok; unit += nclusters) {
        const int sp = unit / tiles, k0 = sp * kqs, k1 = min(kqn, k0 + kqs);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, budget)) {
          atomicOr(a.err, 2u);
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 2 * k0; kb < 2 * k1; kb++) {
          // X by TMA; W halves released by both CTAs' converters at cluster scope
          if (!mbar_wait(&xfull[xs], xph, budget) || !mbar_poll_cluster(&bfull[fs], fph, budget)) {
            atomicOr(a.err, 4u);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(smem_u32(sA + xs * Q8_PA));
          const uint64_t bd = sw128_desc(smem_u32(sB + fs * Q8_PB));
#pragma unroll
          for (int k = 0; k < BK / 16; k++)
            umma_f16_pair(tmem_d, ad + 2 * k, bd + 2 * k, idesc, (kb != 2 * k0 || k != 0) ? 1u : 0u);
          umma_commit_pair(&xempty[xs], 0x3);
          umma_commit_pair(&bempty[fs], 0x3);
          ring_next<Q8_XS>(xs, xph);
          ring_next<Q8_FS>(fs, fph);
        }
        umma_commit_pair(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else if (warp < 6) {
    // Epilogue warps: while a unit's MMAs run they decode the second
    // 64-column half of each raw stage, then read the unit's accumulator.
    const int quarter = warp % 4;
    uint8_t* stg = smem + Q8_OFF_STG + quarter * 2 * 4096;
    int acc = 0;
    uint32_t acc_phase = 0;
    int fs = 0, rs = 0;
    uint32_t fph = 0, rph = 0;
    bool cok = true, waited = false;
    for (int unit = cluster; unit < total; unit += nclusters) {
      const int tile = unit % tiles, sp = unit / tiles;
      int mt, nt;
      pair_tile(a, tile, mt, nt);
      if (cok)
        cok = q8_convert_unit(sp * kqs, min(kqn, (sp + 1) * kqs), (warp - 2) * 32 + lane, 1, lane, sRaw, sScl, sB,
                              rfull, rempty, bfull, bempty, fs, fph, rs, rph, budget, a.err);
      if (!waited) {
        pdl_wait();  // outputs and residual rows may be in use by the previous kernel until it ends
        waited = true;
      }
      const int row = mt * 256 + (int)rank * 128 + quarter * 32 + lane;
      if (!mbar_wait(&tfull[acc], acc_phase, budget)) {
        atomicOr(a.err, 8u);
        break;
      }
      tc_fence_after();
      if constexpr (EPI == EPI_RESID)
        resid_tma_tile(a, &tmR, tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN, row - lane, nt * BN, stg,
                       lane, nsplit > 1 ? unit / tiles : -1);
      else
        epilogue_tile<EPI, HD>(a, tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN, row, nt,
                               (EPI == EPI_QKV || EPI == EPI_SWIGLU) ? stg : nullptr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(cluster_addr(&tempty[acc], 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  } else {
    // Converters (warps 6..9): the first 64-column half of each raw stage,
    // thread t owning weight row t of this CTA's half of the tile.
    const int t = threadIdx.x - 192;
    int fs = 0, rs = 0;
    uint32_t fph = 0, rph = 0;
    for (int unit = cluster; unit < total; unit += nclusters) {
      const int sp = unit / tiles;
      if (!q8_convert_unit(sp * kqs, min(kqn, (sp + 1) * kqs), t, 0, lane, sRaw, sScl, sB, rfull, rempty, bfull,
                           bempty, fs, fph, rs, rph, budget, a.err))
        break;
    }
    if (t == 0)  // every converted stage consumed before exit
      for (int i = 0; i < Q8_FS; i++) {
        if (!mbar_wait(&bempty[fs], fph ^ 1, budget)) atomicOr(a.err, 16u);
        ring_next<Q8_FS>(fs, fph);
      }
  }
  if constexpr (EPI == EPI_RESID)
    if (warp >= 2 && warp < 6 && lane == 0) bulk_wait<0>();  // residual reductions complete before exit
  tc_fence_before();
  __syncwarp();
  __syncthreads();
  cluster_sync();  // both CTAs done with TMEM and each other's barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- scales

__global__ void q8_scales_t_kernel(QTensor t, half* __restrict__ dst, int ldst, int grp, int gstride, int goff) {
  const int blocks = t.cols / 32;
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)t.rows * blocks) return;
  const int b = (int)(i / t.rows), n = (int)(i % t.rows);  // consecutive threads: consecutive rows
  const size_t orow = (size_t)(n / grp) * gstride + goff + (n % grp);
  reinterpret_cast<uint16_t*>(dst)[(size_t)b * ldst + orow] = t.s[(size_t)n * blocks + b];
}

cudaError_t q8_scales_t(const QTensor& t, half* dst, int ldst, int grp, int gstride, int goff, cudaStream_t st) {
  if (t.kind != K_Q8_0 || t.cols % 32) return cudaErrorInvalidValue;
  const size_t n = (size_t)t.rows * (t.cols / 32);
  if (!n) return cudaSuccess;
  q8_scales_t_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(t, dst, ldst, grp, gstride, goff);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- host side

int gemm_q8_ksplit(int M, int N, int K, int num_sms) {
  if (num_sms < 2 || M < 1 || K % 128) return 1;
  const int tiles = ((M + 255) / 256) * ((N + BN - 1) / BN);
  const int pairs = num_sms / 2, kqn = K / 128;
  if (2 * tiles >= pairs) return 1;
  // at least 2 K blocks (256 columns of K) per split, at most 16 splits
  int s = std::min(std::min(pairs / tiles, kqn / 2), 16);
  if (s < 2) return 1;
  const int per = (kqn + s - 1) / s;
  return (kqn + per - 1) / per;  // every split gets at least one K block
}

template <int EPI, int HD>
static cudaError_t launch_q8(const CUtensorMap (&maps)[6], const GemmArgs& a, const Q8Seg& seg, int num_sms,
                             cudaStream_t st, bool pdl) {
  // per device: attribute set once, co-resident CTA pairs queried once
  static std::atomic<int> clusters_fit[64];
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemm_q8_pair_kernel<EPI, HD>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(Q8_THREADS);
  cfg.dynamicSmemBytes = Q8_SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (clusters_fit[dev & 63] == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Q8_SMEM);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(2 * (num_sms / 2));
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (n <= 0) return cudaErrorInvalidConfiguration;
    clusters_fit[dev & 63] = n;
  }
  const int total = a.m_tiles * a.n_tiles * (a.ksplit > 1 ? a.ksplit : 1);
  int clusters = clusters_fit[dev & 63];
  if (clusters > num_sms / 2) clusters = num_sms / 2;
  if (clusters > total) clusters = total;
  cfg.gridDim = dim3(2 * clusters);
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], a, seg);
}

cudaError_t gemm_q8_launch(int epi, const half* A, int lda, const Q8Weights& w, GemmArgs a, int num_sms,
                           cudaStream_t st, bool pdl) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return cudaSuccess;
  if (num_sms < 2 || a.K % 128 || lda % 8 || a.N % 8 || (reinterpret_cast<uintptr_t>(A) & 15) || !w.st ||
      (reinterpret_cast<uintptr_t>(w.st) & 15) || w.nseg < 1 || w.nseg > 3)
    return cudaErrorInvalidValue;
  // operand rows: the tensors stacked, or two interleaved per 128 rows
  Q8Seg seg{};
  seg.nseg = w.nseg;
  seg.interleave = w.interleave;
  if (w.interleave) {
    if (w.nseg != 2 || w.rows[0] != w.rows[1] || w.rows[0] % 128 || 2 * w.rows[0] != a.N)
      return cudaErrorInvalidValue;
  } else {
    int n = 0;
    for (int i = 0; i < w.nseg; i++) {
      if (w.rows[i] < 1 || (i + 1 < w.nseg && w.rows[i] % 128)) return cudaErrorInvalidValue;
      seg.start[i] = n;
      n += w.rows[i];
    }
    if (n != a.N) return cudaErrorInvalidValue;
  }
  CUtensorMap maps[6];  // X, int8 of tensors 0..2, scales, residual / K-split planes
  {
    const uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)a.M}, strides[1] = {(uint64_t)lda * 2};
    const uint32_t box[2] = {64, 128};
    if (!encode_tiled(&maps[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  for (int i = 0; i < 3; i++) {
    const int j = i < w.nseg ? i : 0;
    if (!w.q[j] || (reinterpret_cast<uintptr_t>(w.q[j]) & 15)) return cudaErrorInvalidValue;
    const uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)w.rows[j]}, strides[1] = {(uint64_t)a.K};
    const uint32_t box[2] = {128, 128};
    if (!encode_tiled(&maps[1 + i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w.q[j], dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {(uint64_t)a.N, (uint64_t)(a.K / 32)}, strides[1] = {(uint64_t)a.N * 2};
    const uint32_t box[2] = {128, 4};
    if (!encode_tiled(&maps[4], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.st, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  }
  maps[5] = maps[0];
  if (epi != EPI_RESID || a.ksplit < 2) a.ksplit = 1;
  if (epi == EPI_RESID && a.ksplit > 1) {
    // partial sums F32 [ksplit][M][ldo] in 32 x 32 x 1 boxes
    const int kqn = a.K / 128;
    if (!a.part || (a.ldo % 4) || (reinterpret_cast<uintptr_t>(a.part) & 15) || a.ksplit > kqn ||
        (a.ksplit - 1) * ((kqn + a.ksplit - 1) / a.ksplit) >= kqn)
      return cudaErrorInvalidValue;
    const uint64_t dims[3] = {(uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.ksplit};
    const uint64_t strides[2] = {(uint64_t)a.ldo * 4, (uint64_t)a.M * a.ldo * 4};
    const uint32_t box[3] = {32, 32, 1};
    if (!encode_tiled(&maps[5], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a.part, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  } else if (epi == EPI_RESID) {
    if ((a.ldo % 4) || (reinterpret_cast<uintptr_t>(a.resid) & 15)) return cudaErrorInvalidValue;
    const uint64_t dims[2] = {(uint64_t)a.N, (uint64_t)a.M}, strides[1] = {(uint64_t)a.ldo * 4};
    const uint32_t box[2] = {32, 32};
    if (!encode_tiled(&maps[5], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.resid, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  a.m_tiles = (a.M + 255) / 256;
  a.n_tiles = (a.N + BN - 1) / BN;
  a.group = gemm_pair_group(a.n_tiles);
  switch (epi) {
    case EPI_F32: return launch_q8<EPI_F32, 64>(maps, a, seg, num_sms, st, pdl);
    case EPI_F16: return launch_q8<EPI_F16, 64>(maps, a, seg, num_sms, st, pdl);
    case EPI_RESID: return launch_q8<EPI_RESID, 64>(maps, a, seg, num_sms, st, pdl);
    case EPI_SWIGLU: return launch_q8<EPI_SWIGLU, 64>(maps, a, seg, num_sms, st, pdl);
    case EPI_QKV:
      if (a.hd == 64) return launch_q8<EPI_QKV, 64>(maps, a, seg, num_sms, st, pdl);
      if (a.hd == 128) return launch_q8<EPI_QKV, 128>(maps, a, seg, num_sms, st, pdl);
      return cudaErrorInvalidValue;
  }
  return cudaErrorInvalidValue;
}

}  // namespace laya
