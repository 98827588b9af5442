// Prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   Y[M x N] = X[M x K] . W[N x K]^T   (F16 operands, F32 accumulation)
//
// This replaces the reference's F32 AVX2 kernel Matrix::apply
// (src/tensor.rs:10-102): same contract (W row-major [rows=N][cols=K],
// one output row per token, optional bias), computed as a persistent,
// warp-specialised kernel in two shapes:
//
// gemm_pair_kernel (any M): clusters of two CTAs on two SMs share one
//   256x256 output tile through tcgen05.mma.cta_group::2.  Each CTA stages
//   its own 128 rows of A and 128 rows of B per 64-wide K block (32 KB per
//   stage, 6 stages), so an SM moves a third fewer operand bytes from L2 per
//   FLOP than with single-CTA 128x256 tiles.
// gemm_tc_kernel (a GPU without a second SM): one CTA per 128x256 tile, 4
//   stages of 48 KB.
//
// Roles in both: warp 0 is the TMA producer (128-byte swizzle), warp 1
// allocates 512 TMEM columns (two 256-column accumulators, so the epilogue of
// tile i overlaps the MMAs of tile i+1) and one elected thread issues the
// MMAs, warps 2..5 are the epilogue — tcgen05.ld from TMEM, fused bias /
// residual add (tensor::add, src/tensor.rs:123-128) / SwiGLU
// (src/models/openthai/model.rs:225-230) / QKV + RoPE + KV-cache write, then
// stores to HBM.  Every TMA load reads this GPU's own memory into the issuing
// CTA's own shared memory.
#include <atomic>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>

#include "gemm_epi.cuh"

namespace laya {

constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int GEMM_THREADS = 192;
constexpr int GEMM_SMEM = STAGES * (A_BYTES + B_BYTES) + 1024 + 256;

template <int EPI, int HD>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = a.m_tiles * a.n_tiles;
  const int kblocks = (a.K + BK - 1) / BK;
  const long long budget = a.budget;

  if (warp == 0) {
    if (elect_one()) {
      // The weights never depend on the previous kernel: the first tile's
      // are pulled into L2 before waiting for it (programmatic launch).
      if ((int)blockIdx.x < total)
        for (int kb = 0; kb < min(kblocks, 2 * STAGES); kb++)
          tma_prefetch_2d(&tmB, kb * BK, (int)(blockIdx.x % a.n_tiles) * BN);
      pdl_wait();
      pdl_trigger();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int issued[STAGES];
      for (int s = 0; s < STAGES; s++) issued[s] = -1;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const int mt = tile / a.n_tiles, nt = tile % a.n_tiles;
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&empty[stage], phase ^ 1, budget)) {
            atomicOr(a.err, 1u);
            ok = false;
            break;
          }
          issued[stage] = (int)phase;
          mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, mt * BM);
          tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * BK, nt * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // On a timeout, leave no copy in flight: wait (bounded) for every
      // stage this thread filled to land before the CTA exits.
      if (!ok)
        for (int s = 0; s < STAGES; s++)
          if (issued[s] >= 0) mbar_wait(&full[s], (uint32_t)issued[s], budget);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = idesc_f16_f32(BM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, budget)) {
          atomicOr(a.err, 2u);
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&full[stage], phase, budget)) {
            atomicOr(a.err, 4u);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(smem_u32(sA + stage * A_BYTES));
          const uint64_t bd = sw128_desc(smem_u32(sB + stage * B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; k++)
            umma_f16(tmem_d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // Epilogue: warp w may read TMEM lanes 32*(w%4) .. 32*(w%4)+31.
    pdl_wait();  // outputs and residual rows may be in use by the previous kernel until it ends
    const int quarter = warp % 4;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      const int mt = tile / a.n_tiles, nt = tile % a.n_tiles;
      const int row = mt * BM + quarter * 32 + lane;
      resid_prefetch<EPI>(a, row, nt);
      if (!mbar_wait(&tfull[acc], acc_phase, budget)) {
        atomicOr(a.err, 8u);
        break;
      }
      tc_fence_after();
      epilogue_tile<EPI, HD>(a, tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN, row, nt);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- CTA pair
constexpr int PAIR_STAGES = 6;
constexpr int PA_BYTES = 128 * BK * 2;  // this CTA's 128 rows of the 256-row A tile
constexpr int PB_BYTES = 128 * BK * 2;  // this CTA's 128 rows of the 256-row B tile
constexpr int PAIR_SMEM = PAIR_STAGES * (PA_BYTES + PB_BYTES) + 1024 + 256;
// EPI_RESID stages each epilogue warp's 32x32 F32 chunks (two 4 KB buffers
// per warp) for TMA reduce-add into the residual stream.
constexpr int PAIR_STG = (PAIR_STAGES * (PA_BYTES + PB_BYTES) + 256 + 1023) / 1024 * 1024;
constexpr int PAIR_SMEM_RESID = PAIR_STG + 4 * 2 * 4096 + 1024;
static_assert(PAIR_SMEM <= 227 * 1024 && PAIR_SMEM_RESID <= 227 * 1024, "pair GEMM shared memory");

// Launched in clusters of two CTAs.  Tile t of the cluster's sequence covers
// output rows mt*256 .. +255 (rank r owns mt*256 + 128r ..) and columns
// nt*256 .. +255.  Barriers:
//   full[s]   leader only; one arrival (leader's expect_tx of both CTAs'
//             64 KB) plus the transaction bytes of both CTAs' loads
//   empty[s]  each CTA; arrived by the leader's MMA commit to both CTAs
//   tfull[b]  each CTA; arrived by the leader's commit to both CTAs
//   tempty[b] leader only; 8 arrivals, one per epilogue warp of either CTA

template <int EPI, int HD>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmR, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + PAIR_STAGES * PA_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + PAIR_STAGES * PB_BYTES);
  uint64_t* empty = full + PAIR_STAGES;
  uint64_t* tfull = empty + PAIR_STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIR_STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barrier inits and the allocation visible to both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles = a.m_tiles * a.n_tiles;
  const int kblocks = (a.K + BK - 1) / BK;
  // work unit u = tile u % tiles, K split u / tiles (one split unless EPI_RESID splits K)
  const int nsplit = (EPI == EPI_RESID && a.ksplit > 1) ? a.ksplit : 1;
  const int kbs = (kblocks + nsplit - 1) / nsplit;
  const int total = tiles * nsplit;
  const long long budget = a.budget;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (warp == 0) {
    if (elect_one()) {
      // The weights never depend on the previous kernel: this CTA's rows of
      // the first unit's B tile are pulled into L2 before waiting for it.
      if (cluster < total) {
        const int tile = cluster % tiles, sp = cluster / tiles;
        int mt0, nt0;
        pair_tile(a, tile, mt0, nt0);
        const int kb0 = sp * kbs, kb1 = min(kblocks, kb0 + min(kbs, 2 * PAIR_STAGES));
        for (int kb = kb0; kb < kb1; kb++) tma_prefetch_2d(&tmB, kb * BK, nt0 * 256 + (int)rank * 128);
      }
      pdl_wait();
      pdl_trigger();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = cluster; unit < total && ok; unit += nclusters) {
        const int tile = unit % tiles, sp = unit / tiles;
        int mt, nt;
        pair_tile(a, tile, mt, nt);
        const int kb1 = min(kblocks, (sp + 1) * kbs);
        for (int kb = sp * kbs; kb < kb1; kb++) {
          if (!mbar_wait(&empty[stage], phase ^ 1, budget)) {
            atomicOr(a.err, 1u);
            ok = false;
            break;
          }
          const uint32_t fbar = cluster_addr(&full[stage], 0);
          if (leader) mbar_expect_tx(&full[stage], 2 * (PA_BYTES + PB_BYTES));
          tma_load_2d_pair(sA + stage * PA_BYTES, &tmA, fbar, kb * BK, mt * 256 + rank * 128);
          tma_load_2d_pair(sB + stage * PB_BYTES, &tmB, fbar, kb * BK, nt * 256 + rank * 128);
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every stage's last fill is consumed (its empty barrier
      // completes) before this CTA may exit, so no MMA still reads this
      // CTA's shared memory and no commit arrives here after exit.
      for (int i = 0; i < PAIR_STAGES; i++) {
        if (!mbar_wait(&empty[stage], phase ^ 1, budget)) atomicOr(a.err, 16u);
        if (++stage == PAIR_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      const uint32_t idesc = idesc_f16_f32(256, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int unit = cluster; unit < total && ok; unit += nclusters) {
        const int sp = unit / tiles, kb0 = sp * kbs, kb1 = min(kblocks, kb0 + kbs);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, budget)) {
          atomicOr(a.err, 2u);
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; kb++) {
          if (!mbar_wait(&full[stage], phase, budget)) {
            atomicOr(a.err, 4u);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(smem_u32(sA + stage * PA_BYTES));
          const uint64_t bd = sw128_desc(smem_u32(sB + stage * PB_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; k++)
            umma_f16_pair(tmem_d, ad + 2 * k, bd + 2 * k, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit_pair(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    pdl_wait();  // outputs and residual rows may be in use by the previous kernel until it ends
    const int quarter = warp % 4;
    uint8_t* stg = smem + PAIR_STG + quarter * 2 * 4096;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int unit = cluster; unit < total; unit += nclusters) {
      const int tile = unit % tiles;
      int mt, nt;
      pair_tile(a, tile, mt, nt);
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
  }
  if constexpr (EPI == EPI_RESID)
    if (warp >= 2 && lane == 0) bulk_wait<0>();  // residual reductions complete before exit
  tc_fence_before();
  __syncwarp();
  __syncthreads();
  cluster_sync();  // both CTAs done with TMEM and each other's barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

bool encode_tiled(CUtensorMap* m, int dtype, int rank, const void* base, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, int swizzle) {
  auto fn = encode_fn();
  if (!fn || rank < 1 || rank > 5) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; i++) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; i++) st[i] = strides[i];
  return fn(m, (CUtensorMapDataType)dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, e,
            CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Row-major F16 matrix [rows][cols] as a 2-D TMA map with a box of
// box_rows x 64 columns and 128-byte swizzle.
static bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI, int HD>
static cudaError_t launch_epi(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid,
                              cudaStream_t st, bool pdl) {
  static std::atomic<bool> configured[64];  // per device and instantiation; any host thread may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemm_tc_kernel<EPI, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = GEMM_SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<EPI, HD>, ta, tb, a);
}

template <int EPI, int HD>
static cudaError_t launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tr, const GemmArgs& a,
                               int num_sms, cudaStream_t st, bool pdl) {
  // the residual, QKV and SwiGLU epilogues stage through the per-warp buffers at PAIR_STG
  constexpr int SMEM = (EPI == EPI_RESID || EPI == EPI_QKV || EPI == EPI_SWIGLU) ? PAIR_SMEM_RESID : PAIR_SMEM;
  // Per device: the attribute is set once and the number of CTA pairs that
  // fit at once is queried once, so the persistent grid never exceeds what is
  // co-resident (a pair left for a second wave would double the time).
  static std::atomic<int> clusters_fit[64];
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemm_pair_kernel<EPI, HD>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (clusters_fit[dev & 63] == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
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
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, tr, a);
}

// Row bands per group of the pair kernel's tile walk (pair_tile).  With
// many column tiles (the gate/up GEMM: 64) a group of 8 bands keeps the
// pairs running at once on ~9 weight tiles and 8 row bands, which cut its
// DRAM reads by a fifth at 16 requests (374 -> 298 MB); with few column
// tiles (8 for the down GEMM) the walk by whole row bands already shares
// every weight tile, and grouping raised its reads (325 -> 405 MB).
// LAYA_GEMM_GROUP overrides.
int gemm_pair_group(int n_tiles) {
  static const int forced = [] {
    const char* e = std::getenv("LAYA_GEMM_GROUP");
    return e ? std::atoi(e) : 0;
  }();
  if (forced >= 1) return forced;
  return n_tiles >= 32 ? 8 : 1;
}

int gemm_ksplit(int M, int N, int K, int num_sms) {
  if (M < 1 || num_sms < 2) return 1;
  const int tiles = ((M + 255) / 256) * ((N + BN - 1) / BN);
  const int pairs = num_sms / 2, kblocks = (K + BK - 1) / BK;
  if (2 * tiles >= pairs) return 1;
  // at least 4 K blocks (256 columns of K) per split, at most 16 splits
  int s = std::min(std::min(pairs / tiles, kblocks / 4), 16);
  if (s < 2) return 1;
  const int per = (kblocks + s - 1) / s;
  return (kblocks + per - 1) / per;  // every split gets at least one K block
}

cudaError_t gemm_launch(int epi, const half* A, int lda, const half* B, int ldb, GemmArgs a, int num_sms,
                        cudaStream_t st, bool pdl) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return cudaSuccess;
  if ((lda % 8) || (ldb % 8) || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
    return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  // CTA pairs for every M (a pass of <= 128 rows leaves the second CTA's
  // rows empty, but its weight tiles are split over twice the SMs and the
  // residual GEMMs can split K); one CTA per tile only without a second SM
  if (num_sms >= 2) {
    if (!make_map(&ta, A, a.M, a.K, lda, 128) || !make_map(&tb, B, a.N, a.K, ldb, 128))
      return cudaErrorInvalidValue;
    CUtensorMap tr = ta;
    if (epi != EPI_RESID || a.ksplit < 2) a.ksplit = 1;
    if (epi == EPI_RESID && a.ksplit > 1) {
      // partial sums F32 [ksplit][M][ldo] in 32 x 32 x 1 boxes: rows past M
      // of a plane are clipped, never written into the next plane
      const int kblocks = (a.K + BK - 1) / BK;
      if (!a.part || (a.ldo % 4) || (reinterpret_cast<uintptr_t>(a.part) & 15) || a.ksplit > kblocks ||
          (a.ksplit - 1) * ((kblocks + a.ksplit - 1) / a.ksplit) >= kblocks)
        return cudaErrorInvalidValue;
      const uint64_t dims[3] = {(uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.ksplit};
      const uint64_t strides[2] = {(uint64_t)a.ldo * 4, (uint64_t)a.M * a.ldo * 4};
      const uint32_t box[3] = {32, 32, 1};
      if (!encode_tiled(&tr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a.part, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    } else if (epi == EPI_RESID) {
      // residual F32 [M][ldo] in 32 x 32 boxes, 128-byte swizzle
      if ((a.ldo % 4) || (reinterpret_cast<uintptr_t>(a.resid) & 15)) return cudaErrorInvalidValue;
      const uint64_t dims[2] = {(uint64_t)a.N, (uint64_t)a.M}, strides[1] = {(uint64_t)a.ldo * 4};
      const uint32_t box[2] = {32, 32};
      if (!encode_tiled(&tr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.resid, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    }
    a.m_tiles = (a.M + 255) / 256;
    a.n_tiles = (a.N + BN - 1) / BN;
    a.group = gemm_pair_group(a.n_tiles);
    switch (epi) {
      case EPI_F32: return launch_pair<EPI_F32, 64>(ta, tb, tr, a, num_sms, st, pdl);
      case EPI_F16: return launch_pair<EPI_F16, 64>(ta, tb, tr, a, num_sms, st, pdl);
      case EPI_RESID: return launch_pair<EPI_RESID, 64>(ta, tb, tr, a, num_sms, st, pdl);
      case EPI_SWIGLU: return launch_pair<EPI_SWIGLU, 64>(ta, tb, tr, a, num_sms, st, pdl);
      case EPI_QKV:
        if (a.hd == 64) return launch_pair<EPI_QKV, 64>(ta, tb, tr, a, num_sms, st, pdl);
        if (a.hd == 128) return launch_pair<EPI_QKV, 128>(ta, tb, tr, a, num_sms, st, pdl);
        return cudaErrorInvalidValue;
    }
    return cudaErrorInvalidValue;
  }
  if (epi == EPI_RESID && a.ksplit > 1) return cudaErrorInvalidValue;  // K splits need CTA pairs
  if (!make_map(&ta, A, a.M, a.K, lda, BM) || !make_map(&tb, B, a.N, a.K, ldb, BN)) return cudaErrorInvalidValue;
  a.m_tiles = (a.M + BM - 1) / BM;
  a.n_tiles = (a.N + BN - 1) / BN;
  const int total = a.m_tiles * a.n_tiles;
  const int grid = total < num_sms ? total : num_sms;
  switch (epi) {
    case EPI_F32: return launch_epi<EPI_F32, 64>(ta, tb, a, grid, st, pdl);
    case EPI_F16: return launch_epi<EPI_F16, 64>(ta, tb, a, grid, st, pdl);
    case EPI_RESID: return launch_epi<EPI_RESID, 64>(ta, tb, a, grid, st, pdl);
    case EPI_SWIGLU: return launch_epi<EPI_SWIGLU, 64>(ta, tb, a, grid, st, pdl);
    case EPI_QKV:
      if (a.hd == 64) return launch_epi<EPI_QKV, 64>(ta, tb, a, grid, st, pdl);
      if (a.hd == 128) return launch_epi<EPI_QKV, 128>(ta, tb, a, grid, st, pdl);
      return cudaErrorInvalidValue;
  }
  return cudaErrorInvalidValue;
}

}  // namespace laya
