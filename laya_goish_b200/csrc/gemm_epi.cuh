// Device-side pieces shared by the tcgen05 GEMM kernels (gemm.cu: F16
// operands; gemm_q8.cu: Q8_0 weights decoded in shared memory): the tile
// constants, the fused epilogues that read an accumulator out of TMEM, the
// residual TMA reduction and the CTA-pair tile walk.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemm.h"
#include "ptx.cuh"

namespace laya {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int TMEM_COLS = 512;

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

__device__ __forceinline__ void store_f16x32(half* dst, const float* v, int n) {
  if (n == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint4 u;
      half2 h0 = __floats2half2_rn(v[8 * i], v[8 * i + 1]);
      half2 h1 = __floats2half2_rn(v[8 * i + 2], v[8 * i + 3]);
      half2 h2 = __floats2half2_rn(v[8 * i + 4], v[8 * i + 5]);
      half2 h3 = __floats2half2_rn(v[8 * i + 6], v[8 * i + 7]);
      u.x = *reinterpret_cast<uint32_t*>(&h0);
      u.y = *reinterpret_cast<uint32_t*>(&h1);
      u.z = *reinterpret_cast<uint32_t*>(&h2);
      u.w = *reinterpret_cast<uint32_t*>(&h3);
      reinterpret_cast<uint4*>(dst)[i] = u;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; i++)
      if (i < n) dst[i] = __float2half_rn(v[i]);
  }
}

__device__ __forceinline__ void store_f32x32(float* dst, const float* v, int n) {
  if (n == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
    for (int i = 0; i < 8; i++)
      reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; i++)
      if (i < n) dst[i] = v[i];
  }
}

// Epilogue of one accumulator: this thread owns output row `row` (TMEM lane
// row % 128 of the warp's quarter) and the BN columns of tile column nt.
// Start pulling this thread's residual row segment of tile column nt into L2
// (one bulk prefetch of up to 1 KB), a full tile of MMAs before it is needed.
template <int EPI>
__device__ __forceinline__ void resid_prefetch(const GemmArgs& a, int row, int nt) {
  if constexpr (EPI == EPI_RESID) {
    const int col0 = nt * BN;
    const int n = min(BN, a.N - col0);
    const float* p = a.resid + (size_t)row * a.ldo + col0;
    if (row < a.M && n > 0 && (n & 3) == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0)
      l2_prefetch_bulk(p, (uint32_t)n * 4);
  }
}

// stg (pair kernel, may be null): the warp's 8 KB staging buffer; with it the
// QKV epilogue writes each head's 32 rows through shared memory so that every
// store instruction covers whole 128-byte lines (a lane per row would touch 32
// lines with 16 bytes each).
template <int EPI, int HD>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& a, uint32_t tbase, int row, int nt,
                                              uint8_t* stg = nullptr) {
  const bool live = row < a.M;
  const int col0 = nt * BN;
  if constexpr (EPI == EPI_RESID) {
    // x[row][col0 ..] += acc.  The residual row was prefetched into L2 when
    // the tile started (resid_prefetch); here the eight 16-byte loads of the
    // next 32-column chunk are issued before the current chunk is added, so
    // one L2 round trip overlaps the TMEM read and the stores of the last.
    float* xrow = a.resid + (size_t)row * a.ldo;
    const bool vec = ((a.ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.resid) & 15) == 0);
    float4 cur[8];
    if (live && vec && col0 + 32 <= a.N) {
#pragma unroll
      for (int i = 0; i < 8; i++) cur[i] = reinterpret_cast<const float4*>(xrow + col0)[i];
    }
    for (int c = 0; c < BN / 32; c++) {
      const int cb = col0 + c * 32;
      if (cb >= a.N) break;
      const int n = min(32, a.N - cb);
      float4 nxt[8];
      const bool pre = live && vec && c + 1 < BN / 32 && cb + 64 <= a.N;
      if (pre) {
#pragma unroll
        for (int i = 0; i < 8; i++) nxt[i] = reinterpret_cast<const float4*>(xrow + cb + 32)[i];
      }
      uint32_t r[32];
      __syncwarp();
      tmem_ld32(tbase + c * 32, r);
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
      if (a.bias)
#pragma unroll
        for (int i = 0; i < 32; i++)
          if (i < n) v[i] += a.bias[cb + i];
      if (live) {
        if (vec && n == 32) {
#pragma unroll
          for (int i = 0; i < 8; i++) {
            float4 o = cur[i];
            o.x += v[4 * i];
            o.y += v[4 * i + 1];
            o.z += v[4 * i + 2];
            o.w += v[4 * i + 3];
            reinterpret_cast<float4*>(xrow + cb)[i] = o;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++)
            if (i < n) xrow[cb + i] += v[i];
        }
      }
      if (pre) {
#pragma unroll
        for (int i = 0; i < 8; i++) cur[i] = nxt[i];
      }
    }
  } else if constexpr (EPI == EPI_F32 || EPI == EPI_F16) {
    for (int c = 0; c < BN / 32; c++) {
      const int cb = col0 + c * 32;
      if (cb >= a.N) break;
      uint32_t r[32];
      __syncwarp();
      tmem_ld32(tbase + c * 32, r);
      tmem_ld_wait();
      const int n = min(32, a.N - cb);
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
      if (a.bias)
#pragma unroll
        for (int i = 0; i < 32; i++)
          if (i < n) v[i] += a.bias[cb + i];
      if (live) {
        if constexpr (EPI == EPI_F32) {
          store_f32x32(reinterpret_cast<float*>(a.out) + (size_t)row * a.ldo + cb, v, n);
        } else {
          store_f16x32(reinterpret_cast<half*>(a.out) + (size_t)row * a.ldo + cb, v, n);
        }
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // B rows of tile nt: [0,128) gate rows, [128,256) up rows of FFN
    // columns nt*128 .. nt*128+127 (interleaved at load time).
    // With a staging buffer and a whole tile (128 columns = 256 bytes per
    // row), the rows go through shared memory (16-byte unit j of lane l at
    // l * 256 + (j ^ (l % 8)) * 16) and each store instruction writes two
    // rows' 256 contiguous bytes.
    const int lane = threadIdx.x & 31;
    const bool coop = stg != nullptr && nt * 128 + 128 <= a.N / 2 && (a.ldo % 8) == 0;
    for (int c = 0; c < 4; c++) {
      const int fc = nt * 128 + c * 32;
      if (fc >= a.N / 2) break;
      uint32_t rg[32], ru[32];
      __syncwarp();
      tmem_ld32(tbase + c * 32, rg);
      tmem_ld32(tbase + 128 + c * 32, ru);
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; i++) v[i] = silu_f(__uint_as_float(rg[i])) * __uint_as_float(ru[i]);
      if (coop) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const int j = 4 * c + q;
          half2 h0 = __floats2half2_rn(v[8 * q], v[8 * q + 1]), h1 = __floats2half2_rn(v[8 * q + 2], v[8 * q + 3]);
          half2 h2 = __floats2half2_rn(v[8 * q + 4], v[8 * q + 5]), h3 = __floats2half2_rn(v[8 * q + 6], v[8 * q + 7]);
          uint4 u;
          u.x = *reinterpret_cast<uint32_t*>(&h0);
          u.y = *reinterpret_cast<uint32_t*>(&h1);
          u.z = *reinterpret_cast<uint32_t*>(&h2);
          u.w = *reinterpret_cast<uint32_t*>(&h3);
          *reinterpret_cast<uint4*>(stg + lane * 256 + ((j ^ (lane & 7)) << 4)) = u;
        }
      } else if (live) {
        store_f16x32(reinterpret_cast<half*>(a.out) + (size_t)row * a.ldo + fc, v, min(32, a.N / 2 - fc));
      }
    }
    if (coop) {
      __syncwarp();
      const unsigned long long dmine =
          live ? reinterpret_cast<unsigned long long>(reinterpret_cast<half*>(a.out) + (size_t)row * a.ldo + nt * 128)
               : 0ull;
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int ch = i * 32 + lane, r = ch / 16, j = ch % 16;
        const unsigned long long dr = __shfl_sync(0xffffffffu, dmine, r);
        if (dr)
          *reinterpret_cast<uint4*>(dr + (unsigned long long)j * 16) =
              *reinterpret_cast<const uint4*>(stg + r * 256 + ((j ^ (r & 7)) << 4));
      }
      __syncwarp();
    }
  } else if constexpr (EPI == EPI_QKV) {
    // Columns: [0,qd) q heads, [qd,qd+kd) k heads, [qd+kd,qd+2kd) v heads.
    // One head (hd columns) at a time: bias, rotate-half RoPE for q/k
    // (src/tensor.rs:158-171), then q -> Q rows, k/v -> paged KV cache.
    constexpr int hd = HD;
    const int lane = threadIdx.x & 31;
    int pos = 0, slot = 0;
    if (live) {
      pos = a.pos[row];
      slot = a.slot[row];
    }
    for (int hc = 0; hc < BN; hc += hd) {
      const int cb = col0 + hc;
      if (cb >= a.N) break;  // uniform across the warp
      float v[hd];
#pragma unroll
      for (int c = 0; c < hd / 32; c++) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld32(tbase + hc + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i++) v[c * 32 + i] = __uint_as_float(r[i]);
      }
      if (!live && !stg) continue;
      if (a.bias) {
        const float4* b4 = reinterpret_cast<const float4*>(a.bias + cb);
#pragma unroll
        for (int i = 0; i < hd / 4; i++) {
          const float4 b = __ldg(b4 + i);
          v[4 * i] += b.x;
          v[4 * i + 1] += b.y;
          v[4 * i + 2] += b.z;
          v[4 * i + 3] += b.w;
        }
      }
      const bool is_v = cb >= a.qd + a.kd;
      if (!is_v) {
        // (cos, sin) pairs of positions j, j+1 per 16-byte load.
        const float4* cs = reinterpret_cast<const float4*>(a.rope + (size_t)pos * (hd / 2));
#pragma unroll
        for (int j2 = 0; j2 < hd / 4; j2++) {
          const float4 t = __ldg(cs + j2);
          const int j = 2 * j2;
          const float x0 = v[j], x1 = v[j + hd / 2];
          v[j] = x0 * t.x - x1 * t.y;
          v[j + hd / 2] = x1 * t.x + x0 * t.y;
          const float y0 = v[j + 1], y1 = v[j + 1 + hd / 2];
          v[j + 1] = y0 * t.z - y1 * t.w;
          v[j + 1 + hd / 2] = y1 * t.z + y0 * t.w;
        }
      }
      half* dst = nullptr;
      if (live) {
        if (cb < a.qd) {
          dst = reinterpret_cast<half*>(a.out) + (size_t)row * a.ldo + cb;
        } else {
          const int kvh = is_v ? (cb - a.qd - a.kd) / hd : (cb - a.qd) / hd;
          const int page = slot / a.page_size, off = slot % a.page_size;
          half* base = is_v ? a.vcache : a.kcache;
          dst = base + (((size_t)page * a.kvh + kvh) * a.page_size + off) * hd;
        }
      }
      if (!stg) {
#pragma unroll
        for (int c = 0; c < hd / 32; c++) store_f16x32(dst + c * 32, v + c * 32, 32);
        continue;
      }
      // Through shared memory: lane l's row as hd/8 16-byte chunks, chunk j
      // at l * 2hd + (j ^ (l % 8)) * 16 (conflict-free writes and reads);
      // then each store instruction moves 512 contiguous bytes of rows.
      constexpr int CH = hd / 8;
#pragma unroll
      for (int j = 0; j < CH; j++) {
        half2 h0 = __floats2half2_rn(v[8 * j], v[8 * j + 1]), h1 = __floats2half2_rn(v[8 * j + 2], v[8 * j + 3]);
        half2 h2 = __floats2half2_rn(v[8 * j + 4], v[8 * j + 5]), h3 = __floats2half2_rn(v[8 * j + 6], v[8 * j + 7]);
        uint4 u;
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        u.z = *reinterpret_cast<uint32_t*>(&h2);
        u.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(stg + lane * (2 * hd) + ((j ^ (lane & 7)) << 4)) = u;
      }
      __syncwarp();
      const unsigned long long dmine = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
      for (int i = 0; i < CH; i++) {
        const int c = i * 32 + lane, r = c / CH, j = c % CH;
        const unsigned long long dr = __shfl_sync(0xffffffffu, dmine, r);
        if (dr)
          *reinterpret_cast<uint4*>(dr + (unsigned long long)j * 16) =
              *reinterpret_cast<const uint4*>(stg + r * (2 * hd) + ((j ^ (r & 7)) << 4));
      }
      __syncwarp();
    }
  }
}


// x[rows row_base .. +31][col0 ..] += acc through TMA reduce-add: the warp's
// 32 rows x 32 columns at a time are written to a shared-memory buffer in the
// tensor map's 128-byte swizzle (16-byte unit u of row r at u ^ (r % 8)) and
// one lane issues the reduction.  Each residual element receives exactly one
// addition, so the result does not depend on timing.
// split >= 0: store the tile's partial sums to plane `split` of the 3-D map
// over GemmArgs::part instead of adding them into the residual.
__device__ __forceinline__ void resid_tma_tile(const GemmArgs& a, const CUtensorMap* tmR, uint32_t tbase,
                                               int row_base, int col0, uint8_t* stg, int lane, int split) {
  for (int c = 0; c < BN / 32; c++) {
    const int cb = col0 + c * 32;
    if (cb >= a.N) break;
    uint32_t r[32];
    __syncwarp();
    tmem_ld32(tbase + c * 32, r);
    tmem_ld_wait();
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
    if (a.bias && split <= 0) {
      const int n = min(32, a.N - cb);
#pragma unroll
      for (int i = 0; i < 32; i++)
        if (i < n) v[i] += a.bias[cb + i];
    }
    uint8_t* buf = stg + (c & 1) * 4096;
    if (c >= 2) {
      if (lane == 0) bulk_wait_read<1>();  // the reduction issued from this buffer two chunks ago has read it
      __syncwarp();
    }
#pragma unroll
    for (int u = 0; u < 8; u++)
      *reinterpret_cast<float4*>(buf + lane * 128 + ((u ^ (lane & 7)) << 4)) =
          make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (split >= 0)
        tma_store_3d(tmR, buf, cb, row_base, split);
      else
        tma_reduce_add_2d(tmR, buf, cb, row_base);
      bulk_commit();
    }
  }
  if (lane == 0) bulk_wait_read<0>();  // both buffers free for the next tile
  __syncwarp();
}

// Output tile of tile index t in the pair kernel's walk.  Consecutive
// indices run down a group of `group` row bands before moving to the next
// column tile, so the CTA pairs working at once share a few row bands of A
// and a few column tiles of the weights (group 1: row band by row band).
__device__ __forceinline__ void pair_tile(const GemmArgs& a, int t, int& mt, int& nt) {
  const int G = a.group > 1 ? a.group : 1;
  const int per = G * a.n_tiles;
  const int g0 = (t / per) * G;
  const int gm = min(G, a.m_tiles - g0);
  const int i = t - (t / per) * per;
  nt = i / gm;
  mt = g0 + i % gm;
}

}  // namespace laya
