// Streaming decode GEMV: y = W . x for 1..16 activation rows, W in Q8_0
// (int8 + F16 scale per 32 elements, structure-of-arrays) or F16.  This is
// Matrix::apply (src/tensor.rs:10-102) at decode batch sizes, where the
// weight stream from HBM is the whole cost.
//
// Work unit: a tile of 16 weight rows over all K.  Each CTA (one per SM)
// takes a contiguous range of tiles.  The weights are read from a packed
// image built once per model (gemv3_pack): every stage of every tile (16
// rows x 1 KB of K, plus the Q8_0 scales) is one contiguous 17 KB block,
// already swizzled and with the epilogue's partner rows in place, so one
// producer thread moves it with a single 1-D bulk async copy (a few large
// copies per SM keep HBM busy; many small copies or tensor-map boxes per
// stage do not).  Up to 8 stages are in flight, as many as shared memory
// holds beside the activations; the first are requested before
// griddepcontrol.wait, because weights never depend on the previous kernel.
// The activation rows are staged once per CTA in shared memory as F16 (with
// the RMSNorm applied when it is fused).  Sixteen compute warps split each
// stage's K range and reduce with mma.sync m16n8k16: weights are the 16-row
// A operand (int8 -> F16 exactly through a byte permute), the activation
// rows the 8-column B operand (batch row = column), F32 accumulators; each
// Q8_0 group's partial product is scaled by its F16 scale in F32, in the
// reference's order (scale x sum over the group).  The tensor cores are only
// a reduction engine here: the bound is HBM bandwidth.
//
// A lane's 8 consecutive K elements feed fragment columns {2t, 2t+1, 2t+8,
// 2t+9} of two MMAs; A and B use the same permutation of K, so each lane
// loads 8 contiguous weights per row and 8 contiguous activations.
//
// Rows are placed so that fragment rows g and g+8 (held by the same lane)
// are partners: the RoPE pair (j, j + hd/2) of a q/k head, or the gate and
// up rows of one FFN column.  RoPE + KV-cache append and SwiGLU are
// therefore applied in registers in the epilogue.
#include <atomic>
#include <algorithm>
#include <cstring>


#include "gemv.h"
#include "launch.h"
#include "ptx.cuh"

namespace laya {

constexpr int GV_BYTES = 1024;   // weight bytes per row per stage (Q8_0: 1024 elements, F16: 512)
// Stage image (in HBM and in shared memory): two 8-row halves (tile rows
// 0-7 and 8-15), each [8 planes of 128 B of K][8 rows][128 B] with the
// 16-byte unit u of row r stored at unit u ^ (r % 8) (conflict-free fragment
// loads), then for Q8_0 the halves' scales, [8 rows][32 x F16].
constexpr int GV_HALF_W = 8 * 8 * 128;
constexpr int GV_HALF_S = 8 * 64;
constexpr int GV_STAGE = 18 * 1024;  // shared-memory stride of a stage (1024-byte aligned)
__host__ __device__ constexpr int gv_stage_bytes(bool q8) { return 2 * GV_HALF_W + (q8 ? 2 * GV_HALF_S : 0); }
constexpr int GV_MAX_STAGES = 8;     // ring depth: as many stages as shared memory holds
constexpr int GV_WARPS = 16;                   // compute warps; warp GV_WARPS is the producer
constexpr int GV_THREADS = (GV_WARPS + 2) * 32;  // + producer warp + epilogue warp

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same with a zero accumulator (C = 0).
__device__ __forceinline__ void mma16816_z(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// Four biased bytes b = q + 128 (the packed image stores Q8_0 quants with
// their sign bit flipped) -> two half2 holding q, exactly: b becomes the F16
// 1024 + b (exponent 0x64, b in the mantissa), and 1024 + 128 is subtracted.
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t b, uint32_t& lo, uint32_t& hi) {
  uint32_t l = __byte_perm(b, 0x64646464u, 0x4140);
  uint32_t h = __byte_perm(b, 0x64646464u, 0x4342);
  const half2 off = __float2half2_rn(1152.f);
  half2 hl = __hsub2(*reinterpret_cast<half2*>(&l), off);
  half2 hh = __hsub2(*reinterpret_cast<half2*>(&h), off);
  lo = *reinterpret_cast<uint32_t*>(&hl);
  hi = *reinterpret_cast<uint32_t*>(&hh);
}

__device__ __forceinline__ void named_sync() { asm volatile("bar.sync 1, %0;" ::"n"(GV_WARPS * 32) : "memory"); }

// Source row i (0..15) of tile t: segment and row index, or false when the
// row lies past the matrix (ragged last tile).
__device__ __forceinline__ bool tile_row(const Gemv3Args& a, int t, int i, int& seg, int& row) {
  const int lo = i & 7;
  if (a.mode == GV_SWIGLU) {
    const int c = 8 * t + lo;
    if (a.interleaved) {
      seg = 0;
      row = (c / 128) * 256 + c % 128 + (i >= 8 ? 128 : 0);
      return c < a.seg[0].rows / 2;
    }
    seg = i >= 8 ? 1 : 0;
    row = c;
    return c < a.seg[0].rows;
  }
  if (a.mode == GV_QKV) {
    const int tq = a.qd / 16, tk = a.kd / 16;
    if (t < tq + tk) {
      const bool isk = t >= tq;
      const int tt = isk ? t - tq : t;
      const int per = a.hd / 16;
      const int h = tt / per, u = tt % per;
      seg = isk ? 1 : 0;
      row = h * a.hd + 8 * u + lo + (i >= 8 ? a.hd / 2 : 0);
      return true;
    }
    seg = 2;
    row = (t - tq - tk) * 16 + i;
    return row < a.kd;
  }
  seg = 0;
  row = t * 16 + i;
  return row < a.seg[0].rows;
}

// Byte offset of the weight ring: barriers, cross-warp sums and the staged
// activation rows come first (the ring starts 1024-byte aligned, as the
// 128-byte swizzle requires).
__host__ __device__ constexpr size_t gv_ring_offset(int nb, int K, int nt) {
  return ((size_t)(2 * GV_MAX_STAGES + 4) * 8 + (size_t)2 * GV_WARPS * 32 * 4 * nt * 4 + (size_t)nb * (K + 8) * 2 +
          1023) /
         1024 * 1024;
}

// One 32-element group (chunk c of a stage) as MMA fragments: rows g and
// g+8 of the tile, and the activation rows n*8 + g.
template <int NT>
struct Frag {
  uint32_t ag[4], ah[4];
  float dg, dh;
  uint4 xv[NT];
};

// Per-lane shared-memory offsets of chunk c of a stage (chunk = one 32-element
// group: 32 bytes of each row for Q8_0, 64 for F16): the lane's 8 (Q8_0) or
// 16 (F16) bytes of row g in the first half, its F16 scale of row g (Q8_0),
// and its first K index relative to the stage.
struct ChunkOff {
  int w, s, k;
};
template <bool Q8>
__device__ __forceinline__ ChunkOff chunk_off(int c, int g, int tq) {
  ChunkOff o;
  if constexpr (Q8) {
    const int p = c >> 2, u = ((c & 3) << 1) | (tq >> 1);
    o.w = p * 1024 + g * 128 + ((u ^ g) << 4) + ((tq & 1) << 3);
    o.s = 2 * GV_HALF_W + g * 64 + 2 * c;
  } else {
    const int p = c >> 1, u = ((c & 1) << 2) | tq;
    o.w = p * 1024 + g * 128 + ((u ^ g) << 4);
    o.s = 0;
  }
  o.k = c * 32 + 8 * tq;
  return o;
}

// One chunk of stage `sb` (shared memory) as MMA fragments: rows g and g+8
// of the tile, and the activation rows n*8 + g (rows past the batch repeat
// the last real row; their output columns are never read).
template <int NT, bool Q8>
__device__ __forceinline__ void load_frag(Frag<NT>& f, const uint8_t* sb, const ChunkOff& o, const half* const (&xr)[NT],
                                          int kel0) {
  if constexpr (Q8) {
    const uint2 wg = *reinterpret_cast<const uint2*>(sb + o.w);
    const uint2 wh = *reinterpret_cast<const uint2*>(sb + GV_HALF_W + o.w);
    i8x4_to_h2x2(wg.x, f.ag[0], f.ag[1]);
    i8x4_to_h2x2(wg.y, f.ag[2], f.ag[3]);
    i8x4_to_h2x2(wh.x, f.ah[0], f.ah[1]);
    i8x4_to_h2x2(wh.y, f.ah[2], f.ah[3]);
    // F16 -> F32 is exact for every finite scale
    f.dg = __half2float(*reinterpret_cast<const half*>(sb + o.s));
    f.dh = __half2float(*reinterpret_cast<const half*>(sb + o.s + GV_HALF_S));
  } else {
    const uint4 wg = *reinterpret_cast<const uint4*>(sb + o.w);
    const uint4 wh = *reinterpret_cast<const uint4*>(sb + GV_HALF_W + o.w);
    f.ag[0] = wg.x;
    f.ag[1] = wg.y;
    f.ag[2] = wg.z;
    f.ag[3] = wg.w;
    f.ah[0] = wh.x;
    f.ah[1] = wh.y;
    f.ah[2] = wh.z;
    f.ah[3] = wh.w;
    f.dg = f.dh = 1.f;
  }
#pragma unroll
  for (int n = 0; n < NT; n++) f.xv[n] = *reinterpret_cast<const uint4*>(xr[n] + kel0 + o.k);
}

template <int NT, bool Q8>
__device__ __forceinline__ void mma_frag(const Frag<NT>& f, float (&acc)[NT][4]) {
#pragma unroll
  for (int n = 0; n < NT; n++) {
    if constexpr (Q8) {
      // each Q8_0 group is summed alone, then scaled by its F16 scale
      float p[4];
      mma16816_z(p, f.ag[0], f.ah[0], f.ag[1], f.ah[1], f.xv[n].x, f.xv[n].y);
      mma16816(p, f.ag[2], f.ah[2], f.ag[3], f.ah[3], f.xv[n].z, f.xv[n].w);
      acc[n][0] = fmaf(f.dg, p[0], acc[n][0]);
      acc[n][1] = fmaf(f.dg, p[1], acc[n][1]);
      acc[n][2] = fmaf(f.dh, p[2], acc[n][2]);
      acc[n][3] = fmaf(f.dh, p[3], acc[n][3]);
    } else {
      mma16816(acc[n], f.ag[0], f.ah[0], f.ag[1], f.ah[1], f.xv[n].x, f.xv[n].y);
      mma16816(acc[n], f.ag[2], f.ah[2], f.ag[3], f.ah[3], f.xv[n].z, f.xv[n].w);
    }
  }
}

// Builds stage (t, ks) of the packed image: block b = t * kstages + ks.
// Rows past a matrix and K past its end are zero.
__global__ void gemv3_pack_kernel(const Gemv3Args a, int kstages, uint8_t* __restrict__ dst) {
  const int b = blockIdx.x, t = b / kstages, ks = b % kstages;
  const bool q8 = a.seg[0].kind == K_Q8_0;
  const int K = a.K, row_bytes = q8 ? K : 2 * K;
  uint8_t* out = dst + (size_t)b * gv_stage_bytes(q8);
  for (int i16 = threadIdx.x; i16 < 16 * 64 + (q8 ? 16 * 4 : 0); i16 += blockDim.x) {
    if (i16 < 16 * 64) {
      const int i = i16 / 64, uu = i16 % 64, p = uu / 8, u = uu % 8;
      int seg = 0, row = 0;
      const bool valid = tile_row(a, t, i, seg, row);
      const QTensor& w = seg == 0 ? a.seg[0] : seg == 1 ? a.seg[1] : a.seg[2];
      const int kb = ks * GV_BYTES + p * 128 + u * 16;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (valid && kb < row_bytes) v = *reinterpret_cast<const uint4*>(w.q + (size_t)row * row_bytes + kb);
      if (q8) {  // quants stored biased (q + 128); padding becomes q = 0
        v.x ^= 0x80808080u;
        v.y ^= 0x80808080u;
        v.z ^= 0x80808080u;
        v.w ^= 0x80808080u;
      }
      *reinterpret_cast<uint4*>(out + (i / 8) * GV_HALF_W + p * 1024 + (i % 8) * 128 + ((u ^ (i % 8)) << 4)) = v;
    } else {
      const int j = i16 - 16 * 64, i = j / 4, v4 = j % 4;
      int seg = 0, row = 0;
      const bool valid = tile_row(a, t, i, seg, row);
      const QTensor& w = seg == 0 ? a.seg[0] : seg == 1 ? a.seg[1] : a.seg[2];
      const int grp = ks * 32 + v4 * 8;  // 8 scales per 16 bytes
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (valid && grp < K / 32) v = *reinterpret_cast<const uint4*>(w.s + (size_t)row * (K / 32) + grp);
      *reinterpret_cast<uint4*>(out + 2 * GV_HALF_W + (i / 8) * GV_HALF_S + (i % 8) * 64 + v4 * 16) = v;
    }
  }
}

// Two named barriers besides __syncthreads: 1 = the compute warps,
// 2 = the compute warps and the epilogue warp.
__device__ __forceinline__ void cta_epi_sync() { asm volatile("bar.sync 2, %0;" ::"n"((GV_WARPS + 1) * 32) : "memory"); }

// Work of phase p of a GEMV sequence: this CTA's contiguous tile range.
struct GvPhase {
  int kstages, t0, t1;
};

__device__ __forceinline__ GvPhase gv_phase(const GemvSeq& q, int p, bool q8) {
  const Gemv3Args& a = q.ph[p];
  GvPhase r;
  r.kstages = ((q8 ? a.K : 2 * a.K) + GV_BYTES - 1) / GV_BYTES;
  r.t0 = (int)((long long)blockIdx.x * q.tiles[p] / gridDim.x);
  r.t1 = (int)((long long)(blockIdx.x + 1) * q.tiles[p] / gridDim.x);
  return r;
}

// One launch runs q.n GEMV phases in order (e.g. attention output, gate/up,
// down, the next layer's QKV).  The producer streams every phase's weight
// stages back to back, so the next phase's weights are already in flight
// while the current phase finishes; between phases every CTA waits at a
// grid-wide barrier (q.gbar, zeroed before the launch; the launch is
// cooperative), because a phase reads the previous phase's outputs.
template <int NT, bool Q8>
__global__ void __launch_bounds__(GV_THREADS, 1) gemv3_kernel(const __grid_constant__ GemvSeq q, int nst) {
  // [full | empty | tdone | tfree barriers][cross-warp sums][activation rows][nst-stage ring]
  extern __shared__ uint8_t gsm_raw[];
  // 1024-byte aligned by an integer offset from the shared array, so every
  // pointer below stays a known shared-memory address (shared loads)
  uint8_t* gsm = gsm_raw + ((1024u - (smem_u32(gsm_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(gsm);
  uint64_t* empty = full + GV_MAX_STAGES;
  uint64_t* tdone = empty + GV_MAX_STAGES;  // [2] a tile's partial sums are written (GV_WARPS arrivals)
  uint64_t* tfree = tdone + 2;              // [2] the epilogue has read them (1 arrival)
  float4* red = reinterpret_cast<float4*>(tfree + 2);  // [2][GV_WARPS][NT][32] partial sums
  half* xs = reinterpret_cast<half*>(red + 2 * GV_WARPS * 32 * NT);
  uint8_t* ring = gsm + gv_ring_offset(q.ph[0].nb, q.kmax, NT);
  __shared__ float nred[GV_WARPS][16];
  __shared__ float nscale[16];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long budget = q.ph[0].budget;
  unsigned* err = q.ph[0].err;
  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GV_WARPS);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tdone[b], GV_WARPS);
      mbar_init(&tfree[b], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == GV_WARPS) {
    // ---------------- producer: one thread, one bulk copy per stage, all phases
    if (lane != 0) return;
    int stage = 0;
    uint32_t phase = 0;
    const uint32_t sbytes = (uint32_t)gv_stage_bytes(Q8);
    for (int p = 0; p < q.n; p++) {
      const GvPhase w = gv_phase(q, p, Q8);
      const uint8_t* src = q.ph[p].packed + (size_t)w.t0 * w.kstages * sbytes;
      const int nstg = (w.t1 - w.t0) * w.kstages;  // this CTA's stages of the phase: one contiguous range
      for (int j = 0; j < nstg; j++) {
        if (!mbar_wait_sleep(&empty[stage], phase ^ 1, budget)) atomicOr(err, 32u);
        mbar_expect_tx(&full[stage], sbytes);
        bulk_g2s(ring + stage * GV_STAGE, src + (size_t)j * sbytes, sbytes, &full[stage]);
        if (++stage == nst) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // Every fill is consumed before the CTA exits (no copy left in flight).
    for (int i = 0; i < nst; i++) {
      if (!mbar_wait(&empty[stage], phase ^ 1, budget)) atomicOr(err, 64u);
      if (++stage == nst) {
        stage = 0;
        phase ^= 1;
      }
    }
    return;
  }

  const int g = lane >> 2, tq = lane & 3;
  // Barrier between phases p-1 and p: all of this CTA's outputs of phase p-1
  // are written (compute and epilogue warps meet), then one thread joins
  // the grid-wide count, then everyone proceeds.
  auto grid_sync = [&](int p) {
    cta_epi_sync();
    if (threadIdx.x == 0) {
      // the release is cumulative: the CTA's output stores, ordered before
      // it by the named barrier above, are visible to every CTA whose
      // acquire load below reads the completed count
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(q.gbar) : "memory");
      const unsigned target = (unsigned)p * gridDim.x;
      const long long t0 = clock64();
      unsigned v;
      while (true) {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(q.gbar) : "memory");
        if (v >= target) break;
        if (clock64() - t0 > budget) {
          atomicOr(err, 4096u);
          break;
        }
      }
    }
    cta_epi_sync();
  };

  if (warp == GV_WARPS + 1) {
    // ---------------- epilogue warp: sums the compute warps' partials and
    // writes the outputs.  Each tile's global operands (residual, RoPE
    // factors, bias) are loaded before waiting for its sums, so their
    // latency overlaps the tile's K loop.  Lane (g, tq) holds rows g and g+8
    // for batch rows n*8 + 2tq + e.
    pdl_wait();
    int T = 0;  // tiles handed over so far (all phases)
    for (int p = 0; p < q.n; p++) {
      if (p > 0) grid_sync(p);
      const Gemv3Args& a = q.ph[p];
      const GvPhase w = gv_phase(q, p, Q8);
      const int tqn = a.qd / 16, tkn = a.kd / 16;
      int pos[NT][2], slot[NT][2];
#pragma unroll
      for (int n = 0; n < NT; n++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int b = n * 8 + 2 * tq + e;
          pos[n][e] = (a.mode == GV_QKV && b < a.nb) ? a.pos[b] : 0;
          slot[n][e] = (a.mode == GV_QKV && b < a.nb) ? a.slot[b] : 0;
        }
      unsigned long long best[NT][2];
#pragma unroll
      for (int n = 0; n < NT; n++) best[n][0] = best[n][1] = 0ull;
      for (int t = w.t0; t < w.t1; t++, T++) {
        const int buf = T & 1;
        // operands of tile t
        float yv[NT][2][2];
        float2 cs[NT][2];
        float bg = 0.f, bh = 0.f;
        bool isk = false, isv = false;
        int h = 0, j = 0, r0 = t * 16 + g;
        if (a.mode == GV_QKV) {
          isv = t >= tqn + tkn;
          if (!isv) {
            isk = t >= tqn;
            const int tt = isk ? t - tqn : t, per = a.hd / 16;
            h = tt / per;
            j = 8 * (tt % per) + g;
            const int col0 = (isk ? a.qd : 0) + h * a.hd + j;
            if (a.bias) {
              bg = __ldg(a.bias + col0);
              bh = __ldg(a.bias + col0 + a.hd / 2);
            }
          } else {
            r0 = (t - tqn - tkn) * 16 + g;
            if (a.bias) {
              bg = r0 < a.kd ? __ldg(a.bias + a.qd + a.kd + r0) : 0.f;
              bh = r0 + 8 < a.kd ? __ldg(a.bias + a.qd + a.kd + r0 + 8) : 0.f;
            }
          }
        }
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
          for (int e = 0; e < 2; e++) {
            const int b = n * 8 + 2 * tq + e;
            yv[n][e][0] = yv[n][e][1] = 0.f;
            cs[n][e] = make_float2(1.f, 0.f);
            if (b >= a.nb) continue;
            if (a.mode == GV_PLAIN && a.acc) {
              const float* yb = a.y + (size_t)b * a.ldy;
              if (r0 < a.seg[0].rows) yv[n][e][0] = yb[r0];
              if (r0 + 8 < a.seg[0].rows) yv[n][e][1] = yb[r0 + 8];
            } else if (a.mode == GV_QKV && !isv) {
              cs[n][e] = __ldg(a.rope + (size_t)pos[n][e] * (a.hd / 2) + j);
            }
          }
        if (!mbar_wait_sleep(&tdone[buf], (T >> 1) & 1, budget)) {
          if (lane == 0) atomicOr(err, 512u);
        }
        const float4* rb = red + buf * (GV_WARPS * NT * 32);
        float acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) {
          float4 sum = rb[n * 32 + lane];
#pragma unroll
          for (int ww = 1; ww < GV_WARPS; ww++) {
            const float4 v = rb[(ww * NT + n) * 32 + lane];
            sum.x += v.x;
            sum.y += v.y;
            sum.z += v.z;
            sum.w += v.w;
          }
          acc[n][0] = sum.x;
          acc[n][1] = sum.y;
          acc[n][2] = sum.z;
          acc[n][3] = sum.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfree[buf]);
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
          for (int e = 0; e < 2; e++) {
            const int b = n * 8 + 2 * tq + e;
            if (b >= a.nb) continue;
            const float vg = acc[n][e], vh = acc[n][2 + e];
            if (a.mode == GV_PLAIN) {
              float* yb = a.y + (size_t)b * a.ldy;
              if (r0 < a.seg[0].rows) yb[r0] = yv[n][e][0] + vg;  // yv is 0 unless accumulating
              if (r0 + 8 < a.seg[0].rows) yb[r0 + 8] = yv[n][e][1] + vh;
            } else if (a.mode == GV_ARGMAX) {
              if (r0 < a.seg[0].rows) {
                const unsigned long long kk = pack_logit(vg, r0);
                best[n][e] = kk > best[n][e] ? kk : best[n][e];
              }
              if (r0 + 8 < a.seg[0].rows) {
                const unsigned long long kk = pack_logit(vh, r0 + 8);
                best[n][e] = kk > best[n][e] ? kk : best[n][e];
              }
            } else if (a.mode == GV_SWIGLU) {
              const int c = 8 * t + g;
              const int ffn = a.interleaved ? a.seg[0].rows / 2 : a.seg[0].rows;
              if (c < ffn) a.act[(size_t)b * a.ld_act + c] = __float2half_rn(vg / (1.f + __expf(-vg)) * vh);
            } else {  // GV_QKV
              const int page = slot[n][e] / a.page_size, off = slot[n][e] % a.page_size;
              if (!isv) {
                // rotate-half RoPE (src/tensor.rs:158-171) after the bias
                const float x0 = vg + bg, x1 = vh + bh;
                const float y0 = x0 * cs[n][e].x - x1 * cs[n][e].y, y1 = x1 * cs[n][e].x + x0 * cs[n][e].y;
                half* dst = isk ? a.kcache + (((size_t)page * a.kvh + h) * a.page_size + off) * a.hd
                                : a.q + (size_t)b * a.qd + h * a.hd;
                dst[j] = __float2half_rn(y0);
                dst[j + a.hd / 2] = __float2half_rn(y1);
              } else {
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                  const int r = r0 + 8 * hh;
                  if (r >= a.kd) continue;
                  const float v = (hh ? vh : vg) + (hh ? bh : bg);
                  a.vcache[(((size_t)page * a.kvh + r / a.hd) * a.page_size + off) * a.hd + r % a.hd] =
                      __float2half_rn(v);
                }
              }
            }
          }
      }
      if (a.mode == GV_ARGMAX) {
        // lanes with the same tq hold the same batch rows: reduce over g
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
          for (int e = 0; e < 2; e++) {
            unsigned long long k = best[n][e];
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
              const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
              k = ok > k ? ok : k;
            }
            const int b = n * 8 + 2 * tq + e;
            if (g == 0 && b < a.nb && k) atomicMax(a.best + b, k);
          }
      }
    }
    return;
  }

  // ---------------- compute warps
  const int tid = threadIdx.x;
  constexpr int CPW = Q8 ? 2 : 1;  // chunks per warp in a full stage
  ChunkOff co[CPW];
#pragma unroll
  for (int i = 0; i < CPW; i++) co[i] = chunk_off<Q8>(warp + i * GV_WARPS, g, tq);
  pdl_wait();
  int stage = 0, T = 0;
  uint32_t phase = 0;
  for (int p = 0; p < q.n; p++) {
    if (p > 0) grid_sync(p);
    const Gemv3Args& a = q.ph[p];
    const GvPhase w = gv_phase(q, p, Q8);
    const int K = a.K;
    const int row_bytes = Q8 ? K : 2 * K;
    const int xpitch = K + 8;
    if (!a.xres) {
      // F16 activation rows -> shared memory
      for (int b = 0; b < a.nb; b++)
        for (int k = tid * 8; k < K; k += GV_WARPS * 32 * 8)
          *reinterpret_cast<uint4*>(xs + (size_t)b * xpitch + k) =
              *reinterpret_cast<const uint4*>(a.x + (size_t)b * a.ldx + k);
      named_sync();
    } else if ((size_t)a.nb * K <= (size_t)2 * GV_WARPS * 32 * NT * 4) {
      // x = rmsnorm(xres[b]) * norm_w with one pass over global memory: the
      // residual and the norm weights are loaded together and x * w is
      // kept in F32 in the (idle) partial-sum buffer until the scale is known.
      float* xw = reinterpret_cast<float*>(red);
      for (int b = 0; b < a.nb; b++) {
        float ss = 0.f;
        for (int k = tid * 4; k < K; k += GV_WARPS * 32 * 4) {
          const float4 v = *reinterpret_cast<const float4*>(a.xres + (size_t)b * K + k);
          const float4 wv = *reinterpret_cast<const float4*>(a.norm_w + k);
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
          *reinterpret_cast<float4*>(xw + (size_t)b * K + k) =
              make_float4(v.x * wv.x, v.y * wv.y, v.z * wv.z, v.w * wv.w);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) nred[warp][b] = ss;
      }
      named_sync();
      if (tid < a.nb) {
        float tsum = 0.f;
        for (int i = 0; i < GV_WARPS; i++) tsum += nred[i][tid];
        nscale[tid] = 1.f / sqrtf(tsum / (float)K + a.eps);
      }
      named_sync();
      for (int b = 0; b < a.nb; b++) {
        const float sc = nscale[b];
        for (int k = tid * 4; k < K; k += GV_WARPS * 32 * 4) {
          const float4 t = *reinterpret_cast<const float4*>(xw + (size_t)b * K + k);
          half2 h0 = __floats2half2_rn(t.x * sc, t.y * sc);
          half2 h1 = __floats2half2_rn(t.z * sc, t.w * sc);
          uint2 u2;
          u2.x = *reinterpret_cast<uint32_t*>(&h0);
          u2.y = *reinterpret_cast<uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(xs + (size_t)b * xpitch + k) = u2;
        }
      }
      named_sync();
    } else {
      // x = rmsnorm(xres[b]) * norm_w  (src/models/openthai/model.rs:84-94), F16 rows in shared memory
      for (int b = 0; b < a.nb; b++) {
        float ss = 0.f;
        for (int k = tid * 4; k < K; k += GV_WARPS * 32 * 4) {
          const float4 v = *reinterpret_cast<const float4*>(a.xres + (size_t)b * K + k);
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) nred[warp][b] = ss;
      }
      named_sync();
      if (tid < a.nb) {
        float tsum = 0.f;
        for (int i = 0; i < GV_WARPS; i++) tsum += nred[i][tid];
        nscale[tid] = 1.f / sqrtf(tsum / (float)K + a.eps);
      }
      named_sync();
      for (int k = tid * 4; k < K; k += GV_WARPS * 32 * 4) {
        const float4 wv = *reinterpret_cast<const float4*>(a.norm_w + k);
        for (int b = 0; b < a.nb; b++) {
          const float4 v = *reinterpret_cast<const float4*>(a.xres + (size_t)b * K + k);
          const float sc = nscale[b];
          half2 h0 = __floats2half2_rn(v.x * sc * wv.x, v.y * sc * wv.y);
          half2 h1 = __floats2half2_rn(v.z * sc * wv.z, v.w * sc * wv.w);
          uint2 u2;
          u2.x = *reinterpret_cast<uint32_t*>(&h0);
          u2.y = *reinterpret_cast<uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(xs + (size_t)b * xpitch + k) = u2;
        }
      }
      named_sync();
    }
    // the next kernel may start once every CTA is past its last grid barrier
    if (p == q.n - 1) pdl_trigger();
    const half* xr[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) xr[n] = xs + (size_t)min(n * 8 + g, a.nb - 1) * xpitch;
    for (int t = w.t0; t < w.t1; t++, T++) {
      float acc[NT][4];
#pragma unroll
      for (int n = 0; n < NT; n++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[n][j] = 0.f;
      for (int ks = 0; ks < w.kstages; ks++) {
        if (!mbar_wait_spin(&full[stage], phase, budget)) {
          if (lane == 0) atomicOr(err, 128u);
        }
        const uint8_t* sb = ring + stage * GV_STAGE;
        const int kb = ks * GV_BYTES;
        const int nbytes = min(GV_BYTES, row_bytes - kb);
        const int kel0 = Q8 ? kb : kb / 2;  // first K index of the stage
        // A full stage has 32 (Q8_0) or 16 (F16) groups: warp w takes groups
        // w and w + 16, all loads issued before the MMAs.
        Frag<NT> f[CPW];
        if (nbytes == GV_BYTES) {
#pragma unroll
          for (int i = 0; i < CPW; i++) load_frag<NT, Q8>(f[i], sb, co[i], xr, kel0);
          // the stage's bytes are in registers: hand the slot back to the producer
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[stage]);
#pragma unroll
          for (int i = 0; i < CPW; i++) mma_frag<NT, Q8>(f[i], acc);
        } else {
          // the last stage of a row whose bytes are not a multiple of 1 KB
          const int chunks = nbytes / (Q8 ? 32 : 64);
#pragma unroll
          for (int i = 0; i < CPW; i++)
            if (warp + i * GV_WARPS < chunks) load_frag<NT, Q8>(f[i], sb, co[i], xr, kel0);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[stage]);
#pragma unroll
          for (int i = 0; i < CPW; i++)
            if (warp + i * GV_WARPS < chunks) mma_frag<NT, Q8>(f[i], acc);
        }
        if (++stage == nst) {
          stage = 0;
          phase ^= 1;
        }
      }
      // Hand the partial sums (this warp's share of K) to the epilogue warp.
      const int buf = T & 1;
      if (!mbar_wait_sleep(&tfree[buf], ((T >> 1) & 1) ^ 1, budget)) {
        if (lane == 0) atomicOr(err, 256u);
      }
      float4* rb = red + buf * (GV_WARPS * NT * 32);
#pragma unroll
      for (int n = 0; n < NT; n++) rb[(warp * NT + n) * 32 + lane] = make_float4(acc[n][0], acc[n][1], acc[n][2], acc[n][3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&tdone[buf]);
    }
  }
}

constexpr size_t GV_SMEM_BUDGET = 225 * 1024;  // dynamic shared memory per CTA (one CTA per SM)

// Ring stages that fit beside the staged activations: 2 .. GV_MAX_STAGES,
// or 0 when even two do not fit.
static int stages_for(int nb, int K, int nt) {
  const size_t off = gv_ring_offset(nb, K, nt) + 1024;  // + alignment slack
  if (off + 2 * GV_STAGE > GV_SMEM_BUDGET) return 0;
  return (int)std::min<size_t>(GV_MAX_STAGES, (GV_SMEM_BUDGET - off) / GV_STAGE);
}
static int gemv3_stages(const Gemv3Args& a, int nt) { return stages_for(a.nb, a.K, nt); }

bool gemv3_fits(int nb, int kmax) { return nb >= 1 && nb <= 16 && stages_for(nb, kmax, nb <= 8 ? 1 : 2) >= 2; }

// Weight-side conditions (packing needs only these).
static bool gemv3_weights_ok(const Gemv3Args& a) {
  if (a.K <= 0 || a.K % 256) return false;
  const int nseg = a.mode == GV_QKV ? 3 : (a.mode == GV_SWIGLU && !a.interleaved) ? 2 : 1;
  for (int i = 0; i < nseg; i++) {
    const QTensor& w = a.seg[i];
    if ((w.kind != K_Q8_0 && w.kind != K_F16) || w.kind != a.seg[0].kind || w.cols != a.K || !w.q) return false;
    if (reinterpret_cast<uintptr_t>(w.q) & 15) return false;
    if (w.kind == K_Q8_0 && (!w.s || (reinterpret_cast<uintptr_t>(w.s) & 15))) return false;
  }
  if (a.mode == GV_QKV && (a.hd % 16 || a.qd % 16 || a.kd % 16)) return false;
  return true;
}

bool gemv3_supported(const Gemv3Args& a) {
  if (a.nb < 1 || a.nb > 16 || !gemv3_weights_ok(a)) return false;
  if (a.mode == GV_QKV && (!a.pos || !a.slot || !a.rope)) return false;
  if (gemv3_stages(a, a.nb <= 8 ? 1 : 2) < 2) return false;
  if (a.xres) {
    if (!a.norm_w) return false;
  } else if (!a.x || (a.ldx % 8) || (reinterpret_cast<uintptr_t>(a.x) & 15)) {
    return false;
  }
  return true;
}

static int gemv3_tiles(const Gemv3Args& a) {
  if (a.mode == GV_QKV) return a.qd / 16 + a.kd / 16 + (a.kd + 15) / 16;
  if (a.mode == GV_SWIGLU) return ((a.interleaved ? a.seg[0].rows / 2 : a.seg[0].rows) + 7) / 8;
  return (a.seg[0].rows + 15) / 16;
}

static int gemv3_kstages(const Gemv3Args& a) {
  const int row_bytes = a.seg[0].kind == K_Q8_0 ? a.K : 2 * a.K;
  return (row_bytes + GV_BYTES - 1) / GV_BYTES;
}

size_t gemv3_packed_bytes(const Gemv3Args& a) {
  if (!gemv3_weights_ok(a)) return 0;
  return (size_t)gemv3_tiles(a) * gemv3_kstages(a) * gv_stage_bytes(a.seg[0].kind == K_Q8_0);
}

cudaError_t gemv3_pack(const Gemv3Args& a, uint8_t* dst, cudaStream_t st) {
  if (!gemv3_weights_ok(a)) return cudaErrorInvalidValue;
  const int blocks = gemv3_tiles(a) * gemv3_kstages(a);
  if (blocks <= 0) return cudaSuccess;
  gemv3_pack_kernel<<<blocks, 256, 0, st>>>(a, gemv3_kstages(a), dst);
  return cudaGetLastError();
}

template <int NT, bool Q8>
static cudaError_t gemv3_go(const GemvSeq& q, int num_sms, cudaStream_t st) {
  auto kern = gemv3_kernel<NT, Q8>;
  const int nst = stages_for(q.ph[0].nb, q.kmax, NT);
  if (nst < 2) return cudaErrorInvalidValue;
  const size_t smem = gv_ring_offset(q.ph[0].nb, q.kmax, NT) + 1024 + (size_t)nst * GV_STAGE;
  static std::atomic<bool> configured[64];  // per device; any host thread may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GV_SMEM_BUDGET);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = true;
  }
  // one CTA per SM, each with a contiguous range of every phase's tiles; a
  // multi-phase launch is cooperative (its CTAs wait on one another)
  const int grid = q.n == 1 ? std::min(q.tiles[0], num_sms) : num_sms;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = q.n > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, q, nst);
}

cudaError_t gemv3_launch_seq(const Gemv3Args* ph, int n, unsigned* gbar, int num_sms, cudaStream_t st) {
  if (n < 1 || n > 4 || (n > 1 && !gbar)) return cudaErrorInvalidValue;
  GemvSeq q{};
  q.n = n;
  q.gbar = gbar;
  for (int i = 0; i < n; i++) {
    const Gemv3Args& a = ph[i];
    if (!gemv3_supported(a) || !a.packed || (reinterpret_cast<uintptr_t>(a.packed) & 15)) return cudaErrorInvalidValue;
    if (a.nb != ph[0].nb || a.seg[0].kind != ph[0].seg[0].kind) return cudaErrorInvalidValue;
    q.ph[i] = a;
    q.tiles[i] = gemv3_tiles(a);
    q.kmax = std::max(q.kmax, a.K);
  }
  const int nt = ph[0].nb <= 8 ? 1 : 2;
  if (stages_for(ph[0].nb, q.kmax, nt) < 2) return cudaErrorInvalidValue;
  const bool q8 = ph[0].seg[0].kind == K_Q8_0;
  if (nt == 1) return q8 ? gemv3_go<1, true>(q, num_sms, st) : gemv3_go<1, false>(q, num_sms, st);
  return q8 ? gemv3_go<2, true>(q, num_sms, st) : gemv3_go<2, false>(q, num_sms, st);
}

cudaError_t gemv3_launch(const Gemv3Args& a, int num_sms, cudaStream_t st) {
  if (gemv3_tiles(a) <= 0) return cudaSuccess;
  return gemv3_launch_seq(&a, 1, nullptr, num_sms, st);
}

}  // namespace laya
