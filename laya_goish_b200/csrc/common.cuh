// Shared definitions for the CUDA side of the decision hot path: GGUF
// tensor kinds, the device-resident weight views, and the bit-exact 32-element
// decoders every weight-reading kernel is built on.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace laya {

// GGML tensor types accepted by the reference loader (src/gguf.rs:81-93).
enum Kind : int { K_F32 = 0, K_F16 = 1, K_Q4_0 = 2, K_Q8_0 = 8, K_Q4_K = 12, K_Q6_K = 14 };

// A weight matrix of `rows` x `cols` (N rows of K elements, quantised along
// K) as laid out in HBM.  GGUF blocks are transcoded at upload into
// structure-of-arrays form so that every stream starts 16-byte aligned:
//   F32  : q = float[N][K]
//   F16  : q = half[N][K]
//   Q8_0 : q = int8[N][K],      s = half[N][K/32]
//   Q4_0 : q = uint8[N][K/2],   s = half[N][K/32]   (in-block nibble order)
//   Q4_K : q = the original 144-byte superblocks, [N][K/256][144]
//   Q6_K : q = ql[N][K/2], qh = qh[N][K/4], sc = int8[N][K/16], s = half[N][K/256]
// The decoded values are bit-identical to decoding the original blocks.
struct QTensor {
  int kind;
  int rows, cols;
  const uint8_t* q;
  const uint16_t* s;
  const uint8_t* qh;
  const int8_t* sc;
};

// src/gguf.rs:226-246, as integer bit manipulation so NaN payloads and
// subnormals come out bit-identical.
__host__ __device__ __forceinline__ float bits_f32(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}
__host__ __device__ __forceinline__ float half_bits(uint32_t x) {
  uint32_t sign = (x & 0x8000u) << 16;
  uint32_t e = (x >> 10) & 31u;
  uint32_t m = x & 1023u;
  if (e == 0) {
    if (m == 0) return bits_f32(sign);
    float v = (float)m * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  if (e == 31) return bits_f32(sign | 0x7f800000u | (m << 13));
  return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

#ifdef __CUDACC__
// Order-preserving packing of (logit, row) into 64 bits: larger logits win,
// equal logits resolve to the lower row (the argmax ties-to-lowest rule).
__device__ __forceinline__ unsigned long long pack_logit(float v, int row) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)row);
}
__device__ __forceinline__ int unpack_row(unsigned long long k) { return (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu)); }

// Programmatic dependent launch: a kernel launched with
// cudaLaunchAttributeProgrammaticStreamSerialization may start before the
// previous kernel in the stream has finished.  pdl_wait() blocks until that
// kernel completed and its writes are visible (a no-op for ordinary
// launches); pdl_trigger() lets the next kernel start.  Call pdl_trigger()
// only after pdl_wait(), so at most one kernel ever overlaps.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Decodes elements [k0, k0+32) of row n (k0 % 32 == 0), bit-exact with the
// reference decoder's arithmetic order (src/gguf.rs:250-336): no FMA
// contraction, explicit round-to-nearest multiplies.
__device__ __forceinline__ void dq32(const QTensor& t, int n, int k0, float (&o)[32]) {
  const size_t K = (size_t)t.cols;
  switch (t.kind) {
    case K_F32: {
      const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(t.q) + n * K + k0);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        float4 v = __ldg(p + i);
        o[4 * i] = v.x; o[4 * i + 1] = v.y; o[4 * i + 2] = v.z; o[4 * i + 3] = v.w;
      }
    } break;
    case K_F16: {
      const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(t.q) + n * K + k0);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        uint4 v = __ldg(p + i);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          o[8 * i + 2 * j] = half_bits(w[j] & 0xffffu);
          o[8 * i + 2 * j + 1] = half_bits(w[j] >> 16);
        }
      }
    } break;
    case K_Q8_0: {
      const uint4* p = reinterpret_cast<const uint4*>(t.q + n * K + k0);
      float d = half_bits(__ldg(t.s + n * (K / 32) + k0 / 32));
#pragma unroll
      for (int i = 0; i < 2; i++) {
        uint4 v = __ldg(p + i);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 16; j++) {
          int8_t q = (int8_t)((w[j / 4] >> (8 * (j % 4))) & 0xff);
          o[16 * i + j] = __fmul_rn(d, (float)q);
        }
      }
    } break;
    case K_Q4_0: {
      uint4 v = __ldg(reinterpret_cast<const uint4*>(t.q + n * (K / 2) + k0 / 2));
      float d = half_bits(__ldg(t.s + n * (K / 32) + k0 / 32));
      uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 16; j++) {
        uint32_t c = (w[j / 4] >> (8 * (j % 4))) & 0xff;
        o[j] = __fmul_rn(d, __fsub_rn((float)(c & 15), 8.f));
        o[j + 16] = __fmul_rn(d, __fsub_rn((float)(c >> 4), 8.f));
      }
    } break;
    case K_Q4_K: {
      const uint8_t* blk = t.q + (n * (K / 256) + k0 / 256) * 144;
      int j = (k0 % 256) / 32, g = j / 2, hi = j & 1;
      float d = half_bits(blk[0] | (blk[1] << 8));
      float dm = half_bits(blk[2] | (blk[3] << 8));
      const uint8_t* sc = blk + 4;
      uint32_t s, m;
      if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
      } else {
        s = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      float ds = __fmul_rn(d, (float)s), mm = __fmul_rn(dm, (float)m);
      const uint4* p = reinterpret_cast<const uint4*>(blk + 16 + g * 32);
#pragma unroll
      for (int i = 0; i < 2; i++) {
        uint4 v = __ldg(p + i);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int b = 0; b < 16; b++) {
          uint32_t c = (w[b / 4] >> (8 * (b % 4))) & 0xff;
          uint32_t q = hi ? (c >> 4) : (c & 15);
          o[16 * i + b] = __fsub_rn(__fmul_rn(ds, (float)q), mm);
        }
      }
    } break;
    case K_Q6_K: {
      size_t sb = k0 / 256;
      int e0 = k0 % 256, h = e0 / 128, j = (e0 % 128) / 32;
      const uint8_t* ql = t.q + n * (K / 2) + sb * 128 + h * 64 + (j & 1) * 32;
      const uint8_t* qh = t.qh + n * (K / 4) + sb * 64 + h * 32;
      const int8_t* sc = t.sc + n * (K / 16) + sb * 16 + h * 8 + 2 * j;
      float d = half_bits(__ldg(t.s + n * (K / 256) + sb));
      float d0 = __fmul_rn(d, (float)sc[0]), d1 = __fmul_rn(d, (float)sc[1]);
#pragma unroll
      for (int i = 0; i < 2; i++) {
        uint4 vl = __ldg(reinterpret_cast<const uint4*>(ql) + i);
        uint4 vh = __ldg(reinterpret_cast<const uint4*>(qh) + i);
        uint32_t wl[4] = {vl.x, vl.y, vl.z, vl.w}, wh[4] = {vh.x, vh.y, vh.z, vh.w};
#pragma unroll
        for (int b = 0; b < 16; b++) {
          uint32_t cl = (wl[b / 4] >> (8 * (b % 4))) & 0xff;
          uint32_t ch = (wh[b / 4] >> (8 * (b % 4))) & 0xff;
          uint32_t q = ((j >= 2) ? (cl >> 4) : (cl & 15)) | (((ch >> (2 * j)) & 3) << 4);
          o[16 * i + b] = __fmul_rn(i == 0 ? d0 : d1, __fsub_rn((float)q, 32.f));
        }
      }
    } break;
    default:
#pragma unroll
      for (int i = 0; i < 32; i++) o[i] = 0.f;
  }
}
#endif

}  // namespace laya
