// gguf::decode (src/gguf.rs:250-336) of one GGUF block from its original
// bytes, shared by the kernels that decode raw blocks: same arithmetic order
// as the reference, explicit round-to-nearest (__fmul_rn / __fsub_rn, no
// contraction) so the values are bit-identical.  Block i holds elements
// i*B .. i*B+B-1 (B = 1 for F32/F16, 32 for Q8_0/Q4_0, 256 for Q4_K/Q6_K);
// each decoded element e goes to out(e, value).
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace laya {

struct F32Sink {
  float* o;
  __device__ __forceinline__ void operator()(size_t e, float v) const { o[e] = v; }
};

// Element e of a [rows][cols] matrix -> F16 [rows][ld] (rounded to nearest).
struct F16PadSink {
  half* y;
  int cols, ld;
  __device__ __forceinline__ void operator()(size_t e, float v) const {
    y[(e / cols) * ld + e % cols] = __float2half_rn(v);
  }
};

template <class Sink>
__device__ __forceinline__ void decode_raw_block(int kind, const uint8_t* __restrict__ b, size_t i, const Sink& out) {
  switch (kind) {
    case K_F32: {
      const uint8_t* c = b + i * 4;
      out(i, bits_f32(c[0] | (c[1] << 8) | (c[2] << 16) | ((uint32_t)c[3] << 24)));
    } break;
    case K_F16: {
      const uint8_t* c = b + i * 2;
      out(i, half_bits(c[0] | (c[1] << 8)));
    } break;
    case K_Q8_0: {
      const uint8_t* c = b + i * 34;
      float d = half_bits(c[0] | (c[1] << 8));
      for (int j = 0; j < 32; j++) out(i * 32 + j, __fmul_rn(d, (float)(int8_t)c[2 + j]));
    } break;
    case K_Q4_0: {
      const uint8_t* c = b + i * 18;
      float d = half_bits(c[0] | (c[1] << 8));
      for (int j = 0; j < 16; j++) {
        out(i * 32 + j, __fmul_rn(d, __fsub_rn((float)(c[2 + j] & 15), 8.f)));
        out(i * 32 + j + 16, __fmul_rn(d, __fsub_rn((float)(c[2 + j] >> 4), 8.f)));
      }
    } break;
    case K_Q4_K: {
      const uint8_t* c = b + i * 144;
      float d = half_bits(c[0] | (c[1] << 8)), dm = half_bits(c[2] | (c[3] << 8));
      const uint8_t* sc = c + 4;
      const uint8_t* qs = c + 16;
      const size_t o = i * 256;
      for (int g = 0; g < 4; g++) {
        uint32_t s[2], m[2];
        for (int t = 0; t < 2; t++) {
          int j = g * 2 + t;
          if (j < 4) {
            s[t] = sc[j] & 63;
            m[t] = sc[j + 4] & 63;
          } else {
            s[t] = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4);
            m[t] = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
          }
        }
        for (int j = 0; j < 32; j++) {
          uint32_t q = qs[g * 32 + j];
          out(o + g * 64 + j,
              __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s[0]), (float)(q & 15)), __fmul_rn(dm, (float)m[0])));
          out(o + g * 64 + 32 + j,
              __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s[1]), (float)(q >> 4)), __fmul_rn(dm, (float)m[1])));
        }
      }
    } break;
    case K_Q6_K: {
      const uint8_t* c = b + i * 210;
      const uint8_t* ql = c;
      const uint8_t* qh = c + 128;
      const int8_t* sc = reinterpret_cast<const int8_t*>(c + 192);
      float d = half_bits(c[208] | (c[209] << 8));
      const size_t o = i * 256;
      for (int n = 0; n < 2; n++)
        for (int l = 0; l < 32; l++) {
          int lo = n * 64 + l;
          uint32_t hi = qh[n * 32 + l];
          int si = n * 8 + l / 16;
          uint32_t q[4] = {(ql[lo] & 15u) | ((hi & 3u) << 4), (ql[lo + 32] & 15u) | (((hi >> 2) & 3u) << 4),
                           (uint32_t)(ql[lo] >> 4) | (((hi >> 4) & 3u) << 4),
                           (uint32_t)(ql[lo + 32] >> 4) | (((hi >> 6) & 3u) << 4)};
          for (int j = 0; j < 4; j++)
            out(o + n * 128 + j * 32 + l, __fmul_rn(__fmul_rn(d, (float)sc[si + j * 2]), __fsub_rn((float)q[j], 32.f)));
        }
    } break;
  }
}

}  // namespace laya
