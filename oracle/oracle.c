/*
 * CPU oracle for the Laya Goish decision hot path.  TEST INFRASTRUCTURE ONLY:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it,
 * as the checker.  The CUDA library never links or calls this file.
 *
 * Every function restates a reference function of panudetjt/laya-goish
 * (Rust, no_std) and cites it.  Compile with -ffp-contract=off so that the
 * arithmetic order of the dequantisers stays bit-exact with the reference.
 */
#include "oracle.h"

#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* Weight format: src/gguf.rs                                          */
/* ------------------------------------------------------------------ */

/* src/gguf.rs:226-246 */
float or_half(uint16_t x) {
  uint32_t sign = ((uint32_t)x & 0x8000u) << 16;
  uint32_t e = (x >> 10) & 31;
  uint32_t m = x & 1023;
  uint32_t bits;
  float f;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
      memcpy(&f, &bits, 4);
      return f;
    }
    f = (float)m * (1.0f / 16777216.0f);
    return sign ? -f : f;
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (m << 13);
  } else {
    bits = sign | ((e + 112) << 23) | (m << 13);
  }
  memcpy(&f, &bits, 4);
  return f;
}

static float h16(const uint8_t* b) { return or_half((uint16_t)(b[0] | (b[1] << 8))); }

/* src/gguf.rs:81-93 */
int or_layout(uint32_t kind, int* block, int* size) {
  switch (kind) {
    case 0: *block = 1; *size = 4; return 0;
    case 1: *block = 1; *size = 2; return 0;
    case 2: *block = 32; *size = 18; return 0;
    case 8: *block = 32; *size = 34; return 0;
    case 12: *block = 256; *size = 144; return 0;
    case 14: *block = 256; *size = 210; return 0;
    default: return -1;
  }
}

/* src/gguf.rs:250-336 (same operation order; built without FMA contraction) */
int or_decode(uint32_t kind, const uint8_t* b, size_t nbytes, float* out) {
  int block, size;
  if (or_layout(kind, &block, &size)) return -1;
  size_t nb = nbytes / (size_t)size;
  for (size_t i = 0; i < nb; i++) {
    const uint8_t* c = b + i * (size_t)size;
    float* o = out + i * (size_t)block;
    switch (kind) {
      case 0: memcpy(o, c, 4); break;
      case 1: o[0] = h16(c); break;
      case 8: {
        float d = h16(c);
        for (int j = 0; j < 32; j++) o[j] = d * (float)(int8_t)c[2 + j];
      } break;
      case 2: {
        float d = h16(c);
        for (int j = 0; j < 16; j++) {
          o[j] = d * ((float)(c[2 + j] & 15) - 8.f);
          o[j + 16] = d * ((float)(c[2 + j] >> 4) - 8.f);
        }
      } break;
      case 12: {
        float d = h16(c), dm = h16(c + 2);
        const uint8_t* sc = c + 4;
        const uint8_t* qs = c + 16;
        for (int g = 0; g < 4; g++) {
          uint8_t s[2], m[2];
          for (int t = 0; t < 2; t++) {
            int j = g * 2 + t;
            if (j < 4) {
              s[t] = sc[j] & 63;
              m[t] = sc[j + 4] & 63;
            } else {
              s[t] = (uint8_t)((sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4));
              m[t] = (uint8_t)((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4));
            }
          }
          for (int j = 0; j < 32; j++) {
            uint8_t q = qs[g * 32 + j];
            o[g * 64 + j] = d * (float)s[0] * (float)(q & 15) - dm * (float)m[0];
            o[g * 64 + 32 + j] = d * (float)s[1] * (float)(q >> 4) - dm * (float)m[1];
          }
        }
      } break;
      case 14: {
        const uint8_t* ql = c;
        const uint8_t* qh = c + 128;
        const int8_t* sc = (const int8_t*)(c + 192);
        float d = h16(c + 208);
        for (int n = 0; n < 2; n++)
          for (int l = 0; l < 32; l++) {
            int lo = n * 64 + l;
            uint8_t hi = qh[n * 32 + l];
            int si = n * 8 + l / 16;
            uint8_t q[4] = {
                (uint8_t)((ql[lo] & 15) | ((hi & 3) << 4)),
                (uint8_t)((ql[lo + 32] & 15) | (((hi >> 2) & 3) << 4)),
                (uint8_t)((ql[lo] >> 4) | (((hi >> 4) & 3) << 4)),
                (uint8_t)((ql[lo + 32] >> 4) | (((hi >> 6) & 3) << 4)),
            };
            for (int j = 0; j < 4; j++)
              o[n * 128 + j * 32 + l] = d * (float)sc[si + j * 2] * ((float)q[j] - 32.f);
          }
      } break;
    }
  }
  return 0;
}

/* ---- GGUF container (src/gguf.rs:22-180) ---- */

typedef struct {
  char* key;
  uint32_t type;
  double num;
  char* str;
} or_kv;

typedef struct {
  char* name;
  uint64_t dims[4];
  int nd;
  uint32_t kind;
  uint64_t offset, len;
} or_tinfo;

typedef struct {
  const uint8_t* b;
  size_t n, p;
  or_kv* kv;
  size_t nkv;
  or_tinfo* t;
  size_t nt;
  char* err;
  size_t errlen;
} or_gguf;

static int fail(or_gguf* g, const char* fmt, ...) {
  if (g->err && g->errlen) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g->err, g->errlen, fmt, ap);
    va_end(ap);
  }
  return -1;
}

/* Reader::take (src/gguf.rs:27-32) */
static int take(or_gguf* g, size_t k, const uint8_t** out) {
  if (g->p + k < g->p) return fail(g, "GGUF length overflow");
  if (g->p + k > g->n) return fail(g, "truncated GGUF");
  *out = g->b + g->p;
  g->p += k;
  return 0;
}
static int rd_u32(or_gguf* g, uint32_t* v) {
  const uint8_t* s = NULL;
  if (take(g, 4, &s)) return -1;
  memcpy(v, s, 4);
  return 0;
}
static int rd_u64(or_gguf* g, uint64_t* v) {
  const uint8_t* s = NULL;
  if (take(g, 8, &s)) return -1;
  memcpy(v, s, 8);
  return 0;
}
static int utf8_ok(const uint8_t* s, size_t n) {
  size_t i = 0;
  while (i < n) {
    uint8_t c = s[i];
    size_t k;
    uint32_t cp;
    if (c < 0x80) { i++; continue; }
    if ((c & 0xe0) == 0xc0) { k = 1; cp = c & 0x1f; }
    else if ((c & 0xf0) == 0xe0) { k = 2; cp = c & 0x0f; }
    else if ((c & 0xf8) == 0xf0) { k = 3; cp = c & 0x07; }
    else return 0;
    if (i + k >= n) return 0;
    for (size_t j = 1; j <= k; j++) {
      if ((s[i + j] & 0xc0) != 0x80) return 0;
      cp = (cp << 6) | (s[i + j] & 0x3f);
    }
    if ((k == 1 && cp < 0x80) || (k == 2 && cp < 0x800) || (k == 3 && cp < 0x10000) ||
        cp > 0x10ffff || (cp >= 0xd800 && cp <= 0xdfff))
      return 0;
    i += k + 1;
  }
  return 1;
}
/* Reader::string (src/gguf.rs:39-47) */
static int rd_str(or_gguf* g, char** out) {
  uint64_t n;
  const uint8_t* s = NULL;
  if (rd_u64(g, &n)) return -1;
  if (n > 32u * 1024 * 1024) return fail(g, "GGUF string too large");
  if (take(g, (size_t)n, &s)) return -1;
  if (!utf8_ok(s, (size_t)n)) return fail(g, "invalid GGUF UTF-8");
  if (out) {
    *out = (char*)malloc((size_t)n + 1);
    memcpy(*out, s, (size_t)n);
    (*out)[n] = 0;
  }
  return 0;
}
/* Reader::value (src/gguf.rs:48-79); scalars become doubles, strings are kept,
 * array elements are validated and skipped. */
static int rd_value(or_gguf* g, uint32_t t, int depth, double* num, char** str) {
  const uint8_t* s = NULL;
  if (depth > 4) return fail(g, "GGUF metadata nesting too deep");
  *num = 0;
  switch (t) {
    case 0: if (take(g, 1, &s)) return -1; *num = s[0]; return 0;
    case 1: if (take(g, 1, &s)) return -1; *num = (int8_t)s[0]; return 0;
    case 2: { uint16_t v; if (take(g, 2, &s)) return -1; memcpy(&v, s, 2); *num = v; return 0; }
    case 3: { int16_t v; if (take(g, 2, &s)) return -1; memcpy(&v, s, 2); *num = v; return 0; }
    case 4: { uint32_t v; if (rd_u32(g, &v)) return -1; *num = v; return 0; }
    case 5: { uint32_t v; if (rd_u32(g, &v)) return -1; *num = (int32_t)v; return 0; }
    case 6: { uint32_t v; float f; if (rd_u32(g, &v)) return -1; memcpy(&f, &v, 4); *num = f; return 0; }
    case 7: if (take(g, 1, &s)) return -1; *num = s[0] != 0; return 0;
    case 8: return rd_str(g, str);
    case 9: {
      uint32_t et;
      uint64_t n;
      if (rd_u32(g, &et) || rd_u64(g, &n)) return -1;
      if (n > 1000000) return fail(g, "GGUF array too large");
      for (uint64_t i = 0; i < n; i++) {
        double d;
        char* x = NULL;
        if (rd_value(g, et, depth + 1, &d, &x)) return -1;
        free(x);
      }
      *num = (double)n;
      return 0;
    }
    case 10: { uint64_t v; if (rd_u64(g, &v)) return -1; *num = (double)v; return 0; }
    case 11: { uint64_t v; if (rd_u64(g, &v)) return -1; *num = (double)(int64_t)v; return 0; }
    case 12: { uint64_t v; double d; if (rd_u64(g, &v)) return -1; memcpy(&d, &v, 8); *num = d; return 0; }
    default: return fail(g, "unsupported GGUF metadata type %u", t);
  }
}

static void gguf_free(or_gguf* g) {
  for (size_t i = 0; i < g->nkv; i++) { free(g->kv[i].key); free(g->kv[i].str); }
  for (size_t i = 0; i < g->nt; i++) free(g->t[i].name);
  free(g->kv);
  free(g->t);
}

static const or_kv* gguf_kv(const or_gguf* g, const char* key) {
  for (size_t i = 0; i < g->nkv; i++)
    if (!strcmp(g->kv[i].key, key)) return &g->kv[i];
  return NULL;
}

/* Gguf::open (src/gguf.rs:95-180) */
static int gguf_parse(or_gguf* g) {
  const uint8_t* s = NULL;
  uint32_t ver;
  uint64_t nt, nk;
  if (take(g, 4, &s)) return -1;
  if (memcmp(s, "GGUF", 4)) return fail(g, "not a GGUF file");
  if (rd_u32(g, &ver)) return -1;
  if (ver != 3) return fail(g, "expected GGUF version 3");
  if (rd_u64(g, &nt) || rd_u64(g, &nk)) return -1;
  if (nt > 100000 || nk > 100000) return fail(g, "GGUF table too large");
  g->kv = (or_kv*)calloc(nk ? nk : 1, sizeof(or_kv));
  for (uint64_t i = 0; i < nk; i++) {
    or_kv kv = {0};
    if (rd_str(g, &kv.key)) return -1;
    g->kv[g->nkv++] = kv;
    if (rd_u32(g, &g->kv[g->nkv - 1].type)) return -1;
    if (rd_value(g, g->kv[g->nkv - 1].type, 0, &g->kv[g->nkv - 1].num, &g->kv[g->nkv - 1].str)) return -1;
    for (size_t j = 0; j + 1 < g->nkv; j++)
      if (!strcmp(g->kv[j].key, g->kv[g->nkv - 1].key)) return fail(g, "duplicate GGUF metadata key");
  }
  g->t = (or_tinfo*)calloc(nt ? nt : 1, sizeof(or_tinfo));
  for (uint64_t i = 0; i < nt; i++) {
    or_tinfo* t = &g->t[g->nt];
    uint32_t nd;
    uint64_t count = 1;
    int block, size;
    memset(t, 0, sizeof(*t));
    if (rd_str(g, &t->name)) return -1;
    g->nt++;
    if (rd_u32(g, &nd)) return -1;
    if (nd < 1 || nd > 4) return fail(g, "invalid tensor rank");
    t->nd = (int)nd;
    for (uint32_t k = 0; k < nd; k++) {
      uint64_t d;
      if (rd_u64(g, &d)) return -1;
      if (d == 0) return fail(g, "empty tensor");
      if (count > UINT64_MAX / d) return fail(g, "tensor size overflow");
      count *= d;
      t->dims[k] = d;
    }
    if (rd_u32(g, &t->kind) || rd_u64(g, &t->offset)) return -1;
    if (or_layout(t->kind, &block, &size))
      return fail(g, "unsupported GGML tensor type %u; supported F32/F16/Q4_0/Q8_0/Q4_K/Q6_K", t->kind);
    if (t->dims[0] % (uint64_t)block) return fail(g, "invalid quantized row alignment");
    if (count / (uint64_t)block > UINT64_MAX / (uint64_t)size) return fail(g, "tensor byte size overflow");
    t->len = count / (uint64_t)block * (uint64_t)size;
    for (size_t j = 0; j + 1 < g->nt; j++)
      if (!strcmp(g->t[j].name, t->name)) return fail(g, "duplicate tensor");
  }
  uint64_t align = 32;
  const or_kv* a = gguf_kv(g, "general.alignment");
  if (a) align = (uint64_t)a->num;
  if (align == 0 || (align & (align - 1)) || align > 4096) return fail(g, "invalid GGUF alignment");
  uint64_t base = ((uint64_t)g->p + align - 1) & ~(align - 1);
  for (size_t i = 0; i < g->nt; i++) {
    or_tinfo* t = &g->t[i];
    if (t->offset % align) return fail(g, "unaligned GGUF tensor");
    if (t->offset + base < t->offset) return fail(g, "offset overflow");
    t->offset += base;
    if (t->offset + t->len < t->offset) return fail(g, "length overflow");
    if (t->offset + t->len > g->n) return fail(g, "truncated tensor data");
  }
  return 0;
}

int or_gguf_check(const uint8_t* bytes, size_t n, char* err, size_t errlen) {
  or_gguf g = {0};
  g.b = bytes;
  g.n = n;
  g.err = err;
  g.errlen = errlen;
  int rc = gguf_parse(&g);
  gguf_free(&g);
  return rc;
}

/* ------------------------------------------------------------------ */
/* Kernels: src/tensor.rs                                             */
/* ------------------------------------------------------------------ */

typedef struct {
  const float *x, *w, *bias;
  float* o;
  int k, n, start, end;
} gemm_job;

/* tensor::kernel (src/tensor.rs:58-102): 4 token rows x 1 output column,
 * 8-lane FMA accumulation, in-order horizontal sum, scalar K tail, bias. */
static void* gemm_kernel(void* arg) {
  gemm_job* J = (gemm_job*)arg;
  const float *x = J->x, *w = J->w;
  int k = J->k, n = J->n;
  int r = J->start;
  while (r < J->end) {
    int nr = J->end - r < 4 ? J->end - r : 4;
    for (int c = 0; c < n; c++) {
      __m256 a[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
      int j = 0;
      while (j + 8 <= k) {
        __m256 v = _mm256_loadu_ps(w + (size_t)c * k + j);
        for (int t = 0; t < nr; t++)
          a[t] = _mm256_fmadd_ps(v, _mm256_loadu_ps(x + (size_t)(r + t) * k + j), a[t]);
        j += 8;
      }
      for (int t = 0; t < nr; t++) {
        float lanes[8];
        _mm256_storeu_ps(lanes, a[t]);
        float v = 0.f;
        for (int q = 0; q < 8; q++) v += lanes[q];
        for (int q = j; q < k; q++) v += w[(size_t)c * k + q] * x[(size_t)(r + t) * k + q];
        if (J->bias) v += J->bias[c];
        J->o[(size_t)(r + t) * n + c] = v;
      }
    }
    r += nr;
  }
  return NULL;
}

/* Matrix::apply (src/tensor.rs:10-39): count = min(threads, ceil(m/4)),
 * per = ceil(m/count) token rows per worker, disjoint output rows. */
void or_matrix_apply(const float* w, int rows, int cols, const float* x, int m,
                     const float* bias, int threads, float* out) {
  int count = (m + 3) / 4;
  if (threads < count) count = threads;
  if (count < 1) count = 1;
  int per = (m + count - 1) / count;
  gemm_job jobs[256];
  pthread_t th[256];
  if (count > 256) count = 256;
  for (int t = 0; t < count; t++) {
    int s = t * per, e = (t + 1) * per;
    if (e > m) e = m;
    if (s > m) s = m;
    jobs[t] = (gemm_job){x, w, bias, out, cols, rows, s, e};
  }
  for (int t = 1; t < count; t++) pthread_create(&th[t], NULL, gemm_kernel, &jobs[t]);
  gemm_kernel(&jobs[0]);
  for (int t = 1; t < count; t++) pthread_join(th[t], NULL);
}

/* tensor::softmax (src/tensor.rs:132-140) */
void or_softmax(const float* x, int n, float* p) {
  float m = -INFINITY;
  for (int i = 0; i < n; i++) m = fmaxf(m, x[i]);
  float sum = 0.f;
  for (int i = 0; i < n; i++) {
    p[i] = expf(x[i] - m);
    sum += p[i];
  }
  for (int i = 0; i < n; i++) p[i] /= sum;
}

/* tensor::dot (src/tensor.rs:193-195) */
static float dotf(const float* a, const float* b, int n) {
  float s = 0.f;
  for (int i = 0; i < n; i++) s += a[i] * b[i];
  return s;
}

/* decision::confidence (src/models/laya/decision.rs:155-167) */
float or_confidence(const float* p, int n) {
  if (n < 2) return 1.f;
  double e = 0;
  for (int i = 0; i < n; i++) {
    double x = (double)p[i] > 1e-12 ? (double)p[i] : 1e-12;
    e += x * log(x);
  }
  e = -e;
  double c = 1. - e / log((double)n);
  if (c < 0) c = 0;
  if (c > 1) c = 1;
  return (float)c;
}

/* ------------------------------------------------------------------ */
/* Decoder: src/models/openthai/model.rs with Llama/Qwen2 conventions  */
/* ------------------------------------------------------------------ */

typedef struct {
  float *attn_norm, *ffn_norm;
  float *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  float *bq, *bk, *bv;
} or_layer;

struct or_model {
  or_gguf g;
  int d, L, V, H, KV, hd, ffn, threads, ctx;
  int attn_threads; /* 1 = the reference's single-threaded attention loop */
  float eps, theta;
  const uint8_t* embd;
  uint32_t embd_kind;
  or_layer* layer;
  float* out_norm;
  float* head; /* V x d */
  float temperature[3];
  int has_bucket[3][4];
  float bucket[3][4];
};

static const or_tinfo* find_t(const or_gguf* g, const char* name) {
  for (size_t i = 0; i < g->nt; i++)
    if (!strcmp(g->t[i].name, name)) return &g->t[i];
  return NULL;
}

static float* load_f32(or_model* m, const char* name, uint64_t d0, uint64_t d1, int required, int* bad) {
  const or_tinfo* t = find_t(&m->g, name);
  if (!t) {
    if (required) {
      fail(&m->g, "missing tensor %s", name);
      *bad = 1;
    }
    return NULL;
  }
  uint64_t count = 1;
  for (int i = 0; i < t->nd; i++) count *= t->dims[i];
  if (t->dims[0] != d0 || count != d0 * d1) {
    fail(&m->g, "%s: unexpected shape", name);
    *bad = 1;
    return NULL;
  }
  float* out = (float*)malloc(sizeof(float) * (size_t)count);
  or_decode(t->kind, m->g.b + t->offset, (size_t)t->len, out);
  return out;
}

static double meta_num(const or_gguf* g, const char* arch, const char* k, double def) {
  char key[256];
  snprintf(key, sizeof key, "%s.%s", arch, k);
  const or_kv* kv = gguf_kv(g, key);
  return kv ? kv->num : def;
}

/* Minimal JSON number list / object parser for laya.temperature metadata
 * (src/models/laya/decision.rs:181-213). */
static void parse_temperature(or_model* m) {
  for (int i = 0; i < 3; i++) m->temperature[i] = 1.f;
  memset(m->has_bucket, 0, sizeof m->has_bucket);
  const or_kv* t = gguf_kv(&m->g, "laya.temperature");
  if (t && t->str) {
    const char* s = strchr(t->str, '[');
    for (int i = 0; s && i < 3; i++) {
      char* e;
      double v = strtod(s + 1, &e);
      if (e == s + 1) break;
      m->temperature[i] = (float)v;
      s = strchr(e, ',');
    }
  }
  const or_kv* b = gguf_kv(&m->g, "laya.temperature_by_options");
  if (b && b->str) {
    static const char* kinds[3] = {"choice", "score", "noul"};
    static const char* buckets[4] = {"2", "3-5", "6-10", "11+"};
    for (int k = 0; k < 3; k++)
      for (int j = 0; j < 4; j++) {
        char key[32];
        snprintf(key, sizeof key, "\"%s:%s\"", kinds[k], buckets[j]);
        const char* p = strstr(b->str, key);
        if (!p) continue;
        p = strchr(p + strlen(key), ':');
        if (!p) continue;
        m->bucket[k][j] = (float)strtod(p + 1, NULL);
        m->has_bucket[k][j] = 1;
      }
  }
}

or_model* or_model_load(const uint8_t* bytes, size_t n, int threads, char* err, size_t errlen) {
  or_model* m = (or_model*)calloc(1, sizeof(or_model));
  m->g.b = bytes;
  m->g.n = n;
  m->g.err = err;
  m->g.errlen = errlen;
  m->threads = threads < 1 ? 1 : threads;
  m->attn_threads = 1;
  if (gguf_parse(&m->g)) goto bad;
  const or_kv* arch = gguf_kv(&m->g, "general.architecture");
  if (!arch || !arch->str || (strcmp(arch->str, "llama") && strcmp(arch->str, "qwen2"))) {
    fail(&m->g, "unsupported GGUF architecture %s", arch && arch->str ? arch->str : "");
    goto bad;
  }
  const char* a = arch->str;
  m->L = (int)meta_num(&m->g, a, "block_count", 0);
  m->d = (int)meta_num(&m->g, a, "embedding_length", 0);
  m->H = (int)meta_num(&m->g, a, "attention.head_count", 0);
  m->KV = (int)meta_num(&m->g, a, "attention.head_count_kv", m->H);
  m->ffn = (int)meta_num(&m->g, a, "feed_forward_length", 0);
  m->eps = (float)meta_num(&m->g, a, "attention.layer_norm_rms_epsilon", 1e-5);
  m->theta = (float)meta_num(&m->g, a, "rope.freq_base", 10000.);
  m->ctx = (int)meta_num(&m->g, a, "context_length", 4096);
  if (m->L < 1 || m->d < 1 || m->H < 1 || m->KV < 1 || m->H % m->KV || m->d % m->H || m->ffn < 1) {
    fail(&m->g, "invalid decoder hyperparameters");
    goto bad;
  }
  m->hd = m->d / m->H;
  const or_tinfo* e = find_t(&m->g, "token_embd.weight");
  if (!e || e->dims[0] != (uint64_t)m->d || e->nd != 2) {
    fail(&m->g, "missing or malformed token_embd.weight");
    goto bad;
  }
  m->V = (int)e->dims[1];
  m->embd = m->g.b + e->offset;
  m->embd_kind = e->kind;
  m->layer = (or_layer*)calloc((size_t)m->L, sizeof(or_layer));
  int bad = 0;
  int qd = m->H * m->hd, kd = m->KV * m->hd;
  for (int l = 0; l < m->L && !bad; l++) {
    char nm[128];
    or_layer* y = &m->layer[l];
#define LOADT(field, tail, d0, d1, req) \
  snprintf(nm, sizeof nm, "blk.%d.%s", l, tail); \
  y->field = load_f32(m, nm, d0, d1, req, &bad);
    LOADT(attn_norm, "attn_norm.weight", m->d, 1, 1);
    LOADT(ffn_norm, "ffn_norm.weight", m->d, 1, 1);
    LOADT(wq, "attn_q.weight", m->d, qd, 1);
    LOADT(wk, "attn_k.weight", m->d, kd, 1);
    LOADT(wv, "attn_v.weight", m->d, kd, 1);
    LOADT(wo, "attn_output.weight", qd, m->d, 1);
    LOADT(wg, "ffn_gate.weight", m->d, m->ffn, 1);
    LOADT(wu, "ffn_up.weight", m->d, m->ffn, 1);
    LOADT(wd, "ffn_down.weight", m->ffn, m->d, 1);
    LOADT(bq, "attn_q.bias", qd, 1, 0);
    LOADT(bk, "attn_k.bias", kd, 1, 0);
    LOADT(bv, "attn_v.bias", kd, 1, 0);
#undef LOADT
  }
  if (bad) goto bad;
  m->out_norm = load_f32(m, "output_norm.weight", m->d, 1, 1, &bad);
  m->head = load_f32(m, "output.weight", m->d, m->V, 1, &bad);
  if (bad) goto bad;
  parse_temperature(m);
  return m;
bad:
  or_model_free(m);
  return NULL;
}

void or_model_free(or_model* m) {
  if (!m) return;
  if (m->layer)
    for (int l = 0; l < m->L; l++) {
      or_layer* y = &m->layer[l];
      free(y->attn_norm); free(y->ffn_norm); free(y->wq); free(y->wk); free(y->wv); free(y->wo);
      free(y->wg); free(y->wu); free(y->wd); free(y->bq); free(y->bk); free(y->bv);
    }
  free(m->layer);
  free(m->out_norm);
  free(m->head);
  gguf_free(&m->g);
  free(m);
}

int or_model_dim(const or_model* m, int what) {
  switch (what) {
    case 0: return m->d;
    case 1: return m->L;
    case 2: return m->V;
    case 3: return m->H;
    case 4: return m->KV;
    case 5: return m->hd;
    case 6: return m->ffn;
    case 7: return m->ctx;
  }
  return -1;
}

/* rms (src/models/openthai/model.rs:84-94) with offset 0 and eps from GGUF */
static void rms(const float* x, const float* w, int d, int rows, float eps, float* y) {
  for (int r = 0; r < rows; r++) {
    const float* a = x + (size_t)r * d;
    float scale = 1.f / sqrtf(dotf(a, a, d) / (float)d + eps);
    for (int j = 0; j < d; j++) y[(size_t)r * d + j] = a[j] * scale * w[j];
  }
}

/* Rotate-half RoPE over the full head (src/tensor.rs:158-171; angle formula
 * src/models/openthai/model.rs:264 with rotary dim = head_dim): rope_at. */
static float silu(float x) { return x * (1.f / (1.f + expf(-x))); }

/* K/V of every processed token per layer (post-RoPE K), so a sequence can
 * be extended token by token.  Every row of the forward depends only on its
 * own token and the keys at or before it, and Matrix::apply computes each
 * token row on its own (src/tensor.rs:58-102: a row's lanes and sum order do
 * not depend on which rows share its block), so extending a cached prefix
 * gives the same bits as recomputing the whole sequence. */
struct or_cache {
  int cap, n;
  float *k, *v; /* [L][cap][kd] */
};

or_cache* or_cache_new(const or_model* m, int cap) {
  if (cap < 1 || cap > m->ctx) return NULL;
  or_cache* c = (or_cache*)calloc(1, sizeof(or_cache));
  size_t kd = (size_t)m->KV * m->hd;
  c->cap = cap;
  c->k = (float*)malloc(sizeof(float) * (size_t)m->L * cap * kd);
  c->v = (float*)malloc(sizeof(float) * (size_t)m->L * cap * kd);
  if (!c->k || !c->v) {
    or_cache_free(c);
    return NULL;
  }
  return c;
}

void or_cache_free(or_cache* c) {
  if (!c) return;
  free(c->k);
  free(c->v);
  free(c);
}

int or_cache_len(const or_cache* c) { return c->n; }

int or_cache_truncate(or_cache* c, int n) {
  if (n < 0 || n > c->n) return -1;
  c->n = n;
  return 0;
}

/* Causal GQA attention (src/models/openthai/model.rs:276-294) of s new rows
 * at positions pos0..pos0+s-1 over keys 0..pos; the (row, head) items are
 * independent and split across threads, each computed in the same order as
 * a single-threaded loop. */
typedef struct {
  const float *q, *k, *v;
  float* att;
  int s, pos0, H, hd, qd, kd, grp, first, step;
  float scale;
} attn_job;

static void* attn_worker(void* arg) {
  attn_job* J = (attn_job*)arg;
  int keys = J->pos0 + J->s;
  float* sc = (float*)malloc(sizeof(float) * (size_t)keys);
  float* p = (float*)malloc(sizeof(float) * (size_t)keys);
  for (int it = J->first; it < J->s * J->H; it += J->step) {
    int i = it / J->H, hh = it % J->H, kh = hh / J->grp, pos = J->pos0 + i;
    for (int j = 0; j <= pos; j++)
      sc[j] = dotf(J->q + (size_t)i * J->qd + (size_t)hh * J->hd, J->k + (size_t)j * J->kd + (size_t)kh * J->hd,
                   J->hd) * J->scale;
    or_softmax(sc, pos + 1, p);
    float* o = J->att + (size_t)i * J->qd + (size_t)hh * J->hd;
    for (int z = 0; z < J->hd; z++) o[z] = 0.f;
    for (int j = 0; j <= pos; j++) {
      const float* vv = J->v + (size_t)j * J->kd + (size_t)kh * J->hd;
      for (int z = 0; z < J->hd; z++) o[z] += p[j] * vv[z];
    }
  }
  free(sc);
  free(p);
  return NULL;
}

/* Rotate-half RoPE of s rows starting at position pos0. */
static void rope_at(float* buf, int s, int pos0, int heads, int hd, float theta) {
  int half = hd / 2;
  for (int i = 0; i < s; i++)
    for (int h = 0; h < heads; h++)
      for (int j = 0; j < half; j++) {
        float angle = (float)(pos0 + i) / powf(theta, (float)(2 * j) / (float)hd);
        float co = cosf(angle), si = sinf(angle);
        size_t p = (size_t)i * heads * hd + (size_t)h * hd + j;
        float a = buf[p], b = buf[p + half];
        buf[p] = a * co - b * si;
        buf[p + half] = b * co + a * si;
      }
}

void or_model_attn_threads(or_model* m, int n) { m->attn_threads = n < 1 ? 1 : n; }

/* Timing only: marks positions 0..n-1 as cached with arbitrary K/V values
 * (a seeded pattern of small numbers), so a decode step at context n can be
 * timed without first prefilling n tokens.  Attention does the same work
 * whatever the values are; nothing computed from such a cache is checked. */
int or_cache_fill_timing(or_cache* c, const or_model* m, int n) {
  if (n < 0 || n > c->cap) return -1;
  size_t kd = (size_t)m->KV * m->hd;
  uint32_t st = 12345u;
  for (int l = 0; l < m->L; l++)
    for (size_t i = 0; i < (size_t)n * kd; i++) {
      st = st * 1664525u + 1013904223u;
      float v = (float)((st >> 9) & 1023) / 1024.f - 0.5f;
      c->k[(size_t)l * c->cap * kd + i] = v;
      c->v[(size_t)l * c->cap * kd + i] = -v;
    }
  c->n = n;
  return 0;
}

int or_cache_forward(or_model* m, or_cache* c, const int32_t* ids, int s, const int32_t* read, int nread, float* out) {
  int d = m->d, H = m->H, KV = m->KV, hd = m->hd, ffn = m->ffn;
  int qd = H * hd, kd = KV * hd, grp = H / KV;
  int block, size;
  int pos0 = c->n;
  /* Model::forward input validation (src/models/openthai/model.rs:198-204) */
  if (s < 1 || pos0 + s > c->cap || pos0 + s > m->ctx) return -1;
  for (int i = 0; i < s; i++)
    if (ids[i] < 0 || ids[i] >= m->V) return -1;
  for (int i = 0; i < nread; i++)
    if (read[i] < 0 || read[i] >= s) return -1;
  or_layout(m->embd_kind, &block, &size);
  size_t rowb = (size_t)d / (size_t)block * (size_t)size;
  float* x = (float*)malloc(sizeof(float) * (size_t)s * d);
  float* h = (float*)malloc(sizeof(float) * (size_t)s * d);
  float* q = (float*)malloc(sizeof(float) * (size_t)s * qd);
  float* att = (float*)malloc(sizeof(float) * (size_t)s * qd);
  float* y = (float*)malloc(sizeof(float) * (size_t)s * (ffn > d ? ffn : d));
  float* u = (float*)malloc(sizeof(float) * (size_t)s * ffn);
  /* embedding rows decoded per used id (src/models/openthai/model.rs:205-213) */
  for (int i = 0; i < s; i++) or_decode(m->embd_kind, m->embd + (size_t)ids[i] * rowb, rowb, x + (size_t)i * d);
  float scale = 1.f / sqrtf((float)hd); /* src/tensor.rs:174 */
  int nth = m->attn_threads < s * H ? m->attn_threads : s * H;
  if (nth > 256) nth = 256;
  for (int l = 0; l < m->L; l++) {
    or_layer* b = &m->layer[l];
    float* kl = c->k + ((size_t)l * c->cap) * kd;
    float* vl = c->v + ((size_t)l * c->cap) * kd;
    float* k = kl + (size_t)pos0 * kd;
    float* v = vl + (size_t)pos0 * kd;
    rms(x, b->attn_norm, d, s, m->eps, h);
    or_matrix_apply(b->wq, qd, d, h, s, b->bq, m->threads, q);
    or_matrix_apply(b->wk, kd, d, h, s, b->bk, m->threads, k);
    or_matrix_apply(b->wv, kd, d, h, s, b->bv, m->threads, v);
    rope_at(q, s, pos0, H, hd, m->theta);
    rope_at(k, s, pos0, KV, hd, m->theta);
    attn_job jobs[256];
    pthread_t th[256];
    for (int t = 0; t < nth; t++)
      jobs[t] = (attn_job){q, kl, vl, att, s, pos0, H, hd, qd, kd, grp, t, nth, scale};
    for (int t = 1; t < nth; t++) pthread_create(&th[t], NULL, attn_worker, &jobs[t]);
    attn_worker(&jobs[0]);
    for (int t = 1; t < nth; t++) pthread_join(th[t], NULL);
    or_matrix_apply(b->wo, d, qd, att, s, NULL, m->threads, y);
    for (size_t i = 0; i < (size_t)s * d; i++) x[i] += y[i]; /* tensor::add (src/tensor.rs:123-128) */
    rms(x, b->ffn_norm, d, s, m->eps, h);
    or_matrix_apply(b->wg, ffn, d, h, s, NULL, m->threads, y);
    or_matrix_apply(b->wu, ffn, d, h, s, NULL, m->threads, u);
    for (size_t i = 0; i < (size_t)s * ffn; i++) y[i] = silu(y[i]) * u[i];
    or_matrix_apply(b->wd, d, ffn, y, s, NULL, m->threads, u);
    for (size_t i = 0; i < (size_t)s * d; i++) x[i] += u[i];
  }
  c->n = pos0 + s;
  /* answer-position gather + final norm (src/models/openthai/model.rs:232-240) */
  for (int r = 0; r < nread; r++) memcpy(h + (size_t)r * d, x + (size_t)read[r] * d, sizeof(float) * d);
  rms(h, m->out_norm, d, nread, m->eps, out);
  free(x); free(h); free(q); free(att); free(y); free(u);
  return 0;
}

int or_forward(or_model* m, const int32_t* ids, int s, const int32_t* read, int nread, float* out) {
  if (s < 1 || s > m->ctx) return -1;
  or_cache* c = or_cache_new(m, s);
  if (!c) return -1;
  int rc = or_cache_forward(m, c, ids, s, read, nread, out);
  or_cache_free(c);
  return rc;
}

int or_head(or_model* m, const float* hidden, int rows, const int32_t* cand, int ncand, float* out) {
  int d = m->d;
  if (ncand == 0) {
    or_matrix_apply(m->head, m->V, d, hidden, rows, NULL, m->threads, out);
    return 0;
  }
  float* w = (float*)malloc(sizeof(float) * (size_t)ncand * d);
  for (int c = 0; c < ncand; c++) {
    if (cand[c] < 0 || cand[c] >= m->V) { free(w); return -1; }
    memcpy(w + (size_t)c * d, m->head + (size_t)cand[c] * d, sizeof(float) * d);
  }
  or_matrix_apply(w, ncand, d, hidden, rows, NULL, m->threads, out);
  free(w);
  return 0;
}

static float kind_temperature(const or_model* m, int kind, int k) {
  int bucket = k <= 2 ? 0 : k <= 5 ? 1 : k <= 10 ? 2 : 3;
  float t = m->has_bucket[kind][bucket] ? m->bucket[kind][bucket] : m->temperature[kind];
  return t > 1e-3f ? t : 1e-3f;
}

/* decide_with_cancel per question (src/models/laya/decision.rs:186-268) */
int or_decide(or_model* m, const int32_t* ids, int n, const or_question* q, or_answer* out) {
  int k = q->n_options, L = q->option_len, d = m->d;
  if (k < 1 || k > 16 || L < 1 || (q->kind < 0 || q->kind > 2)) return -1;
  if (q->kind == 2 && k != 2) return -1;
  int base = n + q->suffix_len;
  int total = base + L - 1;
  int32_t* seq = (int32_t*)malloc(sizeof(int32_t) * (size_t)total);
  memcpy(seq, ids, sizeof(int32_t) * (size_t)n);
  if (q->suffix_len) memcpy(seq + n, q->suffix, sizeof(int32_t) * (size_t)q->suffix_len);
  float* logits = out->logits;
  if (L == 1) {
    float* hid = (float*)malloc(sizeof(float) * d);
    int32_t rp = base - 1;
    int rc = or_forward(m, seq, base, &rp, 1, hid);
    if (!rc) rc = or_head(m, hid, 1, q->options, k, logits);
    free(hid);
    if (rc) { free(seq); return rc; }
  } else {
    /* each option is scored by the summed full-vocabulary log-probability
     * of its tokens: the shared prefix seq[0..base-1) once, then per option
     * the last prefix token and the option's first L-1 tokens appended to
     * it (the same rows as one forward over the whole sequence) */
    float* hid = (float*)malloc(sizeof(float) * (size_t)L * d);
    float* row = (float*)malloc(sizeof(float) * (size_t)L * m->V);
    int32_t* rp = (int32_t*)malloc(sizeof(int32_t) * (size_t)L);
    int32_t* tail = (int32_t*)malloc(sizeof(int32_t) * (size_t)L);
    or_cache* c = total <= m->ctx ? or_cache_new(m, total) : NULL;
    int rc0 = c ? 0 : -1;
    if (!rc0 && base > 1) rc0 = or_cache_forward(m, c, seq, base - 1, NULL, 0, NULL);
    if (rc0) { or_cache_free(c); free(hid); free(row); free(rp); free(tail); free(seq); return rc0; }
    for (int o = 0; o < k; o++) {
      const int32_t* opt = q->options + (size_t)o * L;
      tail[0] = seq[base - 1];
      for (int t = 0; t < L - 1; t++) tail[t + 1] = opt[t];
      for (int t = 0; t < L; t++) rp[t] = t;
      or_cache_truncate(c, base - 1);
      int rc = or_cache_forward(m, c, tail, L, rp, L, hid);
      if (!rc) rc = or_head(m, hid, L, NULL, 0, row);
      if (rc) { or_cache_free(c); free(hid); free(row); free(rp); free(tail); free(seq); return rc; }
      double sum = 0;
      for (int t = 0; t < L; t++) {
        const float* r = row + (size_t)t * m->V;
        float mx = -INFINITY;
        for (int c = 0; c < m->V; c++) mx = fmaxf(mx, r[c]);
        double se = 0;
        for (int c = 0; c < m->V; c++) se += exp((double)(r[c] - mx));
        sum += (double)(r[opt[t]] - mx) - log(se);
      }
      logits[o] = (float)sum;
    }
    or_cache_free(c);
    free(hid); free(row); free(rp); free(tail);
  }
  free(seq);
  for (int i = 0; i < k; i++)
    if (!isfinite(logits[i])) return -2; /* src/models/laya/model.rs:412-414 */
  float t = kind_temperature(m, q->kind, k);
  float scaled[16];
  for (int i = 0; i < k; i++) scaled[i] = logits[i] / t;
  float* p = out->probabilities;
  or_softmax(scaled, k, p);
  out->kind = q->kind;
  out->n_options = k;
  out->choice = -1;
  out->score = 0;
  out->noul = 0;
  if (q->kind == 0) {
    int best = 0; /* max_by with ties to the lowest index (decision.rs:233-235) */
    for (int i = 1; i < k; i++)
      if (p[i] > p[best]) best = i;
    out->choice = best;
  } else if (q->kind == 1) {
    double s = 0;
    for (int i = 0; i < k; i++) s += (double)i * (double)p[i];
    out->score = (float)s;
  } else {
    out->noul = p[1];
  }
  out->confidence = q->kind == 2 ? (p[1] > 1.f - p[1] ? p[1] : 1.f - p[1]) : or_confidence(p, k);
  return 0;
}
