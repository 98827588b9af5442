/* CPU oracle of the two OpenThai sequence mixers (TEST INFRASTRUCTURE ONLY).
 *
 * Restates, in F32 and in the reference's loop order, the gated full
 * attention (Full::run, src/models/openthai/model.rs:243-299) and the gated
 * DeltaNet recurrence (Delta::run, src/models/openthai/model.rs:301-363) for
 * a single sequence.  The reference fixes the shapes (hidden 1024; 8 query
 * heads of 256 with 2 KV heads and a 64-dimension rotary part; 16 DeltaNet
 * heads of 128); here they are parameters so that small cases run in tests,
 * with the same layout rules:
 *   - q_proj rows per head: [256 query | 256 gate] (model.rs:248-256);
 *   - q / k RMSNorm per head with weight offset 1 and eps 1e-6 (model.rs:84-94, 257-258);
 *   - rotate-half RoPE on the first `rot` dimensions of a head, pairs (j, j + rot/2),
 *     angle = pos / theta^(2j/rot) (model.rs:259-275);
 *   - DeltaNet in_proj_qkv rows: [q heads | k heads | v heads], each nh x hk
 *     (model.rs:329-331), causal depthwise conv of width 4 then SiLU
 *     (model.rs:309-320), per-head state [key][value] (model.rs:322-352),
 *     output RMSNorm per head with offset 0, then x SiLU(z) (model.rs:356-360).
 * The projections use or_matrix_apply (Matrix::apply, src/tensor.rs:10-39).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

static float ot_dot(const float* a, const float* b, int n) {
  float s = 0.f;
  for (int i = 0; i < n; i++) s += a[i] * b[i];
  return s;
}
static float ot_sigmoid(float x) { return 1.f / (1.f + expf(-x)); }
static float ot_silu(float x) { return x * ot_sigmoid(x); }
static float ot_softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }

/* rms (model.rs:84-94): rows of w's length d, eps 1e-6, weight offset `off` */
static void ot_rms(float* x, const float* w, int d, int rows, float off) {
  for (int r = 0; r < rows; r++) {
    float* a = x + (size_t)r * d;
    float scale = 1.f / sqrtf(ot_dot(a, a, d) / (float)d + 1e-6f);
    for (int j = 0; j < d; j++) a[j] = a[j] * scale * (off + w[j]);
  }
}

/* Gated attention after the projections (model.rs:248-296): qgate [s][H *
 * 2hd] (per head [query | gate]), k / v [s][KV * hd] -> out [s][H * hd],
 * the gated attention output before o_proj. */
int or_ot_full_core(const float* qgate, const float* kin, const float* v, const float* qn, const float* kn, int s,
                    int H, int KV, int hd, int rot, float theta, float* att) {
  if (s < 1 || H < 1 || KV < 1 || H % KV || rot > hd || rot % 2) return -1;
  const int qd = H * hd, kd = KV * hd, grp = H / KV;
  float* q = malloc(sizeof(float) * (size_t)s * qd);
  float* gate = malloc(sizeof(float) * (size_t)s * qd);
  float* k = malloc(sizeof(float) * (size_t)s * kd);
  float* sc = malloc(sizeof(float) * (size_t)s);
  float* p = malloc(sizeof(float) * (size_t)s);
  if (!q || !gate || !k || !sc || !p) return -2;
  for (int i = 0; i < s; i++)
    for (int h = 0; h < H; h++) {
      memcpy(q + (size_t)i * qd + h * hd, qgate + (size_t)i * 2 * qd + h * 2 * hd, sizeof(float) * hd);
      memcpy(gate + (size_t)i * qd + h * hd, qgate + (size_t)i * 2 * qd + h * 2 * hd + hd, sizeof(float) * hd);
    }
  ot_rms(q, qn, hd, s * H, 1.f);
  memcpy(k, kin, sizeof(float) * (size_t)s * kd);
  ot_rms(k, kn, hd, s * KV, 1.f);
  const int half = rot / 2;
  for (int pass = 0; pass < 2; pass++) {
    float* buf = pass == 0 ? q : k;
    const int heads = pass == 0 ? H : KV;
    for (int i = 0; i < s; i++)
      for (int h = 0; h < heads; h++)
        for (int j = 0; j < half; j++) {
          float angle = (float)i / powf(theta, (float)(2 * j) / (float)rot);
          float co = cosf(angle), si = sinf(angle);
          size_t o = (size_t)i * heads * hd + (size_t)h * hd + j;
          float a = buf[o], b = buf[o + half];
          buf[o] = a * co - b * si;
          buf[o + half] = b * co + a * si;
        }
  }
  const float root = sqrtf((float)hd);  /* the reference divides by 16 = sqrt(256) */
  memset(att, 0, sizeof(float) * (size_t)s * qd);
  for (int i = 0; i < s; i++)
    for (int h = 0; h < H; h++) {
      const int kh = h / grp;
      for (int j = 0; j <= i; j++)
        sc[j] = ot_dot(q + (size_t)i * qd + h * hd, k + (size_t)j * kd + kh * hd, hd) / root;
      or_softmax(sc, i + 1, p);
      for (int j = 0; j <= i; j++)
        for (int c = 0; c < hd; c++) att[(size_t)i * qd + h * hd + c] += p[j] * v[(size_t)j * kd + kh * hd + c];
    }
  for (size_t e = 0; e < (size_t)s * qd; e++) att[e] *= ot_sigmoid(gate[e]);
  free(q), free(gate), free(k), free(sc), free(p);
  return 0;
}

int or_ot_full(const float* x, int s, int d, int H, int KV, int hd, int rot, float theta, const float* wq,
               const float* wk, const float* wv, const float* wo, const float* qn, const float* kn, int threads,
               float* out) {
  if (s < 1 || H < 1 || KV < 1 || H % KV || rot > hd || rot % 2) return -1;
  const int qd = H * hd, kd = KV * hd;
  float* qgate = malloc(sizeof(float) * (size_t)s * 2 * qd);
  float* k = malloc(sizeof(float) * (size_t)s * kd);
  float* v = malloc(sizeof(float) * (size_t)s * kd);
  float* att = malloc(sizeof(float) * (size_t)s * qd);
  if (!qgate || !k || !v || !att) return -2;
  or_matrix_apply(wq, 2 * qd, d, x, s, NULL, threads, qgate);
  or_matrix_apply(wk, kd, d, x, s, NULL, threads, k);
  or_matrix_apply(wv, kd, d, x, s, NULL, threads, v);
  int rc = or_ot_full_core(qgate, k, v, qn, kn, s, H, KV, hd, rot, theta, att);
  if (!rc) or_matrix_apply(wo, d, qd, att, s, NULL, threads, out);
  free(qgate), free(k), free(v), free(att);
  return rc;
}

/* The DeltaNet recurrence alone (model.rs:322-355): qkv[s][3 nh hk] after
 * the convolution and SiLU, a / b [s][nh] projections, dt / A_log [nh];
 * out[s][nh hk] before the output norm and gate. */
int or_ot_delta_core(const float* qkv, const float* a, const float* b, const float* dt, const float* alog, int s,
                     int nh, int hk, float* o) {
  if (s < 1 || nh < 1 || hk < 1) return -1;
  const int w = nh * hk, C = 3 * w;
  float* state = malloc(sizeof(float) * (size_t)hk * hk);
  float* delta = malloc(sizeof(float) * (size_t)hk);
  if (!state || !delta) return -2;
  memset(o, 0, sizeof(float) * (size_t)s * w);
  for (int h = 0; h < nh; h++) {
    memset(state, 0, sizeof(float) * (size_t)hk * hk);
    for (int i = 0; i < s; i++) {
      const float* q = qkv + (size_t)i * C + h * hk;
      const float* k = qkv + (size_t)i * C + w + h * hk;
      const float* vv = qkv + (size_t)i * C + 2 * w + h * hk;
      const float qs = 1.f / sqrtf(ot_dot(q, q, hk) + 1e-6f) / sqrtf((float)hk);
      const float ks = 1.f / sqrtf(ot_dot(k, k, hk) + 1e-6f);
      const float decay = expf(-expf(alog[h]) * ot_softplus(a[(size_t)i * nh + h] + dt[h]));
      const float beta = ot_sigmoid(b[(size_t)i * nh + h]);
      for (int e = 0; e < hk * hk; e++) state[e] *= decay;
      memset(delta, 0, sizeof(float) * (size_t)hk);
      for (int j = 0; j < hk; j++) {
        const float key = k[j] * ks;
        for (int c = 0; c < hk; c++) delta[c] += state[(size_t)j * hk + c] * key;
      }
      for (int c = 0; c < hk; c++) delta[c] = (vv[c] - delta[c]) * beta;
      float* oo = o + (size_t)i * w + h * hk;
      for (int j = 0; j < hk; j++) {
        const float key = k[j] * ks, query = q[j] * qs;
        for (int c = 0; c < hk; c++) {
          state[(size_t)j * hk + c] += key * delta[c];
          oo[c] += state[(size_t)j * hk + c] * query;
        }
      }
    }
  }
  free(state), free(delta);
  return 0;
}

/* Delta::run after its projections (model.rs:309-360): raw [s][3w] from
 * in_proj_qkv, z [s][w], a / b [s][nh] -> out [s][w] (w = nh hk) before
 * out_proj: causal width-4 convolution + SiLU, the recurrence, per-head
 * RMSNorm (offset 0) and x SiLU(z). */
int or_ot_delta_mid(const float* raw, const float* z, const float* a, const float* b, const float* conv,
                    const float* dt, const float* alog, const float* normw, int s, int nh, int hk, float* o) {
  if (s < 1 || nh < 1 || hk < 1) return -1;
  const int w = nh * hk, C = 3 * w;
  float* qkv = malloc(sizeof(float) * (size_t)s * C);
  if (!qkv) return -2;
  /* causal depthwise conv (width 4) + SiLU */
  for (int i = 0; i < s; i++)
    for (int c = 0; c < C; c++) {
      float acc = 0.f;
      for (int j = 0; j < 4; j++)
        if (i + j >= 3) acc += raw[(size_t)(i + j - 3) * C + c] * conv[(size_t)c * 4 + j];
      qkv[(size_t)i * C + c] = ot_silu(acc);
    }
  int rc = or_ot_delta_core(qkv, a, b, dt, alog, s, nh, hk, o);
  free(qkv);
  if (rc) return rc;
  ot_rms(o, normw, hk, s * nh, 0.f);
  for (size_t e = 0; e < (size_t)s * w; e++) o[e] *= ot_silu(z[e]);
  return 0;
}

int or_ot_delta(const float* x, int s, int d, int nh, int hk, const float* wqkv, const float* wz, const float* wa,
                const float* wb, const float* wo, const float* conv, const float* dt, const float* alog,
                const float* normw, int threads, float* out) {
  if (s < 1 || nh < 1 || hk < 1) return -1;
  const int w = nh * hk, C = 3 * w;
  float* raw = malloc(sizeof(float) * (size_t)s * C);
  float* z = malloc(sizeof(float) * (size_t)s * w);
  float* a = malloc(sizeof(float) * (size_t)s * nh);
  float* b = malloc(sizeof(float) * (size_t)s * nh);
  float* o = malloc(sizeof(float) * (size_t)s * w);
  if (!raw || !z || !a || !b || !o) return -2;
  or_matrix_apply(wqkv, C, d, x, s, NULL, threads, raw);
  or_matrix_apply(wz, w, d, x, s, NULL, threads, z);
  or_matrix_apply(wa, nh, d, x, s, NULL, threads, a);
  or_matrix_apply(wb, nh, d, x, s, NULL, threads, b);
  int rc = or_ot_delta_mid(raw, z, a, b, conv, dt, alog, normw, s, nh, hk, o);
  if (!rc) or_matrix_apply(wo, d, w, o, s, NULL, threads, out);
  free(raw), free(z), free(a), free(b), free(o);
  return rc;
}
