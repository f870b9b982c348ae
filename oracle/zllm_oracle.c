/*
 * zllm_oracle.c -- TEST INFRASTRUCTURE ONLY (see zllm_oracle.h).
 *
 * A C restatement of the zerollm reference's single-thread plain-JS oracle.  Each function
 * cites the reference file:line it follows.  JS Numbers are IEEE doubles: every expression
 * below is evaluated in double in the JS evaluation order, and every store into a typed
 * array applies the same conversion the typed array applies (f32 round-to-nearest for
 * Float32Array, modular ToInt8 / ToInt32 for Int8Array / Int32Array).
 *
 * Known deviation: Math.exp / Math.cos / Math.sin / Math.pow in V8 are fdlibm ports; this file
 * calls the C library's exp / cos / sin / pow.  Both are faithfully rounded (< 1 ulp); a last-bit
 * difference in a double result changes a stored f32 only when it straddles an f32 rounding
 * boundary.
 */
#include "zllm_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK 32

/* ------------------------------------------------------------------ JS typed-array conversions */
static int32_t js_to_int32(double v) {          /* ECMAScript ToInt32 */
  if (!isfinite(v)) return 0;
  double t = trunc(v);
  double m = fmod(t, 4294967296.0);
  if (m < 0) m += 4294967296.0;
  uint32_t u = (uint32_t)m;
  return (int32_t)u;
}
static int8_t js_to_int8(double v) { return (int8_t)(uint8_t)(uint32_t)js_to_int32(v); }
/* Math.round: nearest integer, ties toward +infinity.  Only called on v >= 0 or NaN here. */
static double js_round_nonneg(double v) {
  if (!(v == v)) return v;
  double f = floor(v);
  double diff = v - f;                 /* exact for |v| < 2^52 */
  return diff >= 0.5 ? f + 1.0 : f;
}

/* ------------------------------------------------------------------ f16 (src/util/f16.js) */
uint16_t zo_f32_to_f16(float x) {            /* f16.js:7-30 */
  uint32_t b; memcpy(&b, &x, 4);
  uint32_t sign = (b >> 16) & 0x8000u;
  int32_t exp = (int32_t)((b >> 23) & 0xffu);
  uint32_t mant = b & 0x7fffffu;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
  exp = exp - 127 + 15;
  if (exp >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    uint32_t m = mant | 0x800000u;
    int shift = 14 - exp;
    uint32_t half = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (half & 1u))) half++;
    return (uint16_t)(sign | half);
  }
  uint32_t half = sign | ((uint32_t)exp << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;
  return (uint16_t)half;
}

float zo_f16_to_f32(uint16_t h) {            /* f16.js:33-40 (values; the table holds them as f32) */
  double sign = (h & 0x8000u) ? -1.0 : 1.0;
  int exp = (h >> 10) & 0x1f;
  int mant = h & 0x3ff;
  if (exp == 0) return (float)(sign * mant * ldexp(1.0, -24));
  if (exp == 0x1f) return mant ? NAN : (float)(sign * INFINITY);
  return (float)(sign * (1.0 + mant / 1024.0) * ldexp(1.0, exp - 15));
}

float zo_bf16_to_f32(uint16_t h) { uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f; }

static float F16TAB[65536];
static int f16tab_ready = 0;
static void f16tab_init(void) {
  if (f16tab_ready) return;
  for (int i = 0; i < 65536; i++) F16TAB[i] = zo_f16_to_f32((uint16_t)i);
  f16tab_ready = 1;
}
static inline double H(const uint8_t *p) { return (double)F16TAB[p[0] | (p[1] << 8)]; }

/* ------------------------------------------------------------------ sizes */
int64_t zo_row_bytes(int type, int64_t cols) {     /* ref-kernels.js:65-77 */
  switch (type) {
    case ZO_F32: return cols * 4;
    case ZO_F16: case ZO_BF16: return cols * 2;
    case ZO_Q8_0: return cols % QK ? -1 : (cols / QK) * 34;
    case ZO_Q4_0: return cols % QK ? -1 : (cols / QK) * 18;
    case ZO_Q5_0: return cols % QK ? -1 : (cols / QK) * 22;
    case ZO_Q4_K: return cols % 256 ? -1 : (cols / 256) * 144;
    case ZO_Q5_K: return cols % 256 ? -1 : (cols / 256) * 176;
    case ZO_Q6_K: return cols % 256 ? -1 : (cols / 256) * 210;
    default: return -1;
  }
}

void zo_unpack_scale_min_k4(const uint8_t *q, int32_t *sc, int32_t *mn) {   /* quant.js:109-118 */
  for (int j = 0; j < 4; j++) {
    sc[j] = q[j] & 63;
    mn[j] = q[j + 4] & 63;
    sc[j + 4] = (q[j + 8] & 0x0f) | ((q[j] >> 6) << 4);
    mn[j + 4] = (q[j + 8] >> 4) | ((q[j + 4] >> 6) << 4);
  }
}

/* ------------------------------------------------------------------ activation quantization */
void zo_quantize_act(const float *x, int64_t n, int8_t *q, float *d, int32_t *s) {  /* ref-kernels.js:44-62 */
  int64_t nb = n / QK;
  for (int64_t b = 0; b < nb; b++) {
    int64_t o = b * QK;
    double amax = 0;
    for (int i = 0; i < QK; i++) { double a = fabs((double)x[o + i]); if (a > amax) amax = a; }
    double scale = amax / 127;
    d[b] = (float)scale;
    double inv = scale != 0 ? 1 / scale : 0;   /* NaN scale is impossible: amax never takes a NaN */
    double sum = 0;
    for (int i = 0; i < QK; i++) {
      double v = (double)x[o + i] * inv;
      double r = v < 0 ? -js_round_nonneg(-v) : js_round_nonneg(v);
      q[o + i] = js_to_int8(r);
      sum += r;
    }
    if (s) s[b] = js_to_int32(sum);
  }
}

/* ------------------------------------------------------------------ dequantization */
int zo_dequant_row(int type, const uint8_t *w, int64_t cols, int64_t row, float *out) {  /* ref-kernels.js:80-120 */
  f16tab_init();
  int64_t rb = zo_row_bytes(type, cols);
  if (rb < 0) return -1;
  const uint8_t *p = w + row * rb;
  switch (type) {
    case ZO_F32: for (int64_t i = 0; i < cols; i++) memcpy(&out[i], p + 4 * i, 4); return 0;
    case ZO_F16: for (int64_t i = 0; i < cols; i++) out[i] = F16TAB[p[2 * i] | (p[2 * i + 1] << 8)]; return 0;
    case ZO_BF16: for (int64_t i = 0; i < cols; i++) out[i] = zo_bf16_to_f32((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8))); return 0;
    case ZO_Q8_0:
      for (int64_t b = 0; b < cols / QK; b++) {
        const uint8_t *o = p + b * 34; double dd = H(o);
        for (int i = 0; i < QK; i++) out[b * QK + i] = (float)(dd * (double)(int8_t)o[2 + i]);
      }
      return 0;
    case ZO_Q4_0:
      for (int64_t b = 0; b < cols / QK; b++) {
        const uint8_t *o = p + b * 18; double dd = H(o);
        for (int j = 0; j < 16; j++) {
          int byte = o[2 + j];
          out[b * QK + j] = (float)(dd * ((byte & 0x0f) - 8));
          out[b * QK + j + 16] = (float)(dd * ((byte >> 4) - 8));
        }
      }
      return 0;
    case ZO_Q5_0:                                   /* quant.js:121-135 */
      for (int64_t b = 0; b < cols / QK; b++) {
        const uint8_t *o = p + b * 22; double dd = H(o);
        uint32_t qh = (uint32_t)o[2] | ((uint32_t)o[3] << 8) | ((uint32_t)o[4] << 16) | ((uint32_t)o[5] << 24);
        for (int j = 0; j < 16; j++) {
          int byte = o[6 + j];
          out[b * 32 + j] = (float)(dd * ((int)((byte & 0x0f) | (((qh >> j) & 1u) << 4)) - 16));
          out[b * 32 + j + 16] = (float)(dd * ((int)((byte >> 4) | (((qh >> (j + 16)) & 1u) << 4)) - 16));
        }
      }
      return 0;
    case ZO_Q4_K: case ZO_Q5_K: {                   /* quant.js:138-175 */
      int five = type == ZO_Q5_K; int bs = five ? 176 : 144; int qs = five ? 48 : 16;
      for (int64_t b = 0; b < cols / 256; b++) {
        const uint8_t *o = p + b * bs;
        double dd = H(o), dmin = H(o + 2);
        int32_t sc[8], mn[8]; zo_unpack_scale_min_k4(o + 4, sc, mn);
        for (int s = 0; s < 8; s++) {
          int chunk = s >> 1, hi = s & 1;
          for (int l = 0; l < 32; l++) {
            int byte = o[qs + chunk * 32 + l];
            int v = hi ? byte >> 4 : byte & 0x0f;
            if (five) v |= ((o[16 + l] >> s) & 1) << 4;
            out[b * 256 + s * 32 + l] = (float)(dd * sc[s] * v - dmin * mn[s]);
          }
        }
      }
      return 0;
    }
    case ZO_Q6_K:                                   /* quant.js:178-202 */
      for (int64_t b = 0; b < cols / 256; b++) {
        const uint8_t *o = p + b * 210;
        double dd = H(o + 208);
        for (int half = 0; half < 2; half++) {
          const uint8_t *ql = o + 64 * half, *qh = o + 128 + 32 * half; const int8_t *sc = (const int8_t *)(o + 192 + 8 * half);
          for (int l = 0; l < 32; l++) {
            int h = qh[l];
            int q1 = ((ql[l] & 0x0f) | (((h >> 0) & 3) << 4)) - 32;
            int q2 = ((ql[l + 32] & 0x0f) | (((h >> 2) & 3) << 4)) - 32;
            int q3 = ((ql[l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
            int q4 = ((ql[l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32;
            int g = l >> 4;
            int64_t e = b * 256 + half * 128;
            out[e + l] = (float)(dd * sc[g] * q1);
            out[e + l + 32] = (float)(dd * sc[g + 2] * q2);
            out[e + l + 64] = (float)(dd * sc[g + 4] * q3);
            out[e + l + 96] = (float)(dd * sc[g + 6] * q4);
          }
        }
      }
      return 0;
    default: return -1;
  }
}

/* ------------------------------------------------------------------ matvec (ref-kernels.js:127-302) */
static float row_dot(int type, const uint8_t *u8, int64_t cols, int64_t r, const float *x,
                     const int8_t *xq, const float *xd, const int32_t *xs, float *tmp) {
  const int64_t nb = cols / QK;
  switch (type) {
    case ZO_Q8_0: {                                   /* :132-152 */
      const uint8_t *o = u8 + r * nb * 34; double acc = 0;
      for (int64_t b = 0; b < nb; b++, o += 34) {
        const int8_t *w = (const int8_t *)(o + 2); const int8_t *a = xq + b * QK;
        int32_t s = 0;
        for (int i = 0; i < QK; i++) s += w[i] * a[i];
        acc += (double)s * H(o) * (double)xd[b];
      }
      return (float)acc;
    }
    case ZO_Q4_0: {                                   /* :153-173 */
      const uint8_t *o = u8 + r * nb * 18; double acc = 0;
      for (int64_t b = 0; b < nb; b++, o += 18) {
        const int8_t *a = xq + b * QK; int32_t s = 0;
        for (int j = 0; j < 16; j++) { int byte = o[2 + j]; s += ((byte & 0x0f) - 8) * a[j] + ((byte >> 4) - 8) * a[j + 16]; }
        acc += (double)s * H(o) * (double)xd[b];
      }
      return (float)acc;
    }
    case ZO_Q5_0: {                                   /* :174-195 */
      const uint8_t *o = u8 + r * nb * 22; double acc = 0;
      for (int64_t b = 0; b < nb; b++, o += 22) {
        const int8_t *a = xq + b * QK;
        uint32_t qh = (uint32_t)o[2] | ((uint32_t)o[3] << 8) | ((uint32_t)o[4] << 16) | ((uint32_t)o[5] << 24);
        int32_t s = 0;
        for (int j = 0; j < 16; j++) {
          int byte = o[6 + j];
          s += ((int)((byte & 0x0f) | (((qh >> j) & 1u) << 4)) - 16) * a[j] + ((int)((byte >> 4) | (((qh >> (j + 16)) & 1u) << 4)) - 16) * a[j + 16];
        }
        acc += (double)s * H(o) * (double)xd[b];
      }
      return (float)acc;
    }
    case ZO_Q4_K: case ZO_Q5_K: {                     /* :196-242 */
      int five = type == ZO_Q5_K; int bs = five ? 176 : 144; int qs = five ? 48 : 16;
      int64_t nsb = cols / 256; double acc = 0;
      for (int64_t sb = 0; sb < nsb; sb++) {
        const uint8_t *o = u8 + (r * nsb + sb) * bs;
        double d = H(o), dmin = H(o + 2);
        int32_t sc[8], mn[8]; zo_unpack_scale_min_k4(o + 4, sc, mn);
        for (int c = 0; c < 4; c++) {
          const uint8_t *q = o + qs + c * 32; const int8_t *a = xq + sb * 256 + c * 64;
          int32_t lo = 0, hi = 0;
          if (five) {
            int sh = 2 * c;
            for (int l = 0; l < 32; l++) {
              int byte = q[l], h5 = o[16 + l];
              lo += ((byte & 0x0f) | (((h5 >> sh) & 1) << 4)) * a[l];
              hi += ((byte >> 4) | (((h5 >> (sh + 1)) & 1) << 4)) * a[32 + l];
            }
          } else {
            for (int l = 0; l < 32; l++) { int byte = q[l]; lo += (byte & 0x0f) * a[l]; hi += (byte >> 4) * a[32 + l]; }
          }
          int64_t b0 = sb * 8 + 2 * c;
          acc += (double)xd[b0] * (d * sc[2 * c] * lo - dmin * mn[2 * c] * (double)xs[b0]);
          acc += (double)xd[b0 + 1] * (d * sc[2 * c + 1] * hi - dmin * mn[2 * c + 1] * (double)xs[b0 + 1]);
        }
      }
      return (float)acc;
    }
    case ZO_Q6_K: {                                   /* :243-277 */
      int64_t nsb = cols / 256; double acc = 0; double gsum[16];
      for (int64_t sb = 0; sb < nsb; sb++) {
        const uint8_t *o = u8 + (r * nsb + sb) * 210;
        double d = H(o + 208);
        for (int half = 0; half < 2; half++) {
          const uint8_t *ql = o + 64 * half, *qh = o + 128 + 32 * half;
          const int8_t *a = xq + sb * 256 + half * 128;
          for (int g = 0; g < 2; g++) {
            int32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
            for (int l = g * 16; l < g * 16 + 16; l++) {
              int h = qh[l], lo0 = ql[l], lo1 = ql[l + 32];
              a0 += (((lo0 & 0x0f) | ((h & 3) << 4)) - 32) * a[l];
              a1 += (((lo1 & 0x0f) | (((h >> 2) & 3) << 4)) - 32) * a[l + 32];
              a2 += (((lo0 >> 4) | (((h >> 4) & 3) << 4)) - 32) * a[l + 64];
              a3 += (((lo1 >> 4) | (((h >> 6) & 3) << 4)) - 32) * a[l + 96];
            }
            gsum[half * 8 + g] = a0; gsum[half * 8 + 2 + g] = a1; gsum[half * 8 + 4 + g] = a2; gsum[half * 8 + 6 + g] = a3;
          }
        }
        for (int g = 0; g < 16; g++) {
          double scale = (double)(int8_t)o[192 + g];
          acc += (double)xd[sb * 8 + (g >> 1)] * d * scale * gsum[g];
        }
      }
      return (float)acc;
    }
    case ZO_F32: {                                    /* :278-288 */
      const uint8_t *o = u8 + r * cols * 4; double acc = 0;
      for (int64_t i = 0; i < cols; i++) { float f; memcpy(&f, o + 4 * i, 4); acc += (double)f * (double)x[i]; }
      return (float)acc;
    }
    case ZO_F16: case ZO_BF16: {                      /* :289-299 */
      zo_dequant_row(type, u8, cols, r, tmp);
      double acc = 0;
      for (int64_t i = 0; i < cols; i++) acc += (double)tmp[i] * (double)x[i];
      return (float)acc;
    }
  }
  return NAN;
}

static int is_quant(int type) { return type != ZO_F32 && type != ZO_F16 && type != ZO_BF16; }

int zo_matvec_q(int type, const uint8_t *w, int64_t cols, const float *x, const int8_t *xq,
                const float *xd, const int32_t *xs, float *y, int64_t r0, int64_t r1, int nthreads) {
  f16tab_init();
  if (zo_row_bytes(type, cols) < 0) return -1;
  int need_tmp = type == ZO_F16 || type == ZO_BF16;
#ifdef _OPENMP
  if (nthreads < 1) nthreads = 1;
#pragma omp parallel num_threads(nthreads)
#endif
  {
    float *tmp = need_tmp ? (float *)malloc(sizeof(float) * (size_t)cols) : NULL;
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
    for (int64_t r = r0; r < r1; r++) y[r] = row_dot(type, w, cols, r, x, xq, xd, xs, tmp);
    free(tmp);
  }
  (void)nthreads;
  return 0;
}

int zo_matvec(int type, const uint8_t *w, int64_t rows, int64_t cols, const float *x,
              float *y, int64_t r0, int64_t r1, int nthreads) {
  (void)rows;
  if (zo_row_bytes(type, cols) < 0) return -1;
  if (!is_quant(type)) return zo_matvec_q(type, w, cols, x, NULL, NULL, NULL, y, r0, r1, nthreads);
  int8_t *q = (int8_t *)malloc((size_t)cols);
  float *d = (float *)malloc(sizeof(float) * (size_t)(cols / QK));
  int32_t *s = (int32_t *)malloc(sizeof(int32_t) * (size_t)(cols / QK));
  zo_quantize_act(x, cols, q, d, s);
  int rc = zo_matvec_q(type, w, cols, x, q, d, s, y, r0, r1, nthreads);
  free(q); free(d); free(s);
  return rc;
}

/* ------------------------------------------------------------------ elementwise */
void zo_rmsnorm(float *out, const float *x, const float *weight, double eps, int n) {  /* ref-kernels.js:305-310 */
  double ss = 0;
  for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
  double s = 1 / sqrt(ss / n + eps);
  for (int i = 0; i < n; i++) out[i] = (float)((double)x[i] * s * (double)weight[i]);
}

void zo_softmax(float *x, int n) {                  /* ref-kernels.js:313-320 */
  double max = -INFINITY;
  for (int i = 0; i < n; i++) if (x[i] > max) max = x[i];
  double sum = 0;
  for (int i = 0; i < n; i++) { double e = exp((double)x[i] - max); x[i] = (float)e; sum += e; }
  double inv = 1 / sum;
  for (int i = 0; i < n; i++) x[i] = (float)((double)x[i] * inv);
}

double zo_silu(double z) { return z / (1 + exp(-z)); }   /* ref-kernels.js:322 */

void zo_rope_tables(int n_rot, double base, int ctx, const float *ff, float *cos_t, float *sin_t) { /* :329-342 */
  int half = n_rot / 2;
  for (int i = 0; i < half; i++) {
    double freq = pow(base, (-2.0 * i) / n_rot);
    if (ff) freq /= (double)ff[i];
    for (int p = 0; p < ctx; p++) {
      cos_t[(int64_t)p * half + i] = (float)cos(p * freq);
      sin_t[(int64_t)p * half + i] = (float)sin(p * freq);
    }
  }
}

void zo_apply_rope(float *v, int n_heads, int head_dim, int n_rot, int neox,
                   const float *cos_t, const float *sin_t, int pos, int h0) {       /* :349-363 */
  int half = n_rot / 2;
  int64_t to = (int64_t)pos * half;
  for (int h = h0; h < n_heads; h++) {
    int o = h * head_dim;
    for (int i = 0; i < half; i++) {
      double c = cos_t[to + i], s = sin_t[to + i];
      int i0 = neox ? o + i : o + 2 * i;
      int i1 = neox ? o + i + half : o + 2 * i + 1;
      double a = v[i0], b = v[i1];
      v[i0] = (float)(a * c - b * s);
      v[i1] = (float)(a * s + b * c);
    }
  }
}

/* ------------------------------------------------------------------ attention for one query head */
void zo_attn_head_f32(const float *qh, const float *k, const float *v, int npos, int hd,
                      int kv_stride, float *scores, float *out) {   /* forward.js:126-139 */
  double scale = 1 / sqrt((double)hd);
  for (int t = 0; t < npos; t++) {
    const float *kk = k + (int64_t)t * kv_stride; double s = 0;
    for (int i = 0; i < hd; i++) s += (double)qh[i] * (double)kk[i];
    scores[t] = (float)(s * scale);
  }
  zo_softmax(scores, npos);
  for (int i = 0; i < hd; i++) out[i] = 0;
  for (int t = 0; t < npos; t++) {
    double p = scores[t]; const float *vv = v + (int64_t)t * kv_stride;
    for (int i = 0; i < hd; i++) out[i] = (float)((double)out[i] + p * (double)vv[i]);
  }
}

void zo_attn_head_f16(const float *qh, const uint16_t *k, const uint16_t *v, int npos, int hd,
                      int kv_stride, float *scores, float *out) {   /* worker.js:320-333 */
  f16tab_init();
  double scale = 1 / sqrt((double)hd);
  for (int t = 0; t < npos; t++) {
    const uint16_t *kk = k + (int64_t)t * kv_stride; double s = 0;
    for (int i = 0; i < hd; i++) s += (double)qh[i] * (double)F16TAB[kk[i]];
    scores[t] = (float)(s * scale);
  }
  zo_softmax(scores, npos);
  for (int i = 0; i < hd; i++) out[i] = 0;
  for (int t = 0; t < npos; t++) {
    double p = scores[t]; const uint16_t *vv = v + (int64_t)t * kv_stride;
    for (int i = 0; i < hd; i++) out[i] = (float)((double)out[i] + p * (double)F16TAB[vv[i]]);
  }
}

/* ------------------------------------------------------------------ model (forward.js:10-158) */
struct zo_model {
  zo_config c;
  zo_weight tok, out;
  const float *out_norm;
  zo_layer *L;
  float *cos_t, *sin_t;
  void *kcache, *vcache;      /* [layer][pos][kvDim], f32 or u16 */
  int pos;
  float *x, *xb, *q, *k, *v, *att, *att_out, *proj, *gate, *up, *hb;
};

zo_model *zo_model_new(const zo_config *cfg, const zo_weight *tok_embd, const zo_weight *output,
                       const float *output_norm, const zo_layer *layers, const float *rope_freqs) {
  f16tab_init();
  zo_model *m = (zo_model *)calloc(1, sizeof(zo_model));
  m->c = *cfg;
  m->tok = *tok_embd;
  m->out = output ? *output : *tok_embd;
  m->out_norm = output_norm;
  m->L = (zo_layer *)malloc(sizeof(zo_layer) * (size_t)cfg->n_layer);
  memcpy(m->L, layers, sizeof(zo_layer) * (size_t)cfg->n_layer);
  int half = cfg->n_rot / 2;
  m->cos_t = (float *)malloc(sizeof(float) * (size_t)cfg->ctx * half);
  m->sin_t = (float *)malloc(sizeof(float) * (size_t)cfg->ctx * half);
  zo_rope_tables(cfg->n_rot, cfg->rope_base, cfg->ctx, rope_freqs, m->cos_t, m->sin_t);
  int64_t kv_dim = (int64_t)cfg->n_head_kv * cfg->head_dim;
  size_t el = cfg->kv_f16 ? 2 : 4;
  size_t kvb = (size_t)cfg->n_layer * cfg->ctx * kv_dim * el;
  m->kcache = calloc(1, kvb); m->vcache = calloc(1, kvb);
  int64_t q_dim = (int64_t)cfg->n_head * cfg->head_dim;
  m->x = (float *)calloc((size_t)cfg->n_embd, 4); m->xb = (float *)calloc((size_t)cfg->n_embd, 4);
  m->q = (float *)calloc((size_t)q_dim, 4); m->k = (float *)calloc((size_t)kv_dim, 4); m->v = (float *)calloc((size_t)kv_dim, 4);
  m->att = (float *)calloc((size_t)cfg->ctx, 4); m->att_out = (float *)calloc((size_t)q_dim, 4);
  m->proj = (float *)calloc((size_t)cfg->n_embd, 4);
  m->gate = (float *)calloc((size_t)cfg->n_ff, 4); m->up = (float *)calloc((size_t)cfg->n_ff, 4); m->hb = (float *)calloc((size_t)cfg->n_ff, 4);
  return m;
}

void zo_model_free(zo_model *m) {
  if (!m) return;
  free(m->L); free(m->cos_t); free(m->sin_t); free(m->kcache); free(m->vcache);
  free(m->x); free(m->xb); free(m->q); free(m->k); free(m->v); free(m->att); free(m->att_out);
  free(m->proj); free(m->gate); free(m->up); free(m->hb); free(m);
}

int zo_model_pos(const zo_model *m) { return m->pos; }
void zo_model_truncate(zo_model *m, int n) { if (n < m->pos) m->pos = n < 0 ? 0 : n; }  /* forward.js:86 */
/* forward.js:78 restorePrefix: after kvSet filled positions [0, n), the model holds n positions */
int zo_model_restore_prefix(zo_model *m, int n) {
  if (n < 0 || n > m->c.ctx) return -1;
  m->pos = n;
  return 0;
}

static void mv(const zo_weight *w, const float *x, float *y, int nthreads) {
  zo_matvec(w->type, w->data, w->rows, w->cols, x, y, 0, w->rows, nthreads);
}

int zo_model_forward(zo_model *m, int token, float *logits, int nthreads) {   /* forward.js:94-158 */
  const zo_config *c = &m->c;
  int pos = m->pos;
  if (pos >= c->ctx) return -1;
  if (!(token >= 0 && token < c->vocab)) return -2;
  int hd = c->head_dim, nh = c->n_head, nkv = c->n_head_kv;
  int64_t kv_dim = (int64_t)nkv * hd;
  int group = nh / nkv;
  zo_dequant_row(m->tok.type, m->tok.data, m->tok.cols, token, m->x);
  for (int l = 0; l < c->n_layer; l++) {
    const zo_layer *L = &m->L[l];
    zo_rmsnorm(m->xb, m->x, L->attn_norm, c->rms_eps, c->n_embd);
    mv(&L->wq, m->xb, m->q, nthreads); mv(&L->wk, m->xb, m->k, nthreads); mv(&L->wv, m->xb, m->v, nthreads);
    if (L->bq) for (int64_t i = 0; i < (int64_t)nh * hd; i++) m->q[i] = (float)((double)m->q[i] + L->bq[i]);
    if (L->bk) for (int64_t i = 0; i < kv_dim; i++) m->k[i] = (float)((double)m->k[i] + L->bk[i]);
    if (L->bv) for (int64_t i = 0; i < kv_dim; i++) m->v[i] = (float)((double)m->v[i] + L->bv[i]);
    if (L->q_norm) for (int h = 0; h < nh; h++) zo_rmsnorm(m->q + h * hd, m->q + h * hd, L->q_norm, c->rms_eps, hd);
    if (L->k_norm) for (int h = 0; h < nkv; h++) zo_rmsnorm(m->k + h * hd, m->k + h * hd, L->k_norm, c->rms_eps, hd);
    zo_apply_rope(m->q, nh, hd, c->n_rot, c->neox, m->cos_t, m->sin_t, pos, 0);
    zo_apply_rope(m->k, nkv, hd, c->n_rot, c->neox, m->cos_t, m->sin_t, pos, 0);
    int64_t lo = (int64_t)l * c->ctx * kv_dim;
    if (c->kv_f16) {                                 /* worker.js:304-306 */
      uint16_t *K = (uint16_t *)m->kcache + lo, *V = (uint16_t *)m->vcache + lo;
      for (int64_t i = 0; i < kv_dim; i++) { K[pos * kv_dim + i] = zo_f32_to_f16(m->k[i]); V[pos * kv_dim + i] = zo_f32_to_f16(m->v[i]); }
    } else {
      float *K = (float *)m->kcache + lo, *V = (float *)m->vcache + lo;
      memcpy(K + pos * kv_dim, m->k, sizeof(float) * (size_t)kv_dim);
      memcpy(V + pos * kv_dim, m->v, sizeof(float) * (size_t)kv_dim);
    }
#ifdef _OPENMP
#pragma omp parallel for num_threads(nthreads < 1 ? 1 : nthreads) schedule(static)
#endif
    for (int h = 0; h < nh; h++) {
      int kvh = h / group;
      float *scores = (float *)malloc(sizeof(float) * (size_t)(pos + 1));
      if (c->kv_f16) {
        const uint16_t *K = (const uint16_t *)m->kcache + lo + kvh * hd, *V = (const uint16_t *)m->vcache + lo + kvh * hd;
        zo_attn_head_f16(m->q + h * hd, K, V, pos + 1, hd, (int)kv_dim, scores, m->att_out + h * hd);
      } else {
        const float *K = (const float *)m->kcache + lo + kvh * hd, *V = (const float *)m->vcache + lo + kvh * hd;
        zo_attn_head_f32(m->q + h * hd, K, V, pos + 1, hd, (int)kv_dim, scores, m->att_out + h * hd);
      }
      free(scores);
    }
    mv(&L->wo, m->att_out, m->proj, nthreads);
    for (int i = 0; i < c->n_embd; i++) m->x[i] = (float)((double)m->x[i] + m->proj[i]);
    zo_rmsnorm(m->xb, m->x, L->ffn_norm, c->rms_eps, c->n_embd);
    mv(&L->gate, m->xb, m->gate, nthreads); mv(&L->up, m->xb, m->up, nthreads);
    for (int i = 0; i < c->n_ff; i++) m->hb[i] = (float)(zo_silu(m->gate[i]) * (double)m->up[i]);
    mv(&L->down, m->hb, m->proj, nthreads);
    for (int i = 0; i < c->n_embd; i++) m->x[i] = (float)((double)m->x[i] + m->proj[i]);
  }
  m->pos = pos + 1;
  if (!logits) return 0;
  zo_rmsnorm(m->xb, m->x, m->out_norm, c->rms_eps, c->n_embd);
  mv(&m->out, m->xb, logits, nthreads);
  return 0;
}

int zo_model_kv_get(zo_model *m, int layer, int is_v, int n, float *out) {
  int64_t kv_dim = (int64_t)m->c.n_head_kv * m->c.head_dim;
  int64_t lo = (int64_t)layer * m->c.ctx * kv_dim;
  if (m->c.kv_f16) {
    const uint16_t *src = (const uint16_t *)(is_v ? m->vcache : m->kcache) + lo;
    for (int64_t i = 0; i < (int64_t)n * kv_dim; i++) out[i] = F16TAB[src[i]];
  } else {
    memcpy(out, (const float *)(is_v ? m->vcache : m->kcache) + lo, sizeof(float) * (size_t)(n * kv_dim));
  }
  return 0;
}

int zo_model_kv_set(zo_model *m, int layer, int is_v, int n, const float *in) {
  int64_t kv_dim = (int64_t)m->c.n_head_kv * m->c.head_dim;
  int64_t lo = (int64_t)layer * m->c.ctx * kv_dim;
  if (m->c.kv_f16) {
    uint16_t *dst = (uint16_t *)(is_v ? m->vcache : m->kcache) + lo;
    for (int64_t i = 0; i < (int64_t)n * kv_dim; i++) dst[i] = zo_f32_to_f16(in[i]);
  } else {
    memcpy((float *)(is_v ? m->vcache : m->kcache) + lo, in, sizeof(float) * (size_t)(n * kv_dim));
  }
  return 0;
}
