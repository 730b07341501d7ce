/*
 * ugb_oracle.c -- CPU restatement of the reference's quantized linear-layer arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see ugb_oracle.h).  Built with -ffp-contract=off so every fp32
 * expression rounds exactly as written (the reference's Rust CPU checks never contract).
 */
#include "ugb_oracle.h"
#include <math.h>
#include <string.h>
#include <stdlib.h>
#include <pthread.h>
#include <unistd.h>

/* ---- fp16 ------------------------------------------------------------------------------ */

float orc_half(uint16_t h) {
  /* frontier_core.rs:60-65 */
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 31u;
  uint32_t frac = h & 1023u;
  float out;
  if (exp == 0) {
    float v = (float)frac * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  uint32_t bits = (exp == 31) ? (sign | 0x7f800000u | (frac << 13))
                              : (sign | ((exp + 112u) << 23) | (frac << 13));
  memcpy(&out, &bits, 4);
  return out;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t *p) { return (uint32_t)rd16(p) | ((uint32_t)rd16(p + 2) << 16); }

/* ---- the reference's other formats (frontier_core.rs:68-101) ------------------------------ */

/* frontier_core.rs:68 IQ4 code book. */
static const int8_t kIq4[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

static uint32_t g_iq3_grid[256];
static int g_iq3_set = 0;

void orc_set_iq3_grid(const uint32_t *grid) {
  memcpy(g_iq3_grid, grid, sizeof g_iq3_grid);
  g_iq3_set = 1;
}

/* IQ4_NL element j (0..31) of an 18-byte block: code-book index = nibble j/16 of byte 2 + j%16
 * (frontier_core.rs:80-82). */
static int iq4nl_value(const uint8_t *blk, int j) {
  return kIq4[(blk[2 + j % 16] >> (4 * (j / 16))) & 15];
}

/* IQ4_XS sub-block scale (sc, 0..63) of sub-block sb and element j (0..255) value index
 * (frontier_core.rs:83-87). */
static int iq4xs_scale(const uint8_t *sb, int s) {
  return ((sb[4 + s / 2] >> (4 * (s % 2))) & 15) | (((rd16(sb + 2) >> (2 * s)) & 3) << 4);
}
static int iq4xs_value(const uint8_t *sb, int j) {
  return kIq4[(sb[8 + (j / 32) * 16 + j % 16] >> (4 * ((j % 32) / 16))) & 15];
}

/* Q6_K element j (0..255): signed 6-bit quant and its int8 scale (frontier_core.rs:88-93). */
static int q6k_quant(const uint8_t *sb, int j) {
  int sub = j / 128, l = j % 32, group = (j % 128) / 32;
  int low = sb[sub * 64 + l + (group % 2) * 32];
  int high = sb[128 + sub * 32 + l];
  return (((low >> (4 * (group / 2))) & 15) | (((high >> (2 * group)) & 3) << 4)) - 32;
}
static int q6k_scale(const uint8_t *sb, int j) {
  int sub = j / 128, l = j % 32, group = (j % 128) / 32;
  return (int8_t)sb[192 + sub * 8 + l / 16 + group * 2];
}

/* IQ3_XXS element j (0..255): signed grid magnitude; the sub-block scale d*(0.5+s)*0.5
 * (frontier_core.rs:94-101). */
static int iq3xxs_value(const uint8_t *sb, int j) {
  int s = j / 32, group = (j % 32) / 8;
  uint32_t aux = rd32(sb + 66 + s * 4);
  uint32_t signs7 = (aux >> (7 * group)) & 127u;
  uint32_t par = (uint32_t)__builtin_popcount(signs7) & 1u;
  uint32_t signs = signs7 | (par << 7);
  int index = sb[2 + s * 8 + group * 2 + (j % 8) / 4];
  int q = (int)((g_iq3_grid[index] >> (8 * (j % 4))) & 255u);
  return (signs & (1u << (j % 8))) ? -q : q;
}
static float iq3xxs_scale(const uint8_t *sb, int s) {
  uint32_t aux = rd32(sb + 66 + s * 4);
  return orc_half(rd16(sb)) * (0.5f + (float)(aux >> 28)) * 0.5f;
}

/* ---- sizes ----------------------------------------------------------------------------- */

/* Block geometry (frontier_core.rs:54-55).  BF16 (30) has no decoder here: only its size is
 * restated, so row_bytes() answers every known-answer case of the reference. */
static int block_of(uint32_t kind, long *elems, long *bytes) {
  switch (kind) {
    case ORC_F32: *elems = 1; *bytes = 4; return 0;
    case ORC_Q8_0: *elems = 32; *bytes = 34; return 0;   /* frontier_core.rs:54 */
    case ORC_Q4_K: *elems = 256; *bytes = 144; return 0; /* ggml block_q4_K */
    case ORC_Q3_K: *elems = 256; *bytes = 110; return 0; /* ggml block_q3_K */
    case 14: *elems = 256; *bytes = 210; return 0;       /* Q6_K */
    case 18: *elems = 256; *bytes = 98; return 0;        /* IQ3_XXS */
    case 20: *elems = 32; *bytes = 18; return 0;         /* IQ4_NL */
    case 23: *elems = 256; *bytes = 136; return 0;       /* IQ4_XS */
    case 30: *elems = 1; *bytes = 2; return 0;           /* BF16 */
    default: return -1;
  }
}

static int has_decoder(uint32_t kind) {
  if (kind == ORC_IQ3_XXS) return g_iq3_set;
  return kind == ORC_F32 || kind == ORC_Q8_0 || kind == ORC_Q4_K || kind == ORC_Q3_K || kind == ORC_Q6_K ||
         kind == ORC_IQ4_NL || kind == ORC_IQ4_XS;
}

long orc_row_bytes(uint32_t kind, long n) {
  /* frontier_core.rs:53-58 */
  long e, b;
  if (block_of(kind, &e, &b)) return -1;
  if (n <= 0 || n % e != 0) return -2;
  return (n / e) * b;
}

/* ---- block decoders -------------------------------------------------------------------- */

/* ggml get_scale_min_k4, restated from the gguf Q4_K.get_scale_min bit map. */
static void q4k_scale_min(const uint8_t *sc12, int j, int *sc, int *mn) {
  if (j < 4) {
    *sc = sc12[j] & 63;
    *mn = sc12[j + 4] & 63;
  } else {
    *sc = (sc12[j + 4] & 0x0F) | ((sc12[j - 4] >> 6) << 4);
    *mn = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
  }
}

/* Q4_K quant of element i (0..255) of a super-block: nibble (i%64)/32 of qs[(i/64)*32+i%32]. */
static int q4k_quant(const uint8_t *sb, int i) {
  const uint8_t *qs = sb + 16;
  return (qs[(i / 64) * 32 + (i % 32)] >> (4 * ((i % 64) / 32))) & 15;
}

/* Q3_K 6-bit signed scale of 16-element sub-block j (0..15), already minus 32. */
static int q3k_scale(const uint8_t *sb, int j) {
  const uint8_t *sc = sb + 96;
  int lo = (sc[j % 8] >> (4 * (j / 8))) & 15;
  int hi = (sc[8 + j % 4] >> (2 * (j / 4))) & 3;
  return (lo | (hi << 4)) - 32;
}

/* Q3_K quant of element i: low 2 bits (qs[(i/128)*32+i%32] >> 2*((i%128)/32)) & 3, minus 4
 * when bit i/32 of hmask[i%32] is clear. */
static int q3k_quant(const uint8_t *sb, int i) {
  const uint8_t *hm = sb;
  const uint8_t *qs = sb + 32;
  int lo = (qs[(i / 128) * 32 + (i % 32)] >> (2 * ((i % 128) / 32))) & 3;
  int h = (hm[i % 32] >> (i / 32)) & 1;
  return lo - (h ? 0 : 4);
}

int orc_dequantize(uint32_t kind, const uint8_t *in, long nbytes, float *out, long n) {
  long rb = orc_row_bytes(kind, n);
  if (rb < 0) return (int)rb;
  if (!has_decoder(kind)) return -1;
  if (rb != nbytes) return -3;
  for (long i = 0; i < n; i++) {
    switch (kind) {
      case ORC_F32: {
        float v;
        memcpy(&v, in + 4 * i, 4);
        out[i] = v;
        break;
      }
      case ORC_Q8_0: { /* frontier_core.rs:79 */
        const uint8_t *p = in + (i / 32) * 34;
        out[i] = orc_half(rd16(p)) * (float)(int8_t)p[2 + i % 32];
        break;
      }
      case ORC_Q4_K: { /* gguf Q4_K.dequantize_blocks: (d*sc)*q - (dmin*m) */
        const uint8_t *sb = in + (i / 256) * 144;
        int j = (int)(i % 256), sc, mn;
        q4k_scale_min(sb + 4, j / 32, &sc, &mn);
        float dl = orc_half(rd16(sb)) * (float)sc;
        float ml = orc_half(rd16(sb + 2)) * (float)mn;
        out[i] = dl * (float)q4k_quant(sb, j) - ml;
        break;
      }
      case ORC_Q3_K: { /* gguf Q3_K.dequantize_blocks: (d*sc)*q */
        const uint8_t *sb = in + (i / 256) * 110;
        int j = (int)(i % 256);
        float dl = orc_half(rd16(sb + 108)) * (float)q3k_scale(sb, j / 16);
        out[i] = dl * (float)q3k_quant(sb, j);
        break;
      }
      case ORC_IQ4_NL: { /* frontier_core.rs:80-82: half(d) * IQ4[q] */
        const uint8_t *p = in + (i / 32) * 18;
        out[i] = orc_half(rd16(p)) * (float)iq4nl_value(p, (int)(i % 32));
        break;
      }
      case ORC_IQ4_XS: { /* frontier_core.rs:83-87: (half(d) * (sc-32)) * IQ4[q] */
        const uint8_t *sb = in + (i / 256) * 136;
        int j = (int)(i % 256);
        out[i] = (orc_half(rd16(sb)) * (float)(iq4xs_scale(sb, j / 32) - 32)) * (float)iq4xs_value(sb, j);
        break;
      }
      case ORC_Q6_K: { /* frontier_core.rs:88-93: (half(d) * sc) * q */
        const uint8_t *sb = in + (i / 256) * 210;
        int j = (int)(i % 256);
        out[i] = (orc_half(rd16(sb + 208)) * (float)q6k_scale(sb, j)) * (float)q6k_quant(sb, j);
        break;
      }
      case ORC_IQ3_XXS: { /* frontier_core.rs:94-101: (scale * q) * sign */
        const uint8_t *sb = in + (i / 256) * 98;
        int j = (int)(i % 256);
        int v = iq3xxs_value(sb, j);
        float mag = iq3xxs_scale(sb, j / 32) * (float)(v < 0 ? -v : v);
        out[i] = v < 0 ? -mag : mag;
        break;
      }
    }
  }
  return 0;
}

/* ---- activation quantiser ----------------------------------------------------------------- */

int orc_quant_act(const float *x, int8_t *q, float *d, int32_t *s, long k) {
  /* gpu_dp4a.cu:23-31 and gpu_prefill.rs:105-106 */
  int bad = 0;
  for (long b = 0; b < k / 32; b++) {
    float a = 0.0f;
    for (int j = 0; j < 32; j++) {
      float v = x[b * 32 + j];
      if (!isfinite(v)) { bad = 1; continue; }
      a = fmaxf(a, fabsf(v));
    }
    d[b] = a / 127.0f;
    float inv = a > 0.0f ? 127.0f / a : 0.0f;
    int32_t sum = 0;
    for (int j = 0; j < 32; j++) {
      float v = x[b * 32 + j];
      int qi = 0;
      if (isfinite(v)) {
        float r = rintf(v * inv); /* round half to even, as __float2int_rn */
        if (r > 127.0f) r = 127.0f;
        if (r < -127.0f) r = -127.0f;
        qi = (int)r;
      }
      q[b * 32 + j] = (int8_t)qi;
      sum += qi;
    }
    s[b] = sum;
  }
  return bad;
}

/* ---- integer block dots ------------------------------------------------------------------- */

static int32_t block_dot(uint32_t kind, const uint8_t *row, const int8_t *q, long b) {
  int32_t acc = 0;
  switch (kind) {
    case ORC_Q8_0: {
      const uint8_t *p = row + b * 34 + 2;
      for (int j = 0; j < 32; j++) acc += (int32_t)(int8_t)p[j] * (int32_t)q[b * 32 + j];
      return acc;
    }
    case ORC_Q4_K: {
      const uint8_t *sb = row + (b / 8) * 144;
      int base = (int)(b % 8) * 32;
      for (int j = 0; j < 32; j++) acc += q4k_quant(sb, base + j) * (int32_t)q[b * 32 + j];
      return acc;
    }
    case ORC_Q3_K: {
      const uint8_t *sb = row + (b / 8) * 110;
      int base = (int)(b % 8) * 32;
      int32_t lo = 0, hi = 0;
      for (int j = 0; j < 16; j++) lo += q3k_quant(sb, base + j) * (int32_t)q[b * 32 + j];
      for (int j = 16; j < 32; j++) hi += q3k_quant(sb, base + j) * (int32_t)q[b * 32 + j];
      int sub = base / 16;
      acc = q3k_scale(sb, sub) * lo + q3k_scale(sb, sub + 1) * hi;
      return acc;
    }
    case ORC_Q6_K: {
      const uint8_t *sb = row + (b / 8) * 210;
      int base = (int)(b % 8) * 32;
      int32_t lo = 0, hi = 0;
      for (int j = 0; j < 16; j++) lo += q6k_quant(sb, base + j) * (int32_t)q[b * 32 + j];
      for (int j = 16; j < 32; j++) hi += q6k_quant(sb, base + j) * (int32_t)q[b * 32 + j];
      return q6k_scale(sb, base) * lo + q6k_scale(sb, base + 16) * hi;
    }
    case ORC_IQ4_NL: {
      const uint8_t *p = row + b * 18;
      for (int j = 0; j < 32; j++) acc += iq4nl_value(p, j) * (int32_t)q[b * 32 + j];
      return acc;
    }
    case ORC_IQ4_XS: {
      const uint8_t *sb = row + (b / 8) * 136;
      int base = (int)(b % 8) * 32;
      for (int j = 0; j < 32; j++) acc += iq4xs_value(sb, base + j) * (int32_t)q[b * 32 + j];
      return acc;
    }
    case ORC_IQ3_XXS: {
      const uint8_t *sb = row + (b / 8) * 98;
      int base = (int)(b % 8) * 32;
      for (int j = 0; j < 32; j++) acc += iq3xxs_value(sb, base + j) * (int32_t)q[b * 32 + j];
      return acc;
    }
  }
  return 0;
}

int orc_block_dots(uint32_t kind, const uint8_t *row, const int8_t *q, long k, int32_t *out) {
  long rb = orc_row_bytes(kind, k);
  if (rb < 0) return (int)rb;
  if (kind == ORC_F32 || !has_decoder(kind)) return -1;
  for (long b = 0; b < k / 32; b++) out[b] = block_dot(kind, row, q, b);
  return 0;
}

/* The scaled row dot; with `absolute` set, the sum of the magnitudes of its block terms instead
 * (the scale against which any reordering of the fp32 sum is judged). */
static float row_dot(uint32_t kind, const uint8_t *row, const int8_t *q, const float *d,
                     const int32_t *s, long k, int absolute) {
  float y = 0.0f;
  for (long b = 0; b < k / 32; b++) {
    int32_t isum = block_dot(kind, row, q, b);
    float term = 0.0f;
    switch (kind) {
      case ORC_Q8_0: {
        float dw = orc_half(rd16(row + b * 34));
        term = (float)isum * (dw * d[b]);
        break;
      }
      case ORC_Q4_K: {
        const uint8_t *sb = row + (b / 8) * 144;
        int sc, mn;
        q4k_scale_min(sb + 4, (int)(b % 8), &sc, &mn);
        float dl = orc_half(rd16(sb)) * (float)sc;
        float ml = orc_half(rd16(sb + 2)) * (float)mn;
        term = d[b] * (dl * (float)isum - ml * (float)s[b]);
        break;
      }
      case ORC_Q3_K: {
        const uint8_t *sb = row + (b / 8) * 110;
        float dsb = orc_half(rd16(sb + 108));
        term = (float)isum * (dsb * d[b]);
        break;
      }
      case ORC_Q6_K: {
        const uint8_t *sb = row + (b / 8) * 210;
        term = (float)isum * (orc_half(rd16(sb + 208)) * d[b]);
        break;
      }
      case ORC_IQ4_NL: {
        term = (float)isum * (orc_half(rd16(row + b * 18)) * d[b]);
        break;
      }
      case ORC_IQ4_XS: {
        const uint8_t *sb = row + (b / 8) * 136;
        float dl = orc_half(rd16(sb)) * (float)(iq4xs_scale(sb, (int)(b % 8)) - 32);
        term = (float)isum * (dl * d[b]);
        break;
      }
      case ORC_IQ3_XXS: {
        const uint8_t *sb = row + (b / 8) * 98;
        term = (float)isum * (iq3xxs_scale(sb, (int)(b % 8)) * d[b]);
        break;
      }
    }
    y += absolute ? fabsf(term) : term;
  }
  return y;
}

typedef struct {
  uint32_t kind;
  const uint8_t *w;
  long row_bytes, k, m, batch, begin, end;
  const int8_t *q;
  const float *d;
  const int32_t *s;
  float *y;
  int absolute;
} mv_span;

/* Rows [begin, end) of the flattened (batch, row) index space. */
static void *mv_span_run(void *arg) {
  const mv_span *t = (const mv_span *)arg;
  long nb = t->k / 32;
  for (long i = t->begin; i < t->end; i++) {
    long v = i / t->m, r = i % t->m;
    t->y[i] = row_dot(t->kind, t->w + r * t->row_bytes, t->q + v * t->k, t->d + v * nb,
                      t->s + v * nb, t->k, t->absolute);
  }
  return NULL;
}

static int matvec_impl(uint32_t kind, const uint8_t *w, long row_bytes, const int8_t *q,
                       const float *d, const int32_t *s, float *y, long k, long m, long batch,
                       int threads, int absolute) {
  long rb = orc_row_bytes(kind, k);
  if (rb < 0) return (int)rb;
  if (kind == ORC_F32 || !has_decoder(kind)) return -1;
  if (rb != row_bytes || m <= 0 || batch <= 0) return -2;
  long total = m * batch;
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (threads > total) threads = (int)total;
  mv_span spans[256];
  pthread_t tids[256];
  for (int t = 0; t < threads; t++) {
    mv_span sp = {kind, w, row_bytes, k, m, batch, total * t / threads,
                  total * (t + 1) / threads, q, d, s, y, absolute};
    spans[t] = sp;
  }
  if (threads == 1) {
    mv_span_run(&spans[0]);
    return 0;
  }
  for (int t = 0; t < threads; t++) pthread_create(&tids[t], NULL, mv_span_run, &spans[t]);
  for (int t = 0; t < threads; t++) pthread_join(tids[t], NULL);
  return 0;
}

int orc_threads(void) {
  const char *env = getenv("UGB_ORACLE_THREADS");
  long n = env ? atol(env) : sysconf(_SC_NPROCESSORS_ONLN);
  if (n < 1) n = 1;
  if (n > 256) n = 256;
  return (int)n;
}

int orc_matvec(uint32_t kind, const uint8_t *w, long row_bytes, const int8_t *q, const float *d,
               const int32_t *s, float *y, long k, long m, long batch) {
  return matvec_impl(kind, w, row_bytes, q, d, s, y, k, m, batch, 1, 0);
}

int orc_matvec_mt(uint32_t kind, const uint8_t *w, long row_bytes, const int8_t *q,
                  const float *d, const int32_t *s, float *y, long k, long m, long batch) {
  return matvec_impl(kind, w, row_bytes, q, d, s, y, k, m, batch, orc_threads(), 0);
}

int orc_matvec_terms_mt(uint32_t kind, const uint8_t *w, long row_bytes, const int8_t *q,
                        const float *d, const int32_t *s, float *y, long k, long m, long batch) {
  return matvec_impl(kind, w, row_bytes, q, d, s, y, k, m, batch, orc_threads(), 1);
}

int orc_matvec_dequant_f32(uint32_t kind, const uint8_t *w, long row_bytes, const float *x,
                           float *y, long k, long m) {
  /* llm.rs:305 `expect += model.q8(t,row,col)*x[col]` */
  long rb = orc_row_bytes(kind, k);
  if (rb < 0) return (int)rb;
  if (!has_decoder(kind)) return -1;
  if (rb != row_bytes) return -2;
  float tmp[256];
  for (long r = 0; r < m; r++) {
    float acc = 0.0f;
    long eb = 1, bb = 4;
    block_of(kind, &eb, &bb);
    for (long b = 0; b < k / eb; b++) {
      orc_dequantize(kind, w + r * row_bytes + b * bb, bb, tmp, eb);
      for (long j = 0; j < eb; j++) acc += tmp[j] * x[b * eb + j];
    }
    y[r] = acc;
  }
  return 0;
}

/* ---- descriptor ABI ------------------------------------------------------------------------ */

static void put64(uint8_t *p, uint64_t v) { for (int i = 0; i < 8; i++) p[i] = (uint8_t)(v >> (8 * i)); }
static void put32(uint8_t *p, uint32_t v) { for (int i = 0; i < 4; i++) p[i] = (uint8_t)(v >> (8 * i)); }

long orc_dispatch_pack(const orc_dispatch *jobs, long count, uint8_t *out, uint32_t *grid_rows4) {
  /* frontier_dispatch.rs:11-31 */
  if (count <= 0 || count > 32) return -1;
  uint32_t rows = 0;
  for (long i = 0; i < count; i++) {
    const orc_dispatch *j = &jobs[i];
    if (j->n == 0 || j->m == 0 || j->row_bytes == 0 || j->n > 16384) return -1;
    uint64_t row_end = (uint64_t)j->m * j->row_bytes, input_bytes = (uint64_t)j->n * 4;
    if (j->weight + row_end < j->weight) return -1;
    if (j->input + input_bytes < j->input) return -1;
    uint64_t out_end = j->output + (uint64_t)j->m * 4;
    if (out_end < j->output) return -1;
    for (long p = 0; p < i; p++) {
      uint64_t end = jobs[p].output + (uint64_t)jobs[p].m * 4;
      if (j->output < end && jobs[p].output < out_end) return -1;
    }
    uint8_t *rec = out + i * 48;
    put64(rec + 0, j->weight);
    put64(rec + 8, j->input);
    put64(rec + 16, j->output);
    put32(rec + 24, j->kind);
    put32(rec + 28, j->n);
    put32(rec + 32, j->m);
    put32(rec + 36, j->row_bytes);
    put32(rec + 40, rows);
    put32(rec + 44, 0);
    uint64_t padded = ((uint64_t)j->m + 3) & ~(uint64_t)3;
    if ((uint64_t)j->m + 3 > 0xffffffffull || rows + padded > 0xffffffffull) return -1;
    rows += (uint32_t)padded;
  }
  *grid_rows4 = rows / 4;
  return count * 48;
}

/* ---- MoE routing ---------------------------------------------------------------------------- */

int orc_moe_route(const float *logits, long n_expert, long top_k, int32_t *ids, float *weights) {
  /* frontier_forward.rs:47-51 softmax */
  float prob[4096];
  int32_t order[4096];
  if (n_expert <= 0 || n_expert > 4096 || top_k <= 0 || top_k > n_expert) return -1;
  float mx = -INFINITY;
  for (long e = 0; e < n_expert; e++) {
    if (!isfinite(logits[e])) return -1;
    mx = fmaxf(mx, logits[e]);
  }
  float sum = 0.0f;
  for (long e = 0; e < n_expert; e++) {
    prob[e] = expf(logits[e] - mx);
    sum += prob[e];
  }
  if (!(sum > 0.0f) || !isfinite(sum)) return -1;
  for (long e = 0; e < n_expert; e++) prob[e] /= sum;
  /* frontier_forward.rs:167: descending probability, ties to the lower id (stable
   * insertion sort over ascending ids keeps the lower id first). */
  for (long e = 0; e < n_expert; e++) {
    long p = e;
    while (p > 0 && prob[order[p - 1]] < prob[e]) { order[p] = order[p - 1]; p--; }
    order[p] = (int32_t)e;
  }
  float top = 0.0f;
  for (long i = 0; i < top_k; i++) top += prob[order[i]];
  if (!(top > 0.0f)) return -1;
  for (long i = 0; i < top_k; i++) {
    ids[i] = order[i];
    weights[i] = prob[order[i]] / top; /* frontier_forward.rs:193 scores[id]/sum */
  }
  return 0;
}

/* ---- prefill repack --------------------------------------------------------------------- */

int orc_prefill_repack_q8_0(const uint8_t *w, long n, long k, long n_pad, int8_t *qa, float *sa) {
  if (k <= 0 || k % 32 || n <= 0 || n_pad < n) return -1;
  long nb = k / 32;
  memset(qa, 0, (size_t)(n_pad * k));
  memset(sa, 0, (size_t)(nb * n_pad) * sizeof(float));
  for (long r = 0; r < n; r++)
    for (long b = 0; b < nb; b++) {
      const uint8_t *p = w + (r * nb + b) * 34;
      sa[b * n_pad + r] = orc_half(rd16(p));
      memcpy(qa + r * k + b * 32, p + 2, 32);
    }
  return 0;
}

float orc_silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

/* ---- prefill GEMM -------------------------------------------------------------------------- */

typedef struct {
  const uint8_t *w;
  const int8_t *q;
  const float *d;
  float *y;
  long n, k, t0, t1;
} pf_span;

static void *pf_span_run(void *arg) {
  const pf_span *s = (const pf_span *)arg;
  long nb = s->k / 32;
  for (long t = s->t0; t < s->t1; t++)
    for (long r = 0; r < s->n; r++) {
      float acc = 0.0f;
      for (long b = 0; b < nb; b++) {
        const uint8_t *p = s->w + (r * nb + b) * 34;
        int32_t dot = 0;
        for (int j = 0; j < 32; j++) dot += (int32_t)(int8_t)p[2 + j] * (int32_t)s->q[t * s->k + b * 32 + j];
        /* gpu_prefill.cu:31-34: fmaf((float)c, d_w * d_x, acc) in block order */
        acc = fmaf((float)dot, orc_half(rd16(p)) * s->d[t * nb + b], acc);
      }
      s->y[t * s->n + r] = acc;
    }
  return NULL;
}

int orc_prefill_gemm_q8_0(const uint8_t *w, long n, long k, const float *x, long m, float *y, int threads) {
  if (n <= 0 || m <= 0 || k <= 0 || k % 32) return -1;
  long nb = k / 32;
  int8_t *q = (int8_t *)malloc((size_t)(m * k));
  float *d = (float *)malloc((size_t)(m * nb) * sizeof(float));
  int32_t *s = (int32_t *)malloc((size_t)(m * nb) * sizeof(int32_t));
  if (!q || !d || !s) { free(q); free(d); free(s); return -2; }
  int bad = 0;
  for (long t = 0; t < m; t++) bad |= orc_quant_act(x + t * k, q + t * k, d + t * nb, s + t * nb, k);
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (threads > m) threads = (int)m;
  pf_span spans[256];
  pthread_t tids[256];
  for (int i = 0; i < threads; i++) {
    spans[i].w = w; spans[i].q = q; spans[i].d = d; spans[i].y = y; spans[i].n = n; spans[i].k = k;
    spans[i].t0 = m * i / threads; spans[i].t1 = m * (i + 1) / threads;
  }
  for (int i = 1; i < threads; i++) pthread_create(&tids[i], NULL, pf_span_run, &spans[i]);
  pf_span_run(&spans[0]);
  for (int i = 1; i < threads; i++) pthread_join(tids[i], NULL);
  free(q); free(d); free(s);
  return bad;
}
