/*
 * memopt_oracle.c — CPU restatement of the reference KV-cache data plane.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels of memopt-transformer-runtime_b200; only tests/, the smoke() entry
 * point and bench.py's CPU-baseline leg may load it.  The product never does.
 *
 * Each function restates one reference kernel (paths relative to the
 * reference project TheRadDani/memopt-transformer-runtime) in scalar C with
 * IEEE fp32 arithmetic (build with -ffp-contract=off, no fast-math) so that
 * integer/byte results are bit-exact with the reference GPU code:
 *   quantize_int4 ........ src/csrc/quantization.cu:104-203
 *   dequantize_int4 ...... src/csrc/quantization.cu:232-270
 *   write_cache .......... src/csrc/kv_cache.cu:228-260
 *   evict_tokens ......... src/csrc/kv_cache.cu:640-1015
 *   evict_cache .......... src/csrc/kv_cache.cu:379-483
 *   paged attention ...... src/csrc/attention.cu:98-339 (computed in fp64)
 * GPU conversion semantics that C leaves undefined are emulated explicitly:
 * float->int is cvt.rzi.s32.f32 (NaN -> 0, saturating), int overflow wraps.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- halves */
float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F;
  uint32_t man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while ((man & 0x400) == 0);
      man &= 0x3FF;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* fp32 -> fp16, round to nearest even (IEEE 754 conversion). */
uint16_t oracle_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) { /* inf or nan */
    if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00 | ((ax >> 13) & 0x3FF));
    return (uint16_t)(sign | 0x7C00);
  }
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00); /* rounds to >= 65520 -> inf */
  if (ax < 0x38800000u) {                                   /* result subnormal or zero */
    if (ax < 0x33000000u) return sign;                      /* < 2^-25: rounds to 0 */
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7FFFFF) | 0x800000;
    const uint32_t shift = 126 - e; /* 14..24 */
    uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1);
    const uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (r & 1))) ++r;
    return (uint16_t)(sign | r);
  }
  uint32_t r = ((ax >> 13) - (112u << 10)); /* rebias exponent */
  const uint32_t rem = ax & 0x1FFF;
  if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) ++r;
  return (uint16_t)(sign | r);
}

/* cvt.rzi.s32.f32 of an already-integral value. */
static int32_t gpu_f2i(float x) {
  if (isnan(x)) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return (int32_t)x;
}

static int32_t wrap_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }

/* ------------------------------------------------------------- INT4 quant */
static float int4_scale(const float* v, int n) {
  float m = 0.f;
  for (int i = 0; i < n; ++i) m = fmaxf(m, fabsf(v[i]));
  return m > 0.f ? m / 7.0f : 1.0f;
}

static uint8_t int4_code(float x, float scale) {
  int32_t iq = wrap_add(gpu_f2i(roundf(x / scale)), 8);
  if (iq < 0) iq = 0;
  if (iq > 15) iq = 15;
  return (uint8_t)iq;
}

/* Flat groups of 64: packed[n/2], scales[n/64] fp32. */
void oracle_quantize_int4(const uint16_t* in, int64_t n, uint8_t* packed, float* scales) {
  for (int64_t g = 0; g < n / 64; ++g) {
    float v[64];
    for (int i = 0; i < 64; ++i) v[i] = oracle_f16_to_f32(in[g * 64 + i]);
    const float s = int4_scale(v, 64);
    scales[g] = s;
    for (int i = 0; i < 32; ++i)
      packed[g * 32 + i] = (uint8_t)(int4_code(v[2 * i], s) | (int4_code(v[2 * i + 1], s) << 4));
  }
}

void oracle_dequantize_int4(const uint8_t* packed, const float* scales, int64_t n, uint16_t* out) {
  for (int64_t g = 0; g < n / 64; ++g) {
    const float s = scales[g];
    for (int i = 0; i < 32; ++i) {
      const uint8_t b = packed[g * 32 + i];
      out[g * 64 + 2 * i] = oracle_f32_to_f16((float)((int)(b & 0xF) - 8) * s);
      out[g * 64 + 2 * i + 1] = oracle_f32_to_f16((float)((int)(b >> 4) - 8) * s);
    }
  }
}

/* ------------------------------------------------------------ write_cache */
/* fp16 pool [NB, BS, H, D]; tokens with slot outside [0, NB*BS) are skipped. */
void oracle_write_cache_f16(const uint16_t* keys, const uint16_t* values, const int32_t* slots,
                            int64_t T, int H, int D, uint16_t* kpool, uint16_t* vpool, int64_t NB,
                            int BS) {
  const int64_t row = (int64_t)H * D;
  for (int64_t t = 0; t < T; ++t) {
    const int32_t s = slots[t];
    if (s < 0 || (int64_t)s >= NB * BS) continue;
    memcpy(kpool + (int64_t)s * row, keys + t * row, row * 2);
    memcpy(vpool + (int64_t)s * row, values + t * row, row * 2);
  }
}

/* INT4 pages: one page per (block, head) of
 * [K codes BS*D/2 | V codes BS*D/2 | K scales BS*(D/64) fp16 | V scales].
 * K row pos: byte i = code(2i) | code(2i+1) << 4 (the reference packing).
 * V row pos: the same bytes, except that for D == 128 byte i is stored at
 * i ^ 32 when bit 1 of pos is set.  K scales [BS][D/64].  V scales, per
 * 16-token tile: [D/64][16] with token r of the tile at slot
 * 2(r & 3) + ((r >> 2) & 1) + 8(r >> 3).  BS is a multiple of 16. */
static int64_t int4_page_bytes(int BS, int D) { return (int64_t)BS * D + (int64_t)BS * (D / 64) * 4; }
static int64_t int4_vrow_byte(int pos, int i, int D) {
  return (int64_t)pos * (D / 2) + ((D == 128 && (pos & 2)) ? (i ^ 32) : i);
}
static int64_t int4_vscale_index(int pos, int g, int G) {
  const int r = pos & 15;
  return ((int64_t)(pos >> 4) * G + g) * 16 + 2 * (r & 3) + ((r >> 2) & 1) + 8 * (r >> 3);
}

void oracle_write_cache_int4(const uint16_t* keys, const uint16_t* values, const int32_t* slots,
                             int64_t T, int H, int D, uint8_t* pages, int64_t NB, int BS) {
  const int gpr = D / 64;
  const int64_t pb = int4_page_bytes(BS, D), codes = (int64_t)BS * (D / 2);
  for (int64_t t = 0; t < T; ++t) {
    const int32_t s = slots[t];
    if (s < 0 || (int64_t)s >= NB * BS) continue;
    const int64_t blk = s / BS;
    const int pos = s % BS;
    for (int h = 0; h < H; ++h) {
      uint8_t* page = pages + (blk * H + h) * pb;
      for (int g = 0; g < gpr; ++g) {
        for (int kv = 0; kv < 2; ++kv) {
          const uint16_t* src = (kv ? values : keys) + (t * H + h) * D + g * 64;
          float v[64];
          for (int i = 0; i < 64; ++i) v[i] = oracle_f16_to_f32(src[i]);
          const float sc = int4_scale(v, 64);
          for (int i = 0; i < 32; ++i) {
            const uint8_t b = (uint8_t)(int4_code(v[2 * i], sc) | (int4_code(v[2 * i + 1], sc) << 4));
            const int bi = g * 32 + i;
            if (kv) page[codes + int4_vrow_byte(pos, bi, D)] = b;
            else page[(int64_t)pos * (D / 2) + bi] = b;
          }
          const uint16_t hs = oracle_f32_to_f16(sc);
          const int64_t si = kv ? int4_vscale_index(pos, g, gpr) : (int64_t)pos * gpr + g;
          memcpy(page + 2 * codes + (int64_t)kv * BS * gpr * 2 + si * 2, &hs, 2);
        }
      }
    }
  }
}

/* ----------------------------------------------------------- evict_tokens */
/* Per (seq, head) threshold as in kv_cache.cu:714-870; returns it via thr_out
 * (nullable, [S*H]).  The pools are fp16 [pool_NB, BS, H, D].  Sequences and
 * heads are processed in (seq, head) order, each fully before the next. */
void oracle_evict_tokens(const float* scores, int S, int H, int L, int32_t* bt, int MB,
                         int32_t* is_block_free, int NBF, uint16_t* kpool, uint16_t* vpool, int BS,
                         int D, float r, int sinks, int32_t* ret_idx, int32_t* ret_cnt,
                         float* thr_out) {
  if (sinks < 0) sinks = 0;
  if (sinks > L) sinks = L;
  const int64_t table = (int64_t)S * MB;
  float* s = (float*)malloc(sizeof(float) * (L > 0 ? L : 1));
  for (int seq = 0; seq < S; ++seq) {
    for (int h = 0; h < H; ++h) {
      const float* src = scores + ((int64_t)seq * H + h) * L;
      for (int t = 0; t < L; ++t) s[t] = t < sinks ? 1e38f : src[t];
      const int keep_c = (int)ceilf(r * (float)L);
      int keep = keep_c < L ? keep_c : L;
      if (keep < 1) keep = 1;
      float mn = 1e38f, mx = -1e38f;
      for (int t = 0; t < L; ++t) {
        mn = fminf(mn, s[t]);
        mx = fmaxf(mx, s[t]);
      }
      float thr;
      if (mn >= mx) {
        thr = mn - 1.0f;
      } else {
        float lo = mn, hi = mx;
        for (int it = 0; it < 32; ++it) {
          const float mid = fmaf(hi - lo, 0.5f, lo);
          int c = 0;
          for (int t = 0; t < L; ++t) c += s[t] >= mid;
          if (c >= keep) lo = mid; else hi = mid;
        }
        thr = lo;
      }
      if (thr_out) thr_out[seq * H + h] = thr;
      int kept = 0;
      for (int t = 0; t < L; ++t) {
        if (!(s[t] < thr)) {
          if (ret_idx) ret_idx[((int64_t)seq * H + h) * L + kept] = t;
          ++kept;
          continue;
        }
        const int lb = t / BS, pos = t % BS;
        const int64_t flat = (int64_t)seq * MB + lb;
        if (flat >= table) continue;
        const int phys = bt[flat];
        if (phys < 0 || phys >= NBF) continue;
        const int64_t base = (((int64_t)phys * BS + pos) * H + h) * D;
        for (int d = t % 32; d < D; d += 32) {
          kpool[base + d] = 0;
          vpool[base + d] = 0;
        }
      }
      if (ret_idx)
        for (int t = kept; t < L; ++t) ret_idx[((int64_t)seq * H + h) * L + t] = -1;
      if (ret_cnt) ret_cnt[seq * H + h] = kept;
      if (BS == 1) { /* the only block size at which a vote can complete */
        for (int t = 0; t < L; t += 32) {
          if (!(s[t] < thr)) continue;
          const int64_t flat = (int64_t)seq * MB + t;
          if (flat >= table) continue;
          const int phys = bt[flat];
          if (phys < 0 || phys >= NBF) continue;
          const int prev = is_block_free[phys]++;
          if (prev + 1 == H) bt[flat] = -1;
        }
      }
    }
  }
  free(s);
}

/* ------------------------------------------------------------ evict_cache */
void oracle_evict_cache(const float* scores, int NB, int BS, int H, int D, uint16_t* kpool,
                        uint16_t* vpool, float r) {
  float* w = (float*)malloc(sizeof(float) * BS);
  for (int b = 0; b < NB; ++b) {
    for (int h = 0; h < H; ++h) {
      for (int p = 0; p < BS; ++p) w[p] = scores[((int64_t)b * BS + p) * H + h];
      int keep = (int)(r * (float)BS);
      if (keep < 1) keep = 1;
      if (keep > BS) keep = BS;
      float thr = -1e38f;
      for (int k = 0; k < keep; ++k) {
        float best = -1e38f;
        int bp = -1;
        for (int p = 0; p < BS; ++p)
          if (w[p] > best) {
            best = w[p];
            bp = p;
          }
        thr = best;
        if (bp >= 0) w[bp] = -1e38f;
      }
      for (int p = 0; p < BS; ++p) {
        if (!(scores[((int64_t)b * BS + p) * H + h] < thr)) continue;
        const int64_t base = (((int64_t)b * BS + p) * H + h) * D;
        memset(kpool + base, 0, (size_t)D * 2);
        memset(vpool + base, 0, (size_t)D * 2);
      }
    }
  }
  free(w);
}

/* ------------------------------------------------------ paged attention */
/* K/V row of (phys, pos, head) as doubles, from an fp16 pool [NB, BS, H, D]
 * (fmt 0) or INT4 pages (fmt 1: codes [NB, H, BS, D/2], fp16 scales
 * [NB, H, BS, D/64], element = (code - 8) * float(scale)). */
typedef struct {
  int fmt;
  const uint16_t *kp, *vp;
  const uint8_t* pages;
  int H, D, BS;
} kv_src;

static void fetch_row(const kv_src* s, int kv, int64_t phys, int pos, int h, double* out) {
  if (s->fmt == 0) {
    const uint16_t* p = (kv ? s->vp : s->kp) + ((phys * s->BS + pos) * s->H + h) * s->D;
    for (int d = 0; d < s->D; ++d) out[d] = oracle_f16_to_f32(p[d]);
  } else {
    const int64_t pb = int4_page_bytes(s->BS, s->D), codes = (int64_t)s->BS * (s->D / 2);
    const int G = s->D / 64;
    const uint8_t* page = s->pages + (phys * s->H + h) * pb;
    const uint8_t* sc = page + 2 * codes + (int64_t)kv * s->BS * G * 2;
    for (int d = 0; d < s->D; ++d) {
      const uint8_t byte = kv ? page[codes + int4_vrow_byte(pos, d / 2, s->D)]
                              : page[(int64_t)pos * (s->D / 2) + d / 2];
      const int code = (d & 1) ? (byte >> 4) : (byte & 0xF);
      const int64_t si = kv ? int4_vscale_index(pos, d / 64, G) : (int64_t)pos * G + d / 64;
      uint16_t hs;
      memcpy(&hs, sc + si * 2, 2);
      out[d] = (double)(code - 8) * (double)oracle_f16_to_f32(hs);
    }
  }
}

/* H query heads over src->H pool (KV) heads: query head h reads KV head
 * h / (H / src->H).  causal = 0: every row of sequence b sees [ctx - W, ctx)
 * (attention.cu semantics); causal = 1: row i of the QL query rows is the
 * token at ctx - QL + i and sees [max(0, c_i - W), c_i), c_i = ctx - QL + i + 1
 * (an extension; the reference is non-causal). */
static void attention_core(const uint16_t* q, const kv_src* src, const int32_t* bt,
                           const int32_t* ctx_lens, int B, int QL, int H, int MB, int64_t NB,
                           int max_seq_len, int window, int causal, double* out) {
  const int KVH = src->H, D = src->D, BS = src->BS;
  const int group = H / KVH;
  if (window <= 0 || window > max_seq_len) window = max_seq_len;
  const double scale = (double)(1.0f / sqrtf((float)D));
  const int64_t rows = (int64_t)B * QL * H;
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t row = 0; row < rows; ++row) {
    const int hq = (int)(row % H);
    const int h = hq / group;
    const int b = (int)(row / ((int64_t)QL * H));
    const int qi = (int)((row / H) % QL);
    double qv[256], kr[256], vr[256], acc[256];
    for (int d = 0; d < D; ++d) {
      qv[d] = oracle_f16_to_f32(q[row * D + d]);
      acc[d] = 0.0;
    }
    int ctx = ctx_lens[b];
    if (causal) ctx = ctx - QL + qi + 1;
    const int ws = window < ctx ? ctx - window : 0;
    double m = -INFINITY, l = 0.0;
    for (int slot = 0; slot < MB; ++slot) {
      const int phys = bt[(int64_t)b * MB + slot];
      if (phys < 0 || (int64_t)phys >= NB) continue;
      const int t0 = slot * BS, t1 = t0 + BS;
      if (t0 >= ctx || t1 <= ws) continue;
      const int e0 = t0 > ws ? t0 : ws, e1 = t1 < ctx ? t1 : ctx;
      for (int t = e0; t < e1; ++t) {
        fetch_row(src, 0, phys, t - t0, h, kr);
        double sdot = 0.0;
        for (int d = 0; d < D; ++d) sdot += qv[d] * kr[d];
        sdot *= scale;
        fetch_row(src, 1, phys, t - t0, h, vr);
        const double mn = sdot > m ? sdot : m;
        const double a = exp(m - mn), p = exp(sdot - mn);
        l = l * a + p;
        for (int d = 0; d < D; ++d) acc[d] = acc[d] * a + p * vr[d];
        m = mn;
      }
    }
    for (int d = 0; d < D; ++d) out[row * D + d] = l > 0.0 ? acc[d] / l : 0.0;
  }
}

void oracle_paged_attention_f16_ex(const uint16_t* q, const uint16_t* kpool, const uint16_t* vpool,
                                   const int32_t* bt, const int32_t* ctx, int B, int QL, int H, int KVH,
                                   int D, int MB, int64_t NB, int BS, int max_seq_len, int window,
                                   int causal, double* out) {
  kv_src s = {0, kpool, vpool, 0, KVH, D, BS};
  attention_core(q, &s, bt, ctx, B, QL, H, MB, NB, max_seq_len, window, causal, out);
}

void oracle_paged_attention_f16(const uint16_t* q, const uint16_t* kpool, const uint16_t* vpool,
                                const int32_t* bt, const int32_t* ctx, int B, int QL, int H, int D,
                                int MB, int64_t NB, int BS, int max_seq_len, int window,
                                double* out) {
  oracle_paged_attention_f16_ex(q, kpool, vpool, bt, ctx, B, QL, H, H, D, MB, NB, BS, max_seq_len, window, 0,
                                out);
}

void oracle_paged_attention_int4_ex(const uint16_t* q, const uint8_t* pages, const int32_t* bt,
                                    const int32_t* ctx, int B, int QL, int H, int KVH, int D, int MB,
                                    int64_t NB, int BS, int max_seq_len, int window, int causal,
                                    double* out) {
  kv_src s = {1, 0, 0, pages, KVH, D, BS};
  attention_core(q, &s, bt, ctx, B, QL, H, MB, NB, max_seq_len, window, causal, out);
}

void oracle_paged_attention_int4(const uint16_t* q, const uint8_t* pages, const int32_t* bt,
                                 const int32_t* ctx, int B, int QL, int H, int D, int MB, int64_t NB,
                                 int BS, int max_seq_len, int window, double* out) {
  oracle_paged_attention_int4_ex(q, pages, bt, ctx, B, QL, H, H, D, MB, NB, BS, max_seq_len, window, 0, out);
}
