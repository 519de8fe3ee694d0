/*
 * dd_oracle.c — CPU ORACLE for the cascade decode-attention path.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library;
 * the product (dendrite_b200/) never calls it.
 *
 * It restates, in plain C, the reference's CPU algorithm for this path:
 *  - ReferenceBackend::decode (crates/dendrite-core/src/attention/backend.rs:206-265):
 *    gather the block table's per-block K/V (:228-234), concatenate along
 *    tokens (:241-242), tile KV heads for GQA with Tensor::repeat (:245-252,
 *    query head h reads KV head h % Hkv), scores = (q . k^T) * scale
 *    (:255-256, scale = 1/sqrt(D) in f32, :37), softmax over tokens (:259),
 *    out = p . v (:262); zeros for an empty table (:218-222).
 *    decode_batch is that loop over queries (:267-283).
 *  - merge_attention_outputs (crates/dendrite-ffi/src/flashinfer/cascade.rs:116-124).
 *  - QuantizedTensor::quantize / dequantize (crates/dendrite-core/src/quantization/fp8.rs:103-152)
 *    with the f32 quotient rounded to a real FP8 E4M3 code (RNE, saturating
 *    at 448 = the reference's clamp); scale = amax * f32(1/448), the affine
 *    multiply candle lowers `tensor / f64` to, or amax / 448 (mode 1).
 *  - MXFP8 (QuantFormat::MXFP8 / block_size 32, crates/dendrite-core/src/quantization/mod.rs:57-59,97,133-140;
 *    no reference code): OCP Microscaling Formats v1.0 — per 32 elements a
 *    shared E8M0 exponent e = max(-127, floor(log2 amax) - 8) and E4M3
 *    elements RNE-saturate(x * 2^-e).
 *
 * Parity status: the reference ships no golden vectors for attention numerics
 * or FP8 codes (its tests check shapes only, backend.rs:376-497, fp8.rs:183-231)
 * and cannot be built here (Rust + candle, no toolchain). The attention
 * restatement is therefore "parity unpinned" against the reference itself; it
 * is cross-checked against torch CPU math in tests/. The E4M3 / E8M0 codecs are
 * pinned against ml_dtypes and torch float8 casts (independent
 * implementations of the same formats) by tests/golden fixtures.
 *
 * Compiled with -ffp-contract=off: Rust (the reference) never fuses a*b+c.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ bf16 */
uint16_t or_f32_to_bf16(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40u); /* quiet NaN */
  b += 0x7fffu + ((b >> 16) & 1u); /* round to nearest even */
  return (uint16_t)(b >> 16);
}

float or_bf16_to_f32(uint16_t h) {
  uint32_t b = (uint32_t)h << 16;
  float f;
  memcpy(&f, &b, 4);
  return f;
}

/* ------------------------------------------------------------- FP8 E4M3 */
/* E4M3 ("fn"): bias 7, no infinities, 0x7F/0xFF NaN, max 448, min subnormal 2^-9. */
float or_e4m3_decode(uint8_t c) {
  const int s = c >> 7, e = (c >> 3) & 15, m = c & 7;
  float v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0) v = ldexpf((float)m, -9);
  else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

/* Round to nearest even, saturate finite overflow (and inf) to +-448. */
uint8_t or_e4m3_encode(float x) {
  if (isnan(x)) return 0x7f;
  const uint8_t sign = signbit(x) ? 0x80 : 0;
  const float a = fabsf(x);
  if (a >= 448.0f) return sign | 0x7e;
  if (a < 0.015625f) { /* below 2^-6: subnormal grid of step 2^-9 */
    const float q = rintf(a * 512.0f); /* exact scaling, RNE; q == 8 is 2^-6 = code 0x08 */
    return sign | (uint8_t)q;
  }
  int ex;
  frexpf(a, &ex);
  int E = ex - 1;                       /* floor(log2 a), -6..8 */
  const float m = ldexpf(a, -E);        /* [1, 2) */
  int mant = (int)rintf((m - 1.0f) * 8.0f);
  if (mant == 8) {
    mant = 0;
    E += 1;
  }
  int code = ((E + 7) << 3) | mant;
  if (code > 0x7e) code = 0x7e;
  return sign | (uint8_t)code;
}

/* E8M0: 2^(c - 127); 255 = NaN. */
float or_e8m0_decode(uint8_t c) {
  if (c == 255) return NAN;
  return ldexpf(1.0f, (int)c - 127);
}

/* Element i of a source buffer in f32 (dtype 2 = f32, 1 = bf16 bits). */
static inline float src_at(const void* src, int dtype, size_t i) {
  return dtype == 2 ? ((const float*)src)[i] : or_bf16_to_f32(((const uint16_t*)src)[i]);
}

float or_head_scale(float amax, int mode) {
  if (!(amax > 0.0f)) return 1.0f;
  return mode == 0 ? amax * (float)(1.0 / 448.0) : amax / 448.0f;
}

/* Per-(K/V, KV head) E4M3 over a pool [P][2][Hkv][16][D]. */
void or_quant_per_head(const void* src, int dtype, int64_t P, int Hkv, int D, int mode,
                       uint8_t* codes, float* scales) {
  const size_t per = (size_t)16 * D;
  const size_t nslices = (size_t)P * 2 * Hkv;
  float amax[64];
  for (int i = 0; i < 2 * Hkv; ++i) amax[i] = 0.0f;
  for (size_t s = 0; s < nslices; ++s) {
    const int kh = (int)(s % (size_t)(2 * Hkv));
    for (size_t e = 0; e < per; ++e) {
      const float a = fabsf(src_at(src, dtype, s * per + e));
      if (a > amax[kh]) amax[kh] = a;
    }
  }
  for (int i = 0; i < 2 * Hkv; ++i) scales[i] = or_head_scale(amax[i], mode);
  for (size_t s = 0; s < nslices; ++s) {
    const float sc = scales[s % (size_t)(2 * Hkv)];
    for (size_t e = 0; e < per; ++e)
      codes[s * per + e] = or_e4m3_encode(src_at(src, dtype, s * per + e) / sc);
  }
}

/* MXFP8 over n elements (n % 32 == 0): codes[n], scales[n/32] (E8M0). */
void or_quant_mx(const void* src, int dtype, int64_t n, uint8_t* codes, uint8_t* scales) {
  for (int64_t b = 0; b < n / 32; ++b) {
    float amax = 0.0f;
    for (int k = 0; k < 32; ++k) {
      const float a = fabsf(src_at(src, dtype, (size_t)(b * 32 + k)));
      if (a > amax) amax = a;
    }
    int e = -127;
    if (amax > 0.0f) {
      int ex;
      frexpf(amax, &ex);
      e = (ex - 1) - 8;
      if (e < -127) e = -127;
    }
    scales[b] = (uint8_t)(e + 127);
    const float inv = ldexpf(1.0f, -e);
    for (int k = 0; k < 32; ++k)
      codes[b * 32 + k] = or_e4m3_encode(src_at(src, dtype, (size_t)(b * 32 + k)) * inv);
  }
}

/* Round trip. format 3 = E4M3 per head (scales f32[2*Hkv]), 4 = MXFP8.
 * out_dtype 1 = bf16 bits (RNE of the f32 product), 2 = f32. */
void or_dequant(const uint8_t* codes, int format, const void* scales, int64_t P, int Hkv, int D,
                void* out, int out_dtype) {
  const size_t n = (size_t)P * 2 * Hkv * 16 * D;
  const size_t per = (size_t)16 * D;
  for (size_t i = 0; i < n; ++i) {
    float sc = format == 3 ? ((const float*)scales)[(i / per) % (size_t)(2 * Hkv)]
                           : or_e8m0_decode(((const uint8_t*)scales)[i / 32]);
    const float v = or_e4m3_decode(codes[i]) * sc;
    if (out_dtype == 2) ((float*)out)[i] = v;
    else ((uint16_t*)out)[i] = or_f32_to_bf16(v);
  }
}

/* ------------------------------------------------------------ attention */
typedef struct {
  int Hq, Hkv, D, gqa_grouped;
  float scale;
  const void* pool; /* [P][2][Hkv][16][D], f32 or bf16 bits */
  int pool_dtype;
  int64_t num_pages;
  const float* q;   /* [B][Hq][D] f32 */
  const int32_t* indptr;
  const uint32_t* ids;
  const int32_t* ntok;
  float* out;       /* [B][Hq][D] */
  float* lse;       /* [B][Hq] natural log, may be NULL */
  int B;
  int next;         /* work counter */
  pthread_mutex_t mu;
  float* ws;        /* caller scratch: ws_per_thread floats per worker, or NULL */
  size_t ws_per_thread;
  int next_ws;      /* next worker's scratch slice */
} decode_job;

/* One query, literally as ReferenceBackend::decode: gather -> cat -> repeat ->
 * matmul -> scale -> softmax -> matmul, all in f32. */
static void decode_one(const decode_job* j, int b, float* scratch_k, float* scratch_v,
                       float* rep_k, float* rep_v, float* sc) {
  const int Hq = j->Hq, Hkv = j->Hkv, D = j->D;
  const int nb_all = j->indptr[b + 1] - j->indptr[b];
  const int ntok = j->ntok[b];
  int nb = (ntok + 15) / 16;
  if (nb > nb_all) nb = nb_all;
  float* out = j->out + (size_t)b * Hq * D;
  if (nb == 0) { /* backend.rs:218-222: no cached context -> zeros */
    memset(out, 0, sizeof(float) * (size_t)Hq * D);
    if (j->lse)
      for (int h = 0; h < Hq; ++h) j->lse[(size_t)b * Hq + h] = -INFINITY;
    return;
  }
  /* gather + cat along tokens: K[Hkv][T][D] */
  int T = 0;
  for (int i = 0; i < nb; ++i) {
    const uint32_t id = j->ids[j->indptr[b] + i];
    const int t_blk = (i == nb - 1 && ntok % 16) ? ntok % 16 : 16;
    if ((int64_t)id >= j->num_pages) continue; /* unknown block: skipped (backend.rs:228-234) */
    for (int h = 0; h < Hkv; ++h)
      for (int t = 0; t < t_blk; ++t) {
        const size_t kb = ((((size_t)id * 2 + 0) * Hkv + h) * 16 + t) * D;
        const size_t vb = ((((size_t)id * 2 + 1) * Hkv + h) * 16 + t) * D;
        for (int d = 0; d < D; ++d) {
          /* layout of the concatenated tensors: [Hkv][Tmax][D], filled at row T + t */
          scratch_k[((size_t)h * (nb * 16) + T + t) * D + d] = src_at(j->pool, j->pool_dtype, kb + d);
          scratch_v[((size_t)h * (nb * 16) + T + t) * D + d] = src_at(j->pool, j->pool_dtype, vb + d);
        }
      }
    T += t_blk;
  }
  const int Tmax = nb * 16;
  if (T == 0) {
    memset(out, 0, sizeof(float) * (size_t)Hq * D);
    if (j->lse)
      for (int h = 0; h < Hq; ++h) j->lse[(size_t)b * Hq + h] = -INFINITY;
    return;
  }
  /* GQA: Tensor::repeat((1, Hq/Hkv, 1, 1)) materialises the tiled copy. */
  const int g = Hq / Hkv;
  for (int h = 0; h < Hq; ++h) {
    const int src = j->gqa_grouped ? h / g : h % Hkv;
    memcpy(rep_k + (size_t)h * T * D, scratch_k + (size_t)src * Tmax * D, sizeof(float) * (size_t)T * D);
    memcpy(rep_v + (size_t)h * T * D, scratch_v + (size_t)src * Tmax * D, sizeof(float) * (size_t)T * D);
  }
  for (int h = 0; h < Hq; ++h) {
    const float* qh = j->q + ((size_t)b * Hq + h) * D;
    const float* kh = rep_k + (size_t)h * T * D;
    const float* vh = rep_v + (size_t)h * T * D;
    float mx = -INFINITY;
    for (int t = 0; t < T; ++t) {
      float acc = 0.0f;
      for (int d = 0; d < D; ++d) acc += qh[d] * kh[(size_t)t * D + d];
      sc[t] = acc * j->scale;
      if (sc[t] > mx) mx = sc[t];
    }
    float sum = 0.0f;
    for (int t = 0; t < T; ++t) {
      sc[t] = expf(sc[t] - mx);
      sum += sc[t];
    }
    for (int t = 0; t < T; ++t) sc[t] /= sum;
    float* oh = out + (size_t)h * D;
    for (int d = 0; d < D; ++d) oh[d] = 0.0f;
    for (int t = 0; t < T; ++t) {
      const float p = sc[t];
      const float* vr = vh + (size_t)t * D;
      for (int d = 0; d < D; ++d) oh[d] += p * vr[d];
    }
    if (j->lse) j->lse[(size_t)b * Hq + h] = mx + logf(sum);
  }
}

static int max_tokens(const decode_job* j) {
  int m = 0;
  for (int b = 0; b < j->B; ++b) {
    const int nb = j->indptr[b + 1] - j->indptr[b];
    const int t = nb * 16;
    if (t > m) m = t;
  }
  return m;
}

/* Scratch floats one worker needs for queries of up to T tokens. */
size_t or_decode_scratch_floats(int Hq, int Hkv, int D, int T) {
  const size_t kvsz = (size_t)Hkv * T * D, repsz = (size_t)Hq * T * D;
  return 2 * (kvsz ? kvsz : 1) + 2 * (repsz ? repsz : 1) + (T ? T : 1);
}

static void* decode_worker(void* arg) {
  decode_job* j = (decode_job*)arg;
  const int T = max_tokens(j);
  const size_t kvsz = (size_t)j->Hkv * T * j->D, repsz = (size_t)j->Hq * T * j->D;
  const size_t need = or_decode_scratch_floats(j->Hq, j->Hkv, j->D, T);
  float* base = NULL;
  int owned = 0;
  if (j->ws && j->ws_per_thread >= need) {
    pthread_mutex_lock(&j->mu);
    base = j->ws + (size_t)j->next_ws++ * j->ws_per_thread;
    pthread_mutex_unlock(&j->mu);
  } else {
    base = (float*)malloc(sizeof(float) * need);
    owned = 1;
  }
  if (base) {
    float* sk = base;
    float* sv = sk + (kvsz ? kvsz : 1);
    float* rk = sv + (kvsz ? kvsz : 1);
    float* rv = rk + (repsz ? repsz : 1);
    float* sc = rv + (repsz ? repsz : 1);
    for (;;) {
      pthread_mutex_lock(&j->mu);
      const int b = j->next++;
      pthread_mutex_unlock(&j->mu);
      if (b >= j->B) break;
      decode_one(j, b, sk, sv, rk, rv, sc);
    }
  }
  if (owned) free(base);
  return NULL;
}

/* ReferenceBackend::decode_batch over B queries with `threads` workers.
 * ws, when not NULL, holds ws_per_thread floats for each worker (at least
 * or_decode_scratch_floats of the batch's longest table), so a timed loop can
 * keep the gather / repeat scratch allocated and touched across calls.
 * Returns 0 on success. */
int or_decode_batch_ws(int B, int Hq, int Hkv, int D, int gqa_grouped, float scale,
                       const void* pool, int pool_dtype, int64_t num_pages, const float* q,
                       const int32_t* indptr, const uint32_t* ids, const int32_t* ntok, float* out,
                       float* lse, int threads, float* ws, size_t ws_per_thread) {
  decode_job j;
  j.Hq = Hq; j.Hkv = Hkv; j.D = D; j.gqa_grouped = gqa_grouped;
  j.scale = scale > 0.0f ? scale : 1.0f / sqrtf((float)D);
  j.pool = pool; j.pool_dtype = pool_dtype; j.num_pages = num_pages;
  j.q = q; j.indptr = indptr; j.ids = ids; j.ntok = ntok; j.out = out; j.lse = lse;
  j.B = B; j.next = 0;
  j.ws = ws; j.ws_per_thread = ws_per_thread; j.next_ws = 0;
  pthread_mutex_init(&j.mu, NULL);
  if (threads < 1) threads = 1;
  if (threads > 1024) threads = 1024;
  pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * threads);
  int started = 0;
  for (int i = 0; i < threads; ++i)
    if (pthread_create(&tid[i], NULL, decode_worker, &j) == 0) ++started;
  if (started == 0) decode_worker(&j);
  for (int i = 0; i < started; ++i) pthread_join(tid[i], NULL);
  free(tid);
  pthread_mutex_destroy(&j.mu);
  return 0;
}

/* The same with per-worker scratch allocated (and first touched) inside. */
int or_decode_batch(int B, int Hq, int Hkv, int D, int gqa_grouped, float scale,
                    const void* pool, int pool_dtype, int64_t num_pages, const float* q,
                    const int32_t* indptr, const uint32_t* ids, const int32_t* ntok, float* out,
                    float* lse, int threads) {
  return or_decode_batch_ws(B, Hq, Hkv, D, gqa_grouped, scale, pool, pool_dtype, num_pages, q,
                            indptr, ids, ntok, out, lse, threads, NULL, 0);
}

/* ReferenceBackend::prefill (crates/dendrite-core/src/attention/backend.rs:
 * 163-204) for batch 1: q [Hq][S][D], k, v [Hkv][S][D] f32. GQA by
 * Tensor::repeat (tiled: head h reads KV head h % Hkv, :176-183); scores
 * q.k^T * scale (:185-187) plus the causal mask, 0 on and below the diagonal
 * and -inf above (create_causal_mask, :146-158); softmax over the keys
 * (max-subtract, exp, sum, divide); @ v. out [Hq][S][D]. */
void or_prefill(int S, int Hq, int Hkv, int D, float scale, const float* q, const float* k,
                const float* v, float* out) {
  const float sc_f = scale > 0.0f ? scale : 1.0f / sqrtf((float)D);
  float* sc = (float*)malloc(sizeof(float) * (S ? S : 1));
  if (!sc) return;
  for (int h = 0; h < Hq; ++h) {
    const int src = h % Hkv;
    const float* kh = k + (size_t)src * S * D;
    const float* vh = v + (size_t)src * S * D;
    for (int i = 0; i < S; ++i) {
      const float* qi = q + ((size_t)h * S + i) * D;
      float mx = -INFINITY;
      for (int jj = 0; jj < S; ++jj) {
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc += qi[d] * kh[(size_t)jj * D + d];
        sc[jj] = acc * sc_f + (jj > i ? -INFINITY : 0.0f);
        if (sc[jj] > mx) mx = sc[jj];
      }
      float sum = 0.0f;
      for (int jj = 0; jj < S; ++jj) {
        sc[jj] = expf(sc[jj] - mx);
        sum += sc[jj];
      }
      for (int jj = 0; jj < S; ++jj) sc[jj] /= sum;
      float* o = out + ((size_t)h * S + i) * D;
      for (int d = 0; d < D; ++d) o[d] = 0.0f;
      for (int jj = 0; jj < S; ++jj)
        for (int d = 0; d < D; ++d) o[d] += sc[jj] * vh[(size_t)jj * D + d];
    }
  }
  free(sc);
}

/* merge_attention_outputs (cascade.rs:116-124), element-wise over n rows of D. */
void or_merge_states(int n, int D, const float* o1, const float* l1, const float* o2,
                     const float* l2, float* o, float* l) {
  for (int r = 0; r < n; ++r) {
    const float max_lse = l1[r] > l2[r] ? l1[r] : l2[r];
    const float e1 = expf(l1[r] - max_lse);
    const float e2 = expf(l2[r] - max_lse);
    const float s = e1 + e2;
    for (int d = 0; d < D; ++d) o[(size_t)r * D + d] = (o1[(size_t)r * D + d] * e1 + o2[(size_t)r * D + d] * e2) / s;
    l[r] = max_lse + logf(s);
  }
}

/* ------------------------------------------------------- array helpers */
void or_e4m3_encode_n(const float* x, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = or_e4m3_encode(x[i]);
}
void or_e4m3_decode_n(const uint8_t* c, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = or_e4m3_decode(c[i]);
}
void or_f32_to_bf16_n(const float* x, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = or_f32_to_bf16(x[i]);
}
