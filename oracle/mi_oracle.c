/* TEST INFRASTRUCTURE ONLY -- the CPU oracle (checker), never the product.
 *
 * Restatement, in plain C, of the reference's arithmetic for the decode hot
 * path. Built with -ffp-contract=off: every `a * b + c` below is two IEEE
 * roundings, exactly like the reference's scalar ops, which its Release build
 * compiles without -march (so without FMA). fmaf() appears only where the
 * reference's AVX2 code issues _mm256_fmadd_ps.
 *
 * Parity is pinned: tests/test_oracle_pin.py compares every function here,
 * bit for bit, with the reference compiled from source (oracle/_ref) and with
 * the known-answer cases of the reference's tests/test_quant.cpp and
 * tests/test_ops_cpu.cpp.
 */
#include "mi_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* IEEE binary16 -> binary32, exact for every input (quant.cpp:24-58 computes
 * the same map; the AVX2 path uses F16C's vcvtph2ps, quant_avx2.cpp:113-117). */
float mio_fp16_to_fp32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      int s = 0;
      while (!(m & 0x400u)) { m <<= 1; s++; }
      bits = sign | ((uint32_t)(113 - s) << 23) | ((m & 0x3ffu) << 13);
    }
  } else if (e == 0x1f) {
    bits = sign | 0x7f800000u | (m << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* binary32 -> binary16, round to nearest even (quant.cpp:70-118). */
uint16_t mio_fp32_to_fp16(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  uint32_t sign = (b >> 16) & 0x8000u;
  uint32_t e8 = (b >> 23) & 0xffu;
  uint32_t m = b & 0x7fffffu;
  if (e8 == 0xff) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0u));
  int32_t e = (int32_t)e8 - 112;
  if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    m |= 0x800000u;
    int shift = 14 - e;
    uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t q = m >> 13, rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) {
    q++;
    if (q == 0x400u) {
      q = 0;
      e++;
      if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    }
  }
  return (uint16_t)(sign | ((uint32_t)e << 10) | q);
}

/* Shared body of the two quantizers (quant.cpp:130-160 and 199-218): per
 * 32-block amax, d = amax/127, id = 1/d (or 0), q = lrintf(x*id) clamped. */
static void quantize_block(const float* xb, float* d_out, int8_t* qs) {
  float amax = 0.0f;
  for (int j = 0; j < 32; j++) {
    float av = fabsf(xb[j]);
    if (av > amax) amax = av;
  }
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  *d_out = d;
  for (int j = 0; j < 32; j++) {
    float scaled = xb[j] * id;
    int32_t q = (int32_t)lrintf(scaled);
    if (q > 127) q = 127;
    if (q < -127) q = -127;
    qs[j] = (int8_t)q;
  }
}

void mio_quantize_row_q8_0_act(const float* x, uint8_t* y, int64_t n) {
  for (int64_t i = 0; i < n / 32; i++) {
    float d;
    quantize_block(x + i * 32, &d, (int8_t*)(y + i * 36 + 4));
    memcpy(y + i * 36, &d, 4);
  }
}

void mio_quantize_row_q8_0(const float* x, uint8_t* y, int64_t n) {
  for (int64_t i = 0; i < n / 32; i++) {
    float d;
    quantize_block(x + i * 32, &d, (int8_t*)(y + i * 34 + 2));
    uint16_t h = mio_fp32_to_fp16(d);
    memcpy(y + i * 34, &h, 2);
  }
}

void mio_dequantize_row_q8_0(const uint8_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n / 32; i++) {
    uint16_t h;
    memcpy(&h, x + i * 34, 2);
    float d = mio_fp16_to_fp32(h);
    const int8_t* qs = (const int8_t*)(x + i * 34 + 2);
    for (int j = 0; j < 32; j++) y[i * 32 + j] = (float)qs[j] * d;
  }
}

int32_t mio_block_isum(const int8_t* x, const int8_t* y) {
  int32_t s = 0;
  for (int j = 0; j < 32; j++) s += (int32_t)x[j] * (int32_t)y[j];
  return s;
}

/* The 8 int32 lanes of one 32-wide block dot, as q8_0_block_dot32x8 leaves
 * them (quant_avx2.cpp:97-105): lane j = sum of bytes 4j..4j+3. With |q| <=
 * 127 the maddubs pair sums never saturate, so plain integer sums are exact. */
void mio_block_lanes(const int8_t* x, const int8_t* y, int32_t lanes[8]) {
  for (int j = 0; j < 8; j++) {
    int32_t s = 0;
    for (int k = 4 * j; k < 4 * j + 4; k++) s += (int32_t)x[k] * (int32_t)y[k];
    lanes[j] = s;
  }
}

/* mi_vec_dot_q8_0_wact_avx2_f16c (quant_avx2.cpp:170-181): eight lane
 * accumulators, each a sequential fmaf over blocks, then hsum_ps
 * (quant_avx2.cpp:74-83) = ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)). */
float mio_vec_dot_q8_0_wact(const uint8_t* w, const uint8_t* a, int64_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t i = 0; i < n / 32; i++) {
    const uint8_t* wb = w + i * 34;
    const uint8_t* ab = a + i * 36;
    uint16_t hd;
    float ad;
    memcpy(&hd, wb, 2);
    memcpy(&ad, ab, 4);
    float dxdy = mio_fp16_to_fp32(hd) * ad;
    int32_t lanes[8];
    mio_block_lanes((const int8_t*)(wb + 2), (const int8_t*)(ab + 4), lanes);
    for (int j = 0; j < 8; j++) acc[j] = fmaf((float)lanes[j], dxdy, acc[j]);
  }
  float s0 = acc[0] + acc[4], s1 = acc[1] + acc[5], s2 = acc[2] + acc[6], s3 = acc[3] + acc[7];
  return (s0 + s1) + (s2 + s3);
}

/* mi_vec_dot_q8_0_wact_scalar (quant.cpp:221-230): one sequential fmaf. */
float mio_vec_dot_q8_0_wact_scalar(const uint8_t* w, const uint8_t* a, int64_t n) {
  float acc = 0.0f;
  for (int64_t i = 0; i < n / 32; i++) {
    const uint8_t* wb = w + i * 34;
    const uint8_t* ab = a + i * 36;
    uint16_t hd;
    float ad;
    memcpy(&hd, wb, 2);
    memcpy(&ad, ab, 4);
    int32_t isum = mio_block_isum((const int8_t*)(wb + 2), (const int8_t*)(ab + 4));
    float dxdy = mio_fp16_to_fp32(hd) * ad;
    acc = fmaf((float)isum, dxdy, acc);
  }
  return acc;
}

/* mi_compute_mul_mat, Q8_0 branch (ops_cpu.cpp:226-237): rows independent. */
void mio_mul_mat_q8_0(const uint8_t* w, int64_t k, int64_t n, const uint8_t* act, int64_t m,
                      float* dst) {
  int64_t wrow = k / 32 * 34, arow = k / 32 * 36;
  for (int64_t i = 0; i < n; i++)
    for (int64_t j = 0; j < m; j++)
      dst[j * n + i] = mio_vec_dot_q8_0_wact(w + i * wrow, act + j * arow, k);
}

/* mi_compute_get_rows, Q8_0 table (ops_cpu.cpp:110-141, quant.cpp:155-163). */
void mio_get_rows_q8_0(const uint8_t* table, int64_t ne0, const int32_t* ids, int64_t n_ids,
                       float* dst) {
  int64_t row = ne0 / 32 * 34;
  for (int64_t j = 0; j < n_ids; j++)
    mio_dequantize_row_q8_0(table + (int64_t)ids[j] * row, dst + j * ne0, ne0);
}

/* mi_compute_rms_norm (ops_cpu.cpp:143-165). */
void mio_rms_norm(const float* x, int64_t ne0, int64_t n_rows, float eps, float* dst) {
  for (int64_t r = 0; r < n_rows; r++) {
    const float* xr = x + r * ne0;
    float sumsq = 0.0f;
    for (int64_t i = 0; i < ne0; i++) sumsq += xr[i] * xr[i];
    float mean = sumsq / (float)ne0;
    float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < ne0; i++) dst[r * ne0 + i] = xr[i] * scale;
  }
}

/* ew_binop with mul / add (ops_cpu.cpp:56-80, 167-175); b_bcast: b is one
 * row broadcast over all rows. */
void mio_mul_row(const float* a, const float* b, int64_t ne0, int64_t n_rows, int b_bcast,
                 float* dst) {
  for (int64_t r = 0; r < n_rows; r++)
    for (int64_t i = 0; i < ne0; i++)
      dst[r * ne0 + i] = a[r * ne0 + i] * b[(b_bcast ? 0 : r) * ne0 + i];
}

void mio_add_row(const float* a, const float* b, int64_t ne0, int64_t n_rows, int b_bcast,
                 float* dst) {
  for (int64_t r = 0; r < n_rows; r++)
    for (int64_t i = 0; i < ne0; i++)
      dst[r * ne0 + i] = a[r * ne0 + i] + b[(b_bcast ? 0 : r) * ne0 + i];
}

float mio_expf(float x) { return expf(x); }

/* mi_compute_silu (ops_cpu.cpp:412-427). */
void mio_silu(const float* x, int64_t n, float* dst) {
  for (int64_t i = 0; i < n; i++) dst[i] = x[i] / (1.0f + expf(-x[i]));
}

/* mi_compute_rope, NEOX pairing (ops_cpu.cpp:270-302). */
void mio_rope_neox(const float* x, int64_t head_dim, int64_t n_head, int64_t n_tokens,
                   int32_t n_past, int32_t n_dims, float freq_base, float* dst) {
  int64_t half = n_dims / 2;
  for (int64_t t = 0; t < n_tokens; t++) {
    int64_t pos = n_past + t;
    for (int64_t h = 0; h < n_head; h++) {
      const float* xr = x + (t * n_head + h) * head_dim;
      float* yr = dst + (t * n_head + h) * head_dim;
      for (int64_t p = 0; p < half; p++) {
        float freq = powf(freq_base, -(float)(2 * p) / (float)n_dims);
        float theta = (float)pos * freq;
        float c = cosf(theta), s = sinf(theta);
        float x0 = xr[p], x1 = xr[p + half];
        yr[p] = x0 * c - x1 * s;
        yr[p + half] = x0 * s + x1 * c;
      }
      for (int64_t i = n_dims; i < head_dim; i++) yr[i] = xr[i];
    }
  }
}

/* mi_compute_attn_qk (ops_cpu.cpp:356-380): scores[i, j, h], d ascending. */
void mio_attn_qk(const float* q, const float* cache_k, int64_t head_dim, int64_t n_head,
                 int64_t n_head_kv, int64_t n_kv, int64_t n_tokens, float* scores) {
  int64_t n_rep = n_head / n_head_kv;
  for (int64_t h = 0; h < n_head; h++) {
    int64_t kvh = h / n_rep;
    for (int64_t i = 0; i < n_kv; i++) {
      const float* kr = cache_k + (i * n_head_kv + kvh) * head_dim;
      for (int64_t j = 0; j < n_tokens; j++) {
        const float* qr = q + (j * n_head + h) * head_dim;
        float acc = 0.0f;
        for (int64_t d = 0; d < head_dim; d++) acc += kr[d] * qr[d];
        scores[(h * n_tokens + j) * n_kv + i] = acc;
      }
    }
  }
}

/* mi_compute_softmax (ops_cpu.cpp:304-346): causal, scale before mask,
 * sequential sum, reciprocal multiply, masked columns zero. */
void mio_softmax(const float* x, int64_t n_kv, int64_t n_tokens, int64_t n_head, int32_t n_past,
                 float scale, float* dst) {
  for (int64_t h = 0; h < n_head; h++) {
    for (int64_t j = 0; j < n_tokens; j++) {
      const float* xr = x + (h * n_tokens + j) * n_kv;
      float* yr = dst + (h * n_tokens + j) * n_kv;
      int64_t allowed = n_past + j + 1;
      if (allowed > n_kv) allowed = n_kv;
      float maxv = -INFINITY;
      for (int64_t i = 0; i < allowed; i++) {
        float v = xr[i] * scale;
        if (v > maxv) maxv = v;
      }
      float sum = 0.0f;
      for (int64_t i = 0; i < allowed; i++) {
        float v = xr[i] * scale;
        float e = expf(v - maxv);
        yr[i] = e;
        sum += e;
      }
      float inv = 1.0f / sum;
      for (int64_t i = 0; i < allowed; i++) yr[i] *= inv;
      for (int64_t i = allowed; i < n_kv; i++) yr[i] = 0.0f;
    }
  }
}

/* mi_compute_attn_kqv (ops_cpu.cpp:386-410): out[o, h, j], t ascending over
 * every position including masked (zero) ones. */
void mio_attn_kqv(const float* probs, const float* cache_v, int64_t head_dim, int64_t n_head,
                  int64_t n_head_kv, int64_t n_kv, int64_t n_tokens, float* dst) {
  int64_t n_rep = n_head / n_head_kv;
  for (int64_t h = 0; h < n_head; h++) {
    int64_t kvh = h / n_rep;
    for (int64_t o = 0; o < head_dim; o++) {
      for (int64_t j = 0; j < n_tokens; j++) {
        const float* pr = probs + (h * n_tokens + j) * n_kv;
        float acc = 0.0f;
        for (int64_t t = 0; t < n_kv; t++) acc += cache_v[(t * n_head_kv + kvh) * head_dim + o] * pr[t];
        dst[(j * n_head + h) * head_dim + o] = acc;
      }
    }
  }
}

int32_t mio_sample_greedy(const float* logits, int32_t n_vocab) {
  int32_t best = 0;
  float bv = logits[0];
  for (int32_t i = 1; i < n_vocab; i++)
    if (logits[i] > bv) {
      bv = logits[i];
      best = i;
    }
  return best;
}

/* rms_norm_and_scale (model_qwen2.cpp:58-60): norm, then multiply by weight. */
static void norm_scale(const float* x, const float* w, int64_t ne0, int64_t n_rows, float eps,
                       float* tmp, float* dst) {
  mio_rms_norm(x, ne0, n_rows, eps, tmp);
  mio_mul_row(tmp, w, ne0, n_rows, 1, dst);
}

static void quantize_rows(const float* x, int64_t ne0, int64_t n_rows, uint8_t* q) {
  for (int64_t r = 0; r < n_rows; r++) mio_quantize_row_q8_0_act(x + r * ne0, q + r * (ne0 / 32 * 36), ne0);
}

/* mi_qwen2_forward's graph (model_qwen2.cpp:133-191 per layer, 236-267
 * around), evaluated node by node in its topological order. */
void mio_qwen2_forward(const mio_hparams* hp, const mio_weights* w, float* const* cache_k,
                       float* const* cache_v, int32_t n_ctx, const int32_t* tokens,
                       int32_t n_tokens, int32_t n_past, int32_t last_logits_only,
                       float* logits, float* layer_out) {
  (void)n_ctx;
  const int64_t T = n_tokens, E = hp->n_embd, H = hp->n_head, HKV = hp->n_head_kv,
                D = hp->head_dim, FF = hp->n_ff, V = hp->n_vocab;
  const int64_t n_kv = n_past + T;
  const float scale = 1.0f / sqrtf((float)hp->head_dim);
  float* x = malloc(sizeof(float) * E * T);
  float* tmp = malloc(sizeof(float) * (FF > E ? FF : E) * T);
  float* normed = malloc(sizeof(float) * E * T);
  uint8_t* qa = malloc((size_t)(FF > E ? FF : E) / 32 * 36 * T);
  float* q = malloc(sizeof(float) * E * T);
  float* k = malloc(sizeof(float) * HKV * D * T);
  float* v = malloc(sizeof(float) * HKV * D * T);
  float* qr = malloc(sizeof(float) * E * T);
  float* kr = malloc(sizeof(float) * HKV * D * T);
  float* scores = malloc(sizeof(float) * n_kv * T * H);
  float* probs = malloc(sizeof(float) * n_kv * T * H);
  float* kqv = malloc(sizeof(float) * E * T);
  float* gate = malloc(sizeof(float) * FF * T);
  float* up = malloc(sizeof(float) * FF * T);
  float* act = malloc(sizeof(float) * FF * T);

  mio_get_rows_q8_0(w->token_embd, E, tokens, T, x);
  for (int l = 0; l < hp->n_layer; l++) {
    const mio_layer* L = &w->layers[l];
    norm_scale(x, L->attn_norm, E, T, hp->rms_eps, tmp, normed);
    quantize_rows(normed, E, T, qa);
    mio_mul_mat_q8_0(L->wq, E, E, qa, T, tmp);
    mio_add_row(tmp, L->bq, E, T, 1, q);
    mio_mul_mat_q8_0(L->wk, E, HKV * D, qa, T, tmp);
    mio_add_row(tmp, L->bk, HKV * D, T, 1, k);
    mio_mul_mat_q8_0(L->wv, E, HKV * D, qa, T, tmp);
    mio_add_row(tmp, L->bv, HKV * D, T, 1, v);
    mio_rope_neox(q, D, H, T, n_past, (int32_t)D, hp->rope_freq_base, qr);
    mio_rope_neox(k, D, HKV, T, n_past, (int32_t)D, hp->rope_freq_base, kr);
    memcpy(cache_k[l] + (int64_t)n_past * HKV * D, kr, sizeof(float) * HKV * D * T);
    memcpy(cache_v[l] + (int64_t)n_past * HKV * D, v, sizeof(float) * HKV * D * T);
    mio_attn_qk(qr, cache_k[l], D, H, HKV, n_kv, T, scores);
    mio_softmax(scores, n_kv, T, H, n_past, scale, probs);
    mio_attn_kqv(probs, cache_v[l], D, H, HKV, n_kv, T, kqv);
    quantize_rows(kqv, E, T, qa);
    mio_mul_mat_q8_0(L->wo, E, E, qa, T, tmp);
    mio_add_row(x, tmp, E, T, 0, x); /* after_attn = residual + attn_proj */
    norm_scale(x, L->ffn_norm, E, T, hp->rms_eps, tmp, normed);
    quantize_rows(normed, E, T, qa);
    mio_mul_mat_q8_0(L->wgate, E, FF, qa, T, gate);
    mio_mul_mat_q8_0(L->wup, E, FF, qa, T, up);
    mio_silu(gate, FF * T, act);
    mio_mul_row(act, up, FF, T, 0, act);
    quantize_rows(act, FF, T, qa);
    mio_mul_mat_q8_0(L->wdown, FF, E, qa, T, tmp);
    mio_add_row(x, tmp, E, T, 0, x);
    if (layer_out) memcpy(layer_out + (int64_t)l * E * T, x, sizeof(float) * E * T);
  }
  norm_scale(x, w->output_norm, E, T, hp->rms_eps, tmp, normed);
  int64_t first = last_logits_only ? T - 1 : 0;
  int64_t m = T - first;
  quantize_rows(normed + first * E, E, m, qa);
  mio_mul_mat_q8_0(w->output, E, V, qa, m, logits);

  free(x); free(tmp); free(normed); free(qa); free(q); free(k); free(v); free(qr); free(kr);
  free(scores); free(probs); free(kqv); free(gate); free(up); free(act);
}
