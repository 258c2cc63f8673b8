/*
 * myl_forward.c — CPU restatement of Myelith's integer decoder forward pass.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product); see
 * myl_forward.h for the reference functions restated here and for the two
 * exact evaluation-order freedoms it uses.
 */
#include "myl_forward.h"

#include <stdlib.h>
#include <string.h>

#include "myl_oracle.h"

typedef __int128 i128;
typedef unsigned __int128 u128;

/* ---- fixed_point.rs:155-169 ----------------------------------------------- */

static i128 rne_i128(i128 value, unsigned shift) {
  if (shift == 0) return value;
  i128 one = 1;
  i128 mask = (one << shift) - 1;
  i128 half = one << (shift - 1);
  i128 q = value >> shift;
  i128 r = value & mask;
  if (r > half || (r == half && (q & 1) != 0)) return q + 1;
  return q;
}

/* ---- rmsnorm.rs:20-24 -------------------------------------------------------- */

int64_t mylo_inv_n_q20(int64_t n) {
  if (n <= 0) return 0; /* the reference asserts n > 0 */
  return (((int64_t)1 << 20) + n / 2) / n;
}

/* ---- fixed_point.rs:117-146: Newton on u64, then round to nearest ----------- */

uint64_t mylo_isqrt_round(uint64_t n) {
  if (n == 0) return 0;
  uint64_t r = n;
  uint64_t next = n / 2 + (n & 1); /* div_ceil(2) */
  while (next < r) {
    r = next;
    next = (r + n / r) / 2;
  }
  while (r > 0 && r > n / r) r -= 1;
  while ((r + 1) <= n / (r + 1)) r += 1;
  uint64_t below = n - r * r;
  uint64_t above = (r + 1) * (r + 1) - n;
  return above < below ? r + 1 : r;
}

/* ---- fixed_point.rs:102-107 ------------------------------------------------- */

int64_t mylo_inv_sqrt_q15(int64_t head_dim) {
  if (head_dim <= 0) return 0; /* the reference asserts head_dim > 0 */
  return (int64_t)mylo_isqrt_round(((uint64_t)1 << 30) / (uint64_t)head_dim);
}

/* ---- rmsnorm.rs:61-153 --------------------------------------------------------
 * ref = max(x_shifts); acc = sum_i x_i^2 << 2*(ref - x_shifts[i]) in i128;
 * M = (acc * inv_n) >> 20; q = smallest even shift with (M >> q) <= max_idx;
 * idx = min(rne(M, q), max_idx); norm_frac = lut_out + lut_in/2 + q/2;
 * per channel: shift = norm_frac + gamma_shift[i] + (x_shift[i] - ref) - out,
 * y = clamp_i16(clamp_i32(rne_i128(x*lut*gamma, shift) or << -shift)). */
int mylo_rmsnorm_i16(const int16_t* x, int64_t n, const uint8_t* x_shifts, const int8_t* gamma,
                     const uint8_t* gamma_shifts, const int16_t* rsqrt_lut, int64_t lut_len,
                     uint8_t lut_input_shift, uint8_t lut_output_frac, int64_t inv_n_q20,
                     uint8_t out_frac_bits, int16_t* out) {
  if (n <= 0 || lut_len <= 0 || (lut_input_shift & 1)) return MYLO_ERR_SHAPE;
  uint8_t ref = x_shifts[0];
  for (int64_t i = 1; i < n; ++i)
    if (x_shifts[i] > ref) ref = x_shifts[i];
  i128 acc = 0;
  for (int64_t i = 0; i < n; ++i) {
    unsigned align = 2u * (unsigned)(uint8_t)(ref - x_shifts[i]);
    i128 sq = (i128)x[i] * (i128)x[i];
    /* sq <= 2^30: the shifted square and the sum stay below 2^127 for the
     * alignments a realistic artifact has; beyond, the reference overflows. */
    if (align > 80) return MYLO_ERR_OVERFLOW;
    acc += sq << align;
  }
  if (acc == 0) {
    memset(out, 0, sizeof(int16_t) * (size_t)n);
    return MYLO_OK;
  }
  i128 prod_m;
  if (__builtin_mul_overflow(acc, (i128)inv_n_q20, &prod_m)) return MYLO_ERR_OVERFLOW;
  i128 m = prod_m >> 20;
  i128 max_idx = (i128)(lut_len - 1);
  unsigned q = 0;
  while ((m >> q) > max_idx) q += 2;
  i128 idx = rne_i128(m, q);
  if (idx > max_idx) idx = max_idx;
  if (idx < 0) idx = 0;
  i128 lut_val = (i128)rsqrt_lut[(int64_t)idx];
  unsigned norm_frac = (unsigned)lut_output_frac + (unsigned)lut_input_shift / 2u + q / 2u;
  for (int64_t i = 0; i < n; ++i) {
    int total = (int)norm_frac + (int)gamma_shifts[i] + ((int)x_shifts[i] - (int)ref);
    int shift = total - (int)out_frac_bits;
    i128 prod = (i128)x[i] * lut_val * (i128)gamma[i];
    i128 v;
    if (shift >= 0) {
      if (shift > 126) return MYLO_ERR_OVERFLOW;
      v = rne_i128(prod, (unsigned)shift);
    } else {
      if (-shift > 127) return MYLO_ERR_OVERFLOW;
      v = (i128)((u128)prod << (unsigned)(-shift)); /* i128 `<<`: wraps */
    }
    if (v < (i128)INT32_MIN) v = INT32_MIN;
    if (v > (i128)INT32_MAX) v = INT32_MAX;
    out[i] = mylo_clamp_i16((int32_t)v);
  }
  return MYLO_OK;
}

/* ---- rope.rs:17-32 ---------------------------------------------------------- */

int mylo_rotate_half_split_i16(const int16_t* vec, int64_t head_dim, const int16_t* cos_row,
                               const int16_t* sin_row, uint8_t frac_bits, int16_t* out) {
  if (head_dim <= 0 || (head_dim & 1) || frac_bits > 30) return MYLO_ERR_SHAPE;
  int64_t half = head_dim / 2;
  for (int64_t j = 0; j < half; ++j) {
    uint32_t c = (uint32_t)(int32_t)cos_row[j], s = (uint32_t)(int32_t)sin_row[j];
    uint32_t x0 = (uint32_t)(int32_t)vec[j], x1 = (uint32_t)(int32_t)vec[j + half];
    /* i32 products and sums (release build: wrapping) */
    int32_t a = (int32_t)(x0 * c - x1 * s);
    int32_t b = (int32_t)(x1 * c + x0 * s);
    out[j] = mylo_clamp_i16(mylo_rshift_round(a, frac_bits));
    out[j + half] = mylo_clamp_i16(mylo_rshift_round(b, frac_bits));
  }
  return MYLO_OK;
}

/* ---- attention.rs:20-27: i64 dot of two int16 vectors ------------------------ */

static int64_t dot_int(const int16_t* a, const int16_t* b, int64_t n) {
  int64_t acc = 0;
  for (int64_t i = 0; i < n; ++i) acc += (int64_t)a[i] * (int64_t)b[i];
  return acc;
}

/* ---- attention.rs:42-94 ------------------------------------------------------ */

static int attention_row(const int16_t* q, const int16_t* k, const int16_t* v, int64_t kv_len,
                         int64_t head_dim, const uint8_t* mask_row, int64_t score_mult,
                         uint8_t score_shift, const int16_t* exp_lut, int64_t exp_len,
                         uint8_t lut_shift, uint8_t prob_frac_bits, int32_t* scores, int64_t* row,
                         int16_t* out) {
  for (int64_t j = 0; j < kv_len; ++j) {
    if (!mask_row || mask_row[j]) {
      uint64_t s = (uint64_t)dot_int(q, k + j * head_dim, head_dim) * (uint64_t)score_mult;
      scores[j] = (int32_t)mylo_rshift_round_i64((int64_t)s, score_shift); /* `as i32` */
    } else {
      scores[j] = INT32_MIN;
    }
  }
  int rc = mylo_softmax_int(scores, kv_len, exp_lut, exp_len, lut_shift, prob_frac_bits, scores);
  if (rc) return rc;
  for (int64_t d = 0; d < head_dim; ++d) row[d] = 0;
  for (int64_t j = 0; j < kv_len; ++j) {
    if (scores[j] == 0) continue;
    const int16_t* vj = v + j * head_dim;
    for (int64_t d = 0; d < head_dim; ++d) row[d] += (int64_t)scores[j] * (int64_t)vj[d];
  }
  for (int64_t d = 0; d < head_dim; ++d)
    out[d] = mylo_clamp_i16_from_i64(mylo_rshift_round_i64(row[d], prob_frac_bits));
  return MYLO_OK;
}

int mylo_attention_int(const int16_t* q, int64_t q_len, const int16_t* k, const int16_t* v,
                       int64_t kv_len, int64_t head_dim, const uint8_t* mask, int64_t score_mult,
                       uint8_t score_shift, const int16_t* exp_lut, int64_t exp_len,
                       uint8_t lut_shift, uint8_t prob_frac_bits, int16_t* out) {
  if (q_len < 0 || kv_len <= 0 || head_dim <= 0 || score_shift > 62 || prob_frac_bits > 30)
    return MYLO_ERR_SHAPE;
  int32_t* scores = (int32_t*)malloc(sizeof(int32_t) * (size_t)kv_len);
  int64_t* row = (int64_t*)malloc(sizeof(int64_t) * (size_t)head_dim);
  int rc = MYLO_OK;
  for (int64_t i = 0; i < q_len && rc == MYLO_OK; ++i)
    rc = attention_row(q + i * head_dim, k, v, kv_len, head_dim, mask ? mask + i * kv_len : NULL,
                       score_mult, score_shift, exp_lut, exp_len, lut_shift, prob_frac_bits, scores,
                       row, out + i * head_dim);
  free(scores);
  free(row);
  return rc;
}

/* ---- exact dot in int32 blocks (equal to dot_scalar, see the header) -------- */

static int64_t dot_blocked(const int8_t* w, const int16_t* x, int64_t n) {
  int64_t acc = 0;
  int64_t i = 0;
  for (; i + 256 <= n; i += 256) {
    int32_t s = 0;
    for (int j = 0; j < 256; ++j) s += (int32_t)w[i + j] * (int32_t)x[i + j];
    acc += s;
  }
  for (; i < n; ++i) acc += (int64_t)w[i] * (int64_t)x[i];
  return acc;
}

/* linear.rs:43-70 / :87-119 on M rows (shifts validated by the caller through
 * check_shifts): y[m][r] = clamp_i16(rescale_i64(dot, w_shift[r] + act, out)). */
static void linear_fast(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                        const uint8_t* w_shifts, uint8_t act_frac, const uint8_t* out_pc,
                        uint8_t out_frac, int16_t* y) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < N; ++r) {
    const int8_t* wr = W + r * K;
    uint8_t in_frac = (uint8_t)(w_shifts[r] + act_frac);
    uint8_t of = out_pc ? out_pc[r] : out_frac;
    for (int64_t m = 0; m < M; ++m) {
      int64_t v = 0;
      mylo_rescale_i64(dot_blocked(wr, x + m * K, K), in_frac, of, &v);
      y[m * N + r] = mylo_clamp_i16_from_i64(v);
    }
  }
}

int mylo_linear_w8a16_pc_fast(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                              const uint8_t* w_shifts, uint8_t act_frac, const uint8_t* out_frac,
                              int16_t* y) {
  if (M < 0 || N < 0 || K <= 0) return MYLO_ERR_SHAPE;
  for (int64_t r = 0; r < N; ++r) {
    unsigned in_frac = (unsigned)w_shifts[r] + act_frac;
    if (in_frac > 255u) return MYLO_ERR_OVERFLOW;
    int d = (int)(int8_t)(uint8_t)in_frac - (int)(int8_t)out_frac[r];
    if (d < -128 || d > 127 || d > 62 || d < -63) return MYLO_ERR_OVERFLOW;
  }
  linear_fast(x, M, W, K, N, w_shifts, act_frac, out_frac, 0, y);
  return MYLO_OK;
}

int mylo_linear_acc_fast(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                         int64_t* acc) {
  if (M < 0 || N < 0 || K <= 0) return MYLO_ERR_SHAPE;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < N; ++r)
    for (int64_t m = 0; m < M; ++m) acc[m * N + r] = dot_blocked(W + r * K, x + m * K, K);
  return MYLO_OK;
}

int mylo_requant_acc(const int64_t* acc, int64_t M, int64_t N, const uint8_t* w_shifts,
                     uint8_t act_frac, const uint8_t* out_frac, int16_t* y) {
  if (M < 0 || N < 0) return MYLO_ERR_SHAPE;
  for (int64_t r = 0; r < N; ++r) {
    unsigned in_frac = (unsigned)w_shifts[r] + act_frac;
    if (in_frac > 255u) return MYLO_ERR_OVERFLOW;
    int d = (int)(int8_t)(uint8_t)in_frac - (int)(int8_t)out_frac[r];
    if (d < -128 || d > 127 || d > 62 || d < -63) return MYLO_ERR_OVERFLOW;
  }
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < M * N; ++e) {
    int64_t r = e % N, v = 0;
    mylo_rescale_i64(acc[e], (uint8_t)(w_shifts[r] + act_frac), out_frac[r], &v);
    y[e] = mylo_clamp_i16_from_i64(v);
  }
  return MYLO_OK;
}

/* The debug-build overflow checks of linear.rs:66 / :115 (u8 add) and of
 * rescale_i64 (i8 difference, shift width) for every row. */
static int check_shifts(int64_t N, const uint8_t* w_shifts, uint8_t act_frac, const uint8_t* out_pc,
                        uint8_t out_frac) {
  for (int64_t r = 0; r < N; ++r) {
    unsigned in_frac = (unsigned)w_shifts[r] + act_frac;
    if (in_frac > 255u) return MYLO_ERR_OVERFLOW;
    int d = (int)(int8_t)(uint8_t)in_frac - (int)(int8_t)(out_pc ? out_pc[r] : out_frac);
    if (d < -128 || d > 127 || d > 62 || d < -63) return MYLO_ERR_OVERFLOW;
  }
  return MYLO_OK;
}

/* i8 difference and width checks of rescale (32) / rescale_i64 (64). */
static int check_rescale(uint8_t in_frac, uint8_t out_frac, int width) {
  int d = (int)(int8_t)in_frac - (int)(int8_t)out_frac;
  if (d < -128 || d > 127) return MYLO_ERR_OVERFLOW;
  if (d >= 0 && d > width - 2) return MYLO_ERR_OVERFLOW;
  if (d < 0 && -d > width - 1) return MYLO_ERR_OVERFLOW;
  return MYLO_OK;
}

#define TRYO(e)                   \
  do {                            \
    int rc_ = (e);                \
    if (rc_ != MYLO_OK) return rc_; \
  } while (0)

static int check_layer(const mylo_model* m, const mylo_layer* L, const uint8_t* out_res) {
  const int64_t H = m->hidden, QD = m->num_heads * m->head_dim, KD = m->num_kv_heads * m->head_dim,
                I = m->intermediate;
  TRYO(check_shifts(QD, L->sq, L->norm_attn_frac, NULL, L->q_frac));
  TRYO(check_shifts(KD, L->sk, L->norm_attn_frac, NULL, L->k_frac));
  TRYO(check_shifts(KD, L->sv, L->norm_attn_frac, NULL, L->v_frac));
  TRYO(check_shifts(I, L->sg, L->norm_mlp_frac, NULL, L->gate_frac));
  TRYO(check_shifts(I, L->su, L->norm_mlp_frac, NULL, L->up_frac));
  TRYO(check_rescale(L->v_frac, L->attn_out_frac, 32));
  for (int64_t i = 0; i < H; ++i) {
    uint8_t acc_attn = L->residual_in_frac[i] < L->residual_mid_frac[i] ? L->residual_in_frac[i]
                                                                          : L->residual_mid_frac[i];
    uint8_t acc_mlp = L->residual_mid_frac[i] < out_res[i] ? L->residual_mid_frac[i] : out_res[i];
    TRYO(check_shifts(1, L->so + i, L->attn_out_frac, NULL, acc_attn));
    TRYO(check_shifts(1, L->sd + i, L->down_in_frac, NULL, acc_mlp));
    TRYO(check_rescale(L->residual_in_frac[i], acc_attn, 64));
    TRYO(check_rescale(acc_attn, L->residual_mid_frac[i], 64));
    TRYO(check_rescale(L->residual_mid_frac[i], acc_mlp, 64));
    TRYO(check_rescale(acc_mlp, out_res[i], 64));
  }
  return MYLO_OK;
}

/* ---- model.rs:401-674: one layer on T tokens (layer-major, see header) ------ */

static int forward_layer(const mylo_model* m, int64_t l, int16_t* k_cache, int16_t* v_cache,
                         int64_t max_pos, int16_t* hidden, int64_t T, int64_t pos0,
                         const uint8_t* out_res) {
  const mylo_layer* L = &m->layers[l];
  const int64_t H = m->hidden, hd = m->head_dim, nq = m->num_heads, nkv = m->num_kv_heads;
  const int64_t QD = nq * hd, KD = nkv * hd, I = m->intermediate, group = nq / nkv;
  const int64_t half = hd / 2, n_pos = m->rope_len / half;
  TRYO(check_layer(m, L, out_res));

  int16_t* xn = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * H));
  int16_t* q = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * QD));
  int16_t* k = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * KD));
  int16_t* v = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * KD));
  int16_t* attn = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * QD));
  int16_t* o = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * H));
  int16_t* resid = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * H));
  int16_t* gate = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * I));
  int16_t* up = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * I));
  uint8_t* acc_attn = (uint8_t*)malloc((size_t)H);
  uint8_t* acc_mlp = (uint8_t*)malloc((size_t)H);
  int rc = MYLO_OK;
  const int64_t inv_n = mylo_inv_n_q20(H);

  /* input_layernorm (model.rs:416-426) */
#pragma omp parallel for schedule(static) reduction(| : rc)
  for (int64_t t = 0; t < T; ++t)
    rc |= mylo_rmsnorm_i16(hidden + t * H, H, L->residual_in_frac, L->ln1_gamma, L->ln1_gamma_shifts,
                           m->rsqrt_lut, m->rsqrt_len, m->rsqrt_input_shift, m->rsqrt_output_frac,
                           inv_n, L->norm_attn_frac, xn + t * H);
  if (rc) goto done;

  /* q/k/v projections and biases (model.rs:438-453) */
  linear_fast(xn, T, L->wq, H, QD, L->sq, L->norm_attn_frac, NULL, L->q_frac, q);
  linear_fast(xn, T, L->wk, H, KD, L->sk, L->norm_attn_frac, NULL, L->k_frac, k);
  linear_fast(xn, T, L->wv, H, KD, L->sv, L->norm_attn_frac, NULL, L->v_frac, v);
  for (int64_t t = 0; t < T && rc == MYLO_OK; ++t) {
    if (L->bq) rc |= mylo_add_bias_i16(q + t * QD, L->bq, L->bq_shifts, QD, L->q_frac);
    if (L->bk) rc |= mylo_add_bias_i16(k + t * KD, L->bk, L->bk_shifts, KD, L->k_frac);
    if (L->bv) rc |= mylo_add_bias_i16(v + t * KD, L->bv, L->bv_shifts, KD, L->v_frac);
  }
  if (rc) goto done;

  /* RoPE at pos % n_pos (model.rs:469-479), KV cache write (model.rs:500-503) */
  for (int64_t t = 0; t < T; ++t) {
    const int64_t pos = pos0 + t, idx = pos % n_pos;
    const int16_t* c = m->cos_lut + idx * half;
    const int16_t* s = m->sin_lut + idx * half;
    int16_t tmp[1024];
    for (int64_t h = 0; h < nq; ++h) {
      mylo_rotate_half_split_i16(q + t * QD + h * hd, hd, c, s, m->rope_frac_bits, tmp);
      memcpy(q + t * QD + h * hd, tmp, sizeof(int16_t) * (size_t)hd);
    }
    for (int64_t h = 0; h < nkv; ++h) {
      mylo_rotate_half_split_i16(k + t * KD + h * hd, hd, c, s, m->rope_frac_bits, tmp);
      int16_t* kc = k_cache + ((l * nkv + h) * max_pos + pos) * hd;
      int16_t* vc = v_cache + ((l * nkv + h) * max_pos + pos) * hd;
      memcpy(kc, tmp, sizeof(int16_t) * (size_t)hd);
      memcpy(vc, v + t * KD + h * hd, sizeof(int16_t) * (size_t)hd);
    }
  }

  /* attention per query head over cache positions <= pos (model.rs:508-558) */
  {
    const int64_t score_mult = mylo_inv_sqrt_q15(hd);
    unsigned ss = (unsigned)L->q_frac + (unsigned)L->k_frac + 15u;
    ss = ss > m->score_frac_bits ? ss - m->score_frac_bits : 0u; /* u16 saturating_sub */
    const uint8_t score_shift = (uint8_t)ss;                   /* `as u8` */
    const uint8_t lut_shift =
        m->score_frac_bits > m->exp_input_frac ? (uint8_t)(m->score_frac_bits - m->exp_input_frac) : 0;
    if (score_shift > 62 || m->prob_frac_bits > 30) {
      rc = MYLO_ERR_OVERFLOW;
      goto done;
    }
#pragma omp parallel reduction(| : rc)
    {
      int32_t* scores = (int32_t*)malloc(sizeof(int32_t) * (size_t)(pos0 + T));
      int64_t* row = (int64_t*)malloc(sizeof(int64_t) * (size_t)hd);
#pragma omp for schedule(dynamic, 4)
      for (int64_t e = 0; e < T * nq; ++e) {
        const int64_t t = e / nq, h = e % nq, kvh = h / group, pos = pos0 + t;
        const int16_t* kc = k_cache + (l * nkv + kvh) * max_pos * hd;
        const int16_t* vc = v_cache + (l * nkv + kvh) * max_pos * hd;
        rc |= attention_row(q + t * QD + h * hd, kc, vc, pos + 1, hd, NULL, score_mult, score_shift,
                            m->exp_lut, m->exp_len, lut_shift, m->prob_frac_bits, scores, row,
                            attn + t * QD + h * hd);
      }
      free(scores);
      free(row);
    }
    if (rc) goto done;
  }

  /* attention output on the V scale -> o_proj input scale (model.rs:563-567) */
  if (L->attn_out_frac != L->v_frac)
    for (int64_t e = 0; e < T * QD; ++e) {
      int32_t r = 0;
      mylo_rescale((int32_t)attn[e], L->v_frac, L->attn_out_frac, &r);
      attn[e] = mylo_clamp_i16(r);
    }

  /* o_proj onto the coarser of the two segment scales, residual add 1
   * (model.rs:576-593) */
  for (int64_t i = 0; i < H; ++i)
    acc_attn[i] = L->residual_in_frac[i] < L->residual_mid_frac[i] ? L->residual_in_frac[i]
                                                                    : L->residual_mid_frac[i];
  linear_fast(attn, T, L->wo, QD, H, L->so, L->attn_out_frac, acc_attn, 0, o);
  for (int64_t t = 0; t < T; ++t)
    for (int64_t i = 0; i < H; ++i) {
      int64_t hres = 0, sum = 0;
      mylo_rescale_i64((int64_t)hidden[t * H + i], L->residual_in_frac[i], acc_attn[i], &hres);
      mylo_rescale_i64(hres + (int64_t)o[t * H + i], acc_attn[i], L->residual_mid_frac[i], &sum);
      resid[t * H + i] = mylo_clamp_i16_from_i64(sum);
    }

  /* post_attention_layernorm (model.rs:596-606) */
#pragma omp parallel for schedule(static) reduction(| : rc)
  for (int64_t t = 0; t < T; ++t)
    rc |= mylo_rmsnorm_i16(resid + t * H, H, L->residual_mid_frac, L->ln2_gamma, L->ln2_gamma_shifts,
                           m->rsqrt_lut, m->rsqrt_len, m->rsqrt_input_shift, m->rsqrt_output_frac,
                           inv_n, L->norm_mlp_frac, xn + t * H);
  if (rc) goto done;

  /* mlp_int onto min(mid, out) (model.rs:612-637, mlp.rs:28-74) */
  for (int64_t i = 0; i < H; ++i)
    acc_mlp[i] = L->residual_mid_frac[i] < out_res[i] ? L->residual_mid_frac[i] : out_res[i];
  linear_fast(xn, T, L->wg, H, I, L->sg, L->norm_mlp_frac, NULL, L->gate_frac, gate);
  linear_fast(xn, T, L->wu, H, I, L->su, L->norm_mlp_frac, NULL, L->up_frac, up);
  rc = mylo_silu_product(gate, up, T * I, m->silu_lut, m->silu_len, L->gate_frac, L->up_frac,
                         L->down_in_frac, m->silu_in_frac, m->silu_lut_offset, m->silu_out_frac, gate,
                         NULL);
  if (rc) goto done;
  linear_fast(gate, T, L->wd, I, H, L->sd, L->down_in_frac, acc_mlp, 0, o);

  /* residual add 2 (model.rs:666-671) */
  for (int64_t t = 0; t < T; ++t)
    for (int64_t i = 0; i < H; ++i) {
      int64_t r = 0, sum = 0;
      mylo_rescale_i64((int64_t)resid[t * H + i], L->residual_mid_frac[i], acc_mlp[i], &r);
      mylo_rescale_i64(r + (int64_t)o[t * H + i], acc_mlp[i], out_res[i], &sum);
      hidden[t * H + i] = mylo_clamp_i16_from_i64(sum);
    }

done:
  free(xn);
  free(q);
  free(k);
  free(v);
  free(attn);
  free(o);
  free(resid);
  free(gate);
  free(up);
  free(acc_attn);
  free(acc_mlp);
  return rc ? (rc & MYLO_ERR_OVERFLOW ? MYLO_ERR_OVERFLOW : MYLO_ERR_SHAPE) : MYLO_OK;
}

/* ---- model.rs:229-311 --------------------------------------------------------- */

int mylo_forward(const mylo_model* m, int16_t* k_cache, int16_t* v_cache, int64_t max_pos,
                 const int32_t* tokens, int64_t T, int64_t pos0, int32_t* logits) {
  const int64_t H = m->hidden, hd = m->head_dim;
  if (T <= 0 || pos0 < 0 || pos0 + T > max_pos || H <= 0 || hd <= 0 || (hd & 1) || hd > 1024 ||
      m->num_kv_heads <= 0 || m->num_heads % m->num_kv_heads || m->num_layers <= 0 ||
      m->rope_len < hd / 2 || m->vocab <= 0)
    return MYLO_ERR_SHAPE;
  for (int64_t t = 0; t < T; ++t)
    if (tokens[t] < 0 || tokens[t] >= m->vocab) return MYLO_ERR_SHAPE;

  int16_t* hidden = (int16_t*)malloc(sizeof(int16_t) * (size_t)(T * H));
  int rc = MYLO_OK;
  /* embedding row rescale onto the first residual segment (model.rs:241-248) */
  const uint8_t* rin0 = m->layers[0].residual_in_frac;
  for (int64_t t = 0; t < T && rc == MYLO_OK; ++t) {
    const int8_t* row = m->embed + (int64_t)tokens[t] * H;
    const uint8_t sh = m->embed_shifts[tokens[t]];
    for (int64_t i = 0; i < H; ++i) {
      int32_t r = 0;
      rc = mylo_rescale((int32_t)row[i], sh, rin0[i], &r);
      if (rc) break;
      hidden[t * H + i] = mylo_clamp_i16(r);
    }
  }
  for (int64_t l = 0; l < m->num_layers && rc == MYLO_OK; ++l) {
    const uint8_t* out_res =
        l + 1 < m->num_layers ? m->layers[l + 1].residual_in_frac : m->final_residual_frac;
    rc = forward_layer(m, l, k_cache, v_cache, max_pos, hidden, T, pos0, out_res);
  }
  if (rc == MYLO_OK && logits) {
    /* final norm (model.rs:264-274) and LM head (model.rs:284-308) */
    int16_t* normed = (int16_t*)malloc(sizeof(int16_t) * (size_t)H);
    rc = mylo_rmsnorm_i16(hidden + (T - 1) * H, H, m->final_residual_frac, m->final_gamma,
                          m->final_gamma_shifts, m->rsqrt_lut, m->rsqrt_len, m->rsqrt_input_shift,
                          m->rsqrt_output_frac, mylo_inv_n_q20(H), m->final_norm_frac, normed);
    if (rc == MYLO_OK) {
      if (m->lm_head16)
        rc = mylo_lm_head_w16a16_i32(normed, 1, m->lm_head16, H, m->vocab, m->lm_head16_shifts,
                                     m->final_norm_frac, m->logit_frac_bits, logits);
      else
        rc = mylo_lm_head_w8a16_i32(normed, 1, m->lm_head, H, m->vocab, m->lm_head_shifts,
                                    m->final_norm_frac, m->logit_frac_bits, logits);
    }
    free(normed);
  }
  free(hidden);
  return rc;
}

/* ---- generate.rs:161-200 (greedy) --------------------------------------------- */

int mylo_generate(const mylo_model* m, int16_t* k_cache, int16_t* v_cache, int64_t max_pos,
                  const int32_t* prompt, int64_t P, int64_t max_new, int32_t* out_tokens,
                  int32_t* step_logits) {
  if (P <= 0 || max_new < 0 || P + max_new > max_pos) return MYLO_ERR_SHAPE;
  int32_t* logits = (int32_t*)malloc(sizeof(int32_t) * (size_t)m->vocab);
  int rc = mylo_forward(m, k_cache, v_cache, max_pos, prompt, P, 0, logits);
  int64_t pos = P;
  for (int64_t s = 0; s < max_new && rc == MYLO_OK; ++s) {
    if (step_logits) memcpy(step_logits + s * m->vocab, logits, sizeof(int32_t) * (size_t)m->vocab);
    int32_t next = (int32_t)mylo_argmax_i32(logits, m->vocab);
    out_tokens[s] = next;
    rc = mylo_forward(m, k_cache, v_cache, max_pos, &next, 1, pos, logits);
    pos += 1;
  }
  free(logits);
  return rc;
}
