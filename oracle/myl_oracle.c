/*
 * myl_oracle.c — CPU restatement of Myelith's W8A16 integer linear path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product); see
 * myl_oracle.h for the list of reference functions restated here.
 *
 * Integer semantics follow the reference's Rust code. Signed right shifts
 * are arithmetic (GCC defines >> on negative values that way, as Rust does);
 * left shifts of signed values go through the unsigned type so that C's
 * undefined behaviour never enters.
 *
 * Loops over output elements are independent (each output element is one
 * dot product followed by its own requant), so they are spread over OpenMP
 * threads; every single element is still computed by one thread in the
 * reference's loop order (dot.rs:403-409), so the result does not depend on
 * the thread count.
 */
#include "myl_oracle.h"

#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- fixed_point.rs:7-35 ---------------------------------------------- */

int8_t mylo_clamp_i8(int32_t x) {
  if (x < -128) return -128;
  if (x > 127) return 127;
  return (int8_t)x;
}

int16_t mylo_clamp_i16(int32_t x) {
  if (x < -32768) return -32768;
  if (x > 32767) return 32767;
  return (int16_t)x;
}

int16_t mylo_clamp_i16_from_i64(int64_t x) {
  if (x < -32768) return -32768;
  if (x > 32767) return 32767;
  return (int16_t)x;
}

int32_t mylo_clamp_i32(int64_t x) {
  if (x < (int64_t)INT32_MIN) return INT32_MIN;
  if (x > (int64_t)INT32_MAX) return INT32_MAX;
  return (int32_t)x;
}

/* ---- fixed_point.rs:39-53: RNE right shift on two's complement --------- */

int32_t mylo_rshift_round(int32_t value, uint8_t shift) {
  if (shift == 0) return value;
  int32_t mask = (int32_t)((1u << shift) - 1u);
  int32_t half = (int32_t)(1u << (shift - 1));
  int32_t quotient = value >> shift;
  int32_t remainder = value & mask;
  if (remainder > half || (remainder == half && (quotient & 1) != 0)) return quotient + 1;
  return quotient;
}

/* ---- fixed_point.rs:57-71 ---------------------------------------------- */

int64_t mylo_rshift_round_i64(int64_t value, uint8_t shift) {
  if (shift == 0) return value;
  int64_t mask = (int64_t)((1ull << shift) - 1ull);
  int64_t half = (int64_t)(1ull << (shift - 1));
  int64_t quotient = value >> shift;
  int64_t remainder = value & mask;
  if (remainder > half || (remainder == half && (quotient & 1) != 0)) return quotient + 1;
  return quotient;
}

/* ---- fixed_point.rs:155-169 (i128 flavour, used by the multiplier mode) - */

static __int128 rshift_round_i128(__int128 value, unsigned shift) {
  if (shift == 0) return value;
  __int128 one = 1;
  __int128 mask = (one << shift) - 1;
  __int128 half = one << (shift - 1);
  __int128 quotient = value >> shift;
  __int128 remainder = value & mask;
  if (remainder > half || (remainder == half && (quotient & 1) != 0)) return quotient + 1;
  return quotient;
}

/* The signed shift `in_frac as i8 - out_frac as i8` (fixed_point.rs:174,
 * :185) with the debug-build panics turned into an error:
 *   - i8 subtraction overflow,
 *   - a right shift whose mask (1 << s) - 1 overflows (s > width - 2),
 *   - a left shift by >= width bits.
 * width is 32 for rescale and 64 for rescale_i64. */
static int signed_shift(uint8_t in_frac, uint8_t out_frac, int width, int* s) {
  int a = (int)(int8_t)in_frac, b = (int)(int8_t)out_frac;
  int d = a - b;
  if (d < -128 || d > 127) return MYLO_ERR_OVERFLOW;
  if (d >= 0 && d > width - 2) return MYLO_ERR_OVERFLOW;
  if (d < 0 && -d > width - 1) return MYLO_ERR_OVERFLOW;
  *s = d;
  return MYLO_OK;
}

/* ---- fixed_point.rs:173-180 -------------------------------------------- */

int mylo_rescale(int32_t acc, uint8_t in_frac, uint8_t out_frac, int32_t* out) {
  int s;
  int rc = signed_shift(in_frac, out_frac, 32, &s);
  if (rc) return rc;
  if (s >= 0) *out = mylo_rshift_round(acc, (uint8_t)s);
  else *out = (int32_t)((uint32_t)acc << (-s));
  return MYLO_OK;
}

/* ---- fixed_point.rs:184-191 -------------------------------------------- */

int mylo_rescale_i64(int64_t acc, uint8_t in_frac, uint8_t out_frac, int64_t* out) {
  int s;
  int rc = signed_shift(in_frac, out_frac, 64, &s);
  if (rc) return rc;
  if (s >= 0) *out = mylo_rshift_round_i64(acc, (uint8_t)s);
  else *out = (int64_t)((uint64_t)acc << (-s));
  return MYLO_OK;
}

/* ---- dot.rs:403-409 ----------------------------------------------------- */

int64_t mylo_dot_scalar(const int8_t* w, const int16_t* x, int64_t n) {
  int64_t acc = 0;
  for (int64_t i = 0; i < n; ++i) acc += (int64_t)w[i] * (int64_t)x[i];
  return acc;
}

/* in_frac = w_shift + act_frac is a u8 addition in linear.rs:66 / :115. */
static int in_frac_of(uint8_t w_shift, uint8_t act_frac, uint8_t* in_frac) {
  unsigned v = (unsigned)w_shift + (unsigned)act_frac;
  if (v > 255u) return MYLO_ERR_OVERFLOW;
  *in_frac = (uint8_t)v;
  return MYLO_OK;
}

/* Validates every (row, out_frac) pair up front so that an error leaves the
 * output untouched; the reference would panic on the first bad row. */
static int check_linear(int64_t M, int64_t K, int64_t N, const uint8_t* w_shifts,
                        uint8_t act_frac, const uint8_t* out_frac_pc, uint8_t out_frac) {
  if (M < 0 || N < 0 || K <= 0) return MYLO_ERR_SHAPE; /* chunks_exact(0) panics */
  for (int64_t r = 0; r < N; ++r) {
    uint8_t in_frac;
    int s;
    if (in_frac_of(w_shifts[r], act_frac, &in_frac)) return MYLO_ERR_OVERFLOW;
    if (signed_shift(in_frac, out_frac_pc ? out_frac_pc[r] : out_frac, 64, &s))
      return MYLO_ERR_OVERFLOW;
  }
  return MYLO_OK;
}

/* ---- linear.rs:43-70 / :87-119 on M rows -------------------------------- */

static void linear_rows(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                        const uint8_t* w_shifts, uint8_t act_frac, const uint8_t* out_frac_pc,
                        uint8_t out_frac, int16_t* y) {
  int64_t total = M * N;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < total; ++e) {
    int64_t m = e / N, r = e % N;
    int64_t acc = mylo_dot_scalar(W + r * K, x + m * K, K);
    uint8_t in_frac = (uint8_t)(w_shifts[r] + act_frac);
    int64_t v = 0;
    mylo_rescale_i64(acc, in_frac, out_frac_pc ? out_frac_pc[r] : out_frac, &v);
    y[e] = mylo_clamp_i16_from_i64(v);
  }
}

int mylo_linear_w8a16(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                      const uint8_t* w_shifts, uint8_t act_frac, uint8_t out_frac, int16_t* y) {
  int rc = check_linear(M, K, N, w_shifts, act_frac, NULL, out_frac);
  if (rc) return rc;
  linear_rows(x, M, W, K, N, w_shifts, act_frac, NULL, out_frac, y);
  return MYLO_OK;
}

int mylo_linear_w8a16_pc(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                         const uint8_t* w_shifts, uint8_t act_frac, const uint8_t* out_frac,
                         int16_t* y) {
  int rc = check_linear(M, K, N, w_shifts, act_frac, out_frac, 0);
  if (rc) return rc;
  linear_rows(x, M, W, K, N, w_shifts, act_frac, out_frac, 0, y);
  return MYLO_OK;
}

/* ---- runtime/src/model.rs:297-307: LM head, i32 clamp ------------------- */

int mylo_lm_head_w8a16_i32(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                           const uint8_t* w_shifts, uint8_t final_norm_frac, uint8_t logit_frac,
                           int32_t* logits) {
  int rc = check_linear(M, K, N, w_shifts, final_norm_frac, NULL, logit_frac);
  if (rc) return rc;
  int64_t total = M * N;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < total; ++e) {
    int64_t m = e / N, r = e % N;
    int64_t acc = mylo_dot_scalar(W + r * K, x + m * K, K);
    int64_t v = 0;
    mylo_rescale_i64(acc, (uint8_t)(w_shifts[r] + final_norm_frac), logit_frac, &v);
    logits[e] = mylo_clamp_i32(v);
  }
  return MYLO_OK;
}

/* ---- LM head path A, runtime/src/model.rs:285-296 ---------------------------
 * int16 weights, i64 products and accumulator, row_frac = shifts[row] +
 * final_norm_frac (u8), rescale_i64 to logit_frac, clamp to i32. */
int mylo_lm_head_w16a16_i32(const int16_t* x, int64_t M, const int16_t* W, int64_t K, int64_t N,
                            const uint8_t* w_shifts, uint8_t final_norm_frac, uint8_t logit_frac,
                            int32_t* logits) {
  int rc = check_linear(M, K, N, w_shifts, final_norm_frac, NULL, logit_frac);
  if (rc) return rc;
  int64_t total = M * N;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < total; ++e) {
    int64_t m = e / N, r = e % N;
    const int16_t* wr = W + r * K;
    const int16_t* xr = x + m * K;
    int64_t acc = 0;
    for (int64_t d = 0; d < K; ++d) acc += (int64_t)wr[d] * (int64_t)xr[d];
    int64_t v = 0;
    mylo_rescale_i64(acc, (uint8_t)(w_shifts[r] + final_norm_frac), logit_frac, &v);
    logits[e] = mylo_clamp_i32(v);
  }
  return MYLO_OK;
}

/* ---- linear_backward, kernels/src/backward.rs:147-211 ------------------------
 * Per token m (the reference takes one token):
 *   ref = max_i w_shifts[i]                      (panics for an empty w_shifts)
 *   acc[j] = sum_i (g[i] * W[i][j]) << (ref - w_shifts[i])     in i128
 *   gx[j]  = clamp_i32(rescale_i64(clamp_i64(rshift_round_i128(acc[j], ref)),
 *                                  g_frac, gx_frac))
 *   gw[i][j] = g[i] * x[j]                       (i64, no scaling)
 * Rust panics in a debug build when a shift reaches the i128 width; this
 * restatement reports that as an overflow (ref >= 128). gw may be NULL. */
int mylo_linear_backward(const int32_t* g, const int16_t* x, int64_t M, const int8_t* W, int64_t K,
                         int64_t N, const uint8_t* w_shifts, uint8_t g_frac, uint8_t gx_frac,
                         int32_t* gx, int64_t* gw) {
  if (M < 0 || K <= 0 || N <= 0) return MYLO_ERR_SHAPE;
  unsigned ref = 0;
  for (int64_t i = 0; i < N; ++i)
    if (w_shifts[i] > ref) ref = w_shifts[i];
  if (ref >= 128) return MYLO_ERR_OVERFLOW;
  int s;
  if (signed_shift(g_frac, gx_frac, 64, &s)) return MYLO_ERR_OVERFLOW;
  int64_t total = M * K;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < total; ++e) {
    int64_t m = e / K, j = e % K;
    __int128 acc = 0;
    for (int64_t i = 0; i < N; ++i) {
      __int128 gi = g[m * N + i];
      if (gi == 0) continue;
      acc += (gi * (__int128)W[i * K + j]) << (ref - w_shifts[i]);
    }
    __int128 q = rshift_round_i128(acc, ref);
    int64_t lim = q > (__int128)INT64_MAX ? INT64_MAX : (q < (__int128)INT64_MIN ? INT64_MIN : (int64_t)q);
    int64_t v = 0;
    mylo_rescale_i64(lim, g_frac, gx_frac, &v);
    gx[e] = mylo_clamp_i32(v);
  }
  if (gw) {
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < M * N; ++e) {
      int64_t m = e / N;
      for (int64_t j = 0; j < K; ++j) gw[e * K + j] = (int64_t)g[e] * (int64_t)x[m * K + j];
    }
  }
  return MYLO_OK;
}

/* ---- multiplier requant (generalisation; pow2 identity fixed_point.rs:365) */

int mylo_linear_w8a16_mult(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                           const int32_t* mult, const uint8_t* shift, int16_t* y) {
  if (M < 0 || N < 0 || K <= 0) return MYLO_ERR_SHAPE;
  for (int64_t r = 0; r < N; ++r)
    if (shift[r] > 126) return MYLO_ERR_OVERFLOW;
  int64_t total = M * N;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < total; ++e) {
    int64_t m = e / N, r = e % N;
    int64_t acc = mylo_dot_scalar(W + r * K, x + m * K, K);
    __int128 p = (__int128)acc * (__int128)mult[r];
    __int128 q = rshift_round_i128(p, shift[r]);
    int16_t out;
    if (q < -32768) out = -32768;
    else if (q > 32767) out = 32767;
    else out = (int16_t)q;
    y[e] = out;
  }
  return MYLO_OK;
}

int mylo_linear_acc_i64(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                        int64_t* acc) {
  if (M < 0 || N < 0 || K <= 0) return MYLO_ERR_SHAPE;
  int64_t total = M * N;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < total; ++e) {
    int64_t m = e / N, r = e % N;
    acc[e] = mylo_dot_scalar(W + r * K, x + m * K, K);
  }
  return MYLO_OK;
}

/* ---- linear.rs:132-145 -------------------------------------------------- */

int mylo_add_bias_i16(int16_t* out, const int16_t* bias, const uint8_t* bias_shifts, int64_t n,
                      uint8_t out_frac) {
  if (n < 0) return MYLO_ERR_SHAPE;
  for (int64_t i = 0; i < n; ++i) {
    int s;
    if (signed_shift(bias_shifts[i], out_frac, 32, &s)) return MYLO_ERR_OVERFLOW;
  }
  for (int64_t i = 0; i < n; ++i) {
    int32_t b = 0;
    mylo_rescale((int32_t)bias[i], bias_shifts[i], out_frac, &b);
    out[i] = mylo_clamp_i16_from_i64((int64_t)out[i] + (int64_t)b);
  }
  return MYLO_OK;
}

/* ---- integer_math.rs:166-170, release (wrapping) i16 arithmetic ---------- */

int16_t mylo_lut_lookup(int16_t x, const int16_t* lut, int64_t lut_len, uint8_t shift,
                        int16_t offset) {
  int16_t idx = (int16_t)(uint16_t)((uint16_t)(int16_t)(x >> shift) + (uint16_t)offset);
  int16_t hi = (int16_t)(uint16_t)((uint16_t)lut_len - 1u);
  if (idx < 0) idx = 0;
  if (idx > hi) idx = hi;
  return lut[idx];
}

/* ---- mlp.rs:49-64 on M rows: the hidden activation h ---------------------- */

int mylo_mlp_hidden(const int16_t* x, int64_t M, const int8_t* W_gate, const int8_t* W_up,
                    int64_t H, int64_t I, const uint8_t* gate_w_shifts, const uint8_t* up_w_shifts,
                    const int16_t* silu_lut, int64_t silu_lut_len, uint8_t in_frac,
                    uint8_t gate_out_frac, uint8_t up_out_frac, uint8_t down_in_frac,
                    uint8_t silu_in_frac, int16_t silu_lut_offset, uint8_t silu_out_frac,
                    int16_t* h, int64_t* silu_wraps) {
  int rc;
  if (M < 0 || H <= 0 || I <= 0 || silu_lut_len <= 0) return MYLO_ERR_SHAPE;
  if ((rc = check_linear(M, H, I, gate_w_shifts, in_frac, NULL, gate_out_frac))) return rc;
  if ((rc = check_linear(M, H, I, up_w_shifts, in_frac, NULL, up_out_frac))) return rc;
  int s;
  if (signed_shift(gate_out_frac, silu_in_frac, 32, &s)) return MYLO_ERR_OVERFLOW;
  uint8_t prod_frac;
  if (in_frac_of(silu_out_frac, up_out_frac, &prod_frac)) return MYLO_ERR_OVERFLOW;
  if (signed_shift(prod_frac, down_in_frac, 64, &s)) return MYLO_ERR_OVERFLOW;

  int16_t* gate = (int16_t*)malloc(sizeof(int16_t) * (size_t)(M * I));
  int16_t* up = (int16_t*)malloc(sizeof(int16_t) * (size_t)(M * I));
  linear_rows(x, M, W_gate, H, I, gate_w_shifts, in_frac, NULL, gate_out_frac, gate);
  linear_rows(x, M, W_up, H, I, up_w_shifts, in_frac, NULL, up_out_frac, up);
  rc = mylo_silu_product(gate, up, M * I, silu_lut, silu_lut_len, gate_out_frac, up_out_frac,
                         down_in_frac, silu_in_frac, silu_lut_offset, silu_out_frac, h, silu_wraps);
  free(gate);
  free(up);
  return rc;
}

/* ---- mlp.rs:52-64: h from the gate and up projections ---------------------- */

int mylo_silu_product(const int16_t* gate, const int16_t* up, int64_t n, const int16_t* silu_lut,
                      int64_t silu_lut_len, uint8_t gate_out_frac, uint8_t up_out_frac,
                      uint8_t down_in_frac, uint8_t silu_in_frac, int16_t silu_lut_offset,
                      uint8_t silu_out_frac, int16_t* h, int64_t* silu_wraps) {
  int s;
  if (n < 0 || silu_lut_len <= 0) return MYLO_ERR_SHAPE;
  if (signed_shift(gate_out_frac, silu_in_frac, 32, &s)) return MYLO_ERR_OVERFLOW;
  uint8_t prod_frac;
  if (in_frac_of(silu_out_frac, up_out_frac, &prod_frac)) return MYLO_ERR_OVERFLOW;
  if (signed_shift(prod_frac, down_in_frac, 64, &s)) return MYLO_ERR_OVERFLOW;
  int64_t wraps = 0;
#pragma omp parallel for schedule(static) reduction(+ : wraps)
  for (int64_t e = 0; e < n; ++e) {
    int32_t g_dom = 0;
    mylo_rescale((int32_t)gate[e], gate_out_frac, silu_in_frac, &g_dom);
    int16_t g16 = (int16_t)(uint16_t)(uint32_t)g_dom; /* `g_dom as i16` */
    int32_t wide_idx = (int32_t)g16 + (int32_t)silu_lut_offset;
    if ((int32_t)g16 != g_dom || wide_idx < -32768 || wide_idx > 32767) ++wraps;
    int16_t activated = mylo_lut_lookup(g16, silu_lut, silu_lut_len, 0, silu_lut_offset);
    int64_t prod = (int64_t)activated * (int64_t)up[e];
    int64_t v = 0;
    mylo_rescale_i64(prod, prod_frac, down_in_frac, &v);
    h[e] = mylo_clamp_i16_from_i64(v);
  }
  if (silu_wraps) *silu_wraps = wraps;
  return MYLO_OK;
}

/* ---- mlp.rs:28-74 on M rows --------------------------------------------- */

int mylo_mlp_int(const int16_t* x, int64_t M, const int8_t* W_gate, const int8_t* W_up,
                 const int8_t* W_down, int64_t H, int64_t I, const uint8_t* gate_w_shifts,
                 const uint8_t* up_w_shifts, const uint8_t* down_w_shifts,
                 const int16_t* silu_lut, int64_t silu_lut_len, uint8_t in_frac,
                 uint8_t gate_out_frac, uint8_t up_out_frac, uint8_t down_in_frac,
                 uint8_t silu_in_frac, int16_t silu_lut_offset, uint8_t silu_out_frac,
                 const uint8_t* out_frac, int16_t* y, int64_t* silu_wraps) {
  int rc;
  if (M < 0 || H <= 0 || I <= 0 || silu_lut_len <= 0) return MYLO_ERR_SHAPE;
  if ((rc = check_linear(M, I, H, down_w_shifts, down_in_frac, out_frac, 0))) return rc;
  int16_t* h = (int16_t*)malloc(sizeof(int16_t) * (size_t)(M * I) + 1);
  rc = mylo_mlp_hidden(x, M, W_gate, W_up, H, I, gate_w_shifts, up_w_shifts, silu_lut, silu_lut_len,
                       in_frac, gate_out_frac, up_out_frac, down_in_frac, silu_in_frac,
                       silu_lut_offset, silu_out_frac, h, silu_wraps);
  if (rc == MYLO_OK) linear_rows(h, M, W_down, I, H, down_w_shifts, down_in_frac, out_frac, 0, y);
  free(h);
  return rc;
}

/* ---- softmax.rs:12-64 ----------------------------------------------------- */

static int32_t exp_lut_lookup(int32_t x, const int16_t* exp_lut, int64_t lut_len, uint8_t lut_shift,
                              int32_t one) {
  if (x <= 0) return one;
  uint32_t idx = (uint32_t)x >> lut_shift;
  if ((int64_t)idx >= lut_len) return 0;
  return (int32_t)exp_lut[idx];
}

int mylo_softmax_int(const int32_t* logits, int64_t n, const int16_t* exp_lut, int64_t lut_len,
                     uint8_t lut_shift, uint8_t frac_bits, int32_t* out) {
  if (n <= 0 || frac_bits > 30) return MYLO_ERR_SHAPE;
  int32_t one = (int32_t)1 << frac_bits;
  int32_t lut_one = lut_len > 0 ? (int32_t)exp_lut[0] : 1;
  int32_t m = logits[0];
  for (int64_t i = 1; i < n; ++i)
    if (logits[i] > m) m = logits[i];
  int64_t s64 = 0;
  for (int64_t i = 0; i < n; ++i) {
    int64_t d = (int64_t)m - (int64_t)logits[i];          /* saturating_sub */
    int32_t diff = d > INT32_MAX ? INT32_MAX : (int32_t)d;
    out[i] = exp_lut_lookup(diff, exp_lut, lut_len, lut_shift, lut_one);
    s64 += out[i];
  }
  if (s64 > INT32_MAX || s64 < INT32_MIN) return MYLO_ERR_OVERFLOW; /* i32 sum */
  int32_t s = (int32_t)s64;
  if (s == 0) {
    int32_t base = one / (int32_t)n;
    int32_t rem = one - base * (int32_t)n;
    for (int64_t i = 0; i < n; ++i) out[i] = base + (i < rem ? 1 : 0);
    return MYLO_OK;
  }
  for (int64_t i = 0; i < n; ++i) {
    int64_t num64 = (int64_t)out[i] * one;
    if (num64 > INT32_MAX || num64 < INT32_MIN) return MYLO_ERR_OVERFLOW; /* e * one in i32 */
    int32_t num = (int32_t)num64;
    int32_t q = num / s, r = num % s;                      /* truncating, as Rust */
    int32_t twice = (r < 0 ? -r : r) * 2, den_abs = s < 0 ? -s : s;
    if (twice > den_abs || (twice == den_abs && (q & 1) != 0)) q = ((num > 0) == (s > 0)) ? q + 1 : q - 1;
    out[i] = q;
  }
  return MYLO_OK;
}

/* ---- MoE layer composed from the reference primitives --------------------
 * (the reference has no MoE; every step below is one of its functions)
 *   logits[e] = clamp_i32(rescale_i64(dot(W_r[e], x), r_shift[e] + act_frac, router_frac))
 *               (runtime/src/model.rs:297-307 semantics)
 *   top-k     = k times argmax_int over the not yet chosen experts (sampling.rs:8-18:
 *               ties go to the lowest index)
 *   p         = softmax_int(logits[top-k], exp_lut, lut_shift, prob_frac) (softmax.rs:24-64)
 *   y_j       = mlp_int(x, expert top-k[j])                          (mlp.rs:28-74)
 *   out[h]    = clamp_i16(rescale_i64(sum_j p_j * y_j[h], prob_frac, 0) + shared[h])
 *               with shared = mlp_int(x, shared expert). */
int mylo_moe_route(const int32_t* logits, int64_t T, int64_t E, int64_t k, const int16_t* exp_lut,
                   int64_t lut_len, uint8_t lut_shift, uint8_t prob_frac, int32_t* topk_idx,
                   int32_t* topk_prob) {
  if (T < 0 || E <= 0 || k <= 0 || k > E || k > 64) return MYLO_ERR_SHAPE;
  for (int64_t t = 0; t < T; ++t) {
    const int32_t* lg = logits + t * E;
    unsigned char chosen[4096];
    if (E > 4096) return MYLO_ERR_SHAPE;
    memset(chosen, 0, (size_t)E);
    int32_t sel[64];
    for (int64_t j = 0; j < k; ++j) {
      int64_t best = -1;
      for (int64_t e = 0; e < E; ++e)
        if (!chosen[e] && (best < 0 || lg[e] > lg[best])) best = e;
      chosen[best] = 1;
      topk_idx[t * k + j] = (int32_t)best;
      sel[j] = lg[best];
    }
    int rc = mylo_softmax_int(sel, k, exp_lut, lut_len, lut_shift, prob_frac, topk_prob + t * k);
    if (rc) return rc;
  }
  return MYLO_OK;
}

int mylo_moe_combine(const int16_t* y_experts, const int32_t* topk_prob, const int16_t* shared,
                     int64_t T, int64_t k, int64_t H, uint8_t prob_frac, int16_t* out) {
  if (T < 0 || k <= 0 || H <= 0 || prob_frac > 62) return MYLO_ERR_SHAPE;
  for (int64_t t = 0; t < T; ++t)
    for (int64_t h = 0; h < H; ++h) {
      int64_t acc = 0;
      for (int64_t j = 0; j < k; ++j)
        acc += (int64_t)topk_prob[t * k + j] * (int64_t)y_experts[(t * k + j) * H + h];
      int64_t v = 0;
      mylo_rescale_i64(acc, prob_frac, 0, &v);
      out[t * H + h] = mylo_clamp_i16_from_i64(v + (int64_t)shared[t * H + h]);
    }
  return MYLO_OK;
}

/* ---- sampling.rs:8-18 ---------------------------------------------------- */

int64_t mylo_argmax_i32(const int32_t* v, int64_t n) {
  int64_t best_i = 0;
  int32_t best_v = v[0];
  for (int64_t i = 1; i < n; ++i)
    if (v[i] > best_v) {
      best_v = v[i];
      best_i = i;
    }
  return best_i;
}

/* ---- prng.rs:7-15 -------------------------------------------------------- */

uint64_t mylo_splitmix64(uint64_t state, uint64_t* out) {
  state += 0x9E3779B97F4A7C15ull;
  uint64_t z = state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  *out = z;
  return state;
}

int mylo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void mylo_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
