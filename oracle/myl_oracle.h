/*
 * myl_oracle.h — CPU restatement of Myelith's W8A16 integer linear path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the CUDA path is
 * compared against (tests, the smoke check and the bench's CPU baseline leg).
 * It is never linked into, loaded by, or called from the product library
 * libmyl_w8a16.so, and the product has no CPU fallback that could route here.
 *
 * Every function restates one function of the reference Rust crate
 * INTEGER_LLM/kernels (paths below are relative to the Myelith project root)
 * with the same integer widths and the same order of operations:
 *
 *   fixed_point.rs:15-35   clamps          fixed_point.rs:39-71  rshift_round{,_i64}
 *   fixed_point.rs:155-169 rshift_round_i128
 *   fixed_point.rs:173-191 rescale{,_i64}  dot.rs:403-409        dot_scalar
 *   linear.rs:43-70        linear_w8a16    linear.rs:87-119      linear_w8a16_pc
 *   linear.rs:132-145      add_bias_i16    integer_math.rs:166   lut_lookup
 *   mlp.rs:28-74           mlp_int (mlp.rs:49-64 mlp_hidden)
 *   runtime/src/model.rs:297-307 LM head (i32 clamp)
 *   sampling.rs:8-18       argmax_int      prng.rs:7-15          splitmix64
 *
 * Where the reference panics (Rust debug build: shape assert, integer
 * overflow in a shift or u8/i8 addition), the oracle returns MYLO_ERR_* and
 * leaves the output untouched. The product library reports the same cases
 * as errors.
 *
 * Parity pin: the self-checks in tests/test_oracle_kat.py replay every
 * known-answer vector of fixed_point.rs, linear.rs and dot.rs, the op golden
 * vector linear_w8a16_identity, and fixtures produced by the reference's own
 * Python restatement (tests/golden/generate.py:37-106), see
 * tests/golden/make_golden.py.
 */
#ifndef MYL_ORACLE_H
#define MYL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MYLO_OK = 0,
  MYLO_ERR_SHAPE = 1,     /* assert_eq! on lengths in linear.rs:51-58, :95-107 */
  MYLO_ERR_OVERFLOW = 2,  /* u8 add / i8 sub / shift-width overflow (debug panic) */
};

/* fixed_point.rs:7-35 */
int8_t  mylo_clamp_i8(int32_t x);
int16_t mylo_clamp_i16(int32_t x);
int16_t mylo_clamp_i16_from_i64(int64_t x);
int32_t mylo_clamp_i32(int64_t x);

/* fixed_point.rs:39-71, :155-169. shift must be < bit width - 1 (see header). */
int32_t mylo_rshift_round(int32_t value, uint8_t shift);
int64_t mylo_rshift_round_i64(int64_t value, uint8_t shift);

/* fixed_point.rs:173-191. Returns MYLO_ERR_OVERFLOW where Rust debug panics. */
int mylo_rescale(int32_t acc, uint8_t in_frac, uint8_t out_frac, int32_t* out);
int mylo_rescale_i64(int64_t acc, uint8_t in_frac, uint8_t out_frac, int64_t* out);

/* dot.rs:403-409: sum_k (i64)w[k] * (i64)x[k] in loop order. */
int64_t mylo_dot_scalar(const int8_t* w, const int16_t* x, int64_t n);

/* linear.rs:43-70 on M independent activation rows (row-major [M][K]).
 * W is flat row-major [N][K]; w_shifts[N]; y is [M][N]. */
int mylo_linear_w8a16(const int16_t* x, int64_t M, const int8_t* W, int64_t K,
                      int64_t N, const uint8_t* w_shifts, uint8_t act_frac,
                      uint8_t out_frac, int16_t* y);

/* linear.rs:87-119: as above with out_frac per output channel. */
int mylo_linear_w8a16_pc(const int16_t* x, int64_t M, const int8_t* W, int64_t K,
                         int64_t N, const uint8_t* w_shifts, uint8_t act_frac,
                         const uint8_t* out_frac, int16_t* y);

/* runtime/src/model.rs:297-307 (LM head, path B): i64 dot, rescale_i64,
 * clamp to i32 instead of i16. */
int mylo_linear_backward(const int32_t* g, const int16_t* x, int64_t M, const int8_t* W, int64_t K,
                         int64_t N, const uint8_t* w_shifts, uint8_t g_frac, uint8_t gx_frac,
                         int32_t* gx, int64_t* gw);
int mylo_lm_head_w16a16_i32(const int16_t* x, int64_t M, const int16_t* W, int64_t K, int64_t N,
                            const uint8_t* w_shifts, uint8_t final_norm_frac, uint8_t logit_frac,
                            int32_t* logits);
int mylo_lm_head_w8a16_i32(const int16_t* x, int64_t M, const int8_t* W, int64_t K,
                           int64_t N, const uint8_t* w_shifts, uint8_t final_norm_frac,
                           uint8_t logit_frac, int32_t* logits);

/* Generalised multiplier requant (no counterpart in the reference linear
 * layer; anchored by the pow2 identity of fixed_point.rs:365-379):
 *   y = clamp_i16( rne_shift_i128( dot * mult[r], shift[r] ) ),
 * shift[r] in [0, 126]. */
int mylo_linear_w8a16_mult(const int16_t* x, int64_t M, const int8_t* W, int64_t K,
                           int64_t N, const int32_t* mult, const uint8_t* shift,
                           int16_t* y);

/* Raw accumulators: acc[M][N] = dot(W[n], x[m]) in i64 (used by the
 * tensor-parallel and split-K parity checks). */
int mylo_linear_acc_i64(const int16_t* x, int64_t M, const int8_t* W, int64_t K,
                        int64_t N, int64_t* acc);

/* linear.rs:132-145. */
int mylo_add_bias_i16(int16_t* out, const int16_t* bias, const uint8_t* bias_shifts,
                      int64_t n, uint8_t out_frac);

/* integer_math.rs:166-170 with Rust release (wrapping) i16 arithmetic. */
int16_t mylo_lut_lookup(int16_t x, const int16_t* lut, int64_t lut_len, uint8_t shift,
                        int16_t offset);

/* mlp.rs:28-74 on M independent rows. W_gate/W_up are [I][H], W_down [H][I].
 * silu_wraps (nullable) receives the number of i16 index wraps
 * ((g_dom as i16) truncation), counted over all rows. */
int mylo_mlp_int(const int16_t* x, int64_t M, const int8_t* W_gate, const int8_t* W_up,
                 const int8_t* W_down, int64_t H, int64_t I, const uint8_t* gate_w_shifts,
                 const uint8_t* up_w_shifts, const uint8_t* down_w_shifts,
                 const int16_t* silu_lut, int64_t silu_lut_len, uint8_t in_frac,
                 uint8_t gate_out_frac, uint8_t up_out_frac, uint8_t down_in_frac,
                 uint8_t silu_in_frac, int16_t silu_lut_offset, uint8_t silu_out_frac,
                 const uint8_t* out_frac, int16_t* y, int64_t* silu_wraps);

/* mlp.rs:49-64: the hidden activation h [M][I] (input of the down projection). */
int mylo_mlp_hidden(const int16_t* x, int64_t M, const int8_t* W_gate, const int8_t* W_up,
                    int64_t H, int64_t I, const uint8_t* gate_w_shifts, const uint8_t* up_w_shifts,
                    const int16_t* silu_lut, int64_t silu_lut_len, uint8_t in_frac,
                    uint8_t gate_out_frac, uint8_t up_out_frac, uint8_t down_in_frac,
                    uint8_t silu_in_frac, int16_t silu_lut_offset, uint8_t silu_out_frac,
                    int16_t* h, int64_t* silu_wraps);

/* mlp.rs:52-64 on n elements: h = clamp_i16(rescale_i64(silu_lut[idx(gate)] * up,
 * silu_out + up_out, down_in)), the SiLU index in wrapping i16 arithmetic. */
int mylo_silu_product(const int16_t* gate, const int16_t* up, int64_t n, const int16_t* silu_lut,
                      int64_t silu_lut_len, uint8_t gate_out_frac, uint8_t up_out_frac,
                      uint8_t down_in_frac, uint8_t silu_in_frac, int16_t silu_lut_offset,
                      uint8_t silu_out_frac, int16_t* h, int64_t* silu_wraps);

/* softmax.rs:24-64 (exp LUT lookup softmax.rs:12-21, RNE division). */
int mylo_softmax_int(const int32_t* logits, int64_t n, const int16_t* exp_lut, int64_t lut_len,
                     uint8_t lut_shift, uint8_t frac_bits, int32_t* out);

/* MoE routing (no counterpart in the reference; composed from its primitives):
 * per token, k times argmax_int over the not yet chosen experts (lowest index
 * wins ties, sampling.rs:8-18), then softmax_int over the k chosen logits. */
int mylo_moe_route(const int32_t* logits, int64_t T, int64_t E, int64_t k, const int16_t* exp_lut,
                   int64_t lut_len, uint8_t lut_shift, uint8_t prob_frac, int32_t* topk_idx,
                   int32_t* topk_prob);

/* MoE combine: out[t][h] = clamp_i16(rescale_i64(sum_j p[t][j] * y[t][j][h], prob_frac, 0)
 *                                    + shared[t][h]); y is [T][k][H]. */
int mylo_moe_combine(const int16_t* y_experts, const int32_t* topk_prob, const int16_t* shared,
                     int64_t T, int64_t k, int64_t H, uint8_t prob_frac, int16_t* out);

/* sampling.rs:8-18: first index of the maximum. */
int64_t mylo_argmax_i32(const int32_t* v, int64_t n);

/* prng.rs:7-15. Returns the new state, writes the output word. */
uint64_t mylo_splitmix64(uint64_t state, uint64_t* out);

/* Number of OpenMP threads the batch functions use (1 when built without). */
int mylo_num_threads(void);
void mylo_set_num_threads(int n);

#ifdef __cplusplus
}
#endif

#endif /* MYL_ORACLE_H */
