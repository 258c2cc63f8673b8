/*
 * myl_forward.h — CPU restatement of Myelith's integer decoder forward pass
 * (Qwen2.5 architecture) around the W8A16 linears.
 *
 * TEST INFRASTRUCTURE ONLY: the checker the CUDA forward is compared against
 * (tests, the smoke check, the bench's parity and CPU-baseline legs). Never
 * linked into or called from libmyl_w8a16.so.
 *
 * Reference functions restated (paths relative to the Myelith project root):
 *
 *   kernels/src/rmsnorm.rs:20-24      inv_n_q20
 *   kernels/src/rmsnorm.rs:61-153     rmsnorm_i16 (i128 sum, max-shift alignment)
 *   kernels/src/fixed_point.rs:102-146 inv_sqrt_q15, isqrt_round
 *   kernels/src/rope.rs:17-32         rotate_half_split_i16
 *   kernels/src/attention.rs:20-27    dot_int
 *   kernels/src/attention.rs:42-94    attention_int
 *   runtime/src/kv_cache.rs:38-51     KVCache::write / read (positions <= pos)
 *   runtime/src/model.rs:229-311      forward_token (embedding, layers, final
 *                                     norm, LM head paths A and B)
 *   runtime/src/model.rs:401-674      forward_layer
 *   runtime/src/generate.rs:161-200   dekodieren_mit_digest (greedy)
 *
 * Arithmetic is the reference's, operation by operation and width by width.
 * Two evaluation-order freedoms are used, both exact:
 *  - the tokens of one prompt run layer by layer (all tokens through layer l,
 *    then layer l+1) instead of token by token. Token p at layer l reads only
 *    the cache entries of positions <= p of layer l (kv_cache.rs:47), which
 *    both orders have written by then, so every value is the same;
 *  - dot products sum the int8*int16 products in int32 blocks of 256 terms
 *    (|block| <= 256*128*32768 = 2^30) added to an int64. Integer addition is
 *    exact and associative (the reference's own reduction-order test,
 *    dot.rs:266), so the sum equals dot_scalar's.
 * Where the reference panics (debug-build shift or integer overflow, shape
 * asserts), the functions return MYLO_ERR_*.
 */
#ifndef MYL_FORWARD_H
#define MYL_FORWARD_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* rmsnorm.rs:20-24 */
int64_t mylo_inv_n_q20(int64_t n);
/* fixed_point.rs:117-146 */
uint64_t mylo_isqrt_round(uint64_t n);
/* fixed_point.rs:102-107 */
int64_t mylo_inv_sqrt_q15(int64_t head_dim);

/* rmsnorm.rs:61-153 on one row of n channels. */
int mylo_rmsnorm_i16(const int16_t* x, int64_t n, const uint8_t* x_shifts, const int8_t* gamma,
                     const uint8_t* gamma_shifts, const int16_t* rsqrt_lut, int64_t lut_len,
                     uint8_t lut_input_shift, uint8_t lut_output_frac, int64_t inv_n_q20,
                     uint8_t out_frac_bits, int16_t* out);

/* rope.rs:17-32: one head vector of length head_dim (even), half-split pairs. */
int mylo_rotate_half_split_i16(const int16_t* vec, int64_t head_dim, const int16_t* cos_row,
                               const int16_t* sin_row, uint8_t frac_bits, int16_t* out);

/* attention.rs:42-94. q [q_len][head_dim], k and v [kv_len][head_dim];
 * mask [q_len][kv_len] bytes (nonzero = attend) or NULL for all true. */
int mylo_attention_int(const int16_t* q, int64_t q_len, const int16_t* k, const int16_t* v,
                       int64_t kv_len, int64_t head_dim, const uint8_t* mask, int64_t score_mult,
                       uint8_t score_shift, const int16_t* exp_lut, int64_t exp_len,
                       uint8_t lut_shift, uint8_t prob_frac_bits, int16_t* out);

/* linear_w8a16_pc (linear.rs:87-119) on M rows with the blocked exact dot:
 * the same outputs as mylo_linear_w8a16_pc, faster (for full-size checks). */
int mylo_linear_w8a16_pc_fast(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                              const uint8_t* w_shifts, uint8_t act_frac, const uint8_t* out_frac,
                              int16_t* y);

/* acc[M][N] = dot(W[n], x[m]) in i64 (blocked exact dot), and the requant of
 * such sums, clamp_i16(rescale_i64(acc, w_shift + act_frac, out_frac[n]))
 * (linear.rs:61-68): the row-parallel check sums the partials of the ranks'
 * K slices and requantises once. */
int mylo_linear_acc_fast(const int16_t* x, int64_t M, const int8_t* W, int64_t K, int64_t N,
                         int64_t* acc);
int mylo_requant_acc(const int64_t* acc, int64_t M, int64_t N, const uint8_t* w_shifts,
                     uint8_t act_frac, const uint8_t* out_frac, int16_t* y);

/* One transformer layer's tensors and calibrated scales (model.rs:62-117). */
typedef struct mylo_layer {
  const int8_t* ln1_gamma;          /* input_layernorm [hidden] */
  const uint8_t* ln1_gamma_shifts;
  const int8_t* ln2_gamma;          /* post_attention_layernorm [hidden] */
  const uint8_t* ln2_gamma_shifts;
  const int8_t* wq;                 /* [heads*head_dim][hidden] */
  const int8_t* wk;                 /* [kv_heads*head_dim][hidden] */
  const int8_t* wv;
  const int8_t* wo;                 /* [hidden][heads*head_dim] */
  const int8_t* wg;                 /* [intermediate][hidden] */
  const int8_t* wu;
  const int8_t* wd;                 /* [hidden][intermediate] */
  const uint8_t *sq, *sk, *sv, *so, *sg, *su, *sd;  /* per-row weight shifts */
  const int16_t *bq, *bk, *bv;      /* int16 biases (NULL: no attention bias) */
  const uint8_t *bq_shifts, *bk_shifts, *bv_shifts;
  uint8_t norm_attn_frac, q_frac, k_frac, v_frac, attn_out_frac;
  uint8_t norm_mlp_frac, gate_frac, up_frac, down_in_frac;
  const uint8_t* residual_in_frac;  /* [hidden] per channel */
  const uint8_t* residual_mid_frac; /* [hidden] */
} mylo_layer;

/* The model (model.rs:120-163) with the spec constants of ModelConfig
 * (model.rs:166-203, read from theta_v/spec.json by loader.rs:654-682). */
typedef struct mylo_model {
  int64_t vocab, hidden, num_layers, num_heads, num_kv_heads, head_dim, intermediate;
  const int8_t* embed;              /* [vocab][hidden] */
  const uint8_t* embed_shifts;      /* [vocab] */
  const int8_t* lm_head;            /* path B [vocab][hidden] (the embedding when tied) */
  const uint8_t* lm_head_shifts;
  const int16_t* lm_head16;         /* path A [vocab][hidden] int16, NULL if absent */
  const uint8_t* lm_head16_shifts;
  const int8_t* final_gamma;
  const uint8_t* final_gamma_shifts;
  uint8_t final_norm_frac;
  const uint8_t* final_residual_frac; /* [hidden] */
  const mylo_layer* layers;         /* [num_layers] */
  const int16_t* cos_lut;           /* [rope_len] = [n_pos][head_dim/2] */
  const int16_t* sin_lut;
  int64_t rope_len;
  const int16_t* exp_lut;
  int64_t exp_len;
  const int16_t* silu_lut;
  int64_t silu_len;
  const int16_t* rsqrt_lut;
  int64_t rsqrt_len;
  uint8_t score_frac_bits, exp_input_frac, prob_frac_bits, rope_frac_bits;
  uint8_t silu_in_frac, silu_out_frac, rsqrt_input_shift, rsqrt_output_frac, logit_frac_bits;
  int16_t silu_lut_offset;
} mylo_model;

/* forward_token (model.rs:229-311) for T consecutive tokens of one sequence at
 * positions pos0 .. pos0+T-1. The KV cache is k_cache/v_cache, each
 * [num_layers][num_kv_heads][max_pos][head_dim] int16 (kv_cache.rs:38-51:
 * entry (layer, head, pos)). logits [vocab] receives the last token's logits
 * (NULL: not computed). */
int mylo_forward(const mylo_model* m, int16_t* k_cache, int16_t* v_cache, int64_t max_pos,
                 const int32_t* tokens, int64_t T, int64_t pos0, int32_t* logits);

/* dekodieren_mit_digest (generate.rs:161-200), greedy: prefill the prompt,
 * then max_new steps of (record logits, argmax_int, record token, forward).
 * out_tokens [max_new]; step_logits [max_new][vocab] receives the logits
 * each step hashed (NULL: not kept). The SHA-256 digest is taken by the
 * caller over, per step, the logits as i32 little-endian then the token as
 * u32 little-endian. */
int mylo_generate(const mylo_model* m, int16_t* k_cache, int16_t* v_cache, int64_t max_pos,
                  const int32_t* prompt, int64_t P, int64_t max_new, int32_t* out_tokens,
                  int32_t* step_logits);

#ifdef __cplusplus
}
#endif

#endif /* MYL_FORWARD_H */
