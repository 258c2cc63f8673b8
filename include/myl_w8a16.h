/*
 * myl_w8a16.h — C ABI of libmyl_w8a16.so, the B200 (sm_100a) implementation of
 * Myelith's W8A16 integer linear layer (int8 weights x int16 activations,
 * exact integer accumulation, power-of-two round-to-nearest-even requant).
 *
 * Every entry point is bit-exact against the reference CPU path. The
 * reference counterpart of each entry point is cited beside it, as
 * <file>:<line> inside the Myelith project (INTEGER_LLM/...).
 *
 * Conventions
 *  - Return value: 0 (MYL_OK) or an MYL_ERR_* code; myl_last_error() gives a
 *    message for the calling thread. The reference panics in the same cases
 *    (shape asserts, debug-build integer overflow); its Rust binding turns a
 *    nonzero status back into a panic.
 *  - W is row-major [out_features][in_features] int8 (one row per output
 *    channel), as QTensor.data holds it (runtime/src/model.rs:28-35).
 *  - Activations are row-major [M][in_features] int16; M is the number of
 *    independent rows (tokens). Every output row equals the reference's
 *    per-token GEMV result (the reference loops forward_token per token).
 *  - Entry points named *_dev take device pointers and a cudaStream_t (passed
 *    as void*), enqueue work and return without synchronising. All other
 *    entry points take host pointers and return after the result is in host
 *    memory.
 *  - A context belongs to one device. Calls on one context are serialised by
 *    the caller (the reference callers are single-threaded).
 *  - There is no CPU fallback: without a usable sm_100 device myl_init fails.
 */
#ifndef MYL_W8A16_H
#define MYL_W8A16_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MYL_ABI_VERSION 1

enum myl_status {
  MYL_OK = 0,
  MYL_ERR_SHAPE = 1,       /* length/shape mismatch: assert_eq! in linear.rs:51-58, :95-107 */
  MYL_ERR_OVERFLOW = 2,    /* u8/i8 overflow or shift >= width in the requant (debug panic) */
  MYL_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  MYL_ERR_ARG = 4,         /* null pointer, bad handle or bad enum */
  MYL_ERR_DEVICE = 5,      /* a kernel reported an error (e.g. a bounded wait ran out) */
  MYL_ERR_UNSUPPORTED = 6, /* device is not sm_100 or a size is beyond a kernel limit */
  MYL_ERR_IO = 7,          /* an artifact file is missing, unreadable or not valid JSON */
  MYL_ERR_CORRUPT = 8,     /* an artifact file disagrees with its manifest (size, hash, dtype),
                              or a wire frame is malformed (magic, length, CRC) */
};

/* Requant modes (myl_requant_create). */
enum myl_rq_mode {
  MYL_RQ_SHIFT_I16 = 0, /* clamp_i16(rescale_i64(acc, w_shift+act_frac, out_frac)) linear.rs:66,115 */
  MYL_RQ_SHIFT_I32 = 1, /* clamp_i32(rescale_i64(...)), the LM head runtime/src/model.rs:303-305 */
  MYL_RQ_MULT_I16 = 2,  /* clamp_i16(rne_i128(acc * mult[r], shift[r])), shift in [0,126] */
};

typedef struct myl_ctx myl_ctx;
typedef struct myl_weight myl_weight;
typedef struct myl_requant myl_requant;

/* Message of the last failed call on this thread ("" if none). */
const char* myl_last_error(void);
int myl_abi_version(void);

/* Replaces CudaBackend::init (kernels/src/backends/cuda.rs:93-107): selects
 * the device, checks for sm_100, creates the stream and workspaces. */
int myl_init(int device, myl_ctx** out);
int myl_destroy(myl_ctx* ctx);
/* Replaces CudaBackend::sm_version / device_id (cuda.rs:109-115). */
int myl_device_info(const myl_ctx* ctx, int* device, int* sm_version, int* num_sms);

/* Uploads one weight matrix once (the reference keeps it in host memory for
 * the model's lifetime, runtime/src/model.rs:28-35). W rows are ldw bytes
 * apart (ldw >= in_features; a column slice of a larger matrix for
 * row-parallel sharding is W + k0 with ldw = full width). */
int myl_weight_register(myl_ctx* ctx, const int8_t* W, int64_t out_features, int64_t in_features,
                        int64_t ldw, const uint8_t* w_shifts, myl_weight** out);
int myl_weight_release(myl_ctx* ctx, myl_weight* w);

/* --- Free-function mirrors (host pointers, synchronous) --------------------- */

/* linear_w8a16 (kernels/src/linear.rs:43-70): y[M][N] int16. */
int myl_linear_w8a16(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                     uint8_t act_frac_bits, uint8_t out_frac_bits, int16_t* y);

/* linear_w8a16_pc (linear.rs:87-119): out_frac_bits[N], one per output channel. */
int myl_linear_w8a16_pc(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                        uint8_t act_frac_bits, const uint8_t* out_frac_bits, int16_t* y);

/* LM head, path B (runtime/src/model.rs:297-307): logits[M][N] int32. */
int myl_lm_head_w8a16_i32(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                          uint8_t final_norm_frac, uint8_t logit_frac, int32_t* logits);

/* LM head, path A (runtime/src/model.rs:285-296): int16 weights [N][K] with
 * one shift per row (loader.rs:124-128), i64 dot, rescale to logit_frac,
 * clamp to i32. The weight is registered with myl_weight16_register and
 * stored as two int8 rows per int16 row (high byte, low byte - 128), so the
 * same GEMV and tensor-core kernels run it; the device form is
 * myl_linear_dev with a MYL_RQ_SHIFT_I32 plan of this weight. */
int myl_weight16_register(myl_ctx* ctx, const int16_t* W, int64_t out_features, int64_t in_features,
                          int64_t ldw, const uint8_t* w_shifts, myl_weight** out);
int myl_lm_head_w16a16_i32(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                           uint8_t final_norm_frac, uint8_t logit_frac, int32_t* logits);

/* Greedy selection (argmax_int, sampling.rs:8-18: lowest index among the
 * maxima) over int32 logits [M][V] (row stride ld, device pointers) whose
 * column j is vocab index index_base + j: keys[m] = v * 2^32 + (2^32 - 1 - i)
 * for the winning logit v at index i, or INT64_MIN when V = 0. The largest key
 * over vocab shards is the global winner, so tensor-parallel ranks combine
 * with one int64 max all-reduce; token = 2^32 - 1 - (key & 0xFFFFFFFF),
 * logit = key >> 32. index_base + V must not exceed 2^32. */
int myl_argmax_keys_dev(myl_ctx* ctx, const int32_t* logits, int64_t M, int64_t V, int64_t ld,
                        int64_t index_base, int64_t* keys, void* stream);

/* linear_w8a16 followed by add_bias_i16 (linear.rs:132-145) as the runtime
 * does for q/k/v (runtime/src/model.rs:438-453), fused into one epilogue:
 * y = clamp_i16(clamp_i16(requant(acc)) + rescale(bias[r], bias_shifts[r], out_frac)). */
int myl_linear_w8a16_bias(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                          uint8_t act_frac_bits, uint8_t out_frac_bits, const int16_t* bias,
                          const uint8_t* bias_shifts, int16_t* y);

/* Multiplier requant: y = clamp_i16(rne_i128(acc * mult[r], shift[r])).
 * No counterpart in the reference linear layer; with mult = 2^m and
 * shift = s + m it equals the pure shift (fixed_point.rs:365-379). */
int myl_linear_w8a16_mult(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                          const int32_t* mult, const uint8_t* shift, int16_t* y);

/* Backend::linear_w8a16 (kernels/src/backend.rs:39-49), same arguments and
 * meaning: one activation row, raw host weight pointer. The weight is
 * uploaded on first use and found again by (W, in, out, w_shifts) address,
 * length and shift table, and by a 64-bit digest of the weight bytes computed
 * on every call (one pass over W, as the reference's own call reads all of W),
 * so a reused address with new contents is uploaded again. Callers that keep
 * weights fixed and want no per-call pass register them (myl_weight_register).
 * myl_backend_forget(ctx, W) drops a cached upload. */
int myl_backend_linear_w8a16(myl_ctx* ctx, const int16_t* x, const int8_t* W, int16_t* out,
                             uint64_t in_features, uint64_t out_features, const uint8_t* w_shifts,
                             uint8_t act_frac, uint8_t out_frac);
int myl_backend_forget(myl_ctx* ctx, const int8_t* W);

/* --- Device path ------------------------------------------------------------- */

/* A requant plan for one weight: per-channel signed total shift (and
 * multiplier), validated on the host and kept on the device.
 *  MYL_RQ_SHIFT_*: act_frac plus out_frac (out_frac_pc[N] if per_channel,
 *                  else out_frac_pc[0]); mult/shift ignored.
 *  MYL_RQ_MULT_I16: mult[N], shift[N]; act_frac/out_frac ignored. */
int myl_requant_create(myl_ctx* ctx, const myl_weight* w, int mode, uint8_t act_frac,
                       const uint8_t* out_frac_pc, int per_channel, const int32_t* mult,
                       const uint8_t* shift, myl_requant** out);
int myl_requant_release(myl_ctx* ctx, myl_requant* rq);
/* Adds the q/k/v bias of add_bias_i16 (linear.rs:132-145) to an int16 plan. */
int myl_requant_set_bias(myl_ctx* ctx, myl_requant* rq, const int16_t* bias,
                         const uint8_t* bias_shifts, uint8_t out_frac);

/* y[M][ldy] = requant(W x) with device pointers. y is int16 for the *_I16
 * modes and int32 for MYL_RQ_SHIFT_I32. x rows are ldx elements apart. */
int myl_linear_dev(myl_ctx* ctx, const myl_weight* w, const myl_requant* rq, const int16_t* x,
                   int64_t M, int64_t ldx, void* y, int64_t ldy, void* stream);

/* acc[M][N] = W x as exact int64 partial sums (no requant). Row-parallel
 * tensor parallelism sums these across ranks, then calls myl_requant_acc_dev. */
int myl_linear_acc_dev(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                       int64_t ldx, int64_t* acc, void* stream);
int myl_requant_acc_dev(myl_ctx* ctx, const myl_requant* rq, const int64_t* acc, int64_t M,
                        void* y, int64_t ldy, void* stream);

/* Row-parallel exchange over peer memory (one process per GPU on one node,
 * buffers shared with myl_ipc_*), replacing the int64 all-reduce:
 *  1. myl_linear_acc_exchange_dev: the GEMM's epilogue stores the exact int64
 *     partial of output row m straight into the receive buffer of the rank
 *     that owns it, o = m / rows_per_rank, as row rank * rows_per_rank +
 *     m % rows_per_rank (dst[o]: [world * rows_per_rank][N] int64, peer
 *     memory over NVLink). rows_per_rank is a multiple of 16 and
 *     M <= world * rows_per_rank.
 *  2. all ranks' step 1 finished (a barrier on the stream, e.g. a one-element
 *     all-reduce);
 *  3. myl_exchange_reduce_dev on every rank: sums the world slabs of its own
 *     rows in recv, requantises (plan rq) and writes the int16/int32 rows into
 *     every rank's output buffer out[o] ([M][ldo]) at their global row;
 *  4. a barrier again before the outputs are read.
 * The sums are exact integers, so the result equals the single-GPU layer bit
 * for bit. At most 8 ranks. */
int myl_linear_acc_exchange_dev(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                                int64_t ldx, int64_t* const* dst, int world, int rank,
                                int64_t rows_per_rank, void* stream);
int myl_exchange_reduce_dev(myl_ctx* ctx, const myl_requant* rq, const int64_t* recv, int world,
                            int rank, int64_t rows_per_rank, int64_t M, void* const* out, int64_t ldo,
                            void* stream);
/* Barrier of steps 2 and 4 on the stream, without a collective library:
 * flags[o] is rank o's array of world 64-bit flag words (peer memory, zero at
 * allocation); this rank stores `epoch` into flags[o][rank] for every o and
 * waits until flags[rank][o] >= epoch for every o. epoch grows by one per
 * call on every rank. The wait is bounded (myl_set_wait_timeout_ns): a peer
 * that does not arrive is reported as MYL_ERR_DEVICE at the next check. */
int myl_exchange_barrier_dev(myl_ctx* ctx, unsigned long long* const* flags, int world, int rank,
                             unsigned long long epoch, void* stream);
/* Expert-parallel MoE over peer memory (no collective library on the data
 * path). Experts are split over the ranks in contiguous shard ranges.
 *  - myl_ep_dispatch_dev: pair q = t * k + j of this rank's tokens (x [T][ldx],
 *    expert ids idx [T][k] from the router) takes slot s = atomicAdd(
 *    counters[o]) on the rank o owning expert idx[q] (system scope, over
 *    NVLink) and stores its row at rows[o] + s * H, idx[q] at ids[o][s] and
 *    rank << 24 | q at src[o][s]. Slots >= capacity are not written and raise
 *    MYL_ERR_DEVICE at the next check (as do expert ids out of range).
 *  - after a barrier, rank o runs its experts on its counters[o] received rows
 *    (myl_moe_experts_dev; the order of the rows does not matter: each output
 *    row depends on its own input row only) and resets its counter;
 *  - myl_ep_return_dev: received row i goes back to back[src >> 24] at row
 *    src & 0xFFFFFF, i.e. in (token, choice) order on its home rank;
 *  - after a barrier, the home rank combines (myl_moe_combine_dev).
 * The arithmetic is the single-GPU layer's, so the output is bit-identical. */
int myl_ep_dispatch_dev(myl_ctx* ctx, const int16_t* x, int64_t T, int64_t ldx, int64_t H,
                        const int32_t* idx, int k, int E, int world, int rank, int16_t* const* rows,
                        int32_t* const* ids, int32_t* const* src, int32_t* const* counters,
                        int64_t capacity, void* stream);
int myl_ep_return_dev(myl_ctx* ctx, const int16_t* y, int64_t count, int64_t H, const int32_t* src,
                      int16_t* const* back, int world, void* stream);

/* Device buffers shared between the processes of one node: allocation with
 * its IPC handle (MYL_IPC_HANDLE_BYTES bytes, to send to the other ranks),
 * opening a peer's handle (not one's own), and their release. */
#define MYL_IPC_HANDLE_BYTES 64
int myl_ipc_alloc(myl_ctx* ctx, size_t bytes, void** ptr, void* handle);
int myl_ipc_open(myl_ctx* ctx, const void* handle, void** ptr);
int myl_ipc_close(myl_ctx* ctx, void* ptr);
int myl_ipc_free(myl_ctx* ctx, void* ptr);

/* Splits int16 activations into the byte planes the tensor-core GEMM reads:
 * two unsigned bytes hi = (x >> 8) + 128 (offset binary) and lo = x & 255,
 * x = 256*hi + lo - 32768; planes are [M][ldp] (ldp a multiple of 16,
 * 16-byte aligned; columns K..ldp-1 hold x = 0, i.e. hi = 128, lo = 0).
 * A producer kernel that writes the planes directly skips this pass. */
int myl_split_hilo_dev(myl_ctx* ctx, const int16_t* x, int64_t M, int64_t K, int64_t ldx,
                       uint8_t* xhi, uint8_t* xlo, int64_t ldp, void* stream);

/* Tensor-core GEMM from byte planes (any M >= 1). rq = NULL stores exact
 * int64 accumulators into y (as myl_linear_acc_dev); otherwise y is the
 * requantised output of rq's mode. */
int myl_linear_planes_dev(myl_ctx* ctx, const myl_weight* w, const myl_requant* rq,
                          const uint8_t* xhi, const uint8_t* xlo, int64_t ldp, int64_t M, void* y,
                          int64_t ldy, void* stream);

/* --- MLP: mlp_int (kernels/src/mlp.rs:28-74) ----------------------------------
 * gate = linear_w8a16(x, W_gate), up = linear_w8a16(x, W_up),
 * h = clamp_i16(rescale_i64(silu_lut[idx(gate)] * up, silu_out + up_out, down_in)),
 * y = linear_w8a16_pc(h, W_down, out_frac[H]).
 * Registration uploads W_gate/W_up interleaved (row 2i = gate_i, 2i+1 = up_i),
 * so one kernel computes both projections and the SiLU product (and, for
 * M > 4, writes h straight into the down projection's byte planes). Every
 * shift is validated as the reference's debug build would. */
typedef struct myl_mlp myl_mlp;
int myl_mlp_register(myl_ctx* ctx, const int8_t* W_gate, const int8_t* W_up, const int8_t* W_down,
                     int64_t hidden, int64_t intermediate, const uint8_t* gate_w_shifts,
                     const uint8_t* up_w_shifts, const uint8_t* down_w_shifts,
                     const int16_t* silu_lut, int64_t silu_lut_len, uint8_t in_frac,
                     uint8_t gate_out_frac, uint8_t up_out_frac, uint8_t down_in_frac,
                     uint8_t silu_in_frac, int16_t silu_lut_offset, uint8_t silu_out_frac,
                     const uint8_t* out_frac, myl_mlp** out);
int myl_mlp_release(myl_ctx* ctx, myl_mlp* mlp);
/* Host pointers: x [M][hidden] -> y [M][hidden]. */
int myl_mlp_int(myl_ctx* ctx, const myl_mlp* mlp, const int16_t* x, int64_t M, int16_t* y);
/* Device pointers on a stream. */
int myl_mlp_dev(myl_ctx* ctx, const myl_mlp* mlp, const int16_t* x, int64_t M, int64_t ldx,
                int16_t* y, int64_t ldy, void* stream);

/* Tensor parallelism over intermediate channels: a rank registers its slice
 * (gate/up rows and down columns of channels [i0, i1)) and gets the exact
 * int64 down-projection partial sums; the caller adds them across ranks and
 * applies the down requant once (myl_mlp_requant_dev), so the result is
 * bit-identical to the unsharded mlp_int. */
int myl_mlp_partial_dev(myl_ctx* ctx, const myl_mlp* mlp, const int16_t* x, int64_t M, int64_t ldx,
                        int64_t* acc, void* stream);
int myl_mlp_requant_dev(myl_ctx* ctx, const myl_mlp* mlp, const int64_t* acc, int64_t M, int16_t* y,
                        int64_t ldy, void* stream);

/* --- linear_backward (kernels/src/backward.rs:147-211) -----------------------------
 * For each of M tokens, with g = dL/dy [N] int32 and x [K] int16:
 *   gx[j] = clamp_i32(rescale_i64(clamp_i64(rne_i128(sum_i (g[i]*W[i][j])
 *                     << (ref - w_shifts[i]), ref)), g_frac, gx_frac)),
 *   ref = max_i w_shifts[i]  (the summands aligned to the largest shift,
 *   rounded once at the end);
 *   gw[i][j] = g[i] * x[j]   int64, [M][N][K] (NULL: not computed).
 * Exact (i64 group sums of equal shift, an i128 accumulator). Limits:
 * w_shifts <= 64, N < 2^24; int16 weights are not supported. */
int myl_linear_backward(myl_ctx* ctx, const myl_weight* w, const int32_t* g, const int16_t* x,
                        int64_t M, uint8_t g_frac, uint8_t gx_frac, int32_t* gx, int64_t* gw);
int myl_linear_backward_dev(myl_ctx* ctx, const myl_weight* w, const int32_t* g, int64_t ldg,
                            const int16_t* x, int64_t ldx, int64_t M, uint8_t g_frac,
                            uint8_t gx_frac, int32_t* gx, int64_t ldgx, int64_t* gw, void* stream);

/* --- MoE layer --------------------------------------------------------------------
 * No counterpart in the reference, which has no MoE; the layer is composed of
 * its primitives only:
 *   logits[t][e] = clamp_i32(rescale_i64(dot(W_router[e], x[t]),
 *                  router_w_shifts[e] + router_in_frac, router_frac))
 *                  (the LM-head linear, runtime/src/model.rs:297-307)
 *   topk[t]      = k times argmax over the experts not yet chosen, ties to the
 *                  lowest index (sampling.rs:8-18)
 *   p[t][j]      = softmax_int(logits[t][topk[t]], exp_lut, exp_lut_shift,
 *                  prob_frac)                        (softmax.rs:24-64)
 *   y[t][j]      = mlp_int(x[t], expert topk[t][j])  (mlp.rs:28-74)
 *   out[t][h]    = clamp_i16(rescale_i64(sum_j p[t][j] * y[t][j][h], prob_frac, 0)
 *                  + shared[t][h])   shared = mlp_int of the shared expert, or 0
 * The experts share the scalar fractions and SiLU table; shifts are per channel.
 * Expert weights: W_gate / W_up [num_local][intermediate][hidden], W_down
 * [num_local][hidden][intermediate], gate/up_w_shifts [num_local][intermediate],
 * down_w_shifts and out_frac [num_local][hidden]; the object holds experts
 * [first_expert, first_expert + num_local) of num_experts (expert parallelism:
 * the router covers all num_experts, each rank holds its share).
 * Limits: top_k <= 8, num_experts <= 256, and every exp_lut entry times
 * 2^prob_frac inside i32 (where softmax_int's i32 product never overflows). */
typedef struct myl_moe myl_moe;
typedef struct myl_moe_spec {
  int64_t hidden, intermediate, num_experts, top_k, first_expert, num_local;
  /* router */
  const int8_t* W_router;          /* [num_experts][hidden] */
  const uint8_t* router_w_shifts;  /* [num_experts] */
  uint8_t router_in_frac, router_frac;
  const int16_t* exp_lut;
  int64_t exp_lut_len;
  uint8_t exp_lut_shift, prob_frac;
  /* experts (mlp_int parameters, see above) */
  const int8_t *W_gate, *W_up, *W_down;
  const uint8_t *gate_w_shifts, *up_w_shifts, *down_w_shifts, *out_frac;
  const int16_t* silu_lut;
  int64_t silu_lut_len;
  uint8_t in_frac, gate_out_frac, up_out_frac, down_in_frac, silu_in_frac, silu_out_frac;
  int16_t silu_lut_offset;
  /* shared expert: borrowed, may be NULL; it must outlive the MoE object */
  const myl_mlp* shared;
} myl_moe_spec;
int myl_moe_register(myl_ctx* ctx, const myl_moe_spec* spec, myl_moe** out);
int myl_moe_release(myl_ctx* ctx, myl_moe* moe);
/* The whole layer on one GPU (num_local == num_experts). Host pointers:
 * x [T][hidden] -> out [T][hidden]. */
int myl_moe_forward(myl_ctx* ctx, const myl_moe* moe, const int16_t* x, int64_t T, int16_t* out);
/* Device pointers on a stream. topk_idx / topk_prob ([T][top_k] int32) may be
 * NULL; when given they receive the routing. */
int myl_moe_dev(myl_ctx* ctx, const myl_moe* moe, const int16_t* x, int64_t T, int64_t ldx,
                int16_t* out, int64_t ldo, int32_t* topk_idx, int32_t* topk_prob, void* stream);
/* The stages, for expert parallelism (device pointers):
 *   route    x [T] -> topk_idx, topk_prob [T][top_k]
 *   experts  rows x [P][hidden] with global expert ids [P], all held by this
 *            object -> y [P][hidden] = mlp_int(x[q], expert ids[q]); an id
 *            outside the object's experts reports MYL_ERR_DEVICE at the next
 *            synchronising call and gives a zero row
 *   shared   myl_mlp_dev of the shared expert on x [T] -> shared_out [T][hidden]
 *   combine  y rows in (token, choice) order [T * top_k][hidden], topk_prob,
 *            shared_out (may be NULL) -> out [T][hidden] */
int myl_moe_route_dev(myl_ctx* ctx, const myl_moe* moe, const int16_t* x, int64_t T, int64_t ldx,
                      int32_t* topk_idx, int32_t* topk_prob, void* stream);
int myl_moe_experts_dev(myl_ctx* ctx, const myl_moe* moe, const int16_t* x, int64_t P, int64_t ldx,
                        const int32_t* expert_ids, int16_t* y, int64_t ldy, void* stream);
int myl_moe_combine_dev(myl_ctx* ctx, const myl_moe* moe, const int16_t* y, int64_t ldy,
                        const int32_t* topk_prob, const int16_t* shared_out, int64_t ld_shared,
                        int64_t T, int16_t* out, int64_t ldo, void* stream);

/* Waits for the context's work and reports kernel-side errors (bounded waits
 * that ran out) as MYL_ERR_DEVICE; the context stays usable afterwards. */
int myl_synchronize(myl_ctx* ctx);

/* Bound of every device-side wait, in nanoseconds (default 2e9). */
int myl_set_wait_timeout_ns(myl_ctx* ctx, uint64_t ns);

/* Kernel selection, for tests and tuning: M <= gemv_max_m (at most 4) runs the
 * CUDA-core GEMV, larger M the tcgen05 GEMM; force_split_k = 0 and
 * force_token_tile = 0 choose automatically (token tile 32, 64 or 128). */
int myl_set_dispatch(myl_ctx* ctx, int gemv_max_m, int force_split_k, int force_token_tile);

/* Caps the SMs the persistent kernels (tensor-core GEMM, balanced GEMV) of
 * this context occupy, so that kernels on other streams (a collective that
 * overlaps the GEMM) find free SMs; 0 = all SMs (the default). */
int myl_set_sm_limit(myl_ctx* ctx, int max_sms);

/* Tensor-core GEMM variant, for tests and tuning: pair_mode = 1 (default) runs
 * 128-token tiles on CTA pairs (one M = 256 MMA over two SMs, each SM loading
 * one activation byte plane), 0 one CTA per 128-channel tile; xbox_rows (16,
 * 32, 64 or 128; 0 = unchanged) is the row count of the activation TMA boxes. */
int myl_set_tc_options(myl_ctx* ctx, int pair_mode, int xbox_rows);

/* Number of this library's kernels launched on the context since init. */
int64_t myl_launch_count(const myl_ctx* ctx);

/* Test hook for failure detection without a GPU fault: while on, every
 * tensor-core launch makes its epilogue wait on a barrier that nothing
 * arrives at; the wait runs out after the wait timeout, the kernel writes an
 * error code, frees its resources and returns, and the next host-synchronising
 * call reports MYL_ERR_DEVICE. The context stays usable. */
int myl_debug_inject_wait_fault(myl_ctx* ctx, int on);

/* --- θ_v artifacts (runtime/src/loader.rs:322-560) --------------------------------
 * myl_artifact_open reads weights_manifest.json and, if present, luts.json of
 * an artifact directory into host memory, rejecting it as the reference
 * does: unsupported dtype, int16 outside the LM head and *_bias, a file whose
 * size disagrees with its shape, a SHA-256 that disagrees with the manifest,
 * a shifts file with the wrong length or hash, a uniform shift outside
 * 0..=255. No device is needed. myl_artifact_register uploads one 2-D tensor
 * as a weight (int16: the LM head's path A, myl_weight16_register). Names are
 * found by manifest key or original name ('.' read as '_', loader.rs:167-170).
 * dtype: 1 = int8, 2 = int16 (little-endian); shape has up to 4 entries. */
typedef struct myl_artifact myl_artifact;
int myl_artifact_open(const char* dir, myl_artifact** out);
int myl_artifact_close(myl_artifact* a);
int64_t myl_artifact_count(const myl_artifact* a);
int myl_artifact_find(const myl_artifact* a, const char* name, int64_t* index);
int myl_artifact_tensor(const myl_artifact* a, int64_t index, const char** key,
                        const char** original_name, int* dtype, int* ndim, int64_t* shape,
                        const void** data, const uint8_t** shifts);
int myl_artifact_register(myl_ctx* ctx, const myl_artifact* a, int64_t index, myl_weight** out);
int myl_artifact_lut(const myl_artifact* a, const char* name, const int16_t** data, int64_t* len);
/* SHA-256 (FIPS 180-4) as the loader checks it (sha2 0.10 in the reference). */
int myl_sha256(const void* data, size_t len, uint8_t* out);

/* --- Pipeline wire format (INTEGER_LLM/pipeline/src/codec.rs) -----------------------
 * Frames carry a stage's int16 activations (or packed token ids) between
 * pipeline stages: "IINTPIPE", nine little-endian u64 fields, the CRC-32
 * (crc32fast 1.3: reflected 0xEDB88320, init and final XOR 0xFFFFFFFF) of the
 * payload, the payload (int16 little-endian) and zero padding to a multiple of
 * 8 bytes (codec.rs:86-111). Decoding rejects, as decode_message does
 * (codec.rs:113-178), a buffer shorter than the header, a wrong magic, a
 * payload length that overflows or runs past the buffer, a CRC mismatch and an
 * odd payload length, each with MYL_ERR_CORRUPT. The encoder writes
 * payload_len = 2 * n whatever meta->payload_len holds, as encode_message does.
 * The _dev forms keep the payload in device memory and compute its CRC on the
 * GPU (they synchronise the stream to report the result). */
#define MYL_WIRE_HEADER_BYTES 84
#define MYL_WIRE_FLAG_STARTS_GENERATION 0x1ull
#define MYL_WIRE_FLAG_ABORT 0x2ull
#define MYL_WIRE_FLAG_TOKEN_INPUT 0x4ull
typedef struct myl_wire_meta {
  uint64_t version, theta_v_hash, request_id, sequence_id, stage_id, token_position;
  uint64_t payload_len, flags, reserved;
  uint32_t crc;
} myl_wire_meta;
/* Frame size in bytes for n int16 values (header + payload + padding). */
uint64_t myl_wire_frame_bytes(uint64_t n_values);
uint32_t myl_crc32(const void* data, uint64_t len);
int myl_wire_encode(const myl_wire_meta* meta, const int16_t* values, uint64_t n, uint8_t* out,
                    uint64_t cap, uint64_t* out_len);
/* values may be NULL with cap 0 to learn n; a payload larger than cap values
 * is MYL_ERR_SHAPE. */
int myl_wire_decode(const uint8_t* buf, uint64_t len, myl_wire_meta* meta, int16_t* values,
                    uint64_t cap, uint64_t* n);
/* CRC-32 of len bytes at a device pointer. */
int myl_crc32_dev(myl_ctx* ctx, const void* data, uint64_t len, uint32_t* crc, void* stream);
/* Header checks on the host, the payload copied once into dev_values, its CRC
 * checked on the GPU. */
int myl_wire_decode_dev(myl_ctx* ctx, const uint8_t* buf, uint64_t len, myl_wire_meta* meta,
                        int16_t* dev_values, uint64_t cap, uint64_t* n, void* stream);
/* Frame from n int16 values at a device pointer: CRC on the GPU, payload
 * copied once into the host frame. */
int myl_wire_encode_dev(myl_ctx* ctx, const myl_wire_meta* meta, const int16_t* dev_values,
                        uint64_t n, uint8_t* out, uint64_t cap, uint64_t* out_len, void* stream);
/* Token ids as the payload of a FLAG_TOKEN_INPUT frame (codec.rs:38-63): two
 * int16 per id (low half, high half); unpacking an odd count is MYL_ERR_SHAPE. */
int myl_wire_pack_tokens(const uint32_t* tokens, uint64_t n, int16_t* out);
int myl_wire_unpack_tokens(const int16_t* values, uint64_t n_values, uint32_t* tokens);

/* --- Integer decoder forward (runtime/src/model.rs, generate.rs) ------------------
 * The model of the reference's IntegerModel (model.rs:120-163): embedding,
 * num_layers transformer layers (forward_layer, model.rs:401-674: RMSNorm,
 * q/k/v with int16 biases, RoPE, KV cache, GQA attention with softmax_int,
 * o_proj onto the coarser residual scale, residual add, RMSNorm, mlp_int,
 * residual add), final RMSNorm and the LM head (path A int16 or path B int8,
 * i32 logits). All tensors are host arrays in the artifact layout (row-major
 * [out][in], one power-of-two shift per row; per-channel residual shifts);
 * myl_model_create validates every shift as the reference's debug build would
 * and uploads the model once. Results are bit-identical to the reference. */
typedef struct myl_layer_spec {
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
  const uint8_t *sq, *sk, *sv, *so, *sg, *su, *sd; /* per-row weight shifts */
  const int16_t *bq, *bk, *bv;      /* int16 biases, NULL: no attention bias */
  const uint8_t *bq_shifts, *bk_shifts, *bv_shifts;
  uint8_t norm_attn_frac, q_frac, k_frac, v_frac, attn_out_frac;
  uint8_t norm_mlp_frac, gate_frac, up_frac, down_in_frac;
  const uint8_t* residual_in_frac;  /* [hidden] per channel */
  const uint8_t* residual_mid_frac; /* [hidden] */
} myl_layer_spec;

typedef struct myl_model_spec {
  int64_t vocab, hidden, num_layers, num_heads, num_kv_heads, head_dim, intermediate;
  const int8_t* embed;              /* [vocab][hidden] */
  const uint8_t* embed_shifts;      /* [vocab] */
  const int8_t* lm_head;            /* path B [vocab][hidden]; NULL: tied to embed */
  const uint8_t* lm_head_shifts;
  const int16_t* lm_head16;         /* path A [vocab][hidden] int16 (used when set) */
  const uint8_t* lm_head16_shifts;
  const int8_t* final_gamma;
  const uint8_t* final_gamma_shifts;
  uint8_t final_norm_frac;
  const uint8_t* final_residual_frac; /* [hidden] */
  const myl_layer_spec* layers;     /* [num_layers] */
  const int16_t* cos_lut;           /* [rope_len] = [n_pos][head_dim/2] */
  const int16_t* sin_lut;
  int64_t rope_len;
  const int16_t* exp_lut;
  int64_t exp_len;
  const int16_t* silu_lut;
  int64_t silu_len;
  const int16_t* rsqrt_lut;
  int64_t rsqrt_len;
  /* ModelConfig (model.rs:166-203) from theta_v/spec.json (loader.rs:654-682) */
  uint8_t score_frac_bits, exp_input_frac, prob_frac_bits, rope_frac_bits;
  uint8_t silu_in_frac, silu_out_frac, rsqrt_input_shift, rsqrt_output_frac, logit_frac_bits;
  int16_t silu_lut_offset;
} myl_model_spec;

typedef struct myl_model myl_model;
typedef struct myl_session myl_session;

/* loader.rs:709-851 build_model: validates and uploads the model. */
int myl_model_create(myl_ctx* ctx, const myl_model_spec* spec, myl_model** out);
int myl_model_release(myl_ctx* ctx, myl_model* model);
/* KV caches of `batch` independent sequences of up to max_positions tokens
 * each (kv_cache.rs:13-36), plus the work buffers of the forward. */
int myl_session_create(myl_ctx* ctx, const myl_model* model, int64_t batch, int64_t max_positions,
                       myl_session** out);
int myl_session_release(myl_ctx* ctx, myl_session* s);
/* Empties the caches: the next token goes to position 0. */
int myl_session_reset(myl_ctx* ctx, myl_session* s);
/* Number of positions the session's sequences hold. */
int64_t myl_session_position(const myl_session* s);

/* forward_token (model.rs:229-311) for T tokens of each of the session's B
 * sequences at the next T positions (host tokens [B][T]); logits [B][vocab]
 * (host, NULL: not computed) receives each sequence's last-token logits. The
 * prompt tokens may come in one call: the result equals T single-token calls. */
int myl_forward(myl_ctx* ctx, const myl_model* model, myl_session* s, const int32_t* tokens,
                int64_t T, int32_t* logits);
/* Greedy generation (generate.rs:76-116 / :161-200): from an empty cache,
 * prefill prompt [B][P], then max_new steps of (argmax_int of the logits,
 * forward of the chosen token). out_tokens [B][max_new]. digests [B][32]
 * (NULL: not computed) receives dekodieren_mit_digest's SHA-256 per sequence:
 * per step the logits as i32 little-endian, then the token as u32
 * little-endian. step_logits [B][max_new][vocab] (NULL: not kept) receives
 * the hashed logits. Without digests and step_logits the decode steps run as
 * one CUDA graph per step with no host synchronisation in between. */
int myl_generate(myl_ctx* ctx, const myl_model* model, myl_session* s, const int32_t* prompt,
                 int64_t P, int64_t max_new, int32_t* out_tokens, uint8_t* digests,
                 int32_t* step_logits);
/* The decode loop of myl_generate alone (generate.rs:101-113), continuing the
 * session after myl_forward of the prompt: max_new greedy steps from the
 * last logits. */
int myl_decode_greedy(myl_ctx* ctx, const myl_model* model, myl_session* s, int64_t max_new,
                      int32_t* out_tokens, uint8_t* digests, int32_t* step_logits);
/* Tensor parallelism over `world` GPUs of one node, one process per GPU
 * (Megatron style, every rank calls the same entry points in the same order):
 * rank r's model holds an even share of the query heads and the KV heads they
 * read (uneven head counts, e.g. 28 heads on 8 ranks, give some ranks one
 * more head and share a KV head between two ranks), of the MLP's intermediate
 * channels (gate/up rows, down columns) and of the vocabulary rows of the LM
 * head; embedding, norms and the residual stream are replicated. The
 * row-parallel projections (o_proj, down) write exact int64 partial sums
 * straight into every rank's receive region over NVLink (peer memory); after a
 * bounded device barrier every rank sums the slabs and requantises once, so
 * the result is bit-identical to the single-GPU model (integer addition is
 * exact and associative). Greedy selection takes the largest
 * (logit, lowest index) key over the ranks' vocabulary shares.
 * Setup: myl_model_create_tp with the whole model spec; a session; a region of
 * myl_session_tp_bytes bytes per rank shared with myl_ipc_alloc/myl_ipc_open;
 * myl_session_set_tp with every rank's region base (index = rank), then a host
 * barrier of the ranks. myl_forward's logits are this rank's vocabulary rows
 * [B][v1 - v0]; digests and step logits are world-1 only. */
int myl_model_create_tp(myl_ctx* ctx, const myl_model_spec* spec, int world, int rank,
                        myl_model** out);
/* info[10] = world, rank, q0, q1, kv0, kv1, i0, i1, v0, v1 (this rank's ranges). */
int myl_model_shard(const myl_model* model, int64_t* info);
int64_t myl_session_tp_bytes(const myl_session* s);
int myl_session_set_tp(myl_ctx* ctx, myl_session* s, void* const* bases);
/* Device time (CUDA events on the launching stream) of the session's last
 * prompt pass (myl_forward or the prefill of myl_generate) and decode loop. */
int myl_session_timing(const myl_session* s, float* prefill_ms, float* decode_ms);

/* Building blocks on the device (the reference functions they restate). */
/* rmsnorm_i16 (rmsnorm.rs:61-153) on M rows [M][ldx] -> [M][ldo]; the
 * parameters are host arrays [n]. */
int myl_rmsnorm_i16(myl_ctx* ctx, const int16_t* x, int64_t M, int64_t n, const uint8_t* x_shifts,
                    const int8_t* gamma, const uint8_t* gamma_shifts, const int16_t* rsqrt_lut,
                    int64_t lut_len, uint8_t lut_input_shift, uint8_t lut_output_frac,
                    int64_t inv_n_q20, uint8_t out_frac_bits, int16_t* out);
/* attention_int (attention.rs:42-94), host arrays: q [q_len][head_dim],
 * k/v [kv_len][head_dim], mask [q_len][kv_len] bytes (nonzero: attend; NULL:
 * all), out [q_len][head_dim]. */
int myl_attention_int(myl_ctx* ctx, const int16_t* q, int64_t q_len, const int16_t* k,
                      const int16_t* v, int64_t kv_len, int64_t head_dim, const uint8_t* mask,
                      int64_t score_mult, uint8_t score_shift, const int16_t* exp_lut,
                      int64_t exp_len, uint8_t lut_shift, uint8_t prob_frac_bits, int16_t* out);

/* --- Allocation-free variant ------------------------------------------------------
 * No counterpart in the reference: its CPU path never allocates device memory.
 *
 * For callers that must not have a library allocate device memory: a runtime
 * that reserves its device budget in its own arena at start-up, so that a long
 * job cannot fail half-way on a late allocation, or a loop that cannot afford
 * the device-wide synchronisation of cudaMalloc/cudaFree.
 *
 * myl_linear_noalloc_dev computes the same result as myl_linear_dev with the
 * tensor-core kernel (for every M), but calls no cudaMalloc, cudaFree or other
 * allocating routine: the activation byte planes live in a fixed array of
 * MYL_NOALLOC_SCRATCH_BYTES inside the library's device image, which every
 * GPU that loads the library holds until the process exits.
 *  - Limits: 2 * M * round_up(in_features, 16) <= MYL_NOALLOC_SCRATCH_BYTES
 *    and in_features <= 65536; larger calls fail with MYL_ERR_UNSUPPORTED.
 *  - The first call on a device looks up the array's device address on that
 *    device; make that first call before any stream capture.
 *  - The array is shared by all calls on a device and keeps the last call's
 *    contents; calls whose work overlaps on the GPU (different streams or
 *    host threads) race on it and must be serialised by the caller.
 *  - Every call runs the tensor-core kernel over one K slice with no tail
 *    split, so a small-M call on a narrow weight (e.g. M = 5, N = 2048: 16
 *    tiles) fills few of the SMs and can take several times as long as
 *    myl_linear_dev, which uses the GEMV or splits K for such shapes.
 *  - The array's device address is looked up once per device index and kept:
 *    the entry point assumes the device's primary context (the one the CUDA
 *    runtime uses) for the life of the process, and no cudaDeviceReset. */
#define MYL_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)
int myl_linear_noalloc_dev(myl_ctx* ctx, const myl_weight* w, const myl_requant* rq,
                           const int16_t* x, int64_t M, int64_t ldx, void* y, int64_t ldy,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MYL_W8A16_H */
