// forward.cuh — the kernels of the integer decoder forward around the W8A16
// linears: embedding, residual add + RMSNorm, RoPE with the KV-cache write,
// and integer attention (scores, softmax_int, probability-weighted values).
//
// Every kernel is bit-exact with the reference (INTEGER_LLM/kernels/src and
// runtime/src/model.rs; file:line at each kernel). Shifts, shift spans and
// table sizes are validated on the host before a launch, so the kernels apply
// them without re-checking.
//
// Layouts (one token row per sequence position, sequences one after another):
//   hidden / residual  [rows][H] int16, rows = B * T (sequence-major)
//   qkv                [rows][ldq] int16: q heads, then k heads, then v heads
//   KV cache           [B][L][n_kv][max_pos][head_dim] int16 (k and v apart),
//                      the reference's (layer, head, position) entries
//                      (runtime/src/kv_cache.rs:38-51)
//   scores             [rows * n_q][lds] int32 (one attention row per query head)
#pragma once

#include "common.cuh"
#include "rownorm.cuh"

namespace myl {

// ---- embedding (model.rs:241-248) -------------------------------------------------
// hidden[r][i] = clamp_i16(rescale(embed[tok][i], embed_shift[tok], rin0[i])).
// One block per token row; a token id outside [0, V) zeroes its row and sets
// DEV_BAD_TOKEN (the reference would index out of bounds).
__global__ void embed_kernel(const int32_t* __restrict__ tokens, int64_t rows,
                             const int8_t* __restrict__ embed, int64_t lde,
                             const uint8_t* __restrict__ embed_shifts,
                             const uint8_t* __restrict__ rin0, int64_t H, int64_t V,
                             int16_t* __restrict__ hidden, int64_t ldh, int* err) {
  pdl_wait();
  pdl_launch();
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int32_t tok = tokens[r];
    int16_t* out = hidden + r * ldh;
    if (tok < 0 || int64_t(tok) >= V) {
      for (int64_t i = threadIdx.x; i < H; i += blockDim.x) out[i] = 0;
      if (threadIdx.x == 0) atomicCAS(err, 0, DEV_BAD_TOKEN);
      continue;
    }
    const int8_t* row = embed + int64_t(tok) * lde;
    const int es = int(int8_t(embed_shifts[tok]));
    for (int64_t i = threadIdx.x; i < H; i += blockDim.x)
      out[i] = clamp16(rescale_i32_s(int32_t(row[i]), es - int(int8_t(rin0[i]))));
  }
}

// One block per row; x [rows][ldx]; out [rows][ldo]. out_sel (nullable): only
// rows with out_sel[r] != 0 are normalised (the final norm of the last token).
__global__ void __launch_bounds__(NORM_THREADS)
    resid_rmsnorm_kernel(const int16_t* __restrict__ x, int64_t ldx, int64_t rows, ResidParams rp,
                         NormParams np, int16_t* __restrict__ out, int64_t ldo,
                         const int64_t* __restrict__ out_rows, int64_t n_out_rows) {
  pdl_wait();
  pdl_launch();
  extern __shared__ int16_t s_row[];  // [H]
  __shared__ __int128 s_part[NORM_THREADS / 32];
  __shared__ int64_t s_lut_val;
  __shared__ int s_nf;
  const int64_t H = np.H;
  const int64_t nrows = out_rows ? n_out_rows : rows;
  for (int64_t rr = blockIdx.x; rr < nrows; rr += gridDim.x) {
    const int64_t r = out_rows ? out_rows[rr] : rr;
    const int16_t* xr = x + r * ldx;
    __int128 acc = 0;
    for (int64_t i = threadIdx.x; i < H; i += NORM_THREADS) {
      int64_t v = xr[i];
      if (rp.add) {
        const int64_t h = rescale_i64_signed(v, rp.s1[i]) + int64_t(rp.add[r * rp.ld_add + i]);
        v = clamp16(rescale_i64_signed(h, rp.s2[i]));
        if (rp.resid_out) rp.resid_out[r * rp.ld_res + i] = int16_t(v);
      }
      s_row[i] = int16_t(v);
      acc += (__int128)(v * v) << np.align2[i];
    }
    acc = warp_sum_i128(acc);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      __int128 a = 0;
      for (int w = 0; w < NORM_THREADS / 32; ++w) a += s_part[w];
      if (a == 0) {
        s_nf = -1000;  // all zero: the row is zeros (rmsnorm.rs:99-101)
        s_lut_val = 0;
      } else {
        const __int128 m = (a * (__int128)np.inv_n) >> 20;
        const __int128 max_idx = np.lut_len - 1;
        int q = 0;
        while ((m >> q) > max_idx) q += 2;
        __int128 idx = rne_i128(m, q);
        if (idx > max_idx) idx = max_idx;
        s_lut_val = np.lut[int64_t(idx)];
        s_nf = np.frac0 + q / 2;
      }
    }
    __syncthreads();
    const int nf = s_nf;
    const int64_t lv = s_lut_val;
    int16_t* orow = out + rr * ldo;
    for (int64_t i = threadIdx.x; i < H; i += NORM_THREADS) {
      int16_t y = 0;
      if (nf != -1000) {
        const int64_t prod = int64_t(s_row[i]) * lv * int64_t(np.gamma[i]);  // |prod| < 2^37
        const int sh = nf + np.sbase[i];
        int64_t v;
        if (sh >= 63) v = 0;  // |prod| < 2^37 rounds to zero
        else if (sh > 0) v = rshift_rne_i64(prod, sh);
        else if (sh == 0) v = prod;
        else {
          // i128 left shift (wrapping), then the i32 clamp (rmsnorm.rs:140-151)
          const __int128 w = (__int128)((unsigned __int128)(__int128)prod << (-sh));
          v = w < (__int128)INT32_MIN ? INT32_MIN : (w > (__int128)INT32_MAX ? INT32_MAX : (int64_t)w);
        }
        y = clamp16(v);
      }
      orow[i] = y;
    }
    __syncthreads();
  }
}

// The residual add and RMSNorm for hidden sizes that are a multiple of 8 up
// to 8 * NORM_THREADS * NORM_NV (block_row_norm), one block per row.
__global__ void __launch_bounds__(NORM_THREADS)
    resid_rmsnorm_vec_kernel(const int16_t* __restrict__ x, int64_t ldx, int64_t rows, ResidParams rp,
                             NormParams np, int16_t* __restrict__ out, int64_t ldo,
                             const int64_t* __restrict__ out_rows, int64_t n_out_rows) {
  pdl_wait();
  pdl_launch();
  __shared__ RowNormSmem sm;
  const int64_t nrows = out_rows ? n_out_rows : rows;
  for (int64_t rr = blockIdx.x; rr < nrows; rr += gridDim.x) {
    const int64_t r = out_rows ? out_rows[rr] : rr;
    int16_t* orow = out + rr * ldo;
    block_row_norm(x + r * ldx, r, rp, np, true, sm,
                   [&](int v, const uint4& y) { *reinterpret_cast<uint4*>(orow + 8 * v) = y; });
  }
}

// The same over clusters of NORM_CL CTAs, one row per cluster at a time
// (H % 8 == 0, H <= 8 * NORM_CL * NORM_CL_THREADS). Launched with the cluster
// dimension NORM_CL; grid.x is a multiple of NORM_CL.
__global__ void __launch_bounds__(NORM_CL_THREADS)
    resid_rmsnorm_cluster_kernel(const int16_t* __restrict__ x, int64_t ldx, int64_t rows, ResidParams rp,
                                 NormParams np, int16_t* __restrict__ out, int64_t ldo,
                                 const int64_t* __restrict__ out_rows, int64_t n_out_rows) {
  pdl_wait();
  pdl_launch();
  __shared__ __int128 s_part[NORM_CL_THREADS / 32];
  // the cluster's CTA sums of a row, pushed here by every CTA (slot = its
  // rank, lo and hi words); two sets by row parity, so that a CTA writing the
  // next row's sum cannot overwrite one still being read (the cluster barrier
  // of every row keeps the CTAs at most one row apart)
  __shared__ __align__(16) unsigned long long s_slot[2][NORM_CL][2];
  __shared__ int64_t s_lv;
  __shared__ int s_nf;
  const int rank = int(cluster_ctarank());
  const int nv = int(np.H / 8);
  const int vpc = (nv + NORM_CL - 1) / NORM_CL;  // vectors per CTA
  const int v = rank * vpc + int(threadIdx.x);
  const bool active = int(threadIdx.x) < vpc && v < nv;
  const bool radd = rp.add || rp.parts;
  const int64_t nrows = out_rows ? n_out_rows : rows;
  int par = 0;
  for (int64_t rr = cluster_id_x(); rr < nrows; rr += cluster_count_x(), par ^= 1) {
    const int64_t r = out_rows ? out_rows[rr] : rr;
    NormVec vec;
    int64_t acc64 = 0;
    __int128 acc128 = 0;
    if (active) {
      norm_vec_load(vec, x + r * ldx, r, v, rp, np);
      norm_vec_resid(vec, radd, acc64, acc128);
      if (radd && rp.resid_out) *reinterpret_cast<uint4*>(rp.resid_out + r * rp.ld_res + 8 * v) = vec.x;
    }
    const __int128 acc = warp_sum_i128((__int128)acc64 + acc128);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < NORM_CL) {  // thread k pushes this CTA's sum into CTA k
      __int128 a = 0;
      for (int w = 0; w < NORM_CL_THREADS / 32; ++w) a += s_part[w];
      const uint32_t remote =
          mapa_shared(static_cast<uint32_t>(__cvta_generic_to_shared(&s_slot[par][rank][0])), threadIdx.x);
      st_shared_cluster_u64(remote, (unsigned long long)a);
      st_shared_cluster_u64(remote + 8, (unsigned long long)(a >> 64));
    }
    cluster_sync_all();  // every CTA's sum has landed in every CTA (release / acquire)
    if (threadIdx.x == 0) {
      __int128 a = 0;
      for (int k = 0; k < NORM_CL; ++k)
        a += (__int128)(((unsigned __int128)s_slot[par][k][1] << 64) | (unsigned __int128)s_slot[par][k][0]);
      int64_t lv;
      int nf;
      norm_scale(a, np, &lv, &nf);
      s_lv = lv;
      s_nf = nf;
    }
    __syncthreads();  // s_lv and s_nf
    if (active) *reinterpret_cast<uint4*>(out + rr * ldo + 8 * v) = norm_vec_out(vec, s_lv, s_nf);
  }
}

// ---- RoPE + KV-cache write (model.rs:469-503, rope.rs:17-32) ----------------------
// Row r = b * T + t is token t of sequence b at position pos = pos0 + t; it
// uses LUT row pos % n_pos. Pair j of a head is (x_j, x_{j+half}):
//   x_j' = clamp_i16(rne(x_j cos - x_{j+half} sin, frac)),
//   x_{j+half}' = clamp_i16(rne(x_{j+half} cos + x_j sin, frac))   (i32, wrapping).
// Query heads are rotated in place; rotated keys and the values go to the
// cache of layer `layer` at position pos.
struct KvCache {
  int16_t* k;
  int16_t* v;
  int64_t seq_stride;   // elements between sequences: L * n_kv * max_pos * hd
  int64_t layer_stride; // n_kv * max_pos * hd
  int64_t head_stride;  // max_pos * hd
};

__device__ __forceinline__ int16_t rope_out(int32_t a, int frac) {
  return clamp16(frac > 0 ? rshift_rne_i32(a, frac) : a);
}

__global__ void rope_kv_kernel(int16_t* __restrict__ qkv, int64_t ldq, int64_t rows, int64_t T,
                               const int64_t* __restrict__ pos0_dev, int nq, int nkv, int hd,
                               const int16_t* __restrict__ cos_l, const int16_t* __restrict__ sin_l,
                               int64_t n_pos, int frac, KvCache kc, int layer) {
  pdl_wait();
  pdl_launch();
  // grid.x: row; grid.y * blockDim.x covers one item per thread: the rotation
  // pairs of the q and k heads, then the values (8 per item when hd % 8 == 0)
  const int half = hd / 2;
  const int n_rot = (nq + nkv) * half;
  const bool vec = (hd & 7) == 0;
  const int n_v = vec ? nkv * hd / 8 : nkv * hd;
  const int e = int(blockIdx.y) * blockDim.x + threadIdx.x;
  if (e >= n_rot + n_v) return;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t b = r / T, t = r % T;
    const int64_t pos = pos0_dev[0] + t;
    int16_t* row = qkv + r * ldq;
    const int64_t cache_off = b * kc.seq_stride + int64_t(layer) * kc.layer_stride + pos * hd;
    if (e < n_rot) {
      const int h = e / half, j = e % half;
      const int64_t idx = pos % n_pos;
      int16_t* v = row + int64_t(h) * hd;  // q heads, then k heads (contiguous in qkv)
      const uint32_t cj = uint32_t(int32_t(cos_l[idx * half + j]));
      const uint32_t sj = uint32_t(int32_t(sin_l[idx * half + j]));
      const uint32_t x0 = uint32_t(int32_t(v[j])), x1 = uint32_t(int32_t(v[j + half]));
      const int16_t o0 = rope_out(int32_t(x0 * cj - x1 * sj), frac);
      const int16_t o1 = rope_out(int32_t(x1 * cj + x0 * sj), frac);
      if (h < nq) {
        v[j] = o0;
        v[j + half] = o1;
      } else {
        int16_t* kd = kc.k + cache_off + int64_t(h - nq) * kc.head_stride;
        kd[j] = o0;
        kd[j + half] = o1;
      }
    } else {
      const int i = e - n_rot;
      const int16_t* vrow = row + int64_t(nq + nkv) * hd;
      if (vec) {
        const int h = (8 * i) / hd, d = (8 * i) % hd;
        *reinterpret_cast<uint4*>(kc.v + cache_off + int64_t(h) * kc.head_stride + d) =
            *reinterpret_cast<const uint4*>(vrow + 8 * i);
      } else {
        const int h = i / hd, d = i % hd;
        kc.v[cache_off + int64_t(h) * kc.head_stride + d] = vrow[i];
      }
    }
  }
}

// ---- attention (attention.rs:42-94, model.rs:508-567) -----------------------------
// Query row (b, t, h) attends the cache entries 0..=pos of KV head h / group.
// Pass 1 (attn_scores_kernel): scores[row][j] = rne_i64(dot(q, k_j) * mult, shift) as i32,
//   and the row maximum (softmax.rs:27) by an atomic max per warp into rowmax.
//   The int16 x int16 dot is exact in two int32 sums: k = 256 kh + kl with kh
//   the signed high byte and kl the unsigned low byte, so
//   dot = 256 * sum q*kh + sum q*kl, |sum q*kh| <= hd * 2^22 and
//   sum q*kl <= hd * 2^23 (both exact in int32 for hd <= 255); each sum is a
//   chain of dp2a (two int16 x int8 products per instruction).
// Pass 2 (attn_pv_*_kernel): softmax_int over the row (softmax.rs:24-64: max,
//   exp LUT of the saturating difference, i32 sum, round-half-even division),
//   then sum_j p_j * v_j in int64 over a chunk of keys; the chunks of a row are
//   added (exact) by the last of its blocks, rounded by prob_frac and clamped
//   (attention.rs:83-90), then rescaled from the V scale to the o_proj input
//   scale (model.rs:563-567). The last block of a row sets its rowmax word back
//   to the empty value for the next call.
struct AttnParams {
  const int16_t* qkv;      // [rows][ldq]
  int64_t ldq;
  int64_t T;               // tokens per sequence in this call
  int64_t rows;            // B * T
  const int64_t* pos0;     // device: position of token 0 of the call
  int nq, nkv, hd;          // this rank's query and KV heads
  int q_head0, kv_head0, G;  // global index of local head 0 / KV head 0, global group size
  KvCache kc;
  int layer;
  int64_t score_mult;
  int score_shift;         // [0, 62]
  int32_t* scores;         // [rows * nq][lds]
  int64_t lds;
  const uint8_t* mask;     // op form only: [rows][kv] bytes (0 = masked), else null
  // row maxima [rows * nq] as max_j (score ^ 0x80000000) over unsigned words:
  // zero (= INT32_MIN) between calls
  unsigned* rowmax;
  // pass 1 with the decode RoPE (T == 1): LUT rows [n_pos][hd / 2], frac bits
  int rope;
  const int16_t* rope_cos;
  const int16_t* rope_sin;
  int64_t n_pos;
  int rope_frac;
  // pass 2
  const int16_t* exp_lut;
  int32_t exp_len;
  int lut_shift;
  int prob_frac;           // [0, 30]
  int out_shift;           // v_frac - attn_out_frac in [-31, 30] (0: no rescale)
  int64_t* part;           // [rows * nq][max_chunks][hd]
  int max_chunks;
  unsigned* counters;      // [rows * nq], zero between calls
  int16_t* out;            // [rows][ldo]: head h at columns h * hd
  int64_t ldo;
};

constexpr int ATT_THREADS = 256;
constexpr int ATT_TPK = 8;                          // pass 1: threads per key
constexpr int ATT_SKEYS = ATT_THREADS / ATT_TPK;    // pass 1: keys per block
constexpr int ATT_MAXG = 8;                         // pass 1: query heads per block (= ATT_TPK)
constexpr int ATT_KCH = 4;                          // pass 1: 8-element chunks per thread (hd <= 256)
constexpr int ATT_CHUNK = 256;                      // pass 2 (many rows): keys per piece
constexpr int ATT_DTHREADS = 512;                   // pass 2 (decode): threads per block
constexpr int ATT_DCHUNK = 512;                     // pass 2 (decode): keys per block
constexpr int ATT_TQ = 64;                          // prefill tiles: query rows per block
constexpr int ATT_TK = 64;                          // prefill tiles: keys per tile
static_assert(ATT_MAXG == ATT_TPK, "one query head per thread of a key after the reduce-scatter");

__device__ __forceinline__ int dp2a_lo_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_lo_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__host__ __device__ constexpr int att_hd8(int hd) { return (hd + 7) & ~7; }
// pass 1 dynamic shared memory: the queries [ATT_MAXG][hd8] and the rotated
// new key [hd8], int16
__host__ __device__ constexpr size_t att_scores_smem(int hd) {
  return size_t((ATT_MAXG + 1) * att_hd8(hd) * 2);
}

// RoPE of one pair (rope.rs:17-32): (x0, x1) -> (x0 c - x1 s, x1 c + x0 s),
// i32 wrapping, round-half-even by frac, clamped to i16.
__device__ __forceinline__ void rope_pair(int16_t a, int16_t b, int16_t c, int16_t s, int frac, int16_t* o0,
                                          int16_t* o1) {
  const uint32_t x0 = uint32_t(int32_t(a)), x1 = uint32_t(int32_t(b));
  const uint32_t cj = uint32_t(int32_t(c)), sj = uint32_t(int32_t(s));
  *o0 = rope_out(int32_t(x0 * cj - x1 * sj), frac);
  *o1 = rope_out(int32_t(x1 * cj + x0 * sj), frac);
}

// The int32 sums of ATT_MAXG heads over the ATT_TPK = 8 threads of a key,
// reduce-scattered: afterwards thread `part` holds the full sum of head `part`.
__device__ __forceinline__ int att_reduce_scatter8(const int (&a)[ATT_MAXG], int part) {
  const bool b2 = part & 4, b1 = part & 2, b0 = part & 1;
  int k4[4], k2[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int keep = b2 ? a[4 + i] : a[i], send = b2 ? a[i] : a[4 + i];
    k4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int keep = b1 ? k4[2 + i] : k4[i], send = b1 ? k4[i] : k4[2 + i];
    k2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  const int keep = b0 ? k2[1] : k2[0], send = b0 ? k2[0] : k2[1];
  return keep + __shfl_xor_sync(0xffffffffu, send, 1);
}

// grid.x: (row group) = ((b * T + t) * nkv + g) * gsub + sub; grid.y: key block of
// ATT_SKEYS keys; sub-groups of ATT_MAXG query heads of the KV head g.
// Thread (key jj, part s) holds the 8-element chunks s, s + 8, ... of key row
// jj in registers as two byte planes, issued before its first product; the
// parts' int32 sums are reduce-scattered so that part s finishes head s.
// With p.rope (decode, T == 1) the RoPE of the row's queries and new key is
// done here (model.rs:469-503): the queries are rotated while staged, the
// block holding key pos rotates the new key into shared memory instead of
// reading the cache, and sub-group 0 of that block writes the key and the
// value row to the cache at pos.
__global__ void __launch_bounds__(ATT_THREADS) attn_scores_kernel(AttnParams p, int gsub) {
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(16) int16_t s_q16[];  // [ATT_MAXG][hd8] queries, then [hd8] new key
  __shared__ int32_t s_mx[ATT_THREADS / 32][ATT_MAXG];
  const int hd = p.hd, hd8 = att_hd8(hd), nc8 = hd8 / 8, half = hd / 2;
  const int gy = int(blockIdx.x);
  const int sub = gy % gsub;
  const int g = (gy / gsub) % p.nkv;
  const int r = gy / gsub / p.nkv;  // token row b * T + t
  const int T = int(p.T);
  const int b = r / T, t = r % T;
  const int64_t pos = p.pos0[0] + t;
  const int64_t len = p.mask ? p.lds : pos + 1;
  const int64_t j0 = int64_t(blockIdx.y) * ATT_SKEYS;
  if (j0 >= len) return;
  // local query heads of KV head g (GQA: global head q reads KV head q / G)
  const int hs = max(0, (p.kv_head0 + g) * p.G - p.q_head0);
  const int he = min(p.nq, (p.kv_head0 + g + 1) * p.G - p.q_head0);
  const int h0 = hs + sub * ATT_MAXG;
  const int nrow = min(ATT_MAXG, he - h0);
  if (nrow <= 0) return;
  const int jj = int(threadIdx.x) / ATT_TPK, part = int(threadIdx.x) % ATT_TPK;
  const int64_t j = j0 + jj;
  const bool live = j < len;
  const bool newkey = p.rope && j == pos;  // rotated in shared memory below
  const int64_t cache_off = int64_t(b) * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                            int64_t(g) * p.kc.head_stride;
  const int16_t* kr = p.kc.k + cache_off + (live ? j : j0) * hd;
  const bool vec = (hd & 7) == 0;
  uint4 kv[ATT_KCH];
#pragma unroll
  for (int i = 0; i < ATT_KCH; ++i) {
    const int w8 = part + ATT_TPK * i;
    kv[i] = make_uint4(0u, 0u, 0u, 0u);
    if (live && !newkey && w8 < nc8) {
      if (vec) {
        kv[i] = *reinterpret_cast<const uint4*>(kr + 8 * w8);
      } else {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        for (int e = 0; e < 8 && 8 * w8 + e < hd; ++e)
          w[e / 2] |= uint32_t(uint16_t(kr[8 * w8 + e])) << (16 * (e & 1));
        kv[i] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  // queries of the sub-group (rotated with p.rope), zero-padded to hd8
  const int16_t* qrow = p.qkv + int64_t(r) * p.ldq;
  int16_t* s_k16 = s_q16 + ATT_MAXG * hd8;
  if (p.rope) {
    const int64_t lrow = (pos % p.n_pos) * half;
    for (int e = threadIdx.x; e < nrow * half; e += ATT_THREADS) {
      const int rr = e / half, d = e % half;
      const int16_t* q = qrow + int64_t(h0 + rr) * hd;
      rope_pair(q[d], q[d + half], p.rope_cos[lrow + d], p.rope_sin[lrow + d], p.rope_frac,
                s_q16 + rr * hd8 + d, s_q16 + rr * hd8 + d + half);
    }
    if (j0 <= pos && pos < j0 + ATT_SKEYS) {
      // the new key of KV head g, and (sub-group 0) key and value to the cache
      const int16_t* k = qrow + int64_t(p.nq + g) * hd;
      int16_t* kc = p.kc.k + cache_off + pos * hd;
      for (int d = threadIdx.x; d < half; d += ATT_THREADS) {
        int16_t o0, o1;
        rope_pair(k[d], k[d + half], p.rope_cos[lrow + d], p.rope_sin[lrow + d], p.rope_frac, &o0, &o1);
        s_k16[d] = o0;
        s_k16[d + half] = o1;
        if (sub == 0) {
          kc[d] = o0;
          kc[d + half] = o1;
        }
      }
      for (int d = hd + threadIdx.x; d < hd8; d += ATT_THREADS) s_k16[d] = 0;
      if (sub == 0) {
        const int16_t* v = qrow + int64_t(p.nq + p.nkv + g) * hd;
        int16_t* vc = p.kc.v + cache_off + pos * hd;
        for (int d = threadIdx.x; d < hd; d += ATT_THREADS) vc[d] = v[d];
      }
    }
    for (int e = threadIdx.x; e < nrow * (hd8 - hd); e += ATT_THREADS)
      s_q16[(e / (hd8 - hd)) * hd8 + hd + e % (hd8 - hd)] = 0;
  } else {
    for (int e = threadIdx.x; e < nrow * hd8; e += ATT_THREADS) {
      const int rr = e / hd8, d = e % hd8;
      s_q16[rr * hd8 + d] = d < hd ? qrow[int64_t(h0 + rr) * hd + d] : int16_t(0);
    }
  }
  __syncthreads();
  if (newkey) {
#pragma unroll
    for (int i = 0; i < ATT_KCH; ++i) {
      const int w8 = part + ATT_TPK * i;
      if (w8 < nc8) kv[i] = *reinterpret_cast<const uint4*>(s_k16 + 8 * w8);
    }
  }
  const uint32_t* s_q = reinterpret_cast<const uint32_t*>(s_q16);
  const int qw = hd8 / 2;
  int acc_h[ATT_MAXG], acc_l[ATT_MAXG];
#pragma unroll
  for (int i = 0; i < ATT_MAXG; ++i) acc_h[i] = acc_l[i] = 0;
#pragma unroll
  for (int i = 0; i < ATT_KCH; ++i) {
    const int w8 = part + ATT_TPK * i;
    if (w8 < nc8) {
      const uint32_t khx = __byte_perm(kv[i].x, kv[i].y, 0x7531), khy = __byte_perm(kv[i].z, kv[i].w, 0x7531);
      const uint32_t klx = __byte_perm(kv[i].x, kv[i].y, 0x6420), kly = __byte_perm(kv[i].z, kv[i].w, 0x6420);
#pragma unroll
      for (int h = 0; h < ATT_MAXG; ++h) {
        if (h < nrow) {
          const uint4 q = *reinterpret_cast<const uint4*>(s_q + h * qw + 4 * w8);
          acc_h[h] = dp2a_hi_ss(q.y, khx, dp2a_lo_ss(q.x, khx, acc_h[h]));
          acc_h[h] = dp2a_hi_ss(q.w, khy, dp2a_lo_ss(q.z, khy, acc_h[h]));
          acc_l[h] = dp2a_hi_su(q.y, klx, dp2a_lo_su(q.x, klx, acc_l[h]));
          acc_l[h] = dp2a_hi_su(q.w, kly, dp2a_lo_su(q.z, kly, acc_l[h]));
        }
      }
    }
  }
  const int ah = att_reduce_scatter8(acc_h, part), al = att_reduce_scatter8(acc_l, part);
  // this thread: head h0 + part of key j
  int32_t sc = INT32_MIN;
  const bool mine = live && part < nrow;
  const int64_t row = int64_t(r) * p.nq + h0 + part;
  if (mine && !(p.mask && !p.mask[int64_t(r) * p.lds + j])) {
    const int64_t dot = int64_t(ah) * 256 + int64_t(al);
    const uint64_t prod = uint64_t(dot) * uint64_t(p.score_mult);  // i64 (wrapping)
    const int64_t s = p.score_shift > 0 ? rshift_rne_i64(int64_t(prod), p.score_shift) : int64_t(prod);
    sc = int32_t(uint32_t(uint64_t(s)));  // `as i32`
  }
  if (mine) p.scores[row * p.lds + j] = sc;
  // the block's maximum per head, one atomic per head and block
  int32_t mx = sc;
#pragma unroll
  for (int o = ATT_TPK; o < 32; o <<= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane < ATT_TPK) s_mx[warp][lane] = mx;
  __syncthreads();
  if (int(threadIdx.x) < nrow) {
    int32_t m = s_mx[0][threadIdx.x];
#pragma unroll
    for (int w = 1; w < ATT_THREADS / 32; ++w) m = max(m, s_mx[w][threadIdx.x]);
    atomicMax(p.rowmax + int64_t(r) * p.nq + h0 + threadIdx.x, uint32_t(m) ^ 0x80000000u);
  }
}

// m16n8k32 integer MMA with the signedness of A and B as template flags.
template <bool AS, bool BS>
__device__ __forceinline__ void mma_i8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  if constexpr (AS && BS)
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else if constexpr (AS && !BS)
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else if constexpr (!AS && BS)
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Pass 1 for many rows (prefill) on the integer MMA path, head_dim 64 or 128:
// block (64 consecutive query rows of one sequence, one query head) walks the
// keys 0..pos in tiles of 64. q = 256 qh + ql and k = 256 kh + kl with the high
// bytes signed and the low bytes unsigned, so
//   dot = 65536 sum qh*kh + 256 (sum qh*kl + sum ql*kh) + sum ql*kl
// from four m16n8k32 MMAs (s8.s8, s8.u8, u8.s8, u8.u8) whose int32 sums are
// exact (|each| <= 255 * 128 * 128 < 2^23). The query planes are staged once,
// the key tile's planes per tile (keys [key][dim] are already the B operand's
// column layout); rows padded to HD + 16 bytes so fragment loads hit distinct
// banks. Warp task = 16 rows x 32 keys; each score is rescaled as in
// attn_scores_kernel and stored for keys <= pos; the row maximum is kept in
// registers over all tiles and written once (this block alone owns the row).
template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_scores_mma_kernel(AttnParams p) {
  pdl_wait();
  pdl_launch();
  static_assert(HD == 64 || HD == 128, "head_dim");
  constexpr int RS = HD + 16;  // padded plane row, bytes
  __shared__ __align__(16) uint8_t s_qh[ATT_TQ][RS], s_ql[ATT_TQ][RS];
  __shared__ __align__(16) uint8_t s_kh[ATT_TK][RS], s_kl[ATT_TK][RS];
  __shared__ int32_t s_mx[2][ATT_TQ];
  const int T = int(p.T);
  const int tiles_per_seq = (T + ATT_TQ - 1) / ATT_TQ;
  const int b = int(blockIdx.x) / tiles_per_seq, t0 = (int(blockIdx.x) % tiles_per_seq) * ATT_TQ;
  const int h = int(blockIdx.y);
  const int nrows = min(ATT_TQ, T - t0);
  const int64_t pos0 = p.pos0[0];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int16_t* kbase = p.kc.k + int64_t(b) * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t((p.q_head0 + h) / p.G - p.kv_head0) * p.kc.head_stride;
  constexpr int DG = HD / 8;  // 16-byte (8-element) vectors per row
  // query planes: 64 rows x DG vectors
  for (int e = threadIdx.x; e < ATT_TQ * DG; e += ATT_THREADS) {
    const int i = e / DG, d8 = e % DG;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (i < nrows) v = *reinterpret_cast<const uint4*>(p.qkv + (int64_t(b) * T + t0 + i) * p.ldq + int64_t(h) * HD + 8 * d8);
    *reinterpret_cast<uint2*>(&s_qh[i][8 * d8]) = make_uint2(__byte_perm(v.x, v.y, 0x7531), __byte_perm(v.z, v.w, 0x7531));
    *reinterpret_cast<uint2*>(&s_ql[i][8 * d8]) = make_uint2(__byte_perm(v.x, v.y, 0x6420), __byte_perm(v.z, v.w, 0x6420));
  }
  // warp task: rows r0..r0+15, keys k0..k0+31 of each tile
  const int r0 = (warp % 4) * 16, kq0 = (warp / 4) * 32;
  const int64_t lenA = r0 + g < nrows ? pos0 + t0 + r0 + g + 1 : 0;  // keys of row r0 + g
  const int64_t lenB = r0 + g + 8 < nrows ? pos0 + t0 + r0 + g + 9 : 0;
  int32_t mxA = INT32_MIN, mxB = INT32_MIN;
  const int64_t kend = pos0 + t0 + nrows;  // the longest row of the block
  for (int64_t j0 = 0; j0 < kend; j0 += ATT_TK) {
    const int nk = int(min(int64_t(ATT_TK), kend - j0));
    __syncthreads();  // the previous key tile is consumed (and the query planes are written)
    {
      constexpr int KIT = ATT_TK * DG / ATT_THREADS;
      uint4 kv[KIT];
#pragma unroll
      for (int q = 0; q < KIT; ++q) {
        const int e = threadIdx.x + q * ATT_THREADS, jj = e / DG, d8 = e % DG;
        kv[q] = jj < nk ? *reinterpret_cast<const uint4*>(kbase + (j0 + jj) * HD + 8 * d8) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int q = 0; q < KIT; ++q) {
        const int e = threadIdx.x + q * ATT_THREADS, jj = e / DG, d8 = e % DG;
        *reinterpret_cast<uint2*>(&s_kh[jj][8 * d8]) =
            make_uint2(__byte_perm(kv[q].x, kv[q].y, 0x7531), __byte_perm(kv[q].z, kv[q].w, 0x7531));
        *reinterpret_cast<uint2*>(&s_kl[jj][8 * d8]) =
            make_uint2(__byte_perm(kv[q].x, kv[q].y, 0x6420), __byte_perm(kv[q].z, kv[q].w, 0x6420));
      }
    }
    __syncthreads();
    int hh[4][4], x[4][4], ll[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) hh[n][i] = x[n][i] = ll[n][i] = 0;
#pragma unroll
    for (int ks = 0; ks < HD / 32; ++ks) {
      const int d = 32 * ks + 4 * c;
      const uint32_t ah0 = *reinterpret_cast<const uint32_t*>(&s_qh[r0 + g][d]);
      const uint32_t ah1 = *reinterpret_cast<const uint32_t*>(&s_qh[r0 + g + 8][d]);
      const uint32_t ah2 = *reinterpret_cast<const uint32_t*>(&s_qh[r0 + g][d + 16]);
      const uint32_t ah3 = *reinterpret_cast<const uint32_t*>(&s_qh[r0 + g + 8][d + 16]);
      const uint32_t al0 = *reinterpret_cast<const uint32_t*>(&s_ql[r0 + g][d]);
      const uint32_t al1 = *reinterpret_cast<const uint32_t*>(&s_ql[r0 + g + 8][d]);
      const uint32_t al2 = *reinterpret_cast<const uint32_t*>(&s_ql[r0 + g][d + 16]);
      const uint32_t al3 = *reinterpret_cast<const uint32_t*>(&s_ql[r0 + g + 8][d + 16]);
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int kn = kq0 + 8 * n + g;
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&s_kh[kn][d]);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&s_kh[kn][d + 16]);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&s_kl[kn][d]);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&s_kl[kn][d + 16]);
        mma_i8_16832<true, true>(hh[n], ah0, ah1, ah2, ah3, bh0, bh1);
        mma_i8_16832<true, false>(x[n], ah0, ah1, ah2, ah3, bl0, bl1);
        mma_i8_16832<false, true>(x[n], al0, al1, al2, al3, bh0, bh1);
        mma_i8_16832<false, false>(ll[n], al0, al1, al2, al3, bl0, bl1);
      }
    }
    // scores of rows r0 + g (i = 0, 1) and r0 + g + 8 (i = 2, 3), keys kq0 + 8n + 2c + (i & 1)
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      int32_t sc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t dot = 65536 * int64_t(hh[n][i]) + 256 * int64_t(x[n][i]) + int64_t(ll[n][i]);
        const uint64_t prod = uint64_t(dot) * uint64_t(p.score_mult);  // i64 (wrapping)
        const int64_t v = p.score_shift > 0 ? rshift_rne_i64(int64_t(prod), p.score_shift) : int64_t(prod);
        sc[i] = int32_t(uint32_t(uint64_t(v)));  // `as i32`
      }
      const int64_t j = j0 + kq0 + 8 * n + 2 * c;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int64_t len = half ? lenB : lenA;
        const int r = r0 + g + 8 * half;
        if (j >= len) continue;
        int32_t* dst = p.scores + ((int64_t(b) * T + t0 + r) * p.nq + h) * p.lds + j;
        int32_t& mx = half ? mxB : mxA;
        mx = max(mx, sc[2 * half]);
        if (j + 1 < len) {
          mx = max(mx, sc[2 * half + 1]);
          if ((p.lds & 1) == 0) {
            *reinterpret_cast<int2*>(dst) = make_int2(sc[2 * half], sc[2 * half + 1]);  // 8-byte aligned
          } else {
            dst[0] = sc[2 * half];
            dst[1] = sc[2 * half + 1];
          }
        } else {
          dst[0] = sc[2 * half];
        }
      }
    }
  }
  // row maxima: the 4 lanes of a row, then the two warps of a row group
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    mxA = max(mxA, __shfl_xor_sync(0xffffffffu, mxA, o));
    mxB = max(mxB, __shfl_xor_sync(0xffffffffu, mxB, o));
  }
  if (c == 0) {
    s_mx[warp / 4][r0 + g] = mxA;
    s_mx[warp / 4][r0 + g + 8] = mxB;
  }
  __syncthreads();
  if (threadIdx.x < nrows) {
    const int32_t m = max(s_mx[0][threadIdx.x], s_mx[1][threadIdx.x]);
    p.rowmax[(int64_t(b) * T + t0 + threadIdx.x) * p.nq + h] = uint32_t(m) ^ 0x80000000u;
  }
}

__device__ __forceinline__ int32_t exp_lookup(int32_t x, const int16_t* lut, int32_t len, int shift,
                                              int32_t one) {
  if (x <= 0) return one;
  const uint32_t idx = uint32_t(x) >> shift;
  if (idx >= uint32_t(len)) return 0;
  return lut[idx];
}

// exp LUT entry of the saturating difference max - s (softmax.rs:33-38)
// (m >= s: m is the row maximum, so the u32 difference is exact)
__device__ __forceinline__ int32_t exp_of(int32_t m, int32_t s, const AttnParams& p, int32_t lut_one) {
  const uint32_t d = min(uint32_t(m) - uint32_t(s), uint32_t(INT32_MAX));
  return exp_lookup(int32_t(d), p.exp_lut, p.exp_len, p.lut_shift, lut_one);
}

// softmax.rs:41-62: the probability of exponential e in a row of `len` keys
// with exponential sum S (key index j for the uniform row of an all-zero sum).
__device__ __forceinline__ int32_t softmax_prob(int32_t e, int32_t S, int64_t j, int64_t len, int32_t one) {
  if (S == 0) {
    const int32_t base = one / int32_t(len), rem = one - base * int32_t(len);
    return base + (j < rem ? 1 : 0);
  }
  const int32_t num = e * one;
  int32_t q = num / S;
  const int32_t rm = num % S;
  const int32_t twice = (rm < 0 ? -rm : rm) * 2, den = S < 0 ? -S : S;
  if (twice > den || (twice == den && (q & 1))) q = ((num > 0) == (S > 0)) ? q + 1 : q - 1;
  return q;
}

// softmax_prob for a positive sum S and a non-negative exponential e with the
// division by S done as a multiplication: with R = ceil(2^63 / S) (one
// division per row), floor(num / S) = floor(2 num R / 2^64) exactly for
// num = e * one < 2^31 and S < 2^31 (the error of R, num / 2^63, stays below
// 1 / S because num * S < 2^62); then the same round-half-even step.
__device__ __forceinline__ uint64_t softmax_recip(int32_t S) {
  return S > 0 ? ((uint64_t(1) << 63) + uint64_t(S) - 1) / uint64_t(S) : 0;
}
__device__ __forceinline__ int32_t softmax_prob_r(int32_t e, int32_t S, uint64_t R, int64_t j, int64_t len,
                                                  int32_t one) {
  if (S <= 0 || e < 0) return softmax_prob(e, S, j, len, one);
  const uint32_t num = uint32_t(e) * uint32_t(one);
  uint32_t q = uint32_t(__umul64hi(uint64_t(num) << 1, R));
  const uint32_t twice = 2 * (num - q * uint32_t(S));  // 2r < 2S < 2^32
  if (twice > uint32_t(S) || (twice == uint32_t(S) && (q & 1))) ++q;
  return int32_t(q);
}

// The sum of the exponentials of a row of `len` scores with maximum m, loads
// issued eight deep; the exponentials of keys [e0, e0 + ne) also go to s_e.
// Ends with the block synchronised (s_e complete). NT: threads of the block.
template <int NT>
__device__ __forceinline__ int32_t attn_row_sum(const int32_t* __restrict__ sc, int64_t len, int32_t m,
                                                const AttnParams& p, int32_t lut_one, int64_t* s_red,
                                                int32_t* s_e, int64_t e0, int ne) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = int(len);  // rows are shorter than 2^31 keys
  const int f0 = int(e0);
  int64_t s = 0;
  for (int j = threadIdx.x; j < n; j += 8 * NT) {
    int32_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int jj = j + u * NT;
      v[u] = jj < n ? sc[jj] : m;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int jj = j + u * NT;
      if (jj < n) {
        const int32_t e = exp_of(m, v[u], p, lut_one);
        s += e;
        if (unsigned(jj - f0) < unsigned(ne)) s_e[jj - f0] = e;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) s_red[warp] = s;
  __syncthreads();
  s = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) s += s_red[w];
  return int32_t(s);  // i32 in the reference; the host bounds len so that it cannot overflow
}

// The chunk combination of pass 2: block c of a row with nch chunks holds
// `tot` (column d < hd). With one chunk it is the row's sum; otherwise the
// partials go to p.part and the last block of the row adds them. That block
// writes the output columns and resets the row's counter and rowmax words.
__device__ __forceinline__ void attn_finish(const AttnParams& p, int64_t row, int64_t c, int64_t nch,
                                            int64_t tot, bool* s_last) {
  const int hd = p.hd;
  const int d = threadIdx.x;
  int64_t* part = p.part + (row * p.max_chunks) * hd;
  if (nch > 1) {
    if (d < hd) part[c * hd + d] = tot;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(p.counters + row, 1u);
      *s_last = (prev + 1 == unsigned(nch));
    }
    __syncthreads();
    if (!*s_last) return;
    __threadfence();
    if (d < hd) {
      int64_t a[4] = {0, 0, 0, 0};
      int64_t cc = 0;
      for (; cc + 4 <= nch; cc += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) a[u] += __ldcg(part + (cc + u) * hd + d);
      }
      for (; cc < nch; ++cc) a[0] += __ldcg(part + cc * hd + d);
      tot = a[0] + a[1] + a[2] + a[3];
    }
  }
  const int64_t r = row / p.nq;
  const int h = int(row % p.nq);
  if (d < hd) {
    int32_t o = clamp16(p.prob_frac > 0 ? rshift_rne_i64(tot, p.prob_frac) : tot);
    if (p.out_shift != 0) o = clamp16(rescale_i32_s(o, p.out_shift));
    p.out[r * p.ldo + int64_t(h) * hd + d] = int16_t(o);
  }
  if (threadIdx.x == 0) {
    if (nch > 1) p.counters[row] = 0;
    p.rowmax[row] = 0u;
  }
}

// grid.x: query row (b * T + t) * nq + h; grid.y: key chunk of `chunk` keys
// (a multiple of ATT_CHUNK). Any head_dim <= 254.
__global__ void __launch_bounds__(ATT_THREADS) attn_pv_kernel(AttnParams p, int64_t chunk) {
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(16) int64_t s_acc[];  // [ATT_THREADS / 32][hd]
  __shared__ int64_t s_red[ATT_THREADS / 32];
  __shared__ int32_t s_p[ATT_CHUNK];
  __shared__ bool s_last;
  const int64_t row = blockIdx.x;
  const int64_t r = row / p.nq;
  const int h = int(row % p.nq);
  const int64_t b = r / p.T, t = r % p.T;
  const int64_t pos = p.pos0[0] + t;
  const int64_t len = p.mask ? p.lds : pos + 1;
  const int64_t nch = (len + chunk - 1) / chunk;
  const int64_t c = blockIdx.y;
  if (c >= nch) return;
  const int32_t* sc = p.scores + row * p.lds;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int32_t m = int32_t(p.rowmax[row] ^ 0x80000000u);
  const int32_t lut_one = p.exp_lut[0];
  const int32_t S = attn_row_sum<ATT_THREADS>(sc, len, m, p, lut_one, s_red, s_p, 0, 0);
  const int32_t one = int32_t(1) << p.prob_frac;
  const int hd = p.hd;
  const int16_t* vbase = p.kc.v + b * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t((p.q_head0 + h) / p.G - p.kv_head0) * p.kc.head_stride;
  int64_t acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0;
  const int64_t jend = min(len, (c + 1) * chunk);
  for (int64_t jc0 = c * chunk; jc0 < jend; jc0 += ATT_CHUNK) {
    const int nj = int(min(int64_t(ATT_CHUNK), jend - jc0));
    __syncthreads();  // s_p of the previous piece is consumed
    if (threadIdx.x < nj) {
      const int64_t j = jc0 + threadIdx.x;
      s_p[threadIdx.x] = softmax_prob(exp_of(m, sc[j], p, lut_one), S, j, len, one);
    }
    __syncthreads();
    // sum_j p_j v_j[d]: warp w takes keys w, w + 8, ...; lane takes d = lane, lane + 32, ...
    for (int jj = warp; jj < nj; jj += ATT_THREADS / 32) {
      const int32_t pj = s_p[jj];
      if (pj == 0) continue;  // attention.rs:79
      const int16_t* vr = vbase + (jc0 + jj) * hd;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < hd) acc[i] += int64_t(pj) * int64_t(vr[d]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < hd) s_acc[warp * hd + d] = acc[i];
  }
  __syncthreads();
  int64_t tot = 0;
  if (threadIdx.x < hd)
    for (int w = 0; w < ATT_THREADS / 32; ++w) tot += s_acc[w * hd + threadIdx.x];
  attn_finish(p, row, c, nch, tot, &s_last);
}

// Pass 2 for head_dim a multiple of 8 (<= 256), many rows: hd / 8 threads per
// value row, each a 16-byte vector, ATT_THREADS * 8 / hd rows in flight per
// step and four steps unrolled; the rows' int64 partial sums meet in shared memory.
__global__ void __launch_bounds__(ATT_THREADS) attn_pv_vec_kernel(AttnParams p, int64_t chunk) {
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(16) int64_t s_acc[];  // [keys per step][hd] = ATT_THREADS * 8
  __shared__ int64_t s_red[ATT_THREADS / 32];
  __shared__ int32_t s_p[ATT_CHUNK];
  __shared__ bool s_last;
  const int64_t row = blockIdx.x;
  const int64_t r = row / p.nq;
  const int h = int(row % p.nq);
  const int64_t b = r / p.T, t = r % p.T;
  const int64_t pos = p.pos0[0] + t;
  const int64_t len = p.mask ? p.lds : pos + 1;
  const int64_t nch = (len + chunk - 1) / chunk;
  const int64_t c = blockIdx.y;
  if (c >= nch) return;
  const int32_t* sc = p.scores + row * p.lds;
  const int32_t m = int32_t(p.rowmax[row] ^ 0x80000000u);
  const int32_t lut_one = p.exp_lut[0];
  const int64_t jfirst = c * chunk;
  const int nfirst = int(min(int64_t(ATT_CHUNK), len - jfirst));
  // the first piece's exponentials come with the sum
  const int32_t S = attn_row_sum<ATT_THREADS>(sc, len, m, p, lut_one, s_red, s_p, jfirst, nfirst);
  const int32_t one = int32_t(1) << p.prob_frac;
  const int hd = p.hd, tpk = hd / 8, kpi = ATT_THREADS / tpk;
  const int kg = threadIdx.x / tpk, dv = threadIdx.x % tpk;
  const int16_t* vbase = p.kc.v + b * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t((p.q_head0 + h) / p.G - p.kv_head0) * p.kc.head_stride + 8 * dv;
  int64_t acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0;
  const int64_t jend = min(len, (c + 1) * chunk);
  for (int64_t jc0 = jfirst; jc0 < jend; jc0 += ATT_CHUNK) {
    const int nj = int(min(int64_t(ATT_CHUNK), jend - jc0));
    if (jc0 != jfirst) __syncthreads();  // s_p of the previous piece is consumed
    if (threadIdx.x < nj) {
      const int64_t j = jc0 + threadIdx.x;
      const int32_t e = jc0 == jfirst ? s_p[threadIdx.x] : exp_of(m, sc[j], p, lut_one);
      s_p[threadIdx.x] = softmax_prob(e, S, j, len, one);
    }
    __syncthreads();
    for (int jj = kg; jj < nj; jj += 4 * kpi) {
      int32_t pp[4];
      uint4 vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j2 = jj + u * kpi;
        pp[u] = j2 < nj ? s_p[j2] : 0;
        vv[u] = pp[u] != 0 ? *reinterpret_cast<const uint4*>(vbase + (jc0 + j2) * hd)
                           : make_uint4(0u, 0u, 0u, 0u);  // attention.rs:79 skips p = 0
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += int64_t(pp[u]) * int64_t(lane16(vv[u], e));
    }
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < 8; ++e) s_acc[kg * hd + 8 * dv + e] = acc[e];
  __syncthreads();
  int64_t tot = 0;
  if (threadIdx.x < hd)
    for (int g = 0; g < kpi; ++g) tot += s_acc[g * hd + threadIdx.x];
  attn_finish(p, row, c, nch, tot, &s_last);
}

// Pass 2 for many rows (prefill), tiled: block (64 consecutive query rows of
// one sequence, one head) walks the keys in tiles of ATT_TK: the tile's value
// rows and the 64 x ATT_TK probabilities are staged in shared memory once and
// used by every row, instead of every row reading every value row. Phase 1:
// each row's exponential sum (a warp per row, from the row maximum of pass 1).
// Phase 2: per tile, p = softmax_prob(...) for keys j <= pos of each row (0
// beyond), then thread (row group, 8-dim group) adds p * v for RPT rows and 8
// dimensions in int64 (hd = 32 * RPT, multiple of 8). Phase 3: round by
// prob_frac, clamp, rescale, store; the rows' maxima are set back to zero.

template <int RPT>
__global__ void __launch_bounds__(ATT_THREADS) attn_pv_tile_kernel(AttnParams p) {
  pdl_wait();
  pdl_launch();
  constexpr int HD = 32 * RPT;
  __shared__ __align__(16) int16_t s_v[ATT_TK][HD];
  __shared__ int32_t s_p[ATT_TQ][ATT_TK + 1];
  __shared__ int32_t s_m[ATT_TQ], s_S[ATT_TQ];
  __shared__ int64_t s_len[ATT_TQ];
  const int T = int(p.T);
  const int tiles_per_seq = (T + ATT_TQ - 1) / ATT_TQ;
  const int b = int(blockIdx.x) / tiles_per_seq, t0 = (int(blockIdx.x) % tiles_per_seq) * ATT_TQ;
  const int h = int(blockIdx.y);
  const int nrows = min(ATT_TQ, T - t0);
  const int64_t pos0 = p.pos0[0];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int32_t lut_one = p.exp_lut[0];
  const int32_t one = int32_t(1) << p.prob_frac;
  auto row_index = [&](int i) { return (int64_t(b) * T + t0 + i) * p.nq + h; };  // scores / rowmax row
  if (threadIdx.x < ATT_TQ) {
    const int i = threadIdx.x;
    s_len[i] = i < nrows ? pos0 + t0 + i + 1 : 0;
    s_m[i] = i < nrows ? int32_t(p.rowmax[row_index(i)] ^ 0x80000000u) : 0;
  }
  __syncthreads();
  // phase 1: exponential sums, warp w takes rows w, w + 8, ...
  for (int i = warp; i < nrows; i += ATT_THREADS / 32) {
    const int32_t* sc = p.scores + row_index(i) * p.lds;
    const int n = int(s_len[i]);
    const int32_t m = s_m[i];
    int64_t S = 0;
    for (int j0 = lane; j0 < n; j0 += 32 * 8) {
      int32_t v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = j0 + 32 * u < n ? sc[j0 + 32 * u] : m;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (j0 + 32 * u < n) S += exp_of(m, v[u], p, lut_one);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    if (lane == 0) s_S[i] = int32_t(S);  // i32 in the reference; the host bounds len
  }
  __syncthreads();
  if (threadIdx.x < nrows) p.rowmax[row_index(threadIdx.x)] = 0u;  // every reader is done
  // phase 2
  constexpr int DG = HD / 8;                 // 8-dim groups
  constexpr int RG = ATT_THREADS / DG;       // row groups (ATT_TQ / RPT)
  static_assert(RG * RPT == ATT_TQ, "row tiling");
  const int dg = threadIdx.x % DG, rg = threadIdx.x / DG;
  int64_t acc[RPT][8];
#pragma unroll
  for (int i = 0; i < RPT; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[i][e] = 0;
  const int16_t* vbase = p.kc.v + int64_t(b) * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t((p.q_head0 + h) / p.G - p.kv_head0) * p.kc.head_stride;
  const int64_t kend = s_len[nrows - 1];  // the longest row of the block
  for (int64_t j0 = 0; j0 < kend; j0 += ATT_TK) {
    const int nk = int(min(int64_t(ATT_TK), kend - j0));
    __syncthreads();  // the previous tile is consumed
    // all loads of the tile first: value rows (16 B) and scores (4 x 4 B) per item
    constexpr int VIT = ATT_TK * DG / ATT_THREADS;       // value vectors per thread
    constexpr int SIT = ATT_TQ * ATT_TK / 4 / ATT_THREADS;  // score quads per thread
    uint4 vreg[VIT];
    int32_t sreg[SIT][4];
#pragma unroll
    for (int q = 0; q < VIT; ++q) {
      const int e = threadIdx.x + q * ATT_THREADS, jj = e / DG, d8 = e % DG;
      vreg[q] = jj < nk ? *reinterpret_cast<const uint4*>(vbase + (j0 + jj) * HD + 8 * d8)
                        : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int q = 0; q < SIT; ++q) {
      const int e = threadIdx.x + q * ATT_THREADS, i = e / (ATT_TK / 4), j4 = 4 * (e % (ATT_TK / 4));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t j = j0 + j4 + u;
        sreg[q][u] = (i < nrows && j < s_len[i]) ? p.scores[row_index(i) * p.lds + j] : 0;
      }
    }
#pragma unroll
    for (int q = 0; q < VIT; ++q) {
      const int e = threadIdx.x + q * ATT_THREADS, jj = e / DG, d8 = e % DG;
      *reinterpret_cast<uint4*>(&s_v[jj][8 * d8]) = vreg[q];
    }
#pragma unroll
    for (int q = 0; q < SIT; ++q) {
      const int e = threadIdx.x + q * ATT_THREADS, i = e / (ATT_TK / 4), j4 = 4 * (e % (ATT_TK / 4));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t j = j0 + j4 + u;
        s_p[i][j4 + u] = (i < nrows && j < s_len[i])
                             ? softmax_prob(exp_of(s_m[i], sreg[q][u], p, lut_one), s_S[i], j, s_len[i], one)
                             : 0;
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int jj = 0; jj < nk; ++jj) {
      const uint4 vv = *reinterpret_cast<const uint4*>(&s_v[jj][8 * dg]);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const int64_t pj = s_p[rg * RPT + i][jj];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][e] += pj * int64_t(lane16(vv, e));
      }
    }
  }
  // phase 3
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg * RPT + i;
    if (r >= nrows) continue;
    int16_t o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      int32_t o = clamp16(p.prob_frac > 0 ? rshift_rne_i64(acc[i][e], p.prob_frac) : acc[i][e]);
      if (p.out_shift != 0) o = clamp16(rescale_i32_s(o, p.out_shift));
      o8[e] = int16_t(o);
    }
    *reinterpret_cast<uint4*>(p.out + (int64_t(b) * T + t0 + r) * p.ldo + int64_t(h) * HD + 8 * dg) = pack16(o8);
  }
}

// The same tiling with the products on the integer MMA path (mma.sync
// m16n8k32, u8 x u8) for head_dim 64 or 128 and p <= 32768 (prob_frac <= 15).
// p = 256 ph + pl and v + 32768 = 256 vh + vl (vh = (v >> 8) + 128, vl =
// v & 255) are unsigned bytes, so per tile
//   sum_j p_j v_j = 65536 HH + 256 (HL + LH) + LL - 32768 sum_j p_j
// with HH = sum ph*vh etc. exact in int32 over 64 keys (<= 6.2e6) and added to
// int64 accumulators after every tile. The probabilities are stored as two
// byte planes [row][key]; the value tile transposed into two byte planes
// [dim][key], so both MMA operands are 4-key words (rows padded to 80 bytes:
// the 8 x 4 words a fragment load touches fall into distinct banks). Warp
// task = 16 rows x 32 dims (4 n-tiles); HD / 64 tasks per warp.
__device__ __forceinline__ void mma_u8u8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int ATT_PK = 80;  // bytes per padded plane row (64 keys)

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_pv_mma_kernel(AttnParams p) {
  pdl_wait();
  pdl_launch();
  static_assert(HD == 64 || HD == 128, "head_dim");
  constexpr int TPW = HD / 64;  // warp tasks per warp
  __shared__ __align__(16) uint8_t s_ph[ATT_TQ][ATT_PK], s_pl[ATT_TQ][ATT_PK];
  __shared__ __align__(16) uint8_t s_vh[HD][ATT_PK], s_vl[HD][ATT_PK];
  __shared__ int32_t s_m[ATT_TQ], s_S[ATT_TQ], s_P[ATT_TQ];
  __shared__ int64_t s_len[ATT_TQ];
  __shared__ uint64_t s_R[ATT_TQ];
  const int T = int(p.T);
  const int tiles_per_seq = (T + ATT_TQ - 1) / ATT_TQ;
  const int b = int(blockIdx.x) / tiles_per_seq, t0 = (int(blockIdx.x) % tiles_per_seq) * ATT_TQ;
  const int h = int(blockIdx.y);
  const int nrows = min(ATT_TQ, T - t0);
  const int64_t pos0 = p.pos0[0];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int32_t lut_one = p.exp_lut[0];
  const int32_t one = int32_t(1) << p.prob_frac;
  auto row_index = [&](int i) { return (int64_t(b) * T + t0 + i) * p.nq + h; };
  if (threadIdx.x < ATT_TQ) {
    const int i = threadIdx.x;
    s_len[i] = i < nrows ? pos0 + t0 + i + 1 : 0;
    s_m[i] = i < nrows ? int32_t(p.rowmax[row_index(i)] ^ 0x80000000u) : 0;
  }
  __syncthreads();
  // phase 1: exponential sums, warp w takes rows w, w + 8, ...
  for (int i = warp; i < nrows; i += ATT_THREADS / 32) {
    const int32_t* sc = p.scores + row_index(i) * p.lds;
    const int n = int(s_len[i]);
    const int32_t m = s_m[i];
    int64_t S = 0;
    for (int j0 = lane; j0 < n; j0 += 32 * 8) {
      int32_t v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = j0 + 32 * u < n ? sc[j0 + 32 * u] : m;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (j0 + 32 * u < n) S += exp_of(m, v[u], p, lut_one);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    if (lane == 0) {
      s_S[i] = int32_t(S);  // i32 in the reference; the host bounds len
      s_R[i] = softmax_recip(int32_t(S));
    }
  }
  __syncthreads();
  if (threadIdx.x < nrows) p.rowmax[row_index(threadIdx.x)] = 0u;  // every reader is done
  const int16_t* vbase = p.kc.v + int64_t(b) * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t((p.q_head0 + h) / p.G - p.kv_head0) * p.kc.head_stride;
  int64_t acc[TPW][4][4];
#pragma unroll
  for (int t = 0; t < TPW; ++t)
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][n][i] = 0;
  const int64_t kend = s_len[nrows - 1];  // the longest row of the block
  for (int64_t j0 = 0; j0 < kend; j0 += ATT_TK) {
    const int nk = int(min(int64_t(ATT_TK), kend - j0));
    __syncthreads();  // the previous tile is consumed
    // loads first: thread (key quad q, 8-dim group d8) reads 4 value vectors;
    // thread (row i, key quad j4) reads 4 scores
    constexpr int DG = HD / 8;
    const int vq = threadIdx.x % 16, vd8 = threadIdx.x / 16;
    const bool vact = vd8 < DG;
    uint4 vreg[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int jj = 4 * vq + u;
      vreg[u] = (vact && jj < nk) ? *reinterpret_cast<const uint4*>(vbase + (j0 + jj) * HD + 8 * vd8)
                                  : make_uint4(0u, 0u, 0u, 0u);
    }
    int32_t sreg[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = threadIdx.x + q * ATT_THREADS, i = e / 16, j4 = 4 * (e % 16);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t j = j0 + j4 + u;
        sreg[q][u] = (i < nrows && j < s_len[i]) ? p.scores[row_index(i) * p.lds + j] : 0;
      }
    }
    // value planes, transposed: word (dim, keys 4vq..4vq+3)
    if (vact) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uint32_t wh = 0, wl = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int32_t v = lane16(vreg[u], e);
          wh |= uint32_t((v >> 8) + 128) << (8 * u);
          wl |= uint32_t(v & 255) << (8 * u);
        }
        *reinterpret_cast<uint32_t*>(&s_vh[8 * vd8 + e][4 * vq]) = wh;
        *reinterpret_cast<uint32_t*>(&s_vl[8 * vd8 + e][4 * vq]) = wl;
      }
    }
    // probability planes and the tile's row sums of p
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = threadIdx.x + q * ATT_THREADS, i = e / 16, j4 = 4 * (e % 16);
      uint32_t wh = 0, wl = 0;
      int32_t psum = 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t j = j0 + j4 + u;
        int32_t pj = 0;
        if (i < nrows && j < s_len[i])
          pj = softmax_prob_r(exp_of(s_m[i], sreg[q][u], p, lut_one), s_S[i], s_R[i], j, s_len[i], one);
        psum += pj;
        wh |= uint32_t(pj >> 8) << (8 * u);
        wl |= uint32_t(pj & 255) << (8 * u);
      }
      *reinterpret_cast<uint32_t*>(&s_ph[i][j4]) = wh;
      *reinterpret_cast<uint32_t*>(&s_pl[i][j4]) = wl;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);  // 16 lanes of a row
      if ((lane & 15) == 0) s_P[i] = psum;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < TPW; ++t) {
      const int task = warp * TPW + t;
      const int r0 = (task % 4) * 16, d0 = (task / 4) * 32;
      int hh[4][4], hl[4][4], ll[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) hh[n][i] = hl[n][i] = ll[n][i] = 0;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const int k0 = 32 * ks + 4 * c;
        const uint32_t ah0 = *reinterpret_cast<const uint32_t*>(&s_ph[r0 + g][k0]);
        const uint32_t ah1 = *reinterpret_cast<const uint32_t*>(&s_ph[r0 + g + 8][k0]);
        const uint32_t ah2 = *reinterpret_cast<const uint32_t*>(&s_ph[r0 + g][k0 + 16]);
        const uint32_t ah3 = *reinterpret_cast<const uint32_t*>(&s_ph[r0 + g + 8][k0 + 16]);
        const uint32_t al0 = *reinterpret_cast<const uint32_t*>(&s_pl[r0 + g][k0]);
        const uint32_t al1 = *reinterpret_cast<const uint32_t*>(&s_pl[r0 + g + 8][k0]);
        const uint32_t al2 = *reinterpret_cast<const uint32_t*>(&s_pl[r0 + g][k0 + 16]);
        const uint32_t al3 = *reinterpret_cast<const uint32_t*>(&s_pl[r0 + g + 8][k0 + 16]);
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int dn = d0 + 8 * n + g;
          const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&s_vh[dn][k0]);
          const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&s_vh[dn][k0 + 16]);
          const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&s_vl[dn][k0]);
          const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&s_vl[dn][k0 + 16]);
          mma_u8u8_16832(hh[n], ah0, ah1, ah2, ah3, bh0, bh1);
          mma_u8u8_16832(hl[n], ah0, ah1, ah2, ah3, bl0, bl1);
          mma_u8u8_16832(hl[n], al0, al1, al2, al3, bh0, bh1);
          mma_u8u8_16832(ll[n], al0, al1, al2, al3, bl0, bl1);
        }
      }
      const int64_t PA = s_P[r0 + g], PB = s_P[r0 + g + 8];
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          acc[t][n][i] += 65536 * int64_t(hh[n][i]) + 256 * int64_t(hl[n][i]) + int64_t(ll[n][i]) -
                          32768 * (i < 2 ? PA : PB);
    }
  }
  // phase 3: lane (g, c) of task t holds rows r0 + g (i = 0, 1) and r0 + g + 8
  // (i = 2, 3), dims d0 + 8n + 2c + (i & 1)
#pragma unroll
  for (int t = 0; t < TPW; ++t) {
    const int task = warp * TPW + t;
    const int r0 = (task % 4) * 16, d0 = (task / 4) * 32;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = r0 + g + 8 * half;
      if (r >= nrows) continue;
      int16_t* orow = p.out + (int64_t(b) * T + t0 + r) * p.ldo + int64_t(h) * HD;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        int16_t o2[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int64_t a = acc[t][n][2 * half + q];
          int32_t o = clamp16(p.prob_frac > 0 ? rshift_rne_i64(a, p.prob_frac) : a);
          if (p.out_shift != 0) o = clamp16(rescale_i32_s(o, p.out_shift));
          o2[q] = int16_t(o);
        }
        *reinterpret_cast<uint32_t*>(orow + d0 + 8 * n + 2 * c) =
            uint32_t(uint16_t(o2[0])) | (uint32_t(uint16_t(o2[1])) << 16);
      }
    }
  }
}

// Pass 2 for few rows (decode), one block per query row for rows of at most
// ATT_RCAP keys (head_dim a multiple of 8, at most 128): the row's statistics
// are computed once, every probability is kept in shared memory, and the
// block's warps walk all value rows (8 loads in flight per thread); no
// cross-block combination, no fence or counter.
constexpr int ATT_RCAP = 4096;
constexpr int ATT_RSHORT = 1024;  // sessions the one-block-per-row kernel is used for

__global__ void __launch_bounds__(ATT_DTHREADS) attn_pv_row_kernel(AttnParams p) {
  pdl_wait();
  pdl_launch();
  __shared__ __align__(16) int64_t s_buf[ATT_DTHREADS * 8];  // probabilities [ATT_RCAP] int32, then the partials
  __shared__ int64_t s_red[ATT_DTHREADS / 32];
  int32_t* s_pr = reinterpret_cast<int32_t*>(s_buf);
  const int row = int(blockIdx.x);
  const int r = row / p.nq, h = row % p.nq;
  const int T = int(p.T);
  const int b = r / T, t = r % T;
  const int len = int(p.pos0[0] + t + 1);
  const int hd = p.hd, tpk = hd / 8, kpi = ATT_DTHREADS / tpk;
  const int kg = int(threadIdx.x) / tpk, dv = int(threadIdx.x) % tpk;
  const int32_t* sc = p.scores + int64_t(row) * p.lds;
  const int32_t m = int32_t(p.rowmax[row] ^ 0x80000000u);
  const int32_t lut_one = p.exp_lut[0];
  const int32_t S = attn_row_sum<ATT_DTHREADS>(sc, len, m, p, lut_one, s_red, s_pr, 0, len);
  if (threadIdx.x == 0) p.rowmax[row] = 0u;  // every thread has read it (the sum's barrier)
  const int32_t one = int32_t(1) << p.prob_frac;
  const uint64_t R = softmax_recip(S);
  for (int j = threadIdx.x; j < len; j += ATT_DTHREADS) s_pr[j] = softmax_prob_r(s_pr[j], S, R, j, len, one);
  __syncthreads();
  const int16_t* vbase = p.kc.v + int64_t(b) * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t((p.q_head0 + h) / p.G - p.kv_head0) * p.kc.head_stride + 8 * dv;
  int64_t acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0;
  for (int j0 = kg; j0 < len; j0 += 8 * kpi) {
    uint4 vv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u * kpi;
      vv[u] = j < len ? *reinterpret_cast<const uint4*>(vbase + int64_t(j) * hd) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u * kpi;
      const int32_t pj = j < len ? s_pr[j] : 0;  // p = 0 adds nothing (attention.rs:79)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += int64_t(pj) * int64_t(lane16(vv[u], e));
    }
  }
  __syncthreads();  // the probabilities are consumed; s_buf takes the partials
#pragma unroll
  for (int e = 0; e < 8; ++e) s_buf[kg * hd + 8 * dv + e] = acc[e];
  __syncthreads();
  if (int(threadIdx.x) < hd) {
    int64_t tot = 0;
    for (int g = 0; g < kpi; ++g) tot += s_buf[g * hd + threadIdx.x];
    int32_t o = clamp16(p.prob_frac > 0 ? rshift_rne_i64(tot, p.prob_frac) : tot);
    if (p.out_shift != 0) o = clamp16(rescale_i32_s(o, p.out_shift));
    p.out[int64_t(r) * p.ldo + int64_t(h) * hd + threadIdx.x] = int16_t(o);
  }
}

// Pass 2 for few rows (decode): ATT_DTHREADS threads, chunks of ATT_DCHUNK
// keys, head_dim a multiple of 8 and at most 128 (so that the
// ATT_DTHREADS / (hd / 8) >= 32 value-row groups cover a chunk in at most 16
// rows each). The chunk's value rows are loaded before the softmax
// statistics, which need the row maximum from pass 1 and one pass over the
// row's scores.
__global__ void __launch_bounds__(ATT_DTHREADS) attn_pv_dec_kernel(AttnParams p) {
  pdl_wait();
  pdl_launch();
  constexpr int VR = ATT_DCHUNK / 32;  // value rows per thread (at most)
  __shared__ __align__(16) int64_t s_acc[ATT_DTHREADS * 8];  // [value-row groups][hd]
  __shared__ int64_t s_red[ATT_DTHREADS / 32];
  __shared__ int32_t s_e[ATT_DCHUNK];
  __shared__ bool s_last;
  const int row = int(blockIdx.x);
  const int r = row / p.nq, h = row % p.nq;
  const int T = int(p.T);
  const int b = r / T, t = r % T;
  const int64_t pos = p.pos0[0] + t;
  const int len = int(p.mask ? p.lds : pos + 1);
  const int nch = (len + ATT_DCHUNK - 1) / ATT_DCHUNK;
  const int c = int(blockIdx.y);
  if (c >= nch) return;
  const int jc0 = c * ATT_DCHUNK;
  const int nj = min(ATT_DCHUNK, len - jc0);
  const int hd = p.hd, tpk = hd / 8, kpi = ATT_DTHREADS / tpk;
  const int kg = int(threadIdx.x) / tpk, dv = int(threadIdx.x) % tpk;
  const int16_t* vbase = p.kc.v + int64_t(b) * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t((p.q_head0 + h) / p.G - p.kv_head0) * p.kc.head_stride +
                         int64_t(jc0) * hd + 8 * dv;
  uint4 vv[VR];
#pragma unroll
  for (int u = 0; u < VR; ++u) {
    const int jj = kg + u * kpi;
    vv[u] = jj < nj ? *reinterpret_cast<const uint4*>(vbase + int64_t(jj) * hd) : make_uint4(0u, 0u, 0u, 0u);
  }
  const int32_t* sc = p.scores + int64_t(row) * p.lds;
  const int32_t m = int32_t(p.rowmax[row] ^ 0x80000000u);
  const int32_t lut_one = p.exp_lut[0];
  const int32_t S = attn_row_sum<ATT_DTHREADS>(sc, len, m, p, lut_one, s_red, s_e, jc0, nj);
  const int32_t one = int32_t(1) << p.prob_frac;
  if (int(threadIdx.x) < nj) s_e[threadIdx.x] = softmax_prob(s_e[threadIdx.x], S, jc0 + threadIdx.x, len, one);
  __syncthreads();
  int64_t acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0;
#pragma unroll
  for (int u = 0; u < VR; ++u) {
    const int jj = kg + u * kpi;
    const int32_t pj = jj < nj ? s_e[jj] : 0;  // p = 0 adds nothing (attention.rs:79)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += int64_t(pj) * int64_t(lane16(vv[u], e));
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) s_acc[kg * hd + 8 * dv + e] = acc[e];
  __syncthreads();
  int64_t tot = 0;
  if (int(threadIdx.x) < hd)
    for (int g = 0; g < kpi; ++g) tot += s_acc[g * hd + threadIdx.x];
  attn_finish(p, row, c, nch, tot, &s_last);
}

// ---- tensor-parallel barrier ----------------------------------------------------
// All ranks call it the same number of times in the same order; each call's
// epoch is this rank's device counter + 1 (so a captured graph replays it
// with a fresh epoch). Optionally first copies `n` int64 values from `src`
// into every rank's slot dst[o] + rank * n. Thread t < world: system fence,
// release store of the epoch into rank t's flag word of this rank, then a
// bounded acquire wait for this rank's flag word of sender t (a peer that
// does not arrive within timeout_ns sets DEV_WAIT_PEER and the kernel returns).
struct TpPeers {
  unsigned long long* flags[MYL_XCHG_MAX];  // each rank's flag words (one per sender)
  int64_t* keys[MYL_XCHG_MAX];              // each rank's key slots [world][B]
};

__global__ void tp_barrier_kernel(TpPeers peers, int world, int rank,
                                  unsigned long long* __restrict__ epoch_ctr,
                                  const int64_t* __restrict__ src, int64_t n, int* err,
                                  uint64_t timeout_ns) {
  pdl_wait();
  pdl_launch();
  const int t = threadIdx.x;
  const unsigned long long epoch = epoch_ctr[0] + 1ull;
  if (src)
    for (int o = 0; o < world; ++o)
      for (int64_t i = t; i < n; i += blockDim.x) peers.keys[o][int64_t(rank) * n + i] = src[i];
  __syncthreads();
  if (t < world) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(peers.flags[t] + rank), "l"(epoch) : "memory");
    const unsigned long long* mine = peers.flags[rank] + t;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
      if (v >= epoch) break;
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicCAS(err, 0, DEV_WAIT_PEER);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (t == 0) epoch_ctr[0] = epoch;
}

// ---- greedy selection into the token stream -----------------------------------------
// keys[b] (select_key) -> token = 2^32 - 1 - (key & 0xFFFFFFFF); written to the
// next-step token buffer and to out_tokens[b * ld_out + step], step from the
// device step counter; the last block advances the position and step counters.
__global__ void greedy_commit_kernel(const int64_t* __restrict__ keys, int64_t B,
                                     int32_t* __restrict__ next_tokens,
                                     int32_t* __restrict__ out_tokens, int64_t ld_out,
                                     int64_t* __restrict__ step, int64_t* __restrict__ pos,
                                     int64_t pos_advance, int nslots) {
  pdl_wait();
  pdl_launch();
  const int64_t s = step[0];
  for (int64_t b = threadIdx.x; b < B; b += blockDim.x) {
    // the largest key over the vocabulary shards' slots [nslots][B]
    int64_t key = keys[b];
    for (int o = 1; o < nslots; ++o) key = max(key, keys[int64_t(o) * B + b]);
    const int32_t tok = int32_t(int64_t(0xFFFFFFFFll) - (key & 0xFFFFFFFFll));
    next_tokens[b] = tok;
    if (out_tokens) out_tokens[b * ld_out + s] = tok;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    step[0] = s + 1;
    pos[0] += pos_advance;
  }
}

}  // namespace myl
