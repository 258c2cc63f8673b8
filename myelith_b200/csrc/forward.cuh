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
// Pass 1 (attn_scores_kernel): scores[row][j] = rne_i64(dot(q, k_j) * mult, shift) as i32.
//   The int16 x int16 dot is exact in two int32 sums: k = 256 kh + kl with kh
//   the signed high byte and kl the unsigned low byte, so
//   dot = 256 * sum q*kh + sum q*kl, |sum q*kh| <= hd * 2^22 and
//   sum q*kl <= hd * 2^23 (both exact in int32 for hd <= 255); each sum is a
//   chain of dp2a (two int16 x int8 products per instruction).
// Pass 2 (attn_pv_kernel): softmax_int over the row (softmax.rs:24-64: max,
//   exp LUT of the saturating difference, i32 sum, round-half-even division),
//   then sum_j p_j * v_j in int64 over a chunk of keys; the chunks of a row are
//   added (exact) by the last of its blocks, rounded by prob_frac and clamped
//   (attention.rs:83-90), then rescaled from the V scale to the o_proj input
//   scale (model.rs:563-567).
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

constexpr int ATT_KEYS = 256;     // keys per block of pass 1 (one per thread)
constexpr int ATT_MAXG = 8;       // query rows per block of pass 1
constexpr int ATT_CHUNK = 256;    // keys per block of pass 2
constexpr int ATT_THREADS = 256;

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

// grid.x: (row group) = ((b * T + t) * nkv + g) * gsub + sub; grid.y: key chunk of ATT_KEYS;
// sub-groups of ATT_MAXG query heads of the KV head g. Dynamic shared memory:
// key planes [ATT_KEYS][hd8 + 8] bytes x 2 (hd8 = head_dim rounded up to 8;
// the 8-byte pad makes the per-key 8-byte reads of a half-warp hit distinct
// banks) and queries [ATT_MAXG][hd8] int16.
__host__ __device__ constexpr int att_hd8(int hd) { return (hd + 7) & ~7; }
__host__ __device__ constexpr size_t att_scores_smem(int hd, int keys = ATT_KEYS) {
  return size_t(2 * keys * (att_hd8(hd) + 8)) + size_t(ATT_MAXG * att_hd8(hd) * 2);
}

__global__ void __launch_bounds__(ATT_THREADS) attn_scores_kernel(AttnParams p, int gsub) {
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(16) uint8_t smem[];
  const int hd = p.hd, hd8 = att_hd8(hd), kst = hd8 + 8, qw = hd8 / 2;
  const int nk = blockDim.x;  // keys per block (<= ATT_KEYS)
  uint8_t* s_kh = smem;
  uint8_t* s_kl = s_kh + nk * kst;
  uint32_t* s_q = reinterpret_cast<uint32_t*>(s_kl + nk * kst);  // [ATT_MAXG][hd8/2]
  const int64_t gy = blockIdx.x;
  const int sub = int(gy % gsub);
  const int g = int((gy / gsub) % p.nkv);
  const int64_t r = gy / gsub / p.nkv;  // token row b * T + t
  const int64_t b = r / p.T, t = r % p.T;
  const int64_t pos = p.pos0[0] + t;
  const int64_t len = p.mask ? p.lds : pos + 1;
  const int64_t j0 = int64_t(blockIdx.y) * nk;
  if (j0 >= len) return;
  // local query heads of KV head g (GQA: global head q reads KV head q / G)
  const int hs = max(0, (p.kv_head0 + g) * p.G - p.q_head0);
  const int he = min(p.nq, (p.kv_head0 + g + 1) * p.G - p.q_head0);
  const int h0 = hs + sub * ATT_MAXG;
  const int nrow = min(ATT_MAXG, he - h0);
  if (nrow <= 0) return;
  // queries of the sub-group as int16 pairs, zero-padded to hd8
  for (int e = threadIdx.x; e < ATT_MAXG * qw; e += nk) {
    const int rr = e / qw, w = e % qw;
    uint32_t v = 0;
    if (rr < nrow) {
      const int16_t* q = p.qkv + r * p.ldq + int64_t(h0 + rr) * hd;
      const int d = 2 * w;
      const uint32_t lo = d < hd ? uint16_t(q[d]) : 0u, hi = d + 1 < hd ? uint16_t(q[d + 1]) : 0u;
      v = lo | (hi << 16);
    }
    s_q[e] = v;
  }
  // key rows j0.. as two byte planes (high byte signed, low byte unsigned),
  // 8 elements per step: one 16-byte load, two byte permutes, two 8-byte stores
  const int16_t* kbase = p.kc.k + b * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t(g) * p.kc.head_stride;
  const int nkeys = int(min(int64_t(nk), len - j0));
  const bool vec = (hd & 7) == 0;
  for (int e = threadIdx.x; e < nk * (hd8 / 8); e += nk) {
    const int jj = e / (hd8 / 8), d = 8 * (e % (hd8 / 8));
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (jj < nkeys) {
      const int16_t* kr = kbase + (j0 + jj) * hd + d;
      if (vec) {
        v = *reinterpret_cast<const uint4*>(kr);
      } else {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        for (int i = 0; i < 8 && d + i < hd; ++i) w[i / 2] |= uint32_t(uint16_t(kr[i])) << (16 * (i & 1));
        v = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    *reinterpret_cast<uint2*>(s_kh + jj * kst + d) =
        make_uint2(__byte_perm(v.x, v.y, 0x7531), __byte_perm(v.z, v.w, 0x7531));
    *reinterpret_cast<uint2*>(s_kl + jj * kst + d) =
        make_uint2(__byte_perm(v.x, v.y, 0x6420), __byte_perm(v.z, v.w, 0x6420));
  }
  __syncthreads();
  const int jj = threadIdx.x;
  if (jj >= nkeys) return;
  int acc_h[ATT_MAXG], acc_l[ATT_MAXG];
#pragma unroll
  for (int i = 0; i < ATT_MAXG; ++i) acc_h[i] = acc_l[i] = 0;
  const uint2* kh8 = reinterpret_cast<const uint2*>(s_kh + jj * kst);
  const uint2* kl8 = reinterpret_cast<const uint2*>(s_kl + jj * kst);
  for (int w8 = 0; w8 < hd8 / 8; ++w8) {
    const uint2 kh = kh8[w8], kl = kl8[w8];
#pragma unroll
    for (int i = 0; i < ATT_MAXG; ++i) {
      if (i < nrow) {
        const uint4 q = *reinterpret_cast<const uint4*>(s_q + i * qw + 4 * w8);
        acc_h[i] = dp2a_hi_ss(q.y, kh.x, dp2a_lo_ss(q.x, kh.x, acc_h[i]));
        acc_h[i] = dp2a_hi_ss(q.w, kh.y, dp2a_lo_ss(q.z, kh.y, acc_h[i]));
        acc_l[i] = dp2a_hi_su(q.y, kl.x, dp2a_lo_su(q.x, kl.x, acc_l[i]));
        acc_l[i] = dp2a_hi_su(q.w, kl.y, dp2a_lo_su(q.z, kl.y, acc_l[i]));
      }
    }
  }
  const int64_t j = j0 + jj;
#pragma unroll
  for (int i = 0; i < ATT_MAXG; ++i) {
    if (i < nrow) {
      const int64_t row = r * p.nq + h0 + i;
      int32_t sc;
      if (p.mask && !p.mask[r * p.lds + j]) {
        sc = INT32_MIN;
      } else {
        const int64_t dot = int64_t(acc_h[i]) * 256 + int64_t(acc_l[i]);
        const uint64_t prod = uint64_t(dot) * uint64_t(p.score_mult);  // i64 (wrapping)
        const int64_t s = p.score_shift > 0 ? rshift_rne_i64(int64_t(prod), p.score_shift) : int64_t(prod);
        sc = int32_t(uint32_t(uint64_t(s)));  // `as i32`
      }
      p.scores[row * p.lds + j] = sc;
    }
  }
}

__device__ __forceinline__ int32_t exp_lookup(int32_t x, const int16_t* lut, int32_t len, int shift,
                                              int32_t one) {
  if (x <= 0) return one;
  const uint32_t idx = uint32_t(x) >> shift;
  if (idx >= uint32_t(len)) return 0;
  return lut[idx];
}

// grid.x: query row (b * T + t) * nq + h; grid.y: key chunk of `chunk` keys
// (a multiple of ATT_CHUNK; one chunk per row when rows are plentiful).
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
  // max over the row
  int32_t m = INT32_MIN;
  for (int64_t j = threadIdx.x; j < len; j += ATT_THREADS) m = max(m, sc[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) s_red[warp] = m;
  __syncthreads();
  m = int32_t(s_red[0]);
  for (int w = 1; w < ATT_THREADS / 32; ++w) m = max(m, int32_t(s_red[w]));
  __syncthreads();
  const int32_t lut_one = p.exp_lut[0];
  // sum of the exponentials (i32 in the reference; the host bounds the row
  // length so that it cannot overflow)
  int64_t s = 0;
  for (int64_t j = threadIdx.x; j < len; j += ATT_THREADS) {
    const int64_t d = int64_t(m) - int64_t(sc[j]);
    s += exp_lookup(d > INT32_MAX ? INT32_MAX : int32_t(d), p.exp_lut, p.exp_len, p.lut_shift, lut_one);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) s_red[warp] = s;
  __syncthreads();
  s = 0;
  for (int w = 0; w < ATT_THREADS / 32; ++w) s += s_red[w];
  const int32_t S = int32_t(s);
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
    // probabilities of this piece (softmax.rs:41-62)
    if (threadIdx.x < nj) {
      const int64_t j = jc0 + threadIdx.x;
      int32_t pj;
      if (S == 0) {
        const int32_t base = one / int32_t(len), rem = one - base * int32_t(len);
        pj = base + (j < rem ? 1 : 0);
      } else {
        const int64_t d = int64_t(m) - int64_t(sc[j]);
        const int32_t e = exp_lookup(d > INT32_MAX ? INT32_MAX : int32_t(d), p.exp_lut, p.exp_len,
                                     p.lut_shift, lut_one);
        const int32_t num = e * one;
        int32_t q = num / S;
        const int32_t rm = num % S;
        const int32_t twice = (rm < 0 ? -rm : rm) * 2, den = S < 0 ? -S : S;
        if (twice > den || (twice == den && (q & 1))) q = ((num > 0) == (S > 0)) ? q + 1 : q - 1;
        pj = q;
      }
      s_p[threadIdx.x] = pj;
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
  int64_t* part = p.part + (row * p.max_chunks) * hd;
  for (int d = threadIdx.x; d < hd; d += ATT_THREADS) {
    int64_t v = 0;
    for (int w = 0; w < ATT_THREADS / 32; ++w) v += s_acc[w * hd + d];
    s_acc[d] = v;  // thread d alone reads column d of every warp, then writes slot d
    if (nch > 1) part[c * hd + d] = v;
  }
  if (nch > 1) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(p.counters + row, 1u);
      s_last = (prev + 1 == unsigned(nch));
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
  } else {
    __syncthreads();
  }
  int16_t* out = p.out + r * p.ldo + int64_t(h) * hd;
  for (int d = threadIdx.x; d < hd; d += ATT_THREADS) {
    int64_t v;
    if (nch > 1) {
      v = 0;
      for (int64_t cc = 0; cc < nch; ++cc) v += __ldcg(part + cc * hd + d);
    } else {
      v = s_acc[d];
    }
    int32_t o = clamp16(p.prob_frac > 0 ? rshift_rne_i64(v, p.prob_frac) : v);
    if (p.out_shift != 0) o = clamp16(rescale_i32_s(o, p.out_shift));
    out[d] = int16_t(o);
  }
  if (nch > 1 && threadIdx.x == 0) p.counters[row] = 0;
}

// The softmax of one attention row (softmax.rs:24-64): its maximum and the
// sum of the exponentials, loads unrolled four deep.
__device__ __forceinline__ void attn_row_stats(const int32_t* __restrict__ sc, int64_t len,
                                               const AttnParams& p, int32_t lut_one, int64_t* s_red,
                                               int32_t* m_out, int32_t* S_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t m = INT32_MIN;
  for (int64_t j = threadIdx.x; j < len; j += 4 * ATT_THREADS) {
    int32_t v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t jj = j + u * ATT_THREADS;
      v[u] = jj < len ? sc[jj] : INT32_MIN;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) m = max(m, v[u]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) s_red[warp] = m;
  __syncthreads();
  m = int32_t(s_red[0]);
  for (int w = 1; w < ATT_THREADS / 32; ++w) m = max(m, int32_t(s_red[w]));
  __syncthreads();
  int64_t s = 0;
  for (int64_t j = threadIdx.x; j < len; j += 4 * ATT_THREADS) {
    int32_t v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t jj = j + u * ATT_THREADS;
      v[u] = jj < len ? sc[jj] : m;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j + u * ATT_THREADS < len) {
        const int64_t d = int64_t(m) - int64_t(v[u]);
        s += exp_lookup(d > INT32_MAX ? INT32_MAX : int32_t(d), p.exp_lut, p.exp_len, p.lut_shift, lut_one);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) s_red[warp] = s;
  __syncthreads();
  s = 0;
  for (int w = 0; w < ATT_THREADS / 32; ++w) s += s_red[w];
  *m_out = m;
  *S_out = int32_t(s);
}

// Pass 2 for head_dim a multiple of 8 (<= 256): hd / 8 threads per value row,
// each a 16-byte vector, ATT_THREADS * 8 / hd rows in flight per step and four
// steps unrolled; the rows' int64 partial sums meet in shared memory.
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
  const int32_t lut_one = p.exp_lut[0];
  int32_t m, S;
  attn_row_stats(sc, len, p, lut_one, s_red, &m, &S);
  const int32_t one = int32_t(1) << p.prob_frac;
  const int hd = p.hd, tpk = hd / 8, kpi = ATT_THREADS / tpk;
  const int kg = threadIdx.x / tpk, dv = threadIdx.x % tpk;
  const int16_t* vbase = p.kc.v + b * p.kc.seq_stride + int64_t(p.layer) * p.kc.layer_stride +
                         int64_t((p.q_head0 + h) / p.G - p.kv_head0) * p.kc.head_stride + 8 * dv;
  int64_t acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0;
  const int64_t jend = min(len, (c + 1) * chunk);
  for (int64_t jc0 = c * chunk; jc0 < jend; jc0 += ATT_CHUNK) {
    const int nj = int(min(int64_t(ATT_CHUNK), jend - jc0));
    __syncthreads();  // s_p of the previous piece is consumed
    if (threadIdx.x < nj) {
      const int64_t j = jc0 + threadIdx.x;
      int32_t pj;
      if (S == 0) {
        const int32_t base = one / int32_t(len), rem = one - base * int32_t(len);
        pj = base + (j < rem ? 1 : 0);
      } else {
        const int64_t d = int64_t(m) - int64_t(sc[j]);
        const int32_t e = exp_lookup(d > INT32_MAX ? INT32_MAX : int32_t(d), p.exp_lut, p.exp_len,
                                     p.lut_shift, lut_one);
        const int32_t num = e * one;
        int32_t q = num / S;
        const int32_t rm = num % S;
        const int32_t twice = (rm < 0 ? -rm : rm) * 2, den = S < 0 ? -S : S;
        if (twice > den || (twice == den && (q & 1))) q = ((num > 0) == (S > 0)) ? q + 1 : q - 1;
        pj = q;
      }
      s_p[threadIdx.x] = pj;
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
  int64_t* part = p.part + (row * p.max_chunks) * hd;
  int64_t tot = 0;
  const int d = threadIdx.x;
  if (d < hd) {
    for (int g = 0; g < kpi; ++g) tot += s_acc[g * hd + d];
    if (nch > 1) part[c * hd + d] = tot;
  }
  if (nch > 1) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(p.counters + row, 1u);
      s_last = (prev + 1 == unsigned(nch));
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (d < hd) {
      tot = 0;
      for (int64_t cc = 0; cc < nch; ++cc) tot += __ldcg(part + cc * hd + d);
    }
  }
  if (d < hd) {
    int32_t o = clamp16(p.prob_frac > 0 ? rshift_rne_i64(tot, p.prob_frac) : tot);
    if (p.out_shift != 0) o = clamp16(rescale_i32_s(o, p.out_shift));
    p.out[r * p.ldo + int64_t(h) * hd + d] = int16_t(o);
  }
  if (nch > 1 && threadIdx.x == 0) p.counters[row] = 0;
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
