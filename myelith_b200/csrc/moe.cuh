// moe.cuh — MoE routing, token permutation and combine around the grouped
// tensor-core GEMM.
//
// The reference has no MoE layer; this one is composed from its primitives:
//   logits[t][e] = clamp_i32(rescale_i64(dot(W_router[e], x[t]), r_shift[e] + in_frac,
//                            router_frac))        (LM-head linear, runtime/src/model.rs:297-307)
//   top-k        = k times argmax over the experts not yet chosen
//                  (sampling.rs:8-18: ties go to the lowest index)
//   p[t][j]      = softmax_int over the k chosen logits (softmax.rs:24-64)
//   y[t][j]      = mlp_int(x[t], expert topk[t][j])    (mlp.rs:28-74)
//   out[t][h]    = clamp_i16(rescale_i64(sum_j p[t][j] * y[t][j][h], prob_frac, 0)
//                            + shared[t][h])
// (token, choice) pairs are permuted so that each expert's rows are
// contiguous (a counting sort by expert). The order inside an expert's
// segment comes from atomics and changes from run to run; every row is
// computed on its own and the combine sums in the fixed order j = 0..k-1, so
// the output does not.
#pragma once

#include "common.cuh"

namespace myl {

constexpr int MOE_MAX_K = 8;
constexpr int MOE_MAX_EXPERTS = 256;

struct MoeRouteParams {
  const int16_t* exp_lut;
  int exp_lut_len;
  int lut_shift;
  int prob_frac;  // the host checks that every e * 2^prob_frac fits in i32
};

// softmax.rs:12-21.
__device__ __forceinline__ int32_t exp_lut_lookup_dev(int32_t x, const MoeRouteParams& p,
                                                      int32_t one) {
  if (x <= 0) return one;
  const uint32_t idx = uint32_t(x) >> p.lut_shift;
  if (idx >= uint32_t(p.exp_lut_len)) return 0;
  return int32_t(p.exp_lut[idx]);
}

// One thread per token: top-k experts (lowest index on ties) and softmax_int
// of their logits (softmax.rs:24-64, Rust's truncating i32 division followed
// by the round-half-even correction).
__global__ void moe_route_kernel(const int32_t* __restrict__ logits, int64_t ldl, int64_t T, int E,
                                 int k, MoeRouteParams p, int32_t* __restrict__ topk_idx,
                                 int32_t* __restrict__ topk_prob) {
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < T;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int32_t* lg = logits + t * ldl;
    uint32_t chosen[MOE_MAX_EXPERTS / 32];
#pragma unroll
    for (int i = 0; i < MOE_MAX_EXPERTS / 32; ++i) chosen[i] = 0u;
    int32_t sel[MOE_MAX_K];
    int idx[MOE_MAX_K];
#pragma unroll
    for (int j = 0; j < MOE_MAX_K; ++j) {
      if (j >= k) break;
      int best = -1;
      int32_t bv = 0;
      for (int e = 0; e < E; ++e) {
        if (chosen[e >> 5] & (1u << (e & 31))) continue;
        const int32_t v = lg[e];
        if (best < 0 || v > bv) {
          best = e;
          bv = v;
        }
      }
      chosen[best >> 5] |= 1u << (best & 31);
      idx[j] = best;
      sel[j] = bv;
    }
    const int32_t one = int32_t(1) << p.prob_frac;
    const int32_t lut_one = p.exp_lut_len > 0 ? int32_t(p.exp_lut[0]) : 1;
    int32_t m = sel[0];
#pragma unroll
    for (int j = 1; j < MOE_MAX_K; ++j)
      if (j < k) m = sel[j] > m ? sel[j] : m;
    int32_t ex[MOE_MAX_K];
    int32_t s = 0;
#pragma unroll
    for (int j = 0; j < MOE_MAX_K; ++j) {
      if (j >= k) break;
      const int64_t d = int64_t(m) - int64_t(sel[j]);  // saturating_sub
      ex[j] = exp_lut_lookup_dev(d > INT32_MAX ? INT32_MAX : int32_t(d), p, lut_one);
      s += ex[j];
    }
#pragma unroll
    for (int j = 0; j < MOE_MAX_K; ++j) {
      if (j >= k) break;
      int32_t q;
      if (s == 0) {
        const int32_t base = one / k, rem = one - base * k;
        q = base + (j < rem ? 1 : 0);
      } else {
        const int32_t num = ex[j] * one;
        q = num / s;
        const int32_t r = num % s;
        const int32_t twice = (r < 0 ? -r : r) * 2, den_abs = s < 0 ? -s : s;
        if (twice > den_abs || (twice == den_abs && (q & 1) != 0))
          q = ((num > 0) == (s > 0)) ? q + 1 : q - 1;
      }
      topk_idx[t * k + j] = idx[j];
      topk_prob[t * k + j] = q;
    }
  }
}

// Rows per expert: counts[e - first] += 1 for every id e in [first, first + E).
// Any other id sets DEV_BAD_EXPERT; its row is left out of the permutation.
__global__ void moe_count_kernel(const int32_t* __restrict__ ids, int64_t P, int first, int E,
                                 int* __restrict__ counts, int* __restrict__ err) {
  __shared__ int hist[MOE_MAX_EXPERTS];
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int64_t q = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; q < P;
       q += int64_t(gridDim.x) * blockDim.x) {
    const int e = ids[q] - first;
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
    else atomicCAS(err, 0, DEV_BAD_EXPERT);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    if (hist[i]) atomicAdd(&counts[i], hist[i]);
}

// Single thread: exclusive scans of the rows per expert and of the units the
// two grouped GEMMs have per expert (tiles_a / tiles_b channel tiles for each
// token tile of BN rows). cursor starts at row_start for the scatter.
__global__ void moe_plan_kernel(const int* __restrict__ counts, int E, int BN, int tiles_a,
                                int tiles_b, int* __restrict__ row_start, int* __restrict__ rows,
                                int* __restrict__ tile_start_a, int* __restrict__ tile_start_b,
                                int* __restrict__ cursor) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int r = 0, ta = 0, tb = 0;
  for (int e = 0; e < E; ++e) {
    const int c = counts[e];
    row_start[e] = r;
    cursor[e] = r;
    rows[e] = c;
    tile_start_a[e] = ta;
    tile_start_b[e] = tb;
    const int mt = (c + BN - 1) / BN;
    r += c;
    ta += mt * tiles_a;
    tb += mt * tiles_b;
  }
  tile_start_a[E] = ta;
  tile_start_b[E] = tb;
}

// Pair q goes to row pos[q] of its expert's segment; that row reads source row
// src[pos[q]] = q / div (div = k when the pairs are (token, choice), 1 when
// every pair is its own row). Pairs with a bad id get pos = -1.
__global__ void moe_scatter_kernel(const int32_t* __restrict__ ids, int64_t P, int first, int E,
                                   int div, int* __restrict__ cursor, int32_t* __restrict__ src,
                                   int32_t* __restrict__ pos) {
  for (int64_t q = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; q < P;
       q += int64_t(gridDim.x) * blockDim.x) {
    const int e = ids[q] - first;
    if (e < 0 || e >= E) {
      pos[q] = -1;
      continue;
    }
    const int row = atomicAdd(&cursor[e], 1);
    src[row] = int32_t(q / div);
    pos[q] = row;
  }
}

// Row p of the planes = source row src[p] of X split as x = 256*hi + lo;
// columns K..ldp-1 are zero.
__global__ void moe_gather_split_kernel(const int16_t* __restrict__ X, int64_t ldx, int64_t P,
                                        int64_t K, const int32_t* __restrict__ src,
                                        int8_t* __restrict__ Xhi, uint8_t* __restrict__ Xlo,
                                        int64_t ldp) {
  const int64_t groups = ldp >> 3;
  const int64_t total = P * groups;
  const bool vec = ((reinterpret_cast<uintptr_t>(X) & 15) == 0) && (ldx % 8 == 0);
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t p = g / groups, k0 = (g % groups) * 8;
    const int16_t* xr = X + int64_t(src[p]) * ldx;
    alignas(16) int16_t v[8];
    if (vec && k0 + 8 <= K) {
      *reinterpret_cast<int4*>(v) = __ldg(reinterpret_cast<const int4*>(xr + k0));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = (k0 + e < K) ? xr[k0 + e] : int16_t(0);
    }
    uint32_t h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h0 |= uint32_t(uint8_t(v[e] >> 8)) << (8 * e);
      l0 |= uint32_t(uint8_t(v[e] & 0xFF)) << (8 * e);
      h1 |= uint32_t(uint8_t(v[e + 4] >> 8)) << (8 * e);
      l1 |= uint32_t(uint8_t(v[e + 4] & 0xFF)) << (8 * e);
    }
    *reinterpret_cast<uint2*>(Xhi + p * ldp + k0) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(Xlo + p * ldp + k0) = make_uint2(l0, l1);
  }
}

// y[q] = y_perm[pos[q]] (a row of zeros where pos[q] < 0).
__global__ void moe_unpermute_kernel(const int16_t* __restrict__ y_perm, int64_t ldyp,
                                     const int32_t* __restrict__ pos, int64_t P, int64_t H,
                                     int16_t* __restrict__ y, int64_t ldy) {
  const int64_t total = P * H;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t q = i / H, h = i % H;
    const int32_t r = pos[q];
    y[q * ldy + h] = r >= 0 ? y_perm[int64_t(r) * ldyp + h] : int16_t(0);
  }
}

// out[t][h] = clamp_i16(rescale_i64(sum_j p[t][j] * y[pos[t][j]][h], prob_frac, 0)
//                       + shared[t][h]); pos == nullptr reads y row t*k + j.
__global__ void moe_combine_kernel(const int16_t* __restrict__ y, int64_t ldyp,
                                   const int32_t* __restrict__ pos, const int32_t* __restrict__ prob,
                                   const int16_t* __restrict__ shared, int64_t ld_shared, int64_t T,
                                   int k, int64_t H, int prob_frac, int16_t* __restrict__ out,
                                   int64_t ldo) {
  const int64_t total = T * H;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / H, h = i % H;
    int64_t acc = 0;
    for (int j = 0; j < k; ++j) {
      const int64_t q = t * k + j;
      const int64_t r = pos ? int64_t(pos[q]) : q;
      if (r >= 0) acc += int64_t(prob[q]) * int64_t(y[r * ldyp + h]);
    }
    int64_t v = rescale_i64_signed(acc, prob_frac);
    if (shared) v += shared[t * ld_shared + h];
    out[t * ldo + h] = int16_t(clamp_i64(v, -32768, 32767));
  }
}

}  // namespace myl
