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
#include "gemm_tc.cuh"

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

// One warp per token: top-k experts (lowest index on ties) and softmax_int
// of their logits (softmax.rs:24-64, Rust's truncating i32 division followed
// by the round-half-even correction). Lane l holds experts l, l + 32, ...; each
// of the k rounds is a warp arg-max over the experts not yet chosen.
__global__ void moe_route_kernel(const int32_t* __restrict__ logits, int64_t ldl, int64_t T, int E,
                                 int k, MoeRouteParams p, int32_t* __restrict__ topk_idx,
                                 int32_t* __restrict__ topk_prob) {
  constexpr int PER = MOE_MAX_EXPERTS / 32;
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t t = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    const int32_t* lg = logits + t * ldl;
    int32_t v[PER];
    unsigned live = 0;  // bit i: expert lane + 32 i exists and is not chosen yet
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? lg[e] : 0;
      if (e < E) live |= 1u << i;
    }
    int32_t sel[MOE_MAX_K];
    int idx[MOE_MAX_K];
#pragma unroll
    for (int j = 0; j < MOE_MAX_K; ++j) {
      if (j >= k) break;
      // this lane's best: highest value, lowest expert id on ties
      int best = INT32_MAX;
      int32_t bv = INT32_MIN;
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (((live >> i) & 1u) && (best == INT32_MAX || v[i] > bv)) {
          bv = v[i];
          best = lane + 32 * i;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const int32_t ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int ob = __shfl_xor_sync(0xffffffffu, best, o);
        if (ob != INT32_MAX && (best == INT32_MAX || ov > bv || (ov == bv && ob < best))) {
          bv = ov;
          best = ob;
        }
      }
      if ((best & 31) == lane) live &= ~(1u << (best >> 5));
      idx[j] = best;
      sel[j] = bv;
    }
    if (lane != 0) continue;
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

// Row p of the planes = source row src[p] of X split into the offset-binary
// byte planes of split_hilo_kernel. blockIdx.y walks rows, threads 8 columns
// each.
__global__ void moe_gather_split_kernel(const int16_t* __restrict__ X, int64_t ldx, int64_t P,
                                        int64_t K, const int32_t* __restrict__ src,
                                        uint8_t* __restrict__ Xhi, uint8_t* __restrict__ Xlo,
                                        int64_t ldp) {
  const bool vec = ((reinterpret_cast<uintptr_t>(X) & 15) == 0) && (ldx % 8 == 0);
  const int64_t k0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (k0 >= ldp) return;
  for (int64_t p = blockIdx.y; p < P; p += gridDim.y) {
    const int16_t* xr = X + int64_t(src[p]) * ldx;
    alignas(16) int16_t v[8];
    if (vec && k0 + 8 <= K) {
      *reinterpret_cast<int4*>(v) = __ldg(reinterpret_cast<const int4*>(xr + k0));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = (k0 + e < K) ? xr[k0 + e] : int16_t(0);
    }
    uint2 hi, lo;
    split8(v, hi, lo);
    *reinterpret_cast<uint2*>(Xhi + p * ldp + k0) = hi;
    *reinterpret_cast<uint2*>(Xlo + p * ldp + k0) = lo;
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
// blockIdx.y walks tokens; a thread owns 8 consecutive h (16-byte accesses
// when every row start is 16-byte aligned, else element by element).
__global__ void moe_combine_kernel(const int16_t* __restrict__ y, int64_t ldyp,
                                   const int32_t* __restrict__ pos, const int32_t* __restrict__ prob,
                                   const int16_t* __restrict__ shared, int64_t ld_shared, int64_t T,
                                   int k, int64_t H, int prob_frac, int16_t* __restrict__ out,
                                   int64_t ldo) {
  const int64_t h0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (h0 >= H) return;
  const bool vec = h0 + 8 <= H && ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(out) |
                                     reinterpret_cast<uintptr_t>(shared)) & 15) == 0 &&
                   ldyp % 8 == 0 && ldo % 8 == 0 && (shared == nullptr || ld_shared % 8 == 0);
  const int n = vec ? 8 : int(H - h0 < 8 ? H - h0 : 8);
  for (int64_t t = blockIdx.y; t < T; t += gridDim.y) {
    int64_t acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0;
    for (int j = 0; j < k; ++j) {
      const int64_t q = t * k + j;
      const int64_t r = pos ? int64_t(pos[q]) : q;
      if (r < 0) continue;
      const int64_t pj = prob[q];
      const int16_t* yr = y + r * ldyp + h0;
      alignas(16) int16_t v[8];
      if (vec) {
        *reinterpret_cast<int4*>(v) = __ldg(reinterpret_cast<const int4*>(yr));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = e < n ? yr[e] : int16_t(0);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += pj * int64_t(v[e]);
    }
    alignas(16) int16_t sv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) sv[e] = 0;
    if (shared) {
      const int16_t* sr = shared + t * ld_shared + h0;
      if (vec) {
        *reinterpret_cast<int4*>(sv) = __ldg(reinterpret_cast<const int4*>(sr));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) sv[e] = e < n ? sr[e] : int16_t(0);
      }
    }
    alignas(16) int16_t o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      o[e] = int16_t(clamp_i64(rescale_i64_signed(acc[e], prob_frac) + sv[e], -32768, 32767));
    int16_t* orow = out + t * ldo + h0;
    if (vec) {
      *reinterpret_cast<int4*>(orow) = *reinterpret_cast<const int4*>(o);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < n) orow[e] = o[e];
    }
  }
}

// ---- expert parallelism over peer memory ----------------------------------------
// Buffers of every rank, passed by value (pointers into peer memory).
struct EpPeers {
  int16_t* rows[MYL_XCHG_MAX];   // received rows [capacity][H]
  int32_t* ids[MYL_XCHG_MAX];    // their expert ids
  int32_t* src[MYL_XCHG_MAX];    // their origin: rank << 24 | pair index
  int32_t* count[MYL_XCHG_MAX];  // slot counter of the receiving rank
  int16_t* back[MYL_XCHG_MAX];   // returned expert outputs [pairs][H] of the home rank
};

// Rank owning expert e when E experts are split in contiguous shard ranges
// (the first E % world ranks hold one more).
__device__ __forceinline__ int ep_owner(int e, int E, int world) {
  const int base = E / world, extra = E % world;
  const int big = extra * (base + 1);
  return e < big ? e / (base + 1) : extra + (e - big) / max(base, 1);
}

// One warp per (token, choice) pair q = t * k + j: a slot on the owner's
// counter (system-scope atomic over NVLink), then the row (H int16), the
// expert id and the origin stored into the owner's buffers. A slot at or
// beyond capacity is not written and raises DEV_BAD_EXPERT.
__global__ void ep_dispatch_kernel(const int16_t* __restrict__ x, int64_t T, int64_t ldx, int64_t H,
                                   const int32_t* __restrict__ idx, int k, int E, int world,
                                   int rank, EpPeers peers, int64_t capacity, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  const int64_t P = T * k;
  for (int64_t q = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); q < P; q += warps) {
    const int e = idx[q];
    if (e < 0 || e >= E) {
      if (lane == 0) atomicCAS(err, 0, DEV_BAD_EXPERT);
      continue;
    }
    const int o = ep_owner(e, E, world);
    int slot = 0;
    if (lane == 0) slot = atomicAdd_system(peers.count[o], 1);
    slot = __shfl_sync(0xffffffffu, slot, 0);
    if (slot >= capacity) {
      if (lane == 0) atomicCAS(err, 0, DEV_BAD_EXPERT);
      continue;
    }
    const int16_t* xr = x + (q / k) * ldx;
    int16_t* dst = peers.rows[o] + int64_t(slot) * H;
    if ((H % 8) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
      for (int64_t c = lane; c < H / 8; c += 32)
        reinterpret_cast<int4*>(dst)[c] = __ldg(reinterpret_cast<const int4*>(xr) + c);
    } else {
      for (int64_t c = lane; c < H; c += 32) dst[c] = xr[c];
    }
    if (lane == 0) {
      peers.ids[o][slot] = e;
      peers.src[o][slot] = (rank << 24) | int32_t(q);
    }
  }
}

// Received row i < count returns to its origin: y[i] -> back[src >> 24] row
// (src & 0xFFFFFF), one warp per row.
__global__ void ep_return_kernel(const int16_t* __restrict__ y, int64_t count, int64_t H,
                                 const int32_t* __restrict__ src, EpPeers peers) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); i < count; i += warps) {
    const int32_t s = src[i];
    int16_t* dst = peers.back[s >> 24] + int64_t(s & 0xFFFFFF) * H;
    const int16_t* yr = y + i * H;
    if ((H % 8) == 0) {
      for (int64_t c = lane; c < H / 8; c += 32)
        reinterpret_cast<int4*>(dst)[c] = __ldg(reinterpret_cast<const int4*>(yr) + c);
    } else {
      for (int64_t c = lane; c < H; c += 32) dst[c] = yr[c];
    }
  }
}

}  // namespace myl
