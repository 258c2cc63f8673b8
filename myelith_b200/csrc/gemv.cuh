// gemv.cuh — decode GEMV for W8A16 (M <= 4 activation rows), HBM-bound.
//
// Computes, per output channel r and activation row m,
//   acc = sum_k W[r,k] * x[m,k]      (exact, dot.rs:403-409)
// and applies the requant epilogue (linear.rs:61-68). Any summation order is
// allowed because the accumulation is exact (|acc| < 2^37 for K <= 32768;
// kernels/src/backends/cuda.rs:17-61 states the same contract).
//
// Layout and schedule
//  - W is the registered device copy: [N][ldw] int8, ldw a multiple of 16,
//    zero-padded beyond K. Each warp takes R output rows at a time (grid-stride
//    over rows, grid sized to the resident blocks); lane l streams the
//    16-byte chunks l, l+32, ... of each row with 128-bit non-coherent loads
//    that bypass L1 (a row's 32 lanes read 512 contiguous bytes).
//  - The activation slice x[:, k0:k0+KS] is staged once per block in shared
//    memory (zero-filled beyond K, split into two 16-byte planes per chunk),
//    so ragged K needs no padding by the caller.
//  - Products use dp2a (two int16 x int8 products per instruction) into int32
//    lanes that are flushed to int64 every U chunks (U*16 products of at most
//    2^22 each stay below 2^31). Lanes are combined with a 64-bit shuffle tree.
//  - gridDim.y > 1 splits K; each slice then writes exact int64 partial sums
//    (EPI_ACC_I64) that reduce_requant_kernel adds and requantises.
#pragma once

#include "common.cuh"

namespace myl {

// Weight rows are read once per call: they bypass L1 and enter L2 as the first
// lines to evict, so a decode step's weight stream (hundreds of MB per layer
// pass) does not push the KV cache, the activations, the LUTs and the kernels'
// code out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ int4 ldg_stream_v4(const void* p, uint64_t pol) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

// Asynchronous bulk prefetch of a contiguous weight range into L2 (no
// registers, no shared memory; bytes a multiple of 16). The GEMV kernels issue
// it for their first rows before the programmatic dependency wait: weights do
// not depend on the previous kernel (they are written only at registration,
// which synchronises), so their first bytes come while that kernel finishes.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, int64_t bytes) {
  while (bytes > 0) {
    const uint32_t b = uint32_t(bytes < 65536 ? bytes : 65536);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(b) : "memory");
    p = static_cast<const int8_t*>(p) + b;
    bytes -= b;
  }
}

__device__ __forceinline__ int dot16_dp2a(const int4 w, const int4 xa, const int4 xb, int acc) {
  // w bytes 4q..4q+3 pair with x words 2q (lo half of w) and 2q+1 (hi half).
  acc = __dp2a_lo(xa.x, w.x, acc);
  acc = __dp2a_hi(xa.y, w.x, acc);
  acc = __dp2a_lo(xa.z, w.y, acc);
  acc = __dp2a_hi(xa.w, w.y, acc);
  acc = __dp2a_lo(xb.x, w.z, acc);
  acc = __dp2a_hi(xb.y, w.z, acc);
  acc = __dp2a_lo(xb.z, w.w, acc);
  acc = __dp2a_hi(xb.w, w.w, acc);
  return acc;
}

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

// MT activation rows, R rows per warp, U chunks per lane in flight, KW warps
// sharing one row group (each takes 1/KW of the chunks; their exact partials
// are added through shared memory).
template <int MT, int R, int U, int KW>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_w8a16_kernel(const int8_t* __restrict__ W, int64_t ldw, int64_t N,
                      const int16_t* __restrict__ X, int64_t ldx, int64_t K, int64_t k_slice,
                      Epilogue ep, int64_t slice_stride) {
  {  // this warp's first rows into L2 (one K slice of R rows)
    const int warp = threadIdx.x >> 5;
    const int64_t row0 = int64_t(blockIdx.x) * (GEMV_WARPS / KW) * R + int64_t(warp / KW) * R;
    if ((threadIdx.x & 31) == 0 && warp % KW == 0 && row0 < N) {
      const int64_t k0 = int64_t(blockIdx.y) * k_slice;
      const int64_t kb = ((min(K - k0, k_slice) + 15) & ~int64_t(15));
      for (int j = 0; j < R && row0 + j < N; ++j) prefetch_l2_bulk(W + (row0 + j) * ldw + k0, kb);
    }
  }
  pdl_wait();
  pdl_launch();
  static_assert(GEMV_WARPS % KW == 0, "warps per row group");
  extern __shared__ __align__(16) int16_t xs[];  // [MT][KS]
  __shared__ int64_t red[GEMV_WARPS][R][MT];
  const int64_t k0 = int64_t(blockIdx.y) * k_slice;
  const int64_t kn = (K - k0) < k_slice ? (K - k0) : k_slice;  // valid elements in slice
  const int KS = int((kn + 15) & ~int64_t(15));                 // staged, multiple of 16
  const int nchunk = KS >> 4;

  // ---- stage x[:, k0:k0+KS] (zero beyond K) ---------------------------------
  // Layout per activation row: plane A = elements 16c..16c+7 of every chunk c,
  // then plane B = elements 16c+8..16c+15, so that lanes reading consecutive
  // chunks read consecutive 16-byte words (no shared-memory bank conflicts).
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(X) & 15) == 0) && (ldx % 8 == 0) && (k0 % 8 == 0);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const int16_t* xr = X + int64_t(m) * ldx + k0;
    int4* dst = reinterpret_cast<int4*>(xs + m * KS);
    const int halves = KS >> 3;  // 8-element halves
    for (int hh = threadIdx.x; hh < halves; hh += GEMV_THREADS) {
      const int i = hh * 8;  // first element of this half
      int4 v;
      if (vec_ok && i + 8 <= kn) {
        v = __ldg(reinterpret_cast<const int4*>(xr + i));
      } else {
        alignas(16) int16_t t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) t[e] = (i + e < kn) ? xr[i + e] : int16_t(0);
        v = *reinterpret_cast<const int4*>(t);
      }
      const int c = hh >> 1;
      dst[(hh & 1) * (KS >> 4) + c] = v;
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Epilogue e = ep;
  if (e.mode == EPI_ACC_I64)
    e.y = static_cast<int64_t*>(e.y) + int64_t(blockIdx.y) * slice_stride;
  constexpr int GROUPS = GEMV_WARPS / KW;  // row groups per block
  const int rg = warp / KW, kw = warp % KW;
  const int cpw = (nchunk + KW - 1) / KW;  // chunks per warp of a row group
  const int c_begin = kw * cpw, c_end = min(nchunk, c_begin + cpw);
  const int64_t block_rows = int64_t(GROUPS) * R;
  const int64_t row_step = int64_t(gridDim.x) * block_rows;

  // Grid-stride loop over row groups (uniform across the block: the grid is
  // sized to the resident blocks, so x is staged once per block).
  for (int64_t base = int64_t(blockIdx.x) * block_rows; base < N; base += row_step) {
    const int64_t row0 = base + int64_t(rg) * R;
    int64_t acc[R][MT];
#pragma unroll
    for (int j = 0; j < R; ++j)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[j][m] = 0;

    const int8_t* wrow[R];
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int64_t r = (row0 + j < N) ? row0 + j : N - 1;  // clamp: duplicate rows are not stored
      wrow[j] = W + r * ldw + k0;
    }

    const uint64_t pol = l2_evict_first_policy();
    for (int c = c_begin + lane; c < c_end; c += 32 * U) {
      int4 wv[U][R];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int cc = c + 32 * u;
#pragma unroll
        for (int j = 0; j < R; ++j)
          wv[u][j] = (cc < c_end) ? ldg_stream_v4(wrow[j] + cc * 16, pol) : make_int4(0, 0, 0, 0);
      }
      int a32[R][MT];
#pragma unroll
      for (int j = 0; j < R; ++j)
#pragma unroll
        for (int m = 0; m < MT; ++m) a32[j][m] = 0;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int cc = c + 32 * u;
        if (cc < c_end) {
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const int4* xp = reinterpret_cast<const int4*>(xs + m * KS);
            const int4 xa = xp[cc], xb = xp[nchunk + cc];
#pragma unroll
            for (int j = 0; j < R; ++j) a32[j][m] = dot16_dp2a(wv[u][j], xa, xb, a32[j][m]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < R; ++j)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[j][m] += a32[j][m];
    }

    // ---- warp reduction (exact, any order), row-group reduction, epilogue ----
#pragma unroll
    for (int j = 0; j < R; ++j)
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        int64_t v = acc[j][m];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        acc[j][m] = v;
      }
    if (KW > 1) {
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < R; ++j)
#pragma unroll
          for (int m = 0; m < MT; ++m) red[warp][j][m] = acc[j][m];
      }
      __syncthreads();
      if (kw == 0) {
#pragma unroll
        for (int j = 0; j < R; ++j)
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            int64_t v = 0;
#pragma unroll
            for (int t = 0; t < KW; ++t) v += red[warp + t][j][m];
            acc[j][m] = v;
          }
      }
      __syncthreads();
    }
    if (kw == 0) {
      if (e.mode == EPI_W16) {
        // Rows row0 (high byte) and row0 + 1 (low byte) of int16 row row0/2 (R == 2).
#pragma unroll
        for (int m = 0; m < MT; ++m)
          if (R == 2 && lane == m && row0 + 1 < N) w16_store(e, m, row0 >> 1, acc[0][m], acc[R - 1][m]);
      } else if (e.mode == EPI_SILU) {
        // Rows row0 (gate) and row0 + 1 (up) of channel pair row0/2 (R == 2).
#pragma unroll
        for (int m = 0; m < MT; ++m)
          if (R == 2 && lane == m && row0 + 1 < N) {
            const int32_t g = int32_t(requant_value(e, row0, acc[0][m]));
            const int32_t u = int32_t(requant_value(e, row0 + 1, acc[R - 1][m]));
            silu_store(e, m, row0 >> 1, silu_combine(e.silu, g, u));
          }
      } else {
#pragma unroll
        for (int j = 0; j < R; ++j)
#pragma unroll
          for (int m = 0; m < MT; ++m)
            if (lane == ((j * MT + m) & 31) && row0 + j < N) epilogue_store(e, m, row0 + j, acc[j][m]);
      }
    }
  }
}

// Balanced GEMV for few rows per warp: warp w of W warps finishes the whole
// row pairs [w*P/W, (w+1)*P/W) (P = ceil(N/2)), so no SM holds more pairs
// than another by more than one per warp, whatever N is; the weight loads of
// a pair are software-pipelined one batch ahead of the products. Used where
// the row-group kernel below would leave SMs with unequal block counts (long K
// and few rows, e.g. the 7B down projection).
// Epilogue of a finished row pair (rows 2p, 2p + 1; 2p + 1 may not exist)
// for activation row m: exact sums a0 (row 2p) and a1 (row 2p + 1).
__device__ __forceinline__ void pair_epilogue_m(const Epilogue& ep, int64_t m, int64_t p, int64_t N,
                                                int64_t a0, int64_t a1) {
  if (ep.mode == EPI_W16) {
    if (2 * p + 1 < N) w16_store(ep, m, p, a0, a1);
  } else if (ep.mode == EPI_SILU) {
    if (2 * p + 1 < N) {
      const int32_t g = int32_t(requant_value(ep, 2 * p, a0));
      const int32_t u = int32_t(requant_value(ep, 2 * p + 1, a1));
      silu_store(ep, m, p, silu_combine(ep.silu, g, u));
    }
  } else {
    epilogue_store(ep, m, 2 * p, a0);
    if (2 * p + 1 < N) epilogue_store(ep, m, 2 * p + 1, a1);
  }
}

template <int MT>
__device__ __forceinline__ void gemv_pair_epilogue(const Epilogue& ep, int64_t p, int64_t N,
                                                   const int64_t (&a)[2][MT]) {
#pragma unroll
  for (int m = 0; m < MT; ++m) pair_epilogue_m(ep, m, p, N, a[0][m], a[1][m]);
}

// The first batch of U chunks per lane of rows w0 and w1 from chunk c on.
template <int U>
__device__ __forceinline__ void gemv_pair_first_batch(const int8_t* __restrict__ w0, const int8_t* __restrict__ w1,
                                                      int c, int c1, uint64_t pol, int4 (&cur)[U][2]) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int cc = c + 32 * u;
    cur[u][0] = cc < c1 ? ldg_stream_v4(w0 + cc * 16, pol) : make_int4(0, 0, 0, 0);
    cur[u][1] = cc < c1 ? ldg_stream_v4(w1 + cc * 16, pol) : make_int4(0, 0, 0, 0);
  }
}

// Exact sums of chunks [c0, c1) of rows w0 and w1 against the staged x,
// loads software-pipelined one batch of U chunks ahead of the products
// (the first batch already in cur when `loaded`).
template <int MT, int U>
__device__ __forceinline__ void gemv_pair_sums(const int8_t* __restrict__ w0,
                                               const int8_t* __restrict__ w1,
                                               const int16_t* __restrict__ xs, int KS, int C, int c0,
                                               int c1, int lane, int64_t (&a)[2][MT], int4 (&cur)[U][2],
                                               bool loaded) {
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int m = 0; m < MT; ++m) a[j][m] = 0;
  int4 nxt[U][2];
  int c = c0 + lane;
  const uint64_t pol = l2_evict_first_policy();
  if (!loaded) gemv_pair_first_batch<U>(w0, w1, c, c1, pol, cur);
  for (; c < c1; c += 32 * U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int cc = c + 32 * (U + u);
      nxt[u][0] = cc < c1 ? ldg_stream_v4(w0 + cc * 16, pol) : make_int4(0, 0, 0, 0);
      nxt[u][1] = cc < c1 ? ldg_stream_v4(w1 + cc * 16, pol) : make_int4(0, 0, 0, 0);
    }
    int a32[2][MT];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int m = 0; m < MT; ++m) a32[j][m] = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int cc = c + 32 * u;
      if (cc < c1) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const int4* xp = reinterpret_cast<const int4*>(xs + m * KS);
          const int4 xa = xp[cc], xb = xp[C + cc];
          a32[0][m] = dot16_dp2a(cur[u][0], xa, xb, a32[0][m]);
          a32[1][m] = dot16_dp2a(cur[u][1], xa, xb, a32[1][m]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int m = 0; m < MT; ++m) a[j][m] += a32[j][m];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      cur[u][0] = nxt[u][0];
      cur[u][1] = nxt[u][1];
    }
  }
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      int64_t v = a[j][m];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      a[j][m] = v;
    }
}

template <int MT, int U>
__global__ void __launch_bounds__(GEMV_THREADS, 2)
    gemv_balanced_kernel(const int8_t* __restrict__ W, int64_t ldw, int64_t N,
                         const int16_t* __restrict__ X, int64_t ldx, int64_t K, Epilogue ep) {
  const int KS = int((K + 15) & ~int64_t(15));
  const int C = KS >> 4;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = int64_t(gridDim.x) * GEMV_WARPS;
  const int64_t wid = int64_t(blockIdx.x) * GEMV_WARPS + (threadIdx.x >> 5);
  const int64_t npairs = (N + 1) / 2;
  const int64_t p_begin = wid * npairs / nwarps, p_end = (wid + 1) * npairs / nwarps;
  // this warp's first row pair: the rest into L2 and the first batch into
  // registers before the programmatic dependency wait
  int4 cur[U][2];
  if (p_begin < p_end) {
    const int8_t* w0 = W + 2 * p_begin * ldw;
    const int8_t* w1 = (2 * p_begin + 1 < N) ? w0 + ldw : w0;
    if (lane == 0) prefetch_l2_bulk(w0, (2 * p_begin + 1 < N ? 2 : 1) * ldw);
    gemv_pair_first_batch<U>(w0, w1, lane, C, l2_evict_first_policy(), cur);
  }
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(16) int16_t xs[];  // [MT][KS], two 16-byte planes per chunk
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(X) & 15) == 0) && (ldx % 8 == 0);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const int16_t* xr = X + int64_t(m) * ldx;
    int4* dst = reinterpret_cast<int4*>(xs + m * KS);
    for (int hh = threadIdx.x; hh < (KS >> 3); hh += GEMV_THREADS) {
      const int i = hh * 8;
      int4 v;
      if (vec_ok && i + 8 <= K) {
        v = __ldg(reinterpret_cast<const int4*>(xr + i));
      } else {
        alignas(16) int16_t t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) t[e] = (i + e < K) ? xr[i + e] : int16_t(0);
        v = *reinterpret_cast<const int4*>(t);
      }
      dst[(hh & 1) * C + (hh >> 1)] = v;
    }
  }
  __syncthreads();

  for (int64_t p = p_begin; p < p_end; ++p) {
    const int64_t r1 = (2 * p + 1 < N) ? 2 * p + 1 : 2 * p;  // odd N: duplicate, not stored
    int64_t a[2][MT];
    gemv_pair_sums<MT, U>(W + 2 * p * ldw, W + r1 * ldw, xs, KS, C, 0, C, lane, a, cur, p == p_begin);
    if (lane == 0) gemv_pair_epilogue<MT>(ep, p, N, a);
  }
}

// Streaming GEMV for one activation row and rows of at most 32 * CPL
// chunks (K <= 512 * CPL; CPL <= 8 keeps the three slots in registers): warp w finishes the whole row pairs
// [w*P/W, (w+1)*P/W) one row at a time, each row's CPL chunks per lane loaded
// in one batch, and the loads of the next two rows in flight while a row's
// products run (three register slots: the pair's even and odd row and the next
// pair's even row). Two blocks per SM, 16 warps: ~7 KB of weight loads in
// flight per warp for K = 3584.
template <int CPL>
__device__ __forceinline__ void gemv_row_load(int4 (&v)[CPL], const int8_t* __restrict__ row, int C, int lane,
                                              uint64_t pol) {
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < C ? ldg_stream_v4(row + 16 * c, pol) : make_int4(0, 0, 0, 0);
  }
}

template <int CPL>
__device__ __forceinline__ int64_t gemv_row_dot(const int4 (&v)[CPL], const int4* __restrict__ xa,
                                                const int4* __restrict__ xb, int C, int lane) {
  // four independent dp2a chains (CPL <= 31 chunks of 16 products of at most
  // 2^22: every partial is exact in int32)
  int a[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    if (c < C) {
      const int4 w = v[i], x0 = xa[c], x1 = xb[c];
      int& p = a[2 * (i & 1)];
      int& q = a[2 * (i & 1) + 1];
      p = __dp2a_lo(x0.x, w.x, p);
      q = __dp2a_lo(x1.x, w.z, q);
      p = __dp2a_hi(x0.y, w.x, p);
      q = __dp2a_hi(x1.y, w.z, q);
      p = __dp2a_lo(x0.z, w.y, p);
      q = __dp2a_lo(x1.z, w.w, q);
      p = __dp2a_hi(x0.w, w.y, p);
      q = __dp2a_hi(x1.w, w.w, q);
    }
  }
  return int64_t(a[0]) + a[1] + a[2] + a[3];
}

template <int CPL>
__global__ void __launch_bounds__(GEMV_THREADS, 2)
    gemv_stream_kernel(const int8_t* __restrict__ W, int64_t ldw, int64_t N,
                       const int16_t* __restrict__ X, int64_t K, Epilogue ep) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = int64_t(gridDim.x) * GEMV_WARPS;
  const int64_t w = int64_t(blockIdx.x) * GEMV_WARPS + (threadIdx.x >> 5);
  const int64_t np = (N + 1) / 2;
  const int64_t p_begin = w * np / nw, p_end = (w + 1) * np / nw;
  const uint64_t pol = l2_evict_first_policy();
  const int KS = int((K + 15) & ~int64_t(15));
  const int C = KS >> 4;
  // the first pair's rows do not depend on the previous kernel: loads issued
  // before the programmatic dependency wait
  int4 e[CPL], o[CPL], n[CPL];
  auto row_ptr = [&](int64_t r) { return W + (r < N ? r : N - 1) * ldw; };  // odd N: duplicate, not stored
  if (p_begin < p_end) {
    gemv_row_load<CPL>(e, row_ptr(2 * p_begin), C, lane, pol);
    gemv_row_load<CPL>(o, row_ptr(2 * p_begin + 1), C, lane, pol);
  }
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(16) int16_t xs[];  // [KS], two 16-byte planes per chunk
  {
    const bool vec_ok = (reinterpret_cast<uintptr_t>(X) & 15) == 0;
    int4* dst = reinterpret_cast<int4*>(xs);
    for (int hh = threadIdx.x; hh < (KS >> 3); hh += GEMV_THREADS) {
      const int i = hh * 8;
      int4 v;
      if (vec_ok && i + 8 <= K) {
        v = __ldg(reinterpret_cast<const int4*>(X + i));
      } else {
        alignas(16) int16_t t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = (i + q < K) ? X[i + q] : int16_t(0);
        v = *reinterpret_cast<const int4*>(t);
      }
      dst[(hh & 1) * C + (hh >> 1)] = v;
    }
  }
  __syncthreads();
  const int4* xa = reinterpret_cast<const int4*>(xs);
  const int4* xb = xa + C;
  for (int64_t p = p_begin; p < p_end; ++p) {
    const bool more = p + 1 < p_end;
    if (more) gemv_row_load<CPL>(n, row_ptr(2 * p + 2), C, lane, pol);
    int64_t a[2][1];
    a[0][0] = gemv_row_dot<CPL>(e, xa, xb, C, lane);
    if (more) gemv_row_load<CPL>(e, row_ptr(2 * p + 3), C, lane, pol);  // e is free: the next odd row
    a[1][0] = gemv_row_dot<CPL>(o, xa, xb, C, lane);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      a[0][0] += __shfl_xor_sync(0xffffffffu, a[0][0], off);
      a[1][0] += __shfl_xor_sync(0xffffffffu, a[1][0], off);
    }
    if (lane == 0) gemv_pair_epilogue<1>(ep, p, N, a);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      o[i] = e[i];
      e[i] = n[i];
    }
  }
}

// GEMV for one activation row and long rows (the down projections): a block
// takes GKS_PAIRS row pairs at a time and each of its warps a quarter of their
// K range, so a weight matrix of few rows still spreads evenly over every
// warp; the quarters' exact sums meet in shared memory. Each warp's next loads
// go out right after its products, before the reduction and the epilogue;
// the first ones before the programmatic dependency wait.
constexpr int GKS_Q = 4;                           // K quarters per row pair
constexpr int GKS_PAIRS = GEMV_WARPS / GKS_Q;      // row pairs per block step

template <int CPL>
__device__ __forceinline__ void gks_load(int4 (&v)[CPL], const int8_t* __restrict__ row, int c0, int c1, int lane,
                                         uint64_t pol) {
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = c0 + lane + 32 * i;
    v[i] = c < c1 ? ldg_stream_v4(row + 16 * c, pol) : make_int4(0, 0, 0, 0);
  }
}

template <int CPL>
__device__ __forceinline__ int64_t gks_dot(const int4 (&v)[CPL], const int4* __restrict__ xa,
                                           const int4* __restrict__ xb, int c0, int c1, int lane) {
  int a[4] = {0, 0, 0, 0};  // CPL <= 31 chunks: every partial exact in int32
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = c0 + lane + 32 * i;
    if (c < c1) {
      const int4 w = v[i], x0 = xa[c], x1 = xb[c];
      int& p = a[2 * (i & 1)];
      int& q = a[2 * (i & 1) + 1];
      p = __dp2a_lo(x0.x, w.x, p);
      q = __dp2a_lo(x1.x, w.z, q);
      p = __dp2a_hi(x0.y, w.x, p);
      q = __dp2a_hi(x1.y, w.z, q);
      p = __dp2a_lo(x0.z, w.y, p);
      q = __dp2a_lo(x1.z, w.w, q);
      p = __dp2a_hi(x0.w, w.y, p);
      q = __dp2a_hi(x1.w, w.w, q);
    }
  }
  return int64_t(a[0]) + a[1] + a[2] + a[3];
}

template <int CPL>
__global__ void __launch_bounds__(GEMV_THREADS, 2)
    gemv_ksplit_kernel(const int8_t* __restrict__ W, int64_t ldw, int64_t N,
                       const int16_t* __restrict__ X, int64_t K, Epilogue ep) {
  __shared__ int64_t red[GEMV_WARPS][2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = warp % GKS_Q, pw = warp / GKS_Q;
  const int KS = int((K + 15) & ~int64_t(15));
  const int C = KS >> 4;
  const int c0 = q * C / GKS_Q, c1 = (q + 1) * C / GKS_Q;  // this warp's chunks, <= 32 * CPL of them
  const int64_t np = (N + 1) / 2;
  const int64_t pstep = int64_t(gridDim.x) * GKS_PAIRS;
  const uint64_t pol = l2_evict_first_policy();
  auto row_ptr = [&](int64_t r) { return W + (r < N ? r : N - 1) * ldw; };  // odd N: duplicate, not stored
  int4 e[CPL], o[CPL];
  int64_t p = int64_t(blockIdx.x) * GKS_PAIRS + pw;
  if (p < np) {  // weights do not depend on the previous kernel
    gks_load<CPL>(e, row_ptr(2 * p), c0, c1, lane, pol);
    gks_load<CPL>(o, row_ptr(2 * p + 1), c0, c1, lane, pol);
  }
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(16) int16_t xs[];  // [KS], two 16-byte planes per chunk
  {
    const bool vec_ok = (reinterpret_cast<uintptr_t>(X) & 15) == 0;
    int4* dst = reinterpret_cast<int4*>(xs);
    for (int hh = threadIdx.x; hh < (KS >> 3); hh += GEMV_THREADS) {
      const int i = hh * 8;
      int4 v;
      if (vec_ok && i + 8 <= K) {
        v = __ldg(reinterpret_cast<const int4*>(X + i));
      } else {
        alignas(16) int16_t t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) t[u] = (i + u < K) ? X[i + u] : int16_t(0);
        v = *reinterpret_cast<const int4*>(t);
      }
      dst[(hh & 1) * C + (hh >> 1)] = v;
    }
  }
  __syncthreads();
  const int4* xa = reinterpret_cast<const int4*>(xs);
  const int4* xb = xa + C;
  for (int64_t base = int64_t(blockIdx.x) * GKS_PAIRS; base < np; base += pstep) {  // uniform per block
    p = base + pw;
    int64_t s0 = 0, s1 = 0;
    if (p < np) {
      s0 = gks_dot<CPL>(e, xa, xb, c0, c1, lane);
      s1 = gks_dot<CPL>(o, xa, xb, c0, c1, lane);
    }
    const int64_t pn = p + pstep;
    if (pn < np) {
      gks_load<CPL>(e, row_ptr(2 * pn), c0, c1, lane, pol);
      gks_load<CPL>(o, row_ptr(2 * pn + 1), c0, c1, lane, pol);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, off);
      s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    }
    if (lane == 0) {
      red[warp][0] = s0;
      red[warp][1] = s1;
    }
    __syncthreads();
    if (q == 0 && lane == 0 && p < np) {
      int64_t a[2][1] = {{0}, {0}};
#pragma unroll
      for (int k = 0; k < GKS_Q; ++k) {
        a[0][0] += red[warp + k][0];
        a[1][0] += red[warp + k][1];
      }
      gemv_pair_epilogue<1>(ep, p, N, a);
    }
    __syncthreads();  // red is rewritten next step
  }
}

// xsum[m] = sum_k x[m][k] (int64), one warp per row: the EPI_W16 correction.
__global__ void x_row_sums_kernel(const int16_t* __restrict__ X, int64_t ldx, int64_t M, int64_t K,
                                  int64_t* __restrict__ xsum) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t m = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); m < M; m += warps) {
    const int16_t* xr = X + m * ldx;
    int64_t s = 0;
    for (int64_t k = lane; k < K; k += 32) s += xr[k];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) xsum[m] = s;
  }
}

// Sums nsplit exact int64 partial slices [nsplit][M][N] (slice_stride apart)
// and applies the epilogue. Summation order is irrelevant (exact integers).
__global__ void reduce_requant_kernel(const int64_t* __restrict__ part, int nsplit,
                                      int64_t slice_stride, int64_t M, int64_t N, Epilogue ep) {
  pdl_wait();
  pdl_launch();
  if (ep.mode == EPI_W16) {  // one thread per (token, int16 weight row)
    const int64_t I = N / 2, total = M * I;
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += int64_t(gridDim.x) * blockDim.x) {
      const int64_t m = e / I, i = e % I;
      int64_t ah = 0, al = 0;
      for (int k = 0; k < nsplit; ++k) {
        ah += part[k * slice_stride + m * N + 2 * i];
        al += part[k * slice_stride + m * N + 2 * i + 1];
      }
      w16_store(ep, m, i, ah, al);
    }
    return;
  }
  if (ep.mode == EPI_SILU) {  // one thread per (token, channel pair)
    const int64_t I = N / 2, total = M * I;
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += int64_t(gridDim.x) * blockDim.x) {
      const int64_t m = e / I, i = e % I;
      int64_t ag = 0, au = 0;
      for (int k = 0; k < nsplit; ++k) {
        ag += part[k * slice_stride + m * N + 2 * i];
        au += part[k * slice_stride + m * N + 2 * i + 1];
      }
      const int32_t g = int32_t(requant_value(ep, 2 * i, ag));
      const int32_t u = int32_t(requant_value(ep, 2 * i + 1, au));
      silu_store(ep, m, i, silu_combine(ep.silu, g, u));
    }
    return;
  }
  if (N < int64_t(blockDim.x)) {
    // Narrow rows (a router's few experts): threads walk the flat
    // (row, column) index so that no thread of a block idles.
    const int64_t total = M * N;
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += int64_t(gridDim.x) * blockDim.x) {
      const int64_t m = e / N, n = e - m * N;
      int64_t s = 0;
      for (int i = 0; i < nsplit; ++i) s += part[i * slice_stride + m * N + n];
      epilogue_store(ep, m, n, s);
    }
    return;
  }
  // Blocks walk (row, 256-column segment) pairs, threads the columns of a
  // segment: one 64-bit division per segment instead of per element.
  const int64_t segs = (N + blockDim.x - 1) / blockDim.x;
  for (int64_t g = blockIdx.x; g < M * segs; g += gridDim.x) {
    const int64_t m = g / segs, n = (g % segs) * blockDim.x + threadIdx.x;
    if (n >= N) continue;
    int64_t s = 0;
    for (int i = 0; i < nsplit; ++i) s += part[i * slice_stride + m * N + n];
    epilogue_store(ep, m, n, s);
  }
}

// Exchange reduce of a row-parallel layer (myl_exchange_reduce_dev): thread g
// sums 8 consecutive columns of one of this rank's rows over the world slabs
// of recv (exact int64), requantises them and stores the 8 results with one
// 16-byte (int16) or two (int32) stores into every rank's output buffer.
// N and ep.ldy are multiples of 8.
__global__ void xchg_reduce_kernel(const int64_t* __restrict__ recv, int world, int64_t slab,
                                   int64_t rows, int64_t N, Epilogue ep) {
  const int64_t per_row = N >> 3, total = rows * per_row;
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = g / per_row, n0 = (g - m * per_row) * 8;
    int64_t s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = 0;
    for (int r = 0; r < world; ++r) {
      const longlong2* p = reinterpret_cast<const longlong2*>(recv + r * slab + m * N + n0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const longlong2 v = __ldg(p + q);
        s[2 * q] += v.x;
        s[2 * q + 1] += v.y;
      }
    }
    int32_t v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = int32_t(requant_value(ep, n0 + j, s[j]));
    const int64_t idx = (ep.xg_row0 + m) * ep.ldy + n0;
    if (ep.out_i32) {
      const int4 a = make_int4(v[0], v[1], v[2], v[3]), b = make_int4(v[4], v[5], v[6], v[7]);
      for (int o = 0; o < ep.xg_world; ++o) {
        int4* d = reinterpret_cast<int4*>(static_cast<int32_t*>(ep.xg_dst[o]) + idx);
        d[0] = a;
        d[1] = b;
      }
    } else {
      int4 h;
      h.x = int((uint32_t(uint16_t(v[0]))) | (uint32_t(uint16_t(v[1])) << 16));
      h.y = int((uint32_t(uint16_t(v[2]))) | (uint32_t(uint16_t(v[3])) << 16));
      h.z = int((uint32_t(uint16_t(v[4]))) | (uint32_t(uint16_t(v[5])) << 16));
      h.w = int((uint32_t(uint16_t(v[6]))) | (uint32_t(uint16_t(v[7])) << 16));
      for (int o = 0; o < ep.xg_world; ++o)
        *reinterpret_cast<int4*>(static_cast<int16_t*>(ep.xg_dst[o]) + idx) = h;
    }
  }
}

// Barrier of the ranks of a peer-memory exchange: thread t < world stores
// `epoch` into rank t's flag word for this rank (system-scope release after
// a system fence, so everything this rank's earlier kernels wrote is visible
// first), then waits until this rank's flag word of sender t has reached the
// epoch (acquire; bounded: a peer that does not arrive within timeout_ns
// sets DEV_WAIT_PEER and the kernel returns).
struct XchgFlags {
  unsigned long long* p[MYL_XCHG_MAX];  // each rank's flag words (one per sender)
};

__global__ void xchg_barrier_kernel(XchgFlags flags, int world, int rank, unsigned long long epoch,
                                    int* err, uint64_t timeout_ns) {
  const int t = threadIdx.x;
  if (t >= world) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flags.p[t] + rank), "l"(epoch) : "memory");
  const unsigned long long* mine = flags.p[rank] + t;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
    if (v >= epoch) return;
    if (globaltimer_ns() - t0 > timeout_ns) {
      atomicCAS(err, 0, DEV_WAIT_PEER);
      return;
    }
    __nanosleep(64);
  }
}

}  // namespace myl
