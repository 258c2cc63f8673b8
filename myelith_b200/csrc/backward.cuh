// backward.cuh — linear_backward (INTEGER_LLM/kernels/src/backward.rs:147-211)
// on CUDA cores, exact.
//
// For each token m and input column j:
//   acc[j] = sum_i (g[i] * W[i][j]) << (ref - w_shifts[i])      (i128)
//   gx[j]  = clamp_i32(rescale_i64(clamp_i64(rne_i128(acc[j], ref)), g_frac, gx_frac))
// with ref = max_i w_shifts[i]; and the outer product gw[i][j] = g[i] * x[j].
//
// The rows are visited in groups of equal shift (a permutation sorted by shift
// is made once per weight): inside a group the products are added in int64
// (|g*w| < 2^38, fewer than 2^24 rows), and each group sum enters the i128
// accumulator once, shifted by the group's alignment. Integer addition is
// exact, so this order gives the reference's sum.
#pragma once

#include "common.cuh"

namespace myl {

struct BwdGroup {
  int align;  // ref - shift of the group's rows (0..64)
  int r0, r1;  // rows [r0, r1) of the permutation
};

// RNE right shift of an i128 by s in [0, 127] (fixed_point.rs:155-169).
__device__ __forceinline__ __int128 rshift_rne_i128(__int128 v, int s) {
  if (s == 0) return v;
  const __int128 one = 1;
  const __int128 q = v >> s;
  const __int128 r = v & ((one << s) - 1);
  const __int128 h = one << (s - 1);
  return q + (((r > h) || (r == h && (q & 1))) ? 1 : 0);
}

constexpr int BWD_THREADS = 128;
constexpr int BWD_COLS = 4;  // input columns per thread (one 4-byte weight load per row)

// blockIdx.x covers BWD_THREADS * BWD_COLS input columns, blockIdx.y MT tokens.
template <int MT>
__global__ void __launch_bounds__(BWD_THREADS)
    linear_backward_gx_kernel(const int8_t* __restrict__ W, int64_t ldw, int64_t K,
                              const int32_t* __restrict__ perm, const BwdGroup* __restrict__ groups,
                              int ngroups, int ref, const int32_t* __restrict__ g, int64_t ldg,
                              int64_t M, int frac_shift, int32_t* __restrict__ gx, int64_t ldgx) {
  const int64_t j0 = (int64_t(blockIdx.x) * BWD_THREADS + threadIdx.x) * BWD_COLS;
  const int64_t m0 = int64_t(blockIdx.y) * MT;
  if (j0 >= K) return;
  __int128 acc[MT][BWD_COLS];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < BWD_COLS; ++c) acc[m][c] = 0;
  const int32_t* grow[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) grow[m] = g + (m0 + m < M ? m0 + m : M - 1) * ldg;
  for (int gi = 0; gi < ngroups; ++gi) {
    const BwdGroup grp = groups[gi];
    int64_t s[MT][BWD_COLS];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int c = 0; c < BWD_COLS; ++c) s[m][c] = 0;
    for (int r = grp.r0; r < grp.r1; ++r) {
      const int64_t i = perm[r];
      // j0 is a multiple of 4 and rows are 16-byte aligned: one 4-byte load
      const char4 w4 = *reinterpret_cast<const char4*>(W + i * ldw + j0);
      const int wv[BWD_COLS] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const int64_t gv = __ldg(grow[m] + i);
#pragma unroll
        for (int c = 0; c < BWD_COLS; ++c) s[m][c] += gv * wv[c];
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int c = 0; c < BWD_COLS; ++c) acc[m][c] += __int128(s[m][c]) << grp.align;
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m0 + m >= M) break;
#pragma unroll
    for (int c = 0; c < BWD_COLS; ++c) {
      if (j0 + c >= K) break;
      const __int128 q = rshift_rne_i128(acc[m][c], ref);
      const int64_t lim = q > __int128(INT64_MAX) ? INT64_MAX
                          : (q < __int128(INT64_MIN) ? INT64_MIN : int64_t(q));
      gx[(m0 + m) * ldgx + j0 + c] =
          int32_t(clamp_i64(rescale_i64_signed(lim, frac_shift), INT32_MIN, INT32_MAX));
    }
  }
}

// gw[m][i][j] = g[m][i] * x[m][j]: one block row per (m, i), threads over j.
__global__ void linear_backward_gw_kernel(const int32_t* __restrict__ g, int64_t ldg,
                                          const int16_t* __restrict__ x, int64_t ldx, int64_t M,
                                          int64_t N, int64_t K, int64_t* __restrict__ gw) {
  for (int64_t row = blockIdx.x; row < M * N; row += gridDim.x) {
    const int64_t m = row / N, i = row % N;
    const int64_t gv = g[m * ldg + i];
    const int16_t* xr = x + m * ldx;
    int64_t* out = gw + row * K;
    for (int64_t j = threadIdx.x; j < K; j += blockDim.x) out[j] = gv * int64_t(xr[j]);
  }
}

}  // namespace myl
