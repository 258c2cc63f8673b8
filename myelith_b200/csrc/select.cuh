// select.cuh — greedy token selection over (a shard of) the LM head's int32
// logits, in a form that combines across vocab-parallel ranks with one int64
// max-reduction.
//
// argmax_int (INTEGER_LLM/kernels/src/sampling.rs:8-18) returns the lowest
// index among the maxima. For logit v at global vocab index i the key
//   key = v * 2^32 + (2^32 - 1 - i)
// orders first by v, then by the lower index, so argmax = the position of the
// largest key, and the largest key over all shards is the global answer:
//   token = 2^32 - 1 - (key & 0xFFFFFFFF),  logit = key >> 32.
#pragma once

#include "common.cuh"

namespace myl {

constexpr int SELECT_THREADS = 256;
constexpr int SELECT_CHUNK = SELECT_THREADS * 16;  // logits per block

__device__ __forceinline__ int64_t select_key(int32_t v, int64_t i) {
  return int64_t(v) * (int64_t(1) << 32) + (int64_t(0xFFFFFFFFll) - i);
}

__global__ void select_init_kernel(int64_t* __restrict__ keys, int64_t M) {
  pdl_wait();
  pdl_launch();
  for (int64_t m = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; m < M;
       m += int64_t(gridDim.x) * blockDim.x)
    keys[m] = INT64_MIN;  // below every key: a shard without logits never wins
}

// blockIdx.x: chunk of SELECT_CHUNK logits of row blockIdx.y (grid-stride over
// rows); the block's largest key goes to keys[row] with atomicMax.
__global__ void __launch_bounds__(SELECT_THREADS)
    select_keys_kernel(const int32_t* __restrict__ logits, int64_t M, int64_t V, int64_t ld,
                       int64_t index_base, int64_t* __restrict__ keys) {
  pdl_wait();
  pdl_launch();
  __shared__ int64_t part[SELECT_THREADS / 32];
  const int64_t j0 = int64_t(blockIdx.x) * SELECT_CHUNK;
  for (int64_t m = blockIdx.y; m < M; m += gridDim.y) {
    const int32_t* row = logits + m * ld;
    int64_t best = INT64_MIN;
#pragma unroll 4
    for (int t = 0; t < SELECT_CHUNK / SELECT_THREADS; ++t) {
      const int64_t j = j0 + int64_t(t) * SELECT_THREADS + threadIdx.x;
      if (j < V) best = max(best, select_key(__ldg(row + j), index_base + j));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      int64_t b = part[0];
      for (int w = 1; w < SELECT_THREADS / 32; ++w) b = max(b, part[w]);
      atomicMax(reinterpret_cast<long long*>(keys + m), static_cast<long long>(b));
    }
    __syncthreads();
  }
}

}  // namespace myl
