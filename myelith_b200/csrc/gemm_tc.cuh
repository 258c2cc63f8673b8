// gemm_tc.cuh — W8A16 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// The reference has no batched GEMM: prefill calls the per-token GEMV
// (INTEGER_LLM/runtime/src/generate.rs:29-31), so every output element here
// must equal linear.rs:61-68 for its (token, channel).
//
// Split-byte exactness. The tensor core multiplies 8-bit operands, the
// activations are int16. Each activation is split as x = 256*hi + lo with
// hi = x >> 8 (signed byte) and lo = x & 255 (unsigned byte), so
//   sum_k w*x = 256 * sum_k w*hi + sum_k w*lo.
// Two kind::i8 MMAs (s8 x s8 and s8 x u8) accumulate the two sums in two int32
// TMEM accumulators. |w*hi| <= 128*128 = 2^14 and |w*lo| <= 128*255 < 2^15, so
// both int32 sums are exact for K <= 65536 (the host enforces K <= 65536 per
// launch; longer K is split into slices whose exact int64 partials are added).
// The epilogue forms 256*S_hi + S_lo in int64, which is the reference's exact
// i64 accumulator, and applies the requant once (fixed_point.rs:184-191).
// The tensor pipe therefore does 2x the algorithmic MACs.
//
// Schedule (one output tile per CTA, 192 threads):
//   warp 0        TMA producer: W tile + X_hi tile + X_lo tile per 128-byte K
//                 step into a STAGES-deep ring of 128B-swizzled smem stages.
//   warp 1        TMEM allocator; lane 0 issues the MMAs (4 K-steps of 32 x 2).
//   warps 2..5    epilogue: tcgen05.ld of both accumulators, combine, requant,
//                 store. Warp w reads TMEM lanes 32*(w%4)..32*(w%4)+31.
// SWAP=false: MMA A = X (128 tokens), B = W (BN channels); lanes = tokens.
// SWAP=true : MMA A = W (128 channels), B = X (BN tokens); lanes = channels
//             (small-M decode / prefill chunks: the weight fills the MMA M).
//
// Every mbarrier wait is bounded (timeout_ns, globaltimer); a wait that runs
// out writes an error code to *err, the CTA drains its own TMA copies and
// MMAs (bounded again), frees TMEM and returns.
#pragma once

#include "common.cuh"

namespace myl {

constexpr int TC_BK = 128;  // K bytes per stage = one 128-byte swizzle row
constexpr int TC_THREADS = 192;

template <int BN, bool SWAP, int STAGES>
struct TcCfg {
  static constexpr int ROWS_W = SWAP ? 128 : BN;
  static constexpr int ROWS_X = SWAP ? BN : 128;
  static constexpr int W_BYTES = ROWS_W * TC_BK;
  static constexpr int X_BYTES = ROWS_X * TC_BK;
  static constexpr int STAGE_BYTES = W_BYTES + 2 * X_BYTES;
  static constexpr int ACC_COLS = 2 * BN;  // hi accumulator | lo accumulator
  static constexpr int TMEM_COLS = ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128
                                   : ACC_COLS <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256,
                "MMA N (M=128) is a multiple of 16 in [16,256]; the epilogue reads 32 columns at a time");
  static_assert(ACC_COLS <= 512, "TMEM has 512 columns");
  // A: SWAP ? W (s8) : X_hi/X_lo; B: SWAP ? X_hi/X_lo : W (s8).
  static constexpr uint32_t IDESC_HI = idesc_i8(128, BN, true, true);
  static constexpr uint32_t IDESC_LO = SWAP ? idesc_i8(128, BN, true, false) : idesc_i8(128, BN, false, true);
};

struct TcSmemCtl {
  uint64_t full[16];
  uint64_t empty[16];
  uint64_t accum_full;
  uint64_t never;  // test hook: nothing ever arrives here
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void tc_fail(int* err, volatile int* abort, int code) {
  *abort = 1;
  atomicCAS(err, 0, code);
}

template <int BN, bool SWAP, int STAGES>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_w8a16_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_xhi,
                         const __grid_constant__ CUtensorMap tm_xlo, int64_t M, int64_t N,
                         int k_tiles_total, int k_tiles_per_split, Epilogue ep,
                         int64_t slice_stride, int* err, uint64_t timeout_ns, int inject_fault) {
  using Cfg = TcCfg<BN, SWAP, STAGES>;
  static_assert(STAGES <= 16, "barrier array size");
  extern __shared__ uint8_t dyn_smem[];
  __shared__ TcSmemCtl ctl;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t smem_base = (smem_addr(dyn_smem) + 1023u) & ~1023u;
  auto sm_w = [&](int s) { return smem_base + uint32_t(s) * Cfg::STAGE_BYTES; };
  auto sm_xh = [&](int s) { return sm_w(s) + Cfg::W_BYTES; };
  auto sm_xl = [&](int s) { return sm_w(s) + Cfg::W_BYTES + Cfg::X_BYTES; };

  const int64_t n0 = SWAP ? int64_t(blockIdx.x) * 128 : int64_t(blockIdx.x) * BN;
  const int64_t m0 = SWAP ? int64_t(blockIdx.y) * BN : int64_t(blockIdx.y) * 128;
  const int kt0 = int(blockIdx.z) * k_tiles_per_split;
  const int kt1 = min(kt0 + k_tiles_per_split, k_tiles_total);
  const int nkt = kt1 - kt0;  // >= 1, guaranteed by the host
  volatile int* abort = &ctl.abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&ctl.full[s]), 1);
      mbar_init(smem_addr(&ctl.empty[s]), 1);
    }
    mbar_init(smem_addr(&ctl.accum_full), 1);
    mbar_init(smem_addr(&ctl.never), 1);
    ctl.abort = 0;
    fence_barrier_init();
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_xhi);
    prefetch_tensormap(&tm_xlo);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(&ctl.tmem_base), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nkt; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = uint32_t(i / STAGES) & 1u;
        if (!mbar_wait_bounded(smem_addr(&ctl.empty[s]), ph ^ 1u, timeout_ns, abort)) {
          tc_fail(err, abort, DEV_WAIT_PRODUCER);
          break;
        }
        const uint32_t fb = smem_addr(&ctl.full[s]);
        mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
        const int32_t kx = (kt0 + i) * TC_BK;
        tma_load_2d(sm_w(s), &tm_w, fb, kx, int32_t(n0));
        tma_load_2d(sm_xh(s), &tm_xhi, fb, kx, int32_t(m0));
        tma_load_2d(sm_xl(s), &tm_xlo, fb, kx, int32_t(m0));
        issued = i + 1;
      }
      if (*abort) {
        // Drain: the last load issued into each stage must land before exit.
        for (int s = 0; s < STAGES && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / STAGES) * STAGES;
          if (!mbar_wait_bounded(smem_addr(&ctl.full[s]), uint32_t(last / STAGES) & 1u, timeout_ns,
                                 nullptr))
            atomicCAS(err, 0, DEV_WAIT_DRAIN);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t d_hi = tmem, d_lo = tmem + BN;
      for (int i = 0; i < nkt; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = uint32_t(i / STAGES) & 1u;
        if (!mbar_wait_bounded(smem_addr(&ctl.full[s]), ph, timeout_ns, abort)) {
          tc_fail(err, abort, DEV_WAIT_MMA);
          break;
        }
        tc_fence_after();
        const uint32_t aw = sm_w(s), axh = sm_xh(s), axl = sm_xl(s);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 32; ++kk) {
          const uint32_t off = uint32_t(kk) * 32u;
          const uint64_t dw = smem_desc_k_sw128(aw + off);
          const uint64_t dxh = smem_desc_k_sw128(axh + off);
          const uint64_t dxl = smem_desc_k_sw128(axl + off);
          const uint32_t accum = (i > 0 || kk > 0) ? 1u : 0u;
          if (SWAP) {
            mma_i8(d_hi, dw, dxh, Cfg::IDESC_HI, accum);
            mma_i8(d_lo, dw, dxl, Cfg::IDESC_LO, accum);
          } else {
            mma_i8(d_hi, dxh, dw, Cfg::IDESC_HI, accum);
            mma_i8(d_lo, dxl, dw, Cfg::IDESC_LO, accum);
          }
        }
        mma_commit(smem_addr(&ctl.empty[s]));  // frees the stage when these MMAs finish
      }
      mma_commit(smem_addr(&ctl.accum_full));
      // The issuer itself sees every MMA finish before TMEM can be released.
      if (!mbar_wait_bounded(smem_addr(&ctl.accum_full), 0u, timeout_ns, nullptr))
        atomicCAS(err, 0, DEV_WAIT_DRAIN);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;
    bool ok = mbar_wait_bounded(smem_addr(&ctl.accum_full), 0u, timeout_ns, abort);
    int code = DEV_WAIT_EPILOGUE;
    if (ok && inject_fault) {
      ok = mbar_wait_bounded(smem_addr(&ctl.never), 0u, timeout_ns, nullptr);
      code = DEV_WAIT_INJECTED;
    }
    if (!ok) {
      tc_fail(err, abort, code);
    } else if (!*abort) {
      tc_fence_after();
      const int row = q * 32 + lane;
      const uint32_t tq = tmem + (uint32_t(q * 32) << 16);
      Epilogue e = ep;
      if (e.mode == EPI_ACC_I64)
        e.y = static_cast<int64_t*>(e.y) + int64_t(blockIdx.z) * slice_stride;
      ChannelRequant rq;
      if (SWAP && n0 + row < N) rq.load(e, n0 + row);
      const bool vec16 = !SWAP && e.mode != EPI_ACC_I64 && !e.out_i32 &&
                         ((reinterpret_cast<uintptr_t>(e.y) & 15) == 0) && (e.ldy % 8 == 0);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t hi[32], lo[32];
        tmem_ld_32x32b_x32(tq + c, hi);
        tmem_ld_32x32b_x32(tq + BN + c, lo);
        tmem_ld_wait();
        if (SWAP) {
          const int64_t n = n0 + row;
          if (n < N) {
            // One unrolled loop per mode keeps the live ranges short.
            if (e.mode == EPI_ACC_I64) {
              int64_t* yp = static_cast<int64_t*>(e.y) + n;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (m0 + c + j < M)
                  yp[(m0 + c + j) * e.ldy] = int64_t(int32_t(hi[j])) * 256 + int64_t(int32_t(lo[j]));
            } else if (e.mode == EPI_SHIFT) {
              const int64_t lo_b = e.out_i32 ? int64_t(INT32_MIN) : -32768;
              const int64_t hi_b = e.out_i32 ? int64_t(INT32_MAX) : 32767;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int64_t m = m0 + c + j;
                if (m < M) {
                  const int64_t a = int64_t(int32_t(hi[j])) * 256 + int64_t(int32_t(lo[j]));
                  const int64_t v = clamp_i64(rescale_i64_signed(a, rq.shift), lo_b, hi_b);
                  if (e.out_i32) static_cast<int32_t*>(e.y)[m * e.ldy + n] = int32_t(v);
                  else static_cast<int16_t*>(e.y)[m * e.ldy + n] = int16_t(v);
                }
              }
            } else {
#pragma unroll 1
              for (int j = 0; j < 32; j += 8) {
                int64_t a[8];
#pragma unroll
                for (int t = 0; t < 8; ++t) a[t] = 0;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj)
                  if (jj >= j && jj < j + 8)
                    a[jj - j] = int64_t(int32_t(hi[jj])) * 256 + int64_t(int32_t(lo[jj]));
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                  const int64_t m = m0 + c + j + t;
                  if (m < M) static_cast<int16_t*>(e.y)[m * e.ldy + n] = int16_t(rq.apply(a[t]));
                }
              }
            }
          }
        } else {
          const int64_t m = m0 + row;
          const int64_t nb = n0 + c;
          int64_t acc[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = int64_t(int32_t(hi[j])) * 256 + int64_t(int32_t(lo[j]));
          if (m < M) {
            if (vec16 && nb + 32 <= N) {
              uint32_t pk[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                ChannelRequant r0, r1;
                r0.load(e, nb + 2 * j);
                r1.load(e, nb + 2 * j + 1);
                const uint32_t a = uint16_t(int16_t(r0.apply(acc[2 * j])));
                const uint32_t b = uint16_t(int16_t(r1.apply(acc[2 * j + 1])));
                pk[j] = a | (b << 16);
              }
              int4* dst = reinterpret_cast<int4*>(static_cast<int16_t*>(e.y) + m * e.ldy + nb);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                dst[v] = make_int4(int(pk[4 * v]), int(pk[4 * v + 1]), int(pk[4 * v + 2]), int(pk[4 * v + 3]));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (nb + j < N) epilogue_store(e, m, nb + j, acc[j]);
            }
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// X int16 [M][ldx] -> X_hi int8 [M][ldp], X_lo uint8 [M][ldp] with
// x = 256*hi + lo; columns K..ldp-1 are written as zero.
__global__ void split_hilo_kernel(const int16_t* __restrict__ X, int64_t ldx, int64_t M, int64_t K,
                                  int8_t* __restrict__ Xhi, uint8_t* __restrict__ Xlo, int64_t ldp) {
  const int64_t groups = ldp >> 3;  // 8 elements per thread step
  const int64_t total = M * groups;
  const bool vec = ((reinterpret_cast<uintptr_t>(X) & 15) == 0) && (ldx % 8 == 0);
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = g / groups, k = (g % groups) * 8;
    const int16_t* xr = X + m * ldx;
    alignas(16) int16_t v[8];
    if (vec && k + 8 <= K) {
      *reinterpret_cast<int4*>(v) = __ldg(reinterpret_cast<const int4*>(xr + k));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = (k + e < K) ? xr[k + e] : int16_t(0);
    }
    uint32_t h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h0 |= (uint32_t(uint8_t(v[e] >> 8))) << (8 * e);
      l0 |= (uint32_t(uint8_t(v[e] & 0xFF))) << (8 * e);
      h1 |= (uint32_t(uint8_t(v[e + 4] >> 8))) << (8 * e);
      l1 |= (uint32_t(uint8_t(v[e + 4] & 0xFF))) << (8 * e);
    }
    *reinterpret_cast<uint2*>(Xhi + m * ldp + k) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(Xlo + m * ldp + k) = make_uint2(l0, l1);
  }
}

}  // namespace myl
