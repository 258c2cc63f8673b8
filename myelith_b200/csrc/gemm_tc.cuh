// gemm_tc.cuh — W8A16 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// The reference has no batched GEMM: prefill calls the per-token GEMV
// (INTEGER_LLM/runtime/src/generate.rs:29-31), so every output element here
// must equal linear.rs:61-68 for its (token, channel).
//
// Split-byte exactness. The tensor core multiplies 8-bit operands, the
// activations are int16. Each activation is split into two unsigned bytes,
// hi = (x >> 8) + 128 (offset binary) and lo = x & 255, so that
// x = 256*hi + lo - 32768 and
//   sum_k w*x = 256*H' + L - 32768*S,  H' = sum_k w*hi, L = sum_k w*lo,
// S = sum_k w (the weight row's sum over the K slice). Both bytes are
// unsigned, so one kind::i8 MMA (s8 weights x u8 activations) with N = 2*BN
// computes H' and L together: the B operand is the x_hi tile followed by the
// x_lo tile, and the accumulator's columns are H' | L. |w*hi|, |w*lo| <= 32640,
// so both int32 sums are exact for K <= 65536 (the host splits longer K into
// slices whose exact int64 partials are added). The epilogue forms
// H = H' - 128*S in wrapping 32-bit arithmetic, which is exact because the
// true H = sum_k w*(x >> 8) fits in int32; S comes from a per-row prefix sum
// over K tiles made at registration. 256*H + L is the reference's exact i64
// accumulator; the requant is applied to it once (fixed_point.rs:184-191).
// The tensor pipe does 2x the algorithmic MACs; one MMA of N = 256 reads 12 KB
// of shared memory per 128 x 256 x 32 step instead of the 16 KB that two
// MMAs of N = 128 sharing the A tile read.
//
// Tiles. The weight is the MMA's A operand (M = 128 output channels, TMEM lane
// = channel) and the activations are B (BN tokens, BN in {32, 64, 128}), so
// each epilogue thread owns one channel and keeps its requant parameters in
// registers, and a warp's stores for one token are 64 contiguous bytes.
//
// Schedule: persistent, one CTA per SM looping over work units
// (channel tile, token tile, K slice), 576 threads:
//   warp 0      TMA producer: W tile + x_hi tile + x_lo tile per 128-byte K
//               step into a STAGES-deep ring of 128B-swizzled smem stages.
//   warp 1      TMEM allocator; lane 0 issues 4 MMAs per K step (8 of half
//               width for a partial token tile) and commits each smem stage
//               back to the producer.
//   warps 2..17 epilogue: tcgen05.ld of H and L, requant, store. Warp w reads
//               TMEM lanes 32*(w%4)..32*(w%4)+31 and a quarter of the BN
//               columns; four warps per SM sub-partition hide the latency of
//               the epilogue's dependent integer steps.
// Two accumulator buffers (2 x (H, L) x BN columns) let the epilogue of one
// unit run while the MMAs of the next unit accumulate into the other buffer.
//
// Every mbarrier wait is bounded (timeout_ns, globaltimer); a wait that runs
// out writes an error code to *err, the CTA drains its own TMA copies and
// MMAs (bounded again), frees TMEM and returns.
#pragma once

#include "common.cuh"

namespace myl {

constexpr int TC_BK = 128;  // K bytes per stage = one 128-byte swizzle row
constexpr int TC_XBOX = 128;  // default activation rows per TMA box (x tensor maps)
constexpr int TC_EPI_WARPS = 16;  // four per TMEM lane quarter, each owning a quarter of the columns
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;

// PAIR: a cluster of two CTAs runs one MMA of M = 256 (cta_group::2); the even
// CTA holds weight rows 0..127 and the x_hi tile, the odd CTA rows 128..255 and
// the x_lo tile, so each SM loads one activation plane instead of two.
template <int BN, int STAGES, bool PAIR = false>
struct TcCfg {
  static constexpr int W_BYTES = 128 * TC_BK;
  static constexpr int X_BYTES = BN * TC_BK;
  static constexpr int STAGE_BYTES = W_BYTES + (PAIR ? 1 : 2) * X_BYTES;
  static constexpr int CT = PAIR ? 256 : 128;  // weight rows (channels) per work unit
  static constexpr int BUF_COLS = 2 * BN;  // H | L of one accumulator buffer
  static constexpr int TMEM_COLS = 2 * BUF_COLS <= 32 ? 32 : 2 * BUF_COLS;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
  static_assert(BN == 32 || BN == 64 || BN == 128, "token tile");
  static_assert(TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation");
  static_assert(STAGES >= 2 && STAGES <= 16, "stage ring");
  static_assert(SMEM_BYTES <= 227 * 1024 - 512, "shared memory");
  // W s8 x [x_hi | x_lo] u8
  static constexpr uint32_t IDESC = idesc_i8(PAIR ? 256 : 128, 2 * BN, true, false);
};

struct TcCtl {
  uint64_t full[16];
  uint64_t empty[16];
  uint64_t tfull[2];   // accumulator buffer b holds a finished unit
  uint64_t tempty[2];  // accumulator buffer b has been read by the epilogue
  uint64_t never;      // test hook: nothing ever arrives here
  uint32_t tmem_base;
  int abort;
};

// One work unit: a 128-channel (256 for a CTA pair) x BN-token output tile
// over one K slice.
struct TcUnit {
  int nt, ks, kt0, nkt;
  int tail_slot;     // >= 0: a K slice of a tail tile, stored as int64 partials
  int64_t m_begin;   // first activation row (token) of the tile
  int64_t m_end;     // rows >= m_end are not stored (end of the group / of M)
  int64_t w_row;     // first weight row of the tile
  int64_t p_off;     // offset of the tile's group into the per-channel parameters
};

// Work decomposition. Dense: units (channel tile, token tile, K slice), channel
// tiles varying fastest (a wave shares a token tile and sweeps the weight).
// Grouped (MoE experts, groups > 0): group g owns activation rows
// [row_start[g], row_start[g] + rows[g]) and weight rows
// [g * group_w_rows, (g + 1) * group_w_rows) of a stacked weight; its units are
// [tile_start[g], tile_start[g + 1]) (device table written by the router), one
// K slice each. A token tile may run past its group's rows into the next
// group's: those columns are computed and not stored.
struct TcWork {
  int tiles_n, tiles_m, ksplit, k_tiles_total, k_tiles_per_split;
  int groups;
  const int* tile_start;
  const int* row_start;
  const int* rows;
  int64_t group_w_rows;
  // Per weight row r, wsum[r * wsum_ld + t] = sum of the row's weights over K
  // tiles [0, t) (wrapping int32): the correction term of the offset-binary hi.
  const int32_t* wsum;
  int64_t wsum_ld;
  // Dense tail split (ksplit == 1): tiles [full_units, full_units + tail_tiles)
  // are the last, incomplete wave; each runs as tail_ks K slices of tail_per K
  // tiles whose int64 partials go to tail_ws[slot][ct / 128][BN][128] (slot =
  // slice * tail_tiles + tile; the middle index is the CTA of a pair) and are
  // added by tail_reduce_kernel, so the final wave is short instead of mostly
  // idle.
  int full_units, tail_tiles, tail_ks, tail_per;
  int64_t* tail_ws;
  // Rows per activation TMA box (the x tensor maps' box height; divides BN).
  int xbox;
  __device__ __forceinline__ int units() const {
    if (groups > 0) return tile_start[groups];
    if (tail_tiles > 0) return full_units + tail_tiles * tail_ks;
    return tiles_n * tiles_m * ksplit;
  }
  // ct: weight rows per unit (128, or 256 for a CTA pair).
  __device__ __forceinline__ TcUnit decode(int u, int BN, int64_t M, int ct) const {
    TcUnit w;
    w.tail_slot = -1;
    if (groups == 0 && tail_tiles > 0 && u >= full_units) {
      const int v = u - full_units;
      const int slice = v / tail_tiles, tl = v % tail_tiles;
      const int t = full_units + tl;
      w.nt = t % tiles_n;
      w.ks = 0;
      w.kt0 = slice * tail_per;
      w.nkt = min(tail_per, k_tiles_total - w.kt0);
      w.m_begin = int64_t(t / tiles_n) * BN;
      w.m_end = M;
      w.w_row = int64_t(w.nt) * ct;
      w.p_off = 0;
      w.tail_slot = slice * tail_tiles + tl;
      return w;
    }
    if (groups == 0) {
      w.nt = u % tiles_n;
      const int r = u / tiles_n;
      const int mt = r % tiles_m;
      w.ks = r / tiles_m;
      w.kt0 = w.ks * k_tiles_per_split;
      w.nkt = min(k_tiles_per_split, k_tiles_total - w.kt0);
      w.m_begin = int64_t(mt) * BN;
      w.m_end = M;
      w.w_row = int64_t(w.nt) * ct;
      w.p_off = 0;
      return w;
    }
    int lo = 0, hi = groups - 1;  // last group with tile_start[g] <= u
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tile_start[mid] <= u) lo = mid;
      else hi = mid - 1;
    }
    const int local = u - tile_start[lo];
    w.nt = local % tiles_n;
    w.ks = 0;
    w.kt0 = 0;
    w.nkt = k_tiles_total;
    w.m_begin = int64_t(row_start[lo]) + int64_t(local / tiles_n) * BN;
    w.m_end = int64_t(row_start[lo]) + rows[lo];
    w.p_off = int64_t(lo) * group_w_rows;
    w.w_row = w.p_off + int64_t(w.nt) * ct;
    return w;
  }
};

__device__ __forceinline__ void tc_fail(int* err, volatile int* abort, int code) {
  *abort = 1;
  atomicCAS(err, 0, code);
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Requant of the exact accumulator V = 256*H + L by a right shift s = 8 + t,
// t in [0, 30], in 32-bit arithmetic. With h = H + (L >> 8) and l = L & 255,
// V = 256*h + l and 0 <= l < 256, so V >> s = h >> t. Round-to-nearest-even
// (fixed_point.rs:57-71) is (V + 2^(s-1) - 1 + odd) >> s with odd = (V >> s) & 1;
// the bias splits as 256*bh + bl with bh = 2^(t-1) - 1, bl = 255 (t >= 1) or
// bh = 0, bl = 127 (t = 0), giving (h + bh + ((l + bl + odd) >> 8)) >> t.
// |h| < 2^30 + 2^23 (K <= 65536), so no step leaves int32.
// The optional per-channel bias (linear.rs:132-145) is added after the first
// clamp and clamped again, as the reference adds it to the clamped output.
struct Requant32 {
  int t, bh, bl, lo_b, hi_b, bias;
  __device__ __forceinline__ void init(int s, bool out_i32, int b) {
    t = s - 8;
    bh = t > 0 ? (1 << (t - 1)) - 1 : 0;
    bl = t > 0 ? 255 : 127;
    lo_b = out_i32 ? INT32_MIN : -32768;
    hi_b = out_i32 ? INT32_MAX : 32767;
    bias = b;
  }
  __device__ __forceinline__ int apply(int32_t H, int32_t L) const {
    const int32_t h = H + (L >> 8);
    const int32_t l = L & 255;
    const int32_t odd = (h >> t) & 1;
    int32_t v = (h + bh + ((l + bl + odd) >> 8)) >> t;
    v = v < lo_b ? lo_b : (v > hi_b ? hi_b : v);
    if (lo_b == -32768) {  // bias only exists for int16 outputs
      v += bias;
      v = v < lo_b ? lo_b : (v > hi_b ? hi_b : v);
    }
    return v;
  }
};

// Loads NC (8, 16 or 32) columns of the H and L accumulators of this thread's lane.
template <int NC>
__device__ __forceinline__ void tmem_ld_pair(uint32_t taddr_h, uint32_t taddr_l, uint32_t (&h)[NC],
                                             uint32_t (&l)[NC]) {
  if constexpr (NC == 32) {
    tmem_ld_32x32b_x32(taddr_h, h);
    tmem_ld_32x32b_x32(taddr_l, l);
  } else if constexpr (NC == 8) {
    tmem_ld_32x32b_x8(taddr_h, h);
    tmem_ld_32x32b_x8(taddr_l, l);
  } else {
    tmem_ld_32x32b_x16(taddr_h, h);
    tmem_ld_32x32b_x16(taddr_l, l);
  }
  tmem_ld_wait();
}

// Writes NC consecutive tokens (rows m0.. of y) of channel n.
template <int NC, typename T, typename F>
__device__ __forceinline__ void store_column(T* yp, int64_t ldy, int64_t m0, int64_t M, F&& value) {
  if (m0 + NC <= M) {
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      *yp = value(j);
      yp += ldy;
    }
  } else {
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      if (m0 + j < M) *yp = value(j);
      yp += ldy;
    }
  }
}

// MODE (EpiMode) is a template parameter so that each instantiation carries
// only its own epilogue: smaller code and fewer registers per kernel.
//
// PAIR (launched as clusters of 2): both CTAs load their halves of each stage
// and count the bytes on the even CTA's full barrier; the even CTA's MMA
// thread issues the M = 256 MMAs and its commits reach the empty and
// accumulator barriers of both CTAs; both epilogues report a drained
// accumulator to the even CTA. A failed wait in either CTA also raises the
// other's abort flag.
template <int BN, int STAGES, int MODE, bool PAIR>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_w8a16_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_xhi,
                         const __grid_constant__ CUtensorMap tm_xlo, int64_t M, int64_t N,
                         TcWork work, Epilogue ep, int64_t slice_stride, int* err,
                         uint64_t timeout_ns, int inject_fault) {
  pdl_wait();
  pdl_launch();
  using Cfg = TcCfg<BN, STAGES, PAIR>;
  extern __shared__ uint8_t dyn_smem[];
  __shared__ TcCtl ctl;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t smem_base = (smem_addr(dyn_smem) + 1023u) & ~1023u;
  auto sm_w = [&](int s) { return smem_base + uint32_t(s) * Cfg::STAGE_BYTES; };
  auto sm_xh = [&](int s) { return sm_w(s) + Cfg::W_BYTES; };  // PAIR: this CTA's plane
  auto sm_xl = [&](int s) { return sm_w(s) + Cfg::W_BYTES + Cfg::X_BYTES; };
  volatile int* abort = &ctl.abort;
  const int units = work.units();
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int u0 = PAIR ? int(cluster_id_x()) : int(blockIdx.x);
  const int ustep = PAIR ? int(cluster_count_x()) : int(gridDim.x);
  auto fail = [&](int code) {
    tc_fail(err, abort, code);
    if (PAIR) st_shared_cluster_u32(mapa_shared(smem_addr(&ctl.abort), rank ^ 1u), 1u);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&ctl.full[s]), 1);
      mbar_init(smem_addr(&ctl.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&ctl.tfull[b]), 1);
      mbar_init(smem_addr(&ctl.tempty[b]), PAIR ? 2 * TC_EPI_WARPS : TC_EPI_WARPS);
    }
    mbar_init(smem_addr(&ctl.never), 1);
    ctl.abort = 0;
    fence_barrier_init();
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_xhi);
    prefetch_tensormap(&tm_xlo);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(smem_addr(&ctl.tmem_base), Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_addr(&ctl.tmem_base), Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncwarp();
  if (PAIR) cluster_sync_all();  // both CTAs' barriers exist before any remote signal
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int g = 0;  // K steps issued by this CTA (ring position)
      bool stop = false;
      for (int u = u0; u < units && !stop; u += ustep) {
        const TcUnit wu = work.decode(u, BN, M, Cfg::CT);
        const int32_t w_row = int32_t(wu.w_row + 128 * int64_t(rank));
        for (int i = 0; i < wu.nkt; ++i, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = uint32_t(g / STAGES) & 1u;
          if (!mbar_wait_bounded(smem_addr(&ctl.empty[s]), ph ^ 1u, timeout_ns, abort)) {
            fail(DEV_WAIT_PRODUCER);
            stop = true;
            break;
          }
          const uint32_t fb = smem_addr(&ctl.full[s]);
          // The activation tiles arrive as boxes of xb rows; a tile with
          // fewer valid tokens (end of M or of an expert's rows) loads only
          // the boxes that hold some, which covers every row its trimmed
          // MMAs read (N = valid rounded up to 16).
          const int xb = work.xbox;
          const int64_t valid = wu.m_end - wu.m_begin;
          const int nbox = valid >= BN ? BN / xb : int((valid + xb - 1) / xb);
          const int32_t kx = (wu.kt0 + i) * TC_BK;
          if (PAIR) {
            // Both CTAs' bytes complete on the even CTA's barrier, which only
            // the even CTA arms (a completion that lands first leaves the
            // phase open: its arrival is still pending).
            const uint32_t fbc = mapa_shared(fb, 0);
            if (leader) mbar_arrive_expect_tx(fb, uint32_t(2 * (Cfg::W_BYTES + nbox * xb * TC_BK)));
            tma_load_2d_pair(sm_w(s), &tm_w, fbc, kx, w_row);
            const CUtensorMap* tmx = leader ? &tm_xhi : &tm_xlo;
            for (int bx = 0; bx < nbox; ++bx)
              tma_load_2d_pair(sm_xh(s) + uint32_t(bx * xb * TC_BK), tmx, fbc, kx,
                               int32_t(wu.m_begin + bx * xb));
          } else {
            mbar_arrive_expect_tx(fb, uint32_t(Cfg::W_BYTES + 2 * nbox * xb * TC_BK));
            tma_load_2d(sm_w(s), &tm_w, fb, kx, w_row);
            for (int bx = 0; bx < nbox; ++bx) {
              const uint32_t off = uint32_t(bx * xb * TC_BK);
              const int32_t row = int32_t(wu.m_begin + bx * xb);
              tma_load_2d(sm_xh(s) + off, &tm_xhi, fb, kx, row);
              tma_load_2d(sm_xl(s) + off, &tm_xlo, fb, kx, row);
            }
          }
        }
      }
      if (PAIR && !*abort) {
        // Every stage's last release (a commit of the even CTA) has landed
        // here before this CTA can leave the cluster.
        for (int s = 0; s < STAGES && s < g; ++s) {
          const int last = s + ((g - 1 - s) / STAGES) * STAGES;
          if (!mbar_wait_bounded(smem_addr(&ctl.empty[s]), uint32_t(last / STAGES) & 1u, timeout_ns,
                                 nullptr))
            atomicCAS(err, 0, DEV_WAIT_DRAIN);
        }
      }
      if (*abort && leader) {
        // Drain: the last load issued into each stage must land before exit.
        for (int s = 0; s < STAGES && s < g; ++s) {
          const int last = s + ((g - 1 - s) / STAGES) * STAGES;
          if (!mbar_wait_bounded(smem_addr(&ctl.full[s]), uint32_t(last / STAGES) & 1u, timeout_ns,
                                 nullptr))
            atomicCAS(err, 0, DEV_WAIT_DRAIN);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && leader) {
      int g = 0, lt = 0;
      bool stop = false;
      for (int u = u0; u < units && !stop; u += ustep, ++lt) {
        const TcUnit wu = work.decode(u, BN, M, Cfg::CT);
        const int nkt = wu.nkt;
        // A full tile runs one MMA of N = 2*BN over [x_hi | x_lo]. A tile with
        // fewer valid tokens than BN (the end of M or of an expert's rows) runs
        // one MMA per byte plane with N = valid rounded up to 16 (kind::i8
        // with M = 128 takes N in multiples of 16); columns above are never read.
        // A pair runs one MMA of N = 2 * that (the x_hi rows from the even CTA,
        // the x_lo rows from the odd one), so L starts at column nmma.
        const int64_t valid = wu.m_end - wu.m_begin;
        const bool full = valid >= BN;
        const uint32_t nmma = full ? uint32_t(BN) : uint32_t((valid + 15) & ~int64_t(15));
        const uint32_t idesc_part = (Cfg::IDESC & ~(0x3Fu << 17)) | ((nmma >> 3) << 17);
        const uint32_t idesc_pair = (Cfg::IDESC & ~(0x3Fu << 17)) | (((2 * nmma) >> 3) << 17);
        const int b = lt & 1;
        const uint32_t tph = uint32_t(lt >> 1) & 1u;
        if (!mbar_wait_bounded(smem_addr(&ctl.tempty[b]), tph ^ 1u, timeout_ns, abort)) {
          fail(DEV_WAIT_MMA);
          break;
        }
        tc_fence_after();
        const uint32_t d_hi = tmem + uint32_t(b * Cfg::BUF_COLS), d_lo = d_hi + BN;
        for (int i = 0; i < nkt; ++i, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = uint32_t(g / STAGES) & 1u;
          if (!mbar_wait_bounded(smem_addr(&ctl.full[s]), ph, timeout_ns, abort)) {
            fail(DEV_WAIT_MMA);
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t aw = sm_w(s), axh = sm_xh(s), axl = sm_xl(s);
#pragma unroll
          for (int kk = 0; kk < TC_BK / 32; ++kk) {
            const uint32_t off = uint32_t(kk) * 32u;
            const uint64_t dw = smem_desc_k_sw128(aw + off);
            const uint32_t accum = (i > 0 || kk > 0) ? 1u : 0u;
            if (PAIR) {
              mma_i8_pair(d_hi, dw, smem_desc_k_sw128(axh + off), idesc_pair, accum);
            } else if (full) {
              mma_i8(d_hi, dw, smem_desc_k_sw128(axh + off), Cfg::IDESC, accum);
            } else {
              mma_i8(d_hi, dw, smem_desc_k_sw128(axh + off), idesc_part, accum);
              mma_i8(d_lo, dw, smem_desc_k_sw128(axl + off), idesc_part, accum);
            }
          }
          // frees the stage (in both CTAs of a pair) when these MMAs finish
          if (PAIR) mma_commit_pair_both(smem_addr(&ctl.empty[s]));
          else mma_commit(smem_addr(&ctl.empty[s]));
        }
        // also signals on abort: the epilogue checks
        if (PAIR) mma_commit_pair_both(smem_addr(&ctl.tfull[b]));
        else mma_commit(smem_addr(&ctl.tfull[b]));
      }
      // The issuer itself sees its last MMAs finish before TMEM can be released.
      if (lt > 0) {
        const int b = (lt - 1) & 1;
        if (!mbar_wait_bounded(smem_addr(&ctl.tfull[b]), uint32_t((lt - 1) >> 1) & 1u, timeout_ns,
                               nullptr))
          atomicCAS(err, 0, DEV_WAIT_DRAIN);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..17) ----------------
    constexpr int QCOLS = BN / 4;                // columns per epilogue warp
    constexpr int NC = QCOLS < 16 ? QCOLS : 16;  // columns per TMEM load
    const int q = warp & 3;
    const int col0 = ((warp - 2) >> 2) * QCOLS;
    const int row = q * 32 + lane;
    int lt = 0;
    for (int u = u0; u < units; u += ustep, ++lt) {
      const TcUnit wu = work.decode(u, BN, M, Cfg::CT);
      const int b = lt & 1;
      const uint32_t tph = uint32_t(lt >> 1) & 1u;
      bool ok = mbar_wait_bounded(smem_addr(&ctl.tfull[b]), tph, timeout_ns, abort);
      int code = DEV_WAIT_EPILOGUE;
      if (ok && inject_fault) {
        ok = mbar_wait_bounded(smem_addr(&ctl.never), 0u, timeout_ns, nullptr);
        code = DEV_WAIT_INJECTED;
      }
      if (!ok) {
        fail(code);
        break;
      }
      if (*abort) break;
      tc_fence_after();
      const int64_t n = int64_t(wu.nt) * Cfg::CT + 128 * int64_t(rank) + row;  // channel in the group
      const int64_t m0 = wu.m_begin + col0;
      const int64_t Mend = wu.m_end;
      const uint32_t tq = tmem + (uint32_t(q * 32) << 16) + uint32_t(b * Cfg::BUF_COLS + col0);
      // Column of L: BN, or for a pair the MMA's N / 2 (valid tokens rounded up to 16).
      const int64_t valid = Mend - wu.m_begin;
      const uint32_t lo_col = (!PAIR || valid >= BN) ? uint32_t(BN)
                                                     : uint32_t((valid + 15) & ~int64_t(15));
      Epilogue e = ep;
      if (MODE == EPI_ACC_I64) e.y = static_cast<int64_t*>(e.y) + int64_t(wu.ks) * slice_stride;
      if (wu.p_off) {  // per-channel parameters of this group
        e.shift = e.shift ? e.shift + wu.p_off : nullptr;
        e.mult = e.mult ? e.mult + wu.p_off : nullptr;
        e.bias = e.bias ? e.bias + wu.p_off : nullptr;
      }
      // Channel parameters, once per unit.
      int shift = 0;
      constexpr int mode = MODE;
      // (EPI_W16 reads the shift of weight row n/2 in w16_store.)
      constexpr bool per_row = mode != EPI_ACC_I64 && mode != EPI_W16;
      if (n < N && per_row) shift = e.shift[n];
      const bool fast = (mode == EPI_SHIFT || mode == EPI_SILU) && shift >= 8 && shift <= 38;
      Requant32 r32;
      r32.init(fast ? shift : 8, e.out_i32 != 0, (n < N && per_row && e.bias) ? e.bias[n] : 0);
      ChannelRequant rq;
      if (n < N && !fast && per_row) rq.load(e, n);
      // H = H' - 128 * S over this unit's K tiles (wrapping; the true H fits).
      uint32_t corr = 0;
      if (n < N) {
        const int32_t* ws = work.wsum + (wu.w_row + 128 * int64_t(rank) + row) * work.wsum_ld;
        corr = (uint32_t(ws[wu.kt0 + wu.nkt]) - uint32_t(ws[wu.kt0])) << 7;
      }
#pragma unroll 1
      for (int c = 0; c < QCOLS; c += NC) {
        if (m0 + c >= Mend) break;  // warp-uniform: no stored token left in this warp's columns
        uint32_t hi[NC], lo[NC];
        tmem_ld_pair<NC>(tq + c, tq + lo_col + c, hi, lo);
#pragma unroll
        for (int j = 0; j < NC; ++j) hi[j] -= corr;
        if (wu.tail_slot >= 0) {  // int64 partial of a tail tile's K slice
          if (n < N) {
            int64_t* tp = work.tail_ws +
                          ((int64_t(wu.tail_slot) * (Cfg::CT / 128) + rank) * BN + col0 + c) * 128 + row;
#pragma unroll
            for (int j = 0; j < NC; ++j)
              tp[int64_t(j) * 128] = int64_t(int32_t(hi[j])) * 256 + int64_t(int32_t(lo[j]));
          }
          continue;
        }
        const int64_t mc = m0 + c;
        if (mode == EPI_W16) {
          // High byte (even row) and offset low byte (odd row) of int16 weight
          // row n/2 sit in adjacent lanes: as for the SiLU pairs, the even lane
          // takes the first NC/2 tokens, the odd lane the last NC/2.
          constexpr int NH = NC / 2;
          const bool even = (row & 1) == 0;
          int64_t a[NC];
#pragma unroll
          for (int j = 0; j < NC; ++j) a[j] = int64_t(int32_t(hi[j])) * 256 + int64_t(int32_t(lo[j]));
          const int64_t mh = mc + (even ? 0 : NH);
          const int64_t jlim = n < N ? Mend - mh : 0;
#pragma unroll
          for (int j = 0; j < NH; ++j) {
            const int64_t mine = even ? a[j] : a[j + NH];
            const int64_t other = __shfl_xor_sync(0xffffffffu, even ? a[j + NH] : a[j], 1);
            if (j < jlim) w16_store(e, mh + j, n >> 1, even ? mine : other, even ? other : mine);
          }
          continue;
        }
        if (mode == EPI_SILU) {
          // Gate (even row) and up (odd row) of channel pair n/2 sit in
          // adjacent lanes. One exchange per token pair gives the even lane
          // (gate, up) of the first NC/2 tokens and the odd lane those of the
          // last NC/2, so every lane computes and stores NC/2 products. The
          // steps run over all NC/2 tokens at a time (independent table loads
          // in flight together).
          constexpr int NH = NC / 2;
          const bool even = (row & 1) == 0;
          int32_t v[NC];
#pragma unroll
          for (int j = 0; j < NC; ++j) {
            v[j] = 0;
            if (n < N)
              v[j] = fast ? r32.apply(int32_t(hi[j]), int32_t(lo[j]))
                          : int32_t(rq.apply(int64_t(int32_t(hi[j])) * 256 + int64_t(int32_t(lo[j]))));
          }
          int32_t g[NH], u[NH];
#pragma unroll
          for (int j = 0; j < NH; ++j) {
            const int32_t mine = even ? v[j] : v[j + NH];
            const int32_t other = __shfl_xor_sync(0xffffffffu, even ? v[j + NH] : v[j], 1);
            g[j] = even ? mine : other;
            u[j] = even ? other : mine;
          }
          const SiluParams& sp = e.silu;
#pragma unroll
          for (int j = 0; j < NH; ++j) g[j] = __ldg(sp.lut + silu_index(sp, g[j]));
          const int64_t mh = mc + (even ? 0 : NH);
          const int64_t jlim = n < N ? Mend - mh : 0;  // tokens mh + j < Mend are stored
          if (e.y == nullptr && sp.h_hi != nullptr && sp.s2 >= 1 && sp.s2 <= 30) {
            uint8_t* ph = sp.h_hi + mh * sp.ldp + (n >> 1);
            uint8_t* pl = sp.h_lo + mh * sp.ldp + (n >> 1);
            const int32_t c2 = (1 << (sp.s2 - 1)) - 1;
            const int ld = int(sp.ldp);  // NH rows of planes: offsets fit in 32 bits
#pragma unroll
            for (int j = 0; j < NH; ++j) {
              // |lut * u| <= 2^30: the one-add rounding stays inside i32
              const int32_t h = max(-32768, min(rne_add_i32(g[j] * u[j], sp.s2, c2), 32767));
              if (j < jlim) {
                ph[j * ld] = uint8_t((h >> 8) + 128);  // offset-binary high byte
                pl[j * ld] = uint8_t(h & 0xFF);
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < NH; ++j)
              if (j < jlim) silu_store(e, mh + j, n >> 1, int16_t(silu_product(sp, g[j], u[j])));
          }
          continue;
        }
        if (n >= N) continue;
        if (mode == EPI_ACC_I64 && e.xb_world > 0) {  // broadcast to every rank's slab
          for (int o = 0; o < e.xb_world; ++o) {
            int64_t* yb = static_cast<int64_t*>(e.xb_dst[o]) + e.xb_rank * e.xb_slab + mc * e.ldy + n;
            store_column<NC>(yb, e.ldy, mc, Mend, [&](int j) {
              return int64_t(int32_t(hi[j])) * 256 + int64_t(int32_t(lo[j]));
            });
          }
        } else if (mode == EPI_ACC_I64) {
          int64_t* yb;
          if (e.xs_world > 0) {  // exchange: the owning rank's receive buffer (peer memory)
            // xs_rows is a multiple of 16 >= NC, so the NC tokens share one owner
            const int64_t o = mc / e.xs_rows;
            yb = static_cast<int64_t*>(e.xs_dst[o]) +
                 (e.xs_rank * e.xs_rows + (mc - o * e.xs_rows)) * e.ldy + n;
          } else {
            yb = static_cast<int64_t*>(e.y) + mc * e.ldy + n;
          }
          store_column<NC>(yb, e.ldy, mc, Mend, [&](int j) {
            return int64_t(int32_t(hi[j])) * 256 + int64_t(int32_t(lo[j]));
          });
        } else if (fast) {
          if (e.out_i32) {
            store_column<NC>(static_cast<int32_t*>(e.y) + mc * e.ldy + n, e.ldy, mc, Mend,
                             [&](int j) { return int32_t(r32.apply(int32_t(hi[j]), int32_t(lo[j]))); });
          } else {
            store_column<NC>(static_cast<int16_t*>(e.y) + mc * e.ldy + n, e.ldy, mc, Mend,
                             [&](int j) { return int16_t(r32.apply(int32_t(hi[j]), int32_t(lo[j]))); });
          }
        } else {
#pragma unroll 1
          for (int j0 = 0; j0 < NC; j0 += 8) {
            int64_t a[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) a[t] = 0;
#pragma unroll
            for (int jj = 0; jj < NC; ++jj)
              if (jj >= j0 && jj < j0 + 8)
                a[jj - j0] = int64_t(int32_t(hi[jj])) * 256 + int64_t(int32_t(lo[jj]));
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const int64_t m = mc + j0 + t;
              if (m < Mend) {
                const int64_t v = rq.apply(a[t]);
                if (e.out_i32) static_cast<int32_t*>(e.y)[m * e.ldy + n] = int32_t(v);
                else static_cast<int16_t*>(e.y)[m * e.ldy + n] = int16_t(v);
              }
            }
          }
        }
      }
      // Hand the buffer back to the MMA issuer (the even CTA's, for a pair).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && !leader) mbar_arrive_cluster(mapa_shared(smem_addr(&ctl.tempty[b]), 0));
        else mbar_arrive(smem_addr(&ctl.tempty[b]));
      }
    }
    tc_fence_before();
  }
  if (PAIR) {
    // Every thread of both CTAs gets here (all waits above are bounded); the
    // even CTA's MMAs are finished and both epilogues are done with TMEM.
    __syncwarp();
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
    else tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// Adds the tail tiles' K-slice partials and applies the final epilogue.
// One thread per (tile, token, channel pair): both rows of the pair, so the
// SiLU mode can combine gate and up. ct: channels per tile (128, or 256 for
// CTA pairs, whose halves are stored one after the other).
__global__ void tail_reduce_kernel(const int64_t* __restrict__ ws, int tail_tiles, int tail_ks,
                                   int first_tile, int tiles_n, int BN, int ct, int64_t M,
                                   int64_t N, Epilogue ep) {
  pdl_wait();
  pdl_launch();
  const int hp = ct / 2;  // channel pairs per tile
  const int halves = ct / 128;
  const int64_t total = int64_t(tail_tiles) * BN * hp;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int pr = int(e % hp);
    const int col = int((e / hp) % BN);
    const int tl = int(e / (int64_t(hp) * BN));
    const int t = first_tile + tl;
    const int64_t m = int64_t(t / tiles_n) * BN + col;
    const int64_t n0 = int64_t(t % tiles_n) * ct + 2 * pr;
    if (m >= M || n0 >= N) continue;
    const int half = (2 * pr) >> 7, r0 = (2 * pr) & 127;
    int64_t a0 = 0, a1 = 0;
    for (int s = 0; s < tail_ks; ++s) {
      const int64_t* p =
          ws + (((int64_t(s) * tail_tiles + tl) * halves + half) * BN + col) * 128 + r0;
      a0 += p[0];
      a1 += p[1];
    }
    if (ep.mode == EPI_W16) {  // rows 2i / 2i + 1: high and offset low byte of int16 row i
      w16_store(ep, m, n0 >> 1, a0, a1);
    } else if (ep.mode == EPI_SILU) {  // N is even: rows 2i / 2i + 1 are gate / up of pair i
      const int32_t g = int32_t(requant_value(ep, n0, a0));
      const int32_t u = int32_t(requant_value(ep, n0 + 1, a1));
      silu_store(ep, m, n0 >> 1, silu_combine(ep.silu, g, u));
    } else {
      epilogue_store(ep, m, n0, a0);
      if (n0 + 1 < N) epilogue_store(ep, m, n0 + 1, a1);
    }
  }
}

// out[r * ld + t] = sum of row r's weights over K tiles [0, t), t = 0..k_tiles,
// in wrapping int32 (only differences over at most 65536 columns are used).
__global__ void weight_tile_sums_kernel(const int8_t* __restrict__ W, int64_t ldp, int64_t N,
                                        int64_t K, int k_tiles, int32_t* __restrict__ out,
                                        int64_t ld) {
  // ldp is a multiple of 16 and the columns K..ldp-1 are zero, so a tile is
  // summed in 16-byte loads (dp4a against ones adds four signed bytes).
  for (int64_t r = blockIdx.x; r < N; r += gridDim.x) {
    const int8_t* wr = W + r * ldp;
    int32_t* o = out + r * ld;
    for (int t = threadIdx.x; t < k_tiles; t += blockDim.x) {
      const int64_t k0 = int64_t(t) * TC_BK;
      const int64_t k1 = k0 + TC_BK < ldp ? k0 + TC_BK : ldp;
      int32_t sum = 0;
      for (int64_t k = k0; k < k1; k += 16) {
        const int4 v = __ldg(reinterpret_cast<const int4*>(wr + k));
        sum = __dp4a(v.x, 0x01010101, sum);
        sum = __dp4a(v.y, 0x01010101, sum);
        sum = __dp4a(v.z, 0x01010101, sum);
        sum = __dp4a(v.w, 0x01010101, sum);
      }
      o[t + 1] = sum;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t acc = 0;
      o[0] = 0;
      for (int t = 1; t <= k_tiles; ++t) {
        acc += uint32_t(o[t]);
        o[t] = int32_t(acc);
      }
    }
    __syncthreads();
  }
}

// X int16 [M][ldx] -> X_hi, X_lo uint8 [M][ldp] with hi = (x >> 8) + 128
// (offset binary) and lo = x & 255, x = 256*hi + lo - 32768; columns
// K..ldp-1 are written as x = 0 (hi = 128, lo = 0), whose weights are zero.
__device__ __forceinline__ void split8(const int16_t (&v)[8], uint2& hi, uint2& lo) {
  uint32_t h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    h0 |= (uint32_t(uint8_t(v[e] >> 8)) ^ 0x80u) << (8 * e);
    l0 |= uint32_t(uint8_t(v[e] & 0xFF)) << (8 * e);
    h1 |= (uint32_t(uint8_t(v[e + 4] >> 8)) ^ 0x80u) << (8 * e);
    l1 |= uint32_t(uint8_t(v[e + 4] & 0xFF)) << (8 * e);
  }
  hi = make_uint2(h0, h1);
  lo = make_uint2(l0, l1);
}

__global__ void split_hilo_kernel(const int16_t* __restrict__ X, int64_t ldx, int64_t M, int64_t K,
                                  uint8_t* __restrict__ Xhi, uint8_t* __restrict__ Xlo, int64_t ldp) {
  pdl_wait();
  pdl_launch();
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
    uint2 hi, lo;
    split8(v, hi, lo);
    *reinterpret_cast<uint2*>(Xhi + m * ldp + k) = hi;
    *reinterpret_cast<uint2*>(Xlo + m * ldp + k) = lo;
  }
}

}  // namespace myl
