// common.cuh — device helpers shared by the W8A16 kernels (sm_100a only).
//
// Requant semantics (the epilogue of every kernel) restate the reference:
//   rshift_round_i64   INTEGER_LLM/kernels/src/fixed_point.rs:57-71
//   rescale_i64        fixed_point.rs:184-191 (negative shift = left shift)
//   clamp_i16_from_i64 fixed_point.rs:23-27, LM head i32 clamp runtime/src/model.rs:305
// The signed total shift s = (w_shift + act_frac) - out_frac is computed and
// range-checked on the host (one int8 per output channel); the device only
// applies it.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libmyl_w8a16 is written for sm_100a (B200) only"
#endif

namespace myl {

// ---- kernel error codes written to the context's device error word --------
enum DeviceError : int {
  DEV_OK = 0,
  DEV_WAIT_PRODUCER = 0x101,  // producer gave up waiting for a free stage
  DEV_WAIT_MMA = 0x102,       // MMA issuer gave up waiting for a loaded stage
  DEV_WAIT_EPILOGUE = 0x103,  // epilogue gave up waiting for the accumulator
  DEV_WAIT_DRAIN = 0x104,     // clean-up gave up waiting for copies / MMAs in flight
  DEV_WAIT_INJECTED = 0x105,  // test hook: a wait on a barrier nothing arrives at
  DEV_WAIT_PEER = 0x106,      // a peer rank did not reach an exchange barrier in time
  DEV_BAD_EXPERT = 0x201,     // an expert id outside the experts this object holds
  DEV_BAD_TOKEN = 0x202,      // a token id outside the vocabulary (device-side ids)
};

// Epilogue modes.
enum EpiMode : int {
  EPI_ACC_I64 = 0,    // store exact int64 partial sums
  EPI_SHIFT = 1,      // reference requant (pure shift)
  EPI_MULT = 2,       // multiplier requant (i128 product)
  EPI_SILU = 3,       // MLP: rows 2i / 2i+1 are gate_i / up_i; store h_i (mlp.rs:49-64)
  EPI_W16 = 4,        // int16 weights: rows 2i / 2i+1 are the high byte and the offset low
                      // byte of row i; store int32 logits (model.rs:285-296)
};

// Parameters of the SiLU-LUT product of mlp.rs:52-64 (validated on the host).
struct SiluParams {
  const int16_t* lut;
  int lut_hi;        // index upper bound: (lut.len() as i16) - 1, Rust release wrapping
  int offset;        // silu_lut_offset (i16)
  int s1;            // gate_out_frac - silu_in_frac, signed, in [-31, 30]
  int s2;            // silu_out_frac + up_out_frac - down_in_frac, signed, in [-63, 62]
  uint8_t* h_hi;     // optional byte planes of h for the down projection: [M][ldp],
  uint8_t* h_lo;     // hi = (h >> 8) + 128, lo = h & 255 (as split_hilo_kernel)
  int64_t ldp;
};

constexpr int MYL_XCHG_MAX = 8;  // ranks of a peer-memory exchange

struct Epilogue {
  int mode;               // EpiMode
  int out_i32;            // 1: clamp to i32 and store int32, 0: clamp to i16, store int16
  const int8_t* shift;    // [N]: signed total shift (EPI_SHIFT, EPI_SILU) / uint8 shift (EPI_MULT)
  const int32_t* mult;    // [N] (EPI_MULT)
  void* y;                // [M][ldy] int16/int32 (requant modes), int64 (EPI_ACC_I64), h (EPI_SILU)
  int64_t ldy;
  const int32_t* bias;    // optional [N]: rescaled bias added after the i16 clamp (linear.rs:132-145)
  SiluParams silu;
  const int64_t* xsum;    // EPI_W16: [M] sum of each activation row over K
  // Exchange of a tensor-parallel row-parallel layer over peer memory.
  // Scatter (EPI_ACC_I64, xs_world > 0): the exact partial of output row m
  // goes to rank o = m / xs_rows, into xs_dst[o] at row xs_rank * xs_rows +
  // m % xs_rows (every receive buffer holds one slab of xs_rows rows per
  // sender). Gather (requant modes, xg_world > 0): the requantised row m goes
  // to every xg_dst[o] at row xg_row0 + m.
  void* xs_dst[MYL_XCHG_MAX];
  int64_t xs_rows;
  int xs_rank, xs_world;
  void* xg_dst[MYL_XCHG_MAX];
  int64_t xg_row0;
  int xg_world;
  // Broadcast (EPI_ACC_I64, xb_world > 0): the exact partial of output (m, n)
  // goes to every rank o, into xb_dst[o] at xb_rank * xb_slab + m * ldy + n
  // (tensor-parallel decode: each rank then sums all slabs locally).
  void* xb_dst[MYL_XCHG_MAX];
  int64_t xb_slab;
  int xb_rank, xb_world;
};

// ---- programmatic dependent launch ---------------------------------------------
// Every kernel of the library starts with pdl_wait(): when it is launched with
// programmatic stream serialization it may be scheduled before its
// predecessor grid has finished, and griddepcontrol.wait holds it until that
// grid has completed and its memory is visible; launched normally, the wait
// returns at once. pdl_launch() then lets the kernel's own successor launch
// early (it waits in turn). Before the wait a kernel writes no global memory
// and reads none that an earlier kernel writes (the GEMVs read their weights,
// which only registration writes, before it).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- requant -----------------------------------------------------------------

// fixed_point.rs:57-71: RNE right shift of a two's-complement value, s in [1, 62].
__device__ __forceinline__ int64_t rshift_rne_i64(int64_t v, int s) {
  const int64_t q = v >> s;
  const int64_t r = v & ((int64_t(1) << s) - 1);
  const int64_t h = int64_t(1) << (s - 1);
  return q + ((r > h) | ((r == h) & (q & 1)));
}

// fixed_point.rs:184-191 with the host-validated signed shift s in [-63, 62].
__device__ __forceinline__ int64_t rescale_i64_signed(int64_t acc, int s) {
  if (s > 0) return rshift_rne_i64(acc, s);
  if (s == 0) return acc;
  return int64_t(uint64_t(acc) << (-s));
}

__device__ __forceinline__ int64_t clamp_i64(int64_t v, int64_t lo, int64_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

// Multiplier mode: rne(acc * m, s) in 128-bit, s in [0, 126], saturated to
// [lo, hi]. The i128 RNE restates fixed_point.rs:155-169.
__device__ __forceinline__ int64_t requant_mult(int64_t acc, int32_t m, int s, int64_t lo,
                                                int64_t hi) {
  __int128 p = (__int128)acc * (__int128)m;
  if (s > 0) {
    const __int128 one = 1;
    const __int128 q = p >> s;
    const __int128 r = p & ((one << s) - 1);
    const __int128 h = one << (s - 1);
    p = q + (((r > h) || (r == h && (q & 1))) ? 1 : 0);
  }
  if (p < (__int128)lo) return lo;
  if (p > (__int128)hi) return hi;
  return (int64_t)p;
}

// fixed_point.rs:39-53 for i32, s in [1, 30].
__device__ __forceinline__ int32_t rshift_rne_i32(int32_t v, int s) {
  const int32_t q = v >> s;
  const int32_t r = v & ((1 << s) - 1);
  const int32_t h = 1 << (s - 1);
  return q + ((r > h) | ((r == h) & (q & 1)));
}

// Round-half-even right shift by s in [1, 30] with one add: for q = v >> s,
// (v + c + (q & 1)) >> s with c = 2^(s-1) - 1 adds 1 to q exactly when the
// remainder is above half, or equal to half with q odd (fixed_point.rs:39-53).
// Needs v + 2^(s-1) inside i32.
__device__ __forceinline__ int32_t rne_add_i32(int32_t v, int s, int32_t c) {
  return (v + c + ((v >> s) & 1)) >> s;
}

// mlp.rs:52-63 for one channel pair: gate g and up u are the clamped int16
// outputs of the two projections. g goes to the LUT domain with rescale (i32,
// fixed_point.rs:173-180), is truncated to i16 and offset with Rust release
// (wrapping) i16 arithmetic, clamped to the table (integer_math.rs:166-170);
// the LUT value times u is rescaled in i64 to the down projection's input
// scale and clamped to i16.
__device__ __forceinline__ int16_t silu_combine(const SiluParams& sp, int32_t g, int32_t u) {
  int32_t gd;
  if (sp.s1 > 0) gd = rshift_rne_i32(g, sp.s1);
  else if (sp.s1 == 0) gd = g;
  else gd = int32_t(uint32_t(g) << (-sp.s1));
  const int16_t g16 = int16_t(uint16_t(uint32_t(gd)));
  int idx = int(int16_t(uint16_t(uint16_t(g16) + uint16_t(sp.offset))));
  idx = idx < 0 ? 0 : idx;
  idx = idx > sp.lut_hi ? sp.lut_hi : idx;
  const int64_t prod = int64_t(sp.lut[idx]) * int64_t(u);
  return int16_t(clamp_i64(rescale_i64_signed(prod, sp.s2), -32768, 32767));
}

// silu_combine split for the tensor-core epilogue, where g and u are already
// clamped to int16: silu_index gives the table index of g (branch-free in
// s1), silu_product rescales lut[idx] * u. |lut * u| <= 2^30 fits in i32, so
// the i64 rescale of mlp.rs:60-62 equals the i32 round-half-even shift for
// s2 in [1, 30]; s2 >= 31 always rounds |prod| <= 2^30 to 0 (2^30 / 2^31 is a
// tie that goes to the even 0); s2 <= 0 takes the i64 path.
__device__ __forceinline__ int silu_index(const SiluParams& sp, int32_t g) {
  const int s = max(sp.s1, 1);
  const int32_t right = rne_add_i32(g, s, (1 << (s - 1)) - 1);  // |g| <= 2^15
  const int32_t gd = sp.s1 > 0 ? right : int32_t(uint32_t(g) << max(-sp.s1, 0));
  const int idx = int(int16_t(uint16_t(uint32_t(gd) + uint32_t(sp.offset))));
  return max(0, min(idx, sp.lut_hi));
}

__device__ __forceinline__ int32_t silu_product(const SiluParams& sp, int32_t lut_value, int32_t u) {
  const int32_t prod = lut_value * u;
  if (sp.s2 > 0) {
    if (sp.s2 >= 31) return 0;
    return max(-32768, min(rshift_rne_i32(prod, sp.s2), 32767));
  }
  return int32_t(clamp_i64(rescale_i64_signed(int64_t(prod), sp.s2), -32768, 32767));
}

// Stores h for (m, channel pair i) (if y is given) and its byte planes (if
// requested).
__device__ __forceinline__ void silu_store(const Epilogue& ep, int64_t m, int64_t i, int16_t h) {
  if (ep.y) static_cast<int16_t*>(ep.y)[m * ep.ldy + i] = h;
  if (ep.silu.h_hi) {
    ep.silu.h_hi[m * ep.silu.ldp + i] = uint8_t((h >> 8) + 128);
    ep.silu.h_lo[m * ep.silu.ldp + i] = uint8_t(h & 0xFF);
  }
}

// Requant of one accumulator of channel n to its clamped output value
// (shift or multiplier mode; the bias, if any, is added after the clamp).
__device__ __forceinline__ int64_t requant_value(const Epilogue& ep, int64_t n, int64_t acc) {
  const int64_t lo = ep.out_i32 ? int64_t(INT32_MIN) : -32768;
  const int64_t hi = ep.out_i32 ? int64_t(INT32_MAX) : 32767;
  int64_t v;
  if (ep.mode == EPI_MULT) v = requant_mult(acc, ep.mult[n], int(uint8_t(ep.shift[n])), lo, hi);
  else v = clamp_i64(rescale_i64_signed(acc, ep.shift[n]), lo, hi);
  if (ep.bias) v = clamp_i64(v + ep.bias[n], lo, hi);
  return v;
}

// EPI_W16: an int16 weight row w = 256*hi + lo with hi = w >> 8 and
// lo_off = (w & 255) - 128 (both int8) gives
//   sum_k w*x = 256*sum hi*x + sum lo_off*x + 128*sum x,
// the exact i64 accumulator of the LM head's path A (model.rs:285-296), which
// is rescaled by the row's shift and clamped to i32 (model.rs:293-295).
__device__ __forceinline__ void w16_store(const Epilogue& ep, int64_t m, int64_t i, int64_t a_hi,
                                          int64_t a_lo) {
  const int64_t acc = a_hi * 256 + a_lo + 128 * ep.xsum[m];
  static_cast<int32_t*>(ep.y)[m * ep.ldy + i] =
      int32_t(clamp_i64(rescale_i64_signed(acc, ep.shift[i]), INT32_MIN, INT32_MAX));
}

// Applies the epilogue to one exact accumulator of output (m, n).
__device__ __forceinline__ void epilogue_store(const Epilogue& ep, int64_t m, int64_t n,
                                               int64_t acc) {
  if (ep.mode == EPI_ACC_I64) {
    if (ep.xb_world > 0) {
      const int64_t idx = ep.xb_rank * ep.xb_slab + m * ep.ldy + n;
      for (int o = 0; o < ep.xb_world; ++o) static_cast<int64_t*>(ep.xb_dst[o])[idx] = acc;
    } else if (ep.xs_world > 0) {
      const int64_t o = m / ep.xs_rows;
      static_cast<int64_t*>(ep.xs_dst[o])[(ep.xs_rank * ep.xs_rows + (m - o * ep.xs_rows)) * ep.ldy + n] =
          acc;
    } else {
      static_cast<int64_t*>(ep.y)[m * ep.ldy + n] = acc;
    }
    return;
  }
  const int64_t v = requant_value(ep, n, acc);
  if (ep.xg_world > 0) {
    const int64_t idx = (ep.xg_row0 + m) * ep.ldy + n;
    for (int o = 0; o < ep.xg_world; ++o) {
      if (ep.out_i32) static_cast<int32_t*>(ep.xg_dst[o])[idx] = int32_t(v);
      else static_cast<int16_t*>(ep.xg_dst[o])[idx] = int16_t(v);
    }
    return;
  }
  if (ep.out_i32) static_cast<int32_t*>(ep.y)[m * ep.ldy + n] = int32_t(v);
  else static_cast<int16_t*>(ep.y)[m * ep.ldy + n] = int16_t(v);
}

// Per-channel requant with the channel's parameters already in registers
// (EPI_SHIFT / EPI_SILU use the shift, EPI_MULT the multiplier too).
struct ChannelRequant {
  int mode, out_i32, shift;
  int32_t mult, bias;
  __device__ __forceinline__ void load(const Epilogue& ep, int64_t n) {
    mode = ep.mode;
    out_i32 = ep.out_i32;
    shift = 0;
    mult = 1;
    bias = ep.bias ? ep.bias[n] : 0;
    if (mode == EPI_MULT) { shift = int(uint8_t(ep.shift[n])); mult = ep.mult[n]; }
    else shift = ep.shift[n];
  }
  __device__ __forceinline__ int64_t apply(int64_t acc) const {
    const int64_t lo = out_i32 ? int64_t(INT32_MIN) : -32768;
    const int64_t hi = out_i32 ? int64_t(INT32_MAX) : 32767;
    const int64_t v = (mode == EPI_MULT) ? requant_mult(acc, mult, shift, lo, hi)
                                         : clamp_i64(rescale_i64_signed(acc, shift), lo, hi);
    return bias ? clamp_i64(v + bias, lo, hi) : v;
  }
};

// ---- PTX wrappers ----------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and leaves the barrier alone) once timeout_ns
// has passed or *abort (if given) became nonzero.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint64_t timeout_ns, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  }
}

// 2D tiled TMA load global -> shared, completion counted on an mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 (5th-generation tensor core, TMEM accumulators) -------------------

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) x B(smem desc)^T, int8 kind, int32 accumulate.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on an mbarrier once all previously issued MMAs of this thread are done.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit words: thread t of the warp receives the 32
// consecutive columns of TMEM lane (lane_base + t).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 8 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms.
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused
// for swizzled K-major, 1), stride byte offset >> 4 [32,46) (1024 B between
// 8-row groups), version 1 [46,48), layout type 2 = 128B swizzle [61,64).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3FFFF) >> 4);
  d |= uint64_t(1) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// ---- CTA pairs (cluster of 2; one MMA of M = 256 spans both SMs) ------------
// In a pair MMA the even CTA issues; each CTA holds half of A (its 128 rows)
// and half of B (N/2 columns) at the same shared-memory offsets, and receives
// its 128 rows x N columns of D in its own TMEM.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// All threads of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (here: the even CTA's). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// MMA completion signal (tcgen05.commit, not a memory load) delivered to the
// mbarrier at the same offset in both CTAs of the pair (CTA mask 0b11).
__device__ __forceinline__ void mma_commit_pair_both(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

// Instruction descriptor, kind::i8: D = s32, A/B signedness, both K-major,
// N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n, bool a_signed, bool b_signed) {
  return (2u << 4) | (uint32_t(a_signed) << 7) | (uint32_t(b_signed) << 10) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

}  // namespace myl
