// rownorm.cuh — the residual add and RMSNorm of one row by one thread block,
// shared by the norm kernels (forward.cuh) and the decode GEMV's prologue
// (gemv.cuh), which normalises the activation row it stages.
//
// rmsnorm_i16: INTEGER_LLM/kernels/src/rmsnorm.rs:61-153; residual adds:
// runtime/src/model.rs:588-593, :666-671. Shifts and spans are validated on
// the host (model.cuh) before any launch.
#pragma once

#include "common.cuh"

namespace myl {

// fixed_point.rs:173-180 (i32 rescale) with the host-validated signed shift
// s = in - out in [-31, 30]; a left shift wraps as in a release build.
__device__ __forceinline__ int32_t rescale_i32_s(int32_t v, int s) {
  if (s > 0) return rshift_rne_i32(v, s);
  if (s == 0) return v;
  return int32_t(uint32_t(v) << (-s));
}

__device__ __forceinline__ int16_t clamp16(int64_t v) {
  return int16_t(v < -32768 ? -32768 : (v > 32767 ? 32767 : v));
}

// fixed_point.rs:155-169 on i128, s in [0, 127].
__device__ __forceinline__ __int128 rne_i128(__int128 v, int s) {
  if (s == 0) return v;
  const __int128 one = 1;
  const __int128 q = v >> s;
  const __int128 r = v & ((one << s) - 1);
  const __int128 h = one << (s - 1);
  return q + (((r > h) || (r == h && (q & 1))) ? 1 : 0);
}

// ---- residual add + RMSNorm -----------------------------------------------------
// Residual add (model.rs:588-593, :666-671), optional:
//   r[i] = clamp_i16(rescale_i64(rescale_i64(h[i], seg_in[i], acc[i]) + add[i], acc[i], seg_out[i]))
//   with s1[i] = seg_in - acc and s2[i] = acc - seg_out (signed, [-63, 62]).
// rmsnorm_i16 (rmsnorm.rs:61-153) of r with the channel shifts of seg_out:
//   ref = max x_shift; acc = sum r_i^2 << align2[i] (i128), align2 = 2 (ref - x_shift[i]);
//   M = (acc * inv_n) >> 20; q = least even shift with (M >> q) <= lut_len - 1;
//   lut_val = lut[min(rne(M, q), lut_len - 1)];
//   y_i = clamp_i16(clamp_i32(shifted(r_i * lut_val * gamma_i, norm_frac + sbase[i]))),
//   norm_frac = lut_out + lut_in / 2 + q / 2, sbase[i] = gamma_shift[i] + x_shift[i] - ref - out.
struct NormParams {
  const uint8_t* align2;   // [H]
  const int8_t* gamma;     // [H]
  const int16_t* sbase;    // [H]
  const int16_t* lut;
  int32_t lut_len;
  int32_t frac0;           // lut_output_frac + lut_input_shift / 2
  int64_t inv_n;
  int64_t H;
};

struct ResidParams {
  const int16_t* add;      // [rows][ld_add], null: no residual add (plain RMSNorm)
  int64_t ld_add;
  const int8_t* s1;        // [H]
  const int8_t* s2;        // [H]
  int16_t* resid_out;      // [rows][ld_res] the new residual stream (may be the input)
  int64_t ld_res;
  // Tensor parallelism: the added projection output is the requant of the
  // exact sum of nparts int64 partial slabs (parts + o * part_slab, rows of H),
  // clamp_i16(rescale_i64(sum, part_shift[i])) (linear.rs:61-68 after the
  // row-parallel sum); `add` is then ignored.
  const int64_t* parts;
  int nparts;
  int64_t part_slab;
  const int8_t* part_shift;
};

constexpr int NORM_THREADS = 256;

__device__ __forceinline__ __int128 warp_sum_i128(__int128 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long lo = (unsigned long long)(v), hi = (unsigned long long)(v >> 64);
    const unsigned long long lo2 = __shfl_xor_sync(0xffffffffu, lo, o);
    const unsigned long long hi2 = __shfl_xor_sync(0xffffffffu, hi, o);
    v += (__int128)(((unsigned __int128)hi2 << 64) | (unsigned __int128)lo2);
  }
  return v;
}

// The same, for hidden sizes that are a multiple of 8 up to 8 * NORM_THREADS *
// NORM_NV: every thread issues all loads of its 16-byte vectors (the row, the
// added projection output, and the per-channel parameters) before using any,
// so one row costs about one memory latency instead of one per element.
constexpr int NORM_NV = 4;

__device__ __forceinline__ int16_t lane16(const uint4& v, int e) {
  const uint32_t w = e < 2 ? v.x : e < 4 ? v.y : e < 6 ? v.z : v.w;
  return int16_t(uint16_t(w >> (16 * (e & 1))));
}
__device__ __forceinline__ int8_t lane8(const uint2& v, int e) {
  return int8_t(uint8_t((e < 4 ? v.x : v.y) >> (8 * (e & 3))));
}
__device__ __forceinline__ uint4 pack16(const int16_t (&a)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = uint32_t(uint16_t(a[2 * i])) | (uint32_t(uint16_t(a[2 * i + 1])) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// rescale_i64 (fixed_point.rs:184-191) with the signed shift s in [-63, 62],
// without branches: a left shift wraps as in a release build, a right shift
// rounds half to even.
__device__ __forceinline__ int64_t rescale_s64(int64_t v, int s) {
  const int l = s < 0 ? -s : 0, rs = s > 0 ? s : 0;
  const int64_t w = int64_t(uint64_t(v) << l);
  const int64_t q = w >> rs;
  const int64_t rem = w - int64_t(uint64_t(q) << rs);  // [0, 2^rs)
  const int64_t half = (int64_t(1) << rs) >> 1;         // 0 when rs = 0
  return q + ((rem > half) | ((rem == half) & (rs > 0) & (q & 1)));
}

// rmsnorm.rs:140-151 for one channel: the product shifted by sh, then the i32
// and i16 clamps. Left shifts (negative sh) go through i128, out of line: they
// are rare, and the code stays small for the single-block decode launches.
__device__ __noinline__ int16_t norm_out_left(int64_t prod, int sh) {
  const __int128 w = (__int128)((unsigned __int128)(__int128)prod << (-sh));
  const int64_t t = w < (__int128)INT32_MIN ? INT32_MIN : (w > (__int128)INT32_MAX ? INT32_MAX : (int64_t)w);
  return clamp16(t);
}
__device__ __forceinline__ int16_t norm_out(int64_t prod, int sh) {
  if (sh >= 63) return 0;  // |prod| < 2^37 rounds to zero
  if (sh > 0) return clamp16(rshift_rne_i64(prod, sh));
  if (sh == 0) return clamp16(prod);
  return norm_out_left(prod, sh);
}

// The root-mean-square normaliser of one row from its square sum: the LUT
// value and norm_frac (rmsnorm.rs:99-125), or nf = -1000 for an all-zero row.
__device__ __noinline__ void norm_scale(__int128 a, const NormParams& np, int64_t* lut_val, int* nf) {
  if (a == 0) {
    *nf = -1000;
    *lut_val = 0;
    return;
  }
  const __int128 m = (a * (__int128)np.inv_n) >> 20;
  const __int128 max_idx = np.lut_len - 1;
  int q = 0;
  while ((m >> q) > max_idx) q += 2;
  __int128 idx = rne_i128(m, q);
  if (idx > max_idx) idx = max_idx;
  *lut_val = np.lut[int64_t(idx)];
  *nf = np.frac0 + q / 2;
}

// One 8-channel vector of a row: its loads (all issued at once), the residual
// add with the square sum, and the normalised output.
struct NormVec {
  uint4 x, a, sb;
  uint2 s1, s2, al, g;
};

__device__ __forceinline__ void norm_vec_load(NormVec& nv, const int16_t* __restrict__ xr, int64_t r,
                                              int v, const ResidParams& rp, const NormParams& np) {
  nv.x = *reinterpret_cast<const uint4*>(xr + 8 * v);
  if (rp.parts) {
    int64_t sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int o = 0; o < rp.nparts; ++o) {
      const longlong2* pp = reinterpret_cast<const longlong2*>(rp.parts + o * rp.part_slab + r * np.H + 8 * v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const longlong2 t2 = __ldcg(pp + q);
        sum[2 * q] += t2.x;
        sum[2 * q + 1] += t2.y;
      }
    }
    const uint2 ps = *reinterpret_cast<const uint2*>(rp.part_shift + 8 * v);
    int16_t a16[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) a16[e] = clamp16(rescale_s64(sum[e], lane8(ps, e)));
    nv.a = pack16(a16);
  } else if (rp.add) {
    nv.a = *reinterpret_cast<const uint4*>(rp.add + r * rp.ld_add + 8 * v);
  }
  if (rp.add || rp.parts) {
    nv.s1 = *reinterpret_cast<const uint2*>(rp.s1 + 8 * v);
    nv.s2 = *reinterpret_cast<const uint2*>(rp.s2 + 8 * v);
  }
  nv.al = *reinterpret_cast<const uint2*>(np.align2 + 8 * v);
  nv.g = *reinterpret_cast<const uint2*>(np.gamma + 8 * v);
  nv.sb = *reinterpret_cast<const uint4*>(np.sbase + 8 * v);
}

// residual add (nv.x becomes the row after the add), then the square sum:
// squares (< 2^31) shifted by at most 20 bits are summed in int64 (8192 of
// them stay below 2^63), wider alignments in i128
__device__ __forceinline__ void norm_vec_resid(NormVec& nv, bool radd, int64_t& acc64, __int128& acc128) {
  int16_t val[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    int64_t t = lane16(nv.x, e);
    if (radd) {
      const int64_t h = rescale_s64(t, lane8(nv.s1, e)) + int64_t(lane16(nv.a, e));
      t = clamp16(rescale_s64(h, lane8(nv.s2, e)));
    }
    val[e] = int16_t(t);
    const int a = uint8_t(lane8(nv.al, e));
    if (a <= 20) acc64 += (t * t) << a;
    else acc128 += (__int128)(t * t) << a;
  }
  nv.x = pack16(val);
}

__device__ __forceinline__ uint4 norm_vec_out(const NormVec& nv, int64_t lv, int nf) {
  int16_t y[8];
#pragma unroll
  for (int e = 0; e < 8; ++e)
    y[e] = nf == -1000 ? int16_t(0)
                       : norm_out(int64_t(lane16(nv.x, e)) * lv * int64_t(lane8(nv.g, e)), nf + lane16(nv.sb, e));
  return pack16(y);
}

// Shared memory of block_row_norm.
struct RowNormSmem {
  __int128 part[NORM_THREADS / 32];
  int64_t lut_val;
  int nf;
};

// Residual add and RMSNorm of row r by the whole block (blockDim.x ==
// NORM_THREADS; H % 8 == 0, H <= 8 * NORM_THREADS * NORM_NV). xr is the row of
// the residual stream; rp the optional residual add (as ResidParams, row r of
// `add` or of the partial slabs); with write_resid the row after the add goes
// to rp.resid_out. Each normalised 8-element vector v goes to store(v, packed).
template <class Store>
__device__ __forceinline__ void block_row_norm(const int16_t* __restrict__ xr, int64_t r,
                                               const ResidParams& rp, const NormParams& np,
                                               bool write_resid, RowNormSmem& sm, Store store) {
  const int nv = int(np.H / 8);
  NormVec vecs[NORM_NV];
  const bool radd = rp.add || rp.parts;
#pragma unroll
  for (int k = 0; k < NORM_NV; ++k) {
    const int v = threadIdx.x + k * NORM_THREADS;
    if (v < nv) norm_vec_load(vecs[k], xr, r, v, rp, np);
  }
  int64_t acc64 = 0;
  __int128 acc128 = 0;
#pragma unroll
  for (int k = 0; k < NORM_NV; ++k) {
    const int v = threadIdx.x + k * NORM_THREADS;
    if (v < nv) {
      norm_vec_resid(vecs[k], radd, acc64, acc128);
      if (radd && write_resid && rp.resid_out)
        *reinterpret_cast<uint4*>(rp.resid_out + r * rp.ld_res + 8 * v) = vecs[k].x;
    }
  }
  __int128 acc = (__int128)acc64 + acc128;
  acc = warp_sum_i128(acc);
  if ((threadIdx.x & 31) == 0) sm.part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    __int128 a = 0;
    for (int w = 0; w < NORM_THREADS / 32; ++w) a += sm.part[w];
    int64_t lv;
    int nf;
    norm_scale(a, np, &lv, &nf);
    sm.lut_val = lv;
    sm.nf = nf;
  }
  __syncthreads();
  const int nf = sm.nf;
  const int64_t lv = sm.lut_val;
#pragma unroll
  for (int k = 0; k < NORM_NV; ++k) {
    const int v = threadIdx.x + k * NORM_THREADS;
    if (v < nv) store(v, norm_vec_out(vecs[k], lv, nf));
  }
  __syncthreads();  // sm is reused by the next row
}

// ---- one row over a cluster of CTAs (few rows: decode) ---------------------------
// A row's vectors are split over the NORM_CL CTAs of a cluster (NORM_CL_THREADS
// threads each, one vector per thread); each CTA's int128 square sum is read
// pushed into every CTA of the cluster through distributed shared memory, so
// the per-row work is spread over NORM_CL SMs instead of one.
constexpr int NORM_CL = 8;
constexpr int NORM_CL_THREADS = 128;

__device__ __forceinline__ void st_shared_cluster_u64(uint32_t cluster_addr, unsigned long long v) {
  asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(cluster_addr), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_shared_cluster_u64(uint32_t cluster_addr) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(cluster_addr) : "memory");
  return v;
}

}  // namespace myl
