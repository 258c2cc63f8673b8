// myl_w8a16.cu — libmyl_w8a16.so: C ABI, weight registry and kernel dispatch.
//
// The ABI (include/myl_w8a16.h) replaces the CUDA slot of the reference's
// Backend trait (INTEGER_LLM/kernels/src/backends/cuda.rs:80-261) and the free
// functions the runtime calls (kernels/src/linear.rs:43, :87; the LM-head loop
// of runtime/src/model.rs:297-307). There is no CPU path in this library.
//
// Dispatch for y = requant(W x), x with M rows:
//   M <= gemv_max_m (default 4)  CUDA-core GEMV (gemv.cuh), HBM-bound decode.
//   otherwise                    split x into hi/lo byte planes and run the
//                                persistent tcgen05 split-byte GEMM (gemm_tc.cuh)
//                                on 128-channel x BN-token tiles, BN = 32/64/128.
//   Too few tiles for the 148 SMs, or K > 65536, splits K; the slices write
//   exact int64 partials that reduce_requant_kernel adds and requantises.
#include "../../include/myl_w8a16.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "moe.cuh"
#include "backward.cuh"
#include "select.cuh"
#include "wire.cuh"
#include "forward.cuh"

using namespace myl;

// ---------------------------------------------------------------------------------
// errors

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CUDA_TRY(expr)                                                                     \
  do {                                                                                     \
    cudaError_t e_ = (expr);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      return fail(MYL_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_),    \
                  __FILE__, __LINE__);                                                     \
  } while (0)

#define TRY(expr)                  \
  do {                             \
    int rc_ = (expr);              \
    if (rc_ != MYL_OK) return rc_; \
  } while (0)

// ---------------------------------------------------------------------------------
// objects

struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
};

struct myl_weight {
  int64_t N = 0, K = 0, ldp = 0;  // device copy is [N][ldp] int8, ldp = round_up(K, 16)
  int8_t* d_W = nullptr;
  int32_t* d_wsum = nullptr;       // [N][wsum_ld]: per-row prefix sums over 128-byte K tiles
  // int16 weights (myl_weight16_register): N = 2 * n16 int8 rows, row 2i = high
  // byte and row 2i + 1 = low byte - 128 of int16 row i; w_shifts has n16 entries.
  bool w16 = false;
  int64_t n16 = 0;
  // linear_backward: rows sorted by shift and the groups of equal shift,
  // made on the first backward call.
  int bwd_ref = -1;
  int bwd_ngroups = 0;
  int32_t* d_bwd_perm = nullptr;
  BwdGroup* d_bwd_groups = nullptr;
  int64_t wsum_ld = 0;             // K tiles + 1
  std::vector<uint8_t> w_shifts;
  CUtensorMap tm128{};             // TMA map with a 128-row box (one channel tile)
  // Backend-trait cache key: the host address, and a digest of the bytes
  // (checked on every hit, so a reused address with new contents re-registers).
  const int8_t* host_W = nullptr;
  const uint8_t* host_shifts = nullptr;
  uint64_t host_digest = 0;
};

struct myl_requant {
  int64_t N = 0;
  int mode = 0;
  int8_t* d_shift = nullptr;
  int32_t* d_mult = nullptr;
  int32_t* d_bias = nullptr;  // rescaled bias (myl_requant_set_bias)
};

struct myl_mlp {
  int64_t H = 0, I = 0;
  myl_weight* w_gu = nullptr;    // [2I][H]: row 2i = gate_i, row 2i+1 = up_i
  myl_weight* w_down = nullptr;  // [H][I]
  int8_t* d_shift_gu = nullptr;  // [2I] signed total shifts of the gate/up rows
  int8_t* d_shift_down = nullptr;  // [H]
  int16_t* d_lut = nullptr;
  int lut_hi = 0, offset = 0, s1 = 0, s2 = 0;
};

constexpr int MYL_PIPE = 8;  // chunks of a pipelined host-pointer call

struct myl_ctx {
  int device = 0, sm = 0, num_sms = 0;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;
  int* h_err = nullptr;  // pinned
  uint64_t timeout_ns = 2000000000ull;
  int gemv_max_m = 4, force_split_k = 0, force_tile = 0, inject_fault = 0;
  int sm_limit = 0;  // persistent grids use at most this many SMs (0: all)
  int xbox = TC_XBOX;  // activation rows per TMA box of the tensor-core GEMM
  int pair_mode = 1;   // CTA-pair GEMM (M = 256 MMAs): 0 off, 1 for 128-token tiles
  int pair_slots = 0;  // co-resident CTA pairs of the pair kernel (0: not yet queried)
  int pdl = 0;         // launch with programmatic stream serialization (the forward's chains)
  int64_t launches = 0;
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  DevBuf x, y, rq, planes, part, h, hplanes, moe, xsum, crc;
  // Host-pointer calls on page-locked memory: copy-in and copy-out streams
  // and one event pair per chunk.
  cudaStream_t s_in = nullptr, s_out = nullptr;
  cudaEvent_t ev_in[MYL_PIPE] = {}, ev_comp[MYL_PIPE] = {};
  // The workspace buffers are shared by every call on the context; calls on
  // different streams are ordered through this event.
  cudaEvent_t ws_event = nullptr;
  cudaStream_t ws_last = nullptr;
  bool ws_used = false;
  std::unordered_map<const int8_t*, myl_weight*> backend_cache;
};

// SMs the persistent kernels may occupy (myl_set_sm_limit leaves the rest to
// kernels on other streams, e.g. a collective overlapping the GEMM).
static int sms(const myl_ctx* ctx) {
  return ctx->sm_limit > 0 ? std::min(ctx->sm_limit, ctx->num_sms) : ctx->num_sms;
}

// Launch configuration; with ctx->pdl the kernel may start while its
// predecessor on the stream finishes (every kernel begins with pdl_wait()).
struct LaunchCfg {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  LaunchCfg(const myl_ctx* ctx, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
            unsigned cluster_x = 0) {
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    unsigned n = 0;
    if (cluster_x) {
      attr[n].id = cudaLaunchAttributeClusterDimension;
      attr[n].val.clusterDim.x = cluster_x;
      attr[n].val.clusterDim.y = 1;
      attr[n].val.clusterDim.z = 1;
      ++n;
    }
    if (ctx->pdl) {
      attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[n].val.programmaticStreamSerializationAllowed = 1;
      ++n;
    }
    cfg.numAttrs = n;
  }
};

static bool capturing(cudaStream_t st) {
  cudaStreamCaptureStatus s = cudaStreamCaptureStatusNone;
  return cudaStreamIsCapturing(st, &s) == cudaSuccess && s != cudaStreamCaptureStatusNone;
}

static int ws_acquire(myl_ctx* ctx, cudaStream_t st) {
  if (ctx->ws_used && ctx->ws_last != st && !capturing(st))
    CUDA_TRY(cudaStreamWaitEvent(st, ctx->ws_event, 0));
  return MYL_OK;
}

static int ws_release(myl_ctx* ctx, cudaStream_t st) {
  if (capturing(st)) return MYL_OK;
  CUDA_TRY(cudaEventRecord(ctx->ws_event, st));
  ctx->ws_last = st;
  ctx->ws_used = true;
  return MYL_OK;
}

// Bumped whenever a workspace buffer moves, so that a captured CUDA graph
// holding the old address is captured again before its next replay.
static uint64_t g_ws_epoch = 1;

static int ensure(DevBuf& b, size_t bytes) {
  if (b.cap >= bytes) return MYL_OK;
  ++g_ws_epoch;
  if (b.p) CUDA_TRY(cudaFree(b.p));
  b.p = nullptr;
  b.cap = 0;
  size_t cap = std::max<size_t>(bytes, 4096);
  CUDA_TRY(cudaMalloc(&b.p, cap));
  b.cap = cap;
  return MYL_OK;
}

static int encode_map(myl_ctx* ctx, CUtensorMap* map, const void* base, int64_t cols, int64_t rows,
                      int64_t ld_bytes, int box_rows) {
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld_bytes)};
  cuuint32_t box[2] = {cuuint32_t(TC_BK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = ctx->encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MYL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return MYL_OK;
}

// ---------------------------------------------------------------------------------
// requant parameter validation (host). Restates the overflow behaviour of the
// reference's debug build: u8 addition w_shift + act_frac (linear.rs:66),
// i8 subtraction and shift widths in rescale_i64 (fixed_point.rs:184-191,
// :57-71).

static int signed_total_shift(uint8_t w_shift, uint8_t act_frac, uint8_t out_frac, int8_t* s) {
  unsigned in_frac = unsigned(w_shift) + unsigned(act_frac);
  if (in_frac > 255u) return fail(MYL_ERR_OVERFLOW, "w_shift + act_frac = %u overflows u8", in_frac);
  int d = int(int8_t(uint8_t(in_frac))) - int(int8_t(out_frac));
  if (d < -128 || d > 127) return fail(MYL_ERR_OVERFLOW, "in_frac - out_frac overflows i8");
  if (d > 62) return fail(MYL_ERR_OVERFLOW, "right shift %d overflows the i64 mask", d);
  if (d < -63) return fail(MYL_ERR_OVERFLOW, "left shift %d exceeds i64 width", -d);
  *s = int8_t(d);
  return MYL_OK;
}

static int64_t out_features(const myl_weight* w) { return w->w16 ? w->n16 : w->N; }

static int shift_plan(const myl_weight* w, uint8_t act_frac, const uint8_t* out_frac, int per_channel,
                      std::vector<int8_t>& s) {
  s.resize(size_t(out_features(w)));
  for (int64_t r = 0; r < out_features(w); ++r)
    TRY(signed_total_shift(w->w_shifts[size_t(r)], act_frac, per_channel ? out_frac[r] : out_frac[0],
                           &s[size_t(r)]));
  return MYL_OK;
}

// ---------------------------------------------------------------------------------
// kernel launchers

using GemvFn = void (*)(const int8_t*, int64_t, int64_t, const int16_t*, int64_t, int64_t, int64_t,
                        Epilogue, int64_t);

template <int MT, int R, int U, int KW>
static void* gemv_ptr() {
  return reinterpret_cast<void*>(&gemv_w8a16_kernel<MT, R, U, KW>);
}

struct GemvVariant {
  void* fn;
  int R, KW;
};

// Rows per warp R, 16-byte chunks per lane in flight U and warps per row group
// KW, from measurements on B200: two rows per warp and ~128 KB of loads in
// flight per SM; long rows (K >= 8192) want twice the chunks per lane; when
// the rows alone give too few warp jobs (N/R*KW below ~40 warps per SM) the
// warps of a block share rows and split K.
static GemvVariant gemv_variant(int M, int64_t K, int64_t N, int num_sms) {
  const int64_t chunks = (K + 15) / 16;
  int kw = 1;
  while (kw < 8 && (N / 2) * kw < int64_t(40) * num_sms && chunks / (kw * 2) >= 64) kw *= 2;
  switch (M) {
    case 1:
      if (K >= 8192) {
        if (kw >= 8) return {gemv_ptr<1, 2, 8, 8>(), 2, 8};
        if (kw == 4) return {gemv_ptr<1, 2, 8, 4>(), 2, 4};
        if (kw == 2) return {gemv_ptr<1, 2, 8, 2>(), 2, 2};
        return {gemv_ptr<1, 2, 8, 1>(), 2, 1};
      }
      if (kw >= 4) return {gemv_ptr<1, 2, 4, 4>(), 2, 4};
      if (kw == 2) return {gemv_ptr<1, 2, 4, 2>(), 2, 2};
      return {gemv_ptr<1, 2, 4, 1>(), 2, 1};
    case 2:
      if (kw >= 4) return {gemv_ptr<2, 2, 4, 4>(), 2, 4};
      if (kw == 2) return {gemv_ptr<2, 2, 4, 2>(), 2, 2};
      return {gemv_ptr<2, 2, 4, 1>(), 2, 1};
    case 3:
      if (kw >= 4) return {gemv_ptr<3, 2, 2, 4>(), 2, 4};
      if (kw == 2) return {gemv_ptr<3, 2, 2, 2>(), 2, 2};
      return {gemv_ptr<3, 2, 2, 1>(), 2, 1};
    default:
      if (kw >= 4) return {gemv_ptr<4, 2, 2, 4>(), 2, 4};
      if (kw == 2) return {gemv_ptr<4, 2, 2, 2>(), 2, 2};
      return {gemv_ptr<4, 2, 2, 1>(), 2, 1};
  }
}

// Per-(device, kernel) launch facts cached across calls: the dynamic shared
// memory attribute (device state) and the resident blocks per SM.
struct LaunchCache {
  std::mutex mu;
  std::map<std::pair<int, const void*>, std::pair<int, int>> smem_occ;  // -> (smem set, blocks/SM)
};
static LaunchCache g_launch_cache;

static int kernel_smem_occupancy(int device, const void* fn, int threads, size_t smem,
                                 int* resident) {
  std::lock_guard<std::mutex> lock(g_launch_cache.mu);
  const auto key = std::make_pair(device, fn);
  auto it = g_launch_cache.smem_occ.find(key);
  if (it != g_launch_cache.smem_occ.end() && it->second.first == int(smem)) {
    if (resident) *resident = it->second.second;
    return MYL_OK;
  }
  CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  int r = 0;
  CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, fn, threads, smem));
  g_launch_cache.smem_occ[key] = {int(smem), r};
  if (resident) *resident = r;
  return MYL_OK;
}

static constexpr int GEMV_SMEM_BUDGET = 100 * 1024;

static inline int64_t round_up16(int64_t v) { return (v + 15) & ~int64_t(15); }

template <int MT, int U>
static void* gemv_balanced_ptr() {
  return reinterpret_cast<void*>(&gemv_balanced_kernel<MT, U>);
}

// The balanced GEMV (one K slice): grid = resident blocks x SMs, every warp
// an equal share of whole row pairs.
static int launch_gemv_balanced(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                                int64_t ldx, const Epilogue& ep, cudaStream_t st) {
  int64_t K = w->K, N = w->N;
  void* fn = nullptr;
  switch (M) {
    case 1: fn = gemv_balanced_ptr<1, 6>(); break;  // 124 registers, two blocks per SM
    default: fn = gemv_balanced_ptr<2, 4>(); break;
  }
  const size_t smem = size_t(M) * size_t(round_up16(K)) * 2;
  int resident = 0;
  TRY(kernel_smem_occupancy(ctx->device, fn, GEMV_THREADS, smem, &resident));
  const unsigned grid = unsigned(std::max(1, resident) * sms(ctx));
  const int8_t* dW = w->d_W;
  int64_t ldw = w->ldp;
  Epilogue e = ep;
  void* args[] = {(void*)&dW, (void*)&ldw, (void*)&N, (void*)&x, (void*)&ldx, (void*)&K, (void*)&e};
  LaunchCfg lc(ctx, dim3(grid), dim3(GEMV_THREADS), smem, st);
  CUDA_TRY(cudaLaunchKernelExC(&lc.cfg, fn, args));
  ctx->launches++;
  return MYL_OK;
}

// The balanced kernel wins where the row-group kernel's blocks would fall
// unevenly on the SMs: one or two activation rows and at most two row pairs
// per warp of a full wave (measured on B200: 7B down projection 22.3 -> 18.8 us,
// the gate/up shape with four pairs per warp stays on the row-group kernel).
static bool use_balanced_gemv(const myl_ctx* ctx, const myl_weight* w, int64_t M) {
  if (M > 2 || std::getenv("MYL_GEMV_CLASSIC")) return false;
  const int64_t npairs = (w->N + 1) / 2, warps = int64_t(sms(ctx)) * 2 * GEMV_WARPS;
  return npairs <= 2 * warps;
}

template <int CPL>
static void* gemv_stream_ptr() {
  return reinterpret_cast<void*>(&gemv_stream_kernel<CPL>);
}

// The streaming GEMV (one activation row, rows of at most 8 * 32 chunks):
// grid = resident blocks x SMs, every warp an equal share of whole row pairs.
// Returns false (nothing launched) for other shapes.
static bool gemv_stream_fits(const myl_weight* w, int64_t M) {
  return M == 1 && (w->K + 15) / 16 <= 8 * 32 && !std::getenv("MYL_GEMV_CLASSIC");
}

static int launch_gemv_stream(myl_ctx* ctx, const myl_weight* w, const int16_t* x, const Epilogue& ep,
                              cudaStream_t st) {
  int64_t K = w->K, N = w->N;
  const int64_t C = (K + 15) / 16;
  void* fn = C <= 64    ? gemv_stream_ptr<2>()
           : C <= 128 ? gemv_stream_ptr<4>()
           : C <= 224 ? gemv_stream_ptr<7>()  // K = 3584: no idle chunk slot
                      : gemv_stream_ptr<8>();
  const size_t smem = size_t(round_up16(K)) * 2;
  int resident = 0;
  TRY(kernel_smem_occupancy(ctx->device, fn, GEMV_THREADS, smem, &resident));
  const int64_t pairs = (N + 1) / 2;
  const unsigned grid = unsigned(std::min<int64_t>(std::max(1, resident) * int64_t(sms(ctx)),
                                                   (pairs + GEMV_WARPS - 1) / GEMV_WARPS));
  const int8_t* dW = w->d_W;
  int64_t ldw = w->ldp;
  Epilogue e = ep;
  void* args[] = {(void*)&dW, (void*)&ldw, (void*)&N, (void*)&x, (void*)&K, (void*)&e};
  LaunchCfg lc(ctx, dim3(grid), dim3(GEMV_THREADS), smem, st);
  CUDA_TRY(cudaLaunchKernelExC(&lc.cfg, fn, args));
  ctx->launches++;
  return MYL_OK;
}

// The K-quarter GEMV (one activation row, rows of 257 to 384 chunks, e.g. the
// 0.5B down projection): grid = the resident blocks, balanced so that every
// block runs the same number of row-pair steps. (For the 7B down projection,
// 1184 chunks, it measured 23.8 us against the balanced kernel's 19.)
static int launch_gemv_ksplit(myl_ctx* ctx, const myl_weight* w, const int16_t* x, const Epilogue& ep,
                              cudaStream_t st) {
  int64_t K = w->K, N = w->N;
  void* fn = reinterpret_cast<void*>(&gemv_ksplit_kernel<3>);
  const size_t smem = size_t(round_up16(K)) * 2;
  int resident = 0;
  TRY(kernel_smem_occupancy(ctx->device, fn, GEMV_THREADS, smem, &resident));
  const int64_t steps_total = ((N + 1) / 2 + GKS_PAIRS - 1) / GKS_PAIRS;
  const int64_t slots = int64_t(std::max(1, resident)) * sms(ctx);
  const int64_t iters = (steps_total + slots - 1) / slots;
  const unsigned grid = unsigned((steps_total + iters - 1) / iters);
  const int8_t* dW = w->d_W;
  int64_t ldw = w->ldp;
  Epilogue e = ep;
  void* args[] = {(void*)&dW, (void*)&ldw, (void*)&N, (void*)&x, (void*)&K, (void*)&e};
  LaunchCfg lc(ctx, dim3(grid), dim3(GEMV_THREADS), smem, st);
  CUDA_TRY(cudaLaunchKernelExC(&lc.cfg, fn, args));
  ctx->launches++;
  return MYL_OK;
}

static int launch_gemv(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M, int64_t ldx,
                       const Epilogue& ep_final, cudaStream_t st) {
  if (ctx->force_split_k == 0 && gemv_stream_fits(w, M)) return launch_gemv_stream(ctx, w, x, ep_final, st);
  if (ctx->force_split_k == 0 && M == 1 && (w->K + 15) / 16 <= GKS_Q * 32 * 3 && !std::getenv("MYL_GEMV_CLASSIC"))
    return launch_gemv_ksplit(ctx, w, x, ep_final, st);
  GemvVariant v = gemv_variant(int(M), w->K, w->N, sms(ctx));
  const int64_t K = w->K;
  const int64_t ks_max = (GEMV_SMEM_BUDGET / (2 * M)) & ~int64_t(15);
  int ksplit = int((round_up16(K) + ks_max - 1) / ks_max);
  if (ctx->force_split_k > 0) ksplit = ctx->force_split_k;
  if (ksplit == 1 && ctx->force_split_k == 0 && use_balanced_gemv(ctx, w, M))
    return launch_gemv_balanced(ctx, w, x, M, ldx, ep_final, st);
  int64_t k_slice = round_up16((K + ksplit - 1) / ksplit);
  ksplit = int((K + k_slice - 1) / k_slice);
  const size_t smem = size_t(M) * size_t(k_slice) * 2;
  int resident = 0;
  TRY(kernel_smem_occupancy(ctx->device, v.fn, GEMV_THREADS, smem, &resident));
  const int64_t rows_per_block = int64_t(GEMV_WARPS / v.KW) * v.R;
  const int64_t row_blocks = (w->N + rows_per_block - 1) / rows_per_block;
  // Balanced grid: every block runs the same number of row-group iterations.
  const int64_t per_slice = std::max<int64_t>(1, int64_t(std::max(resident, 1)) * sms(ctx) / ksplit);
  const int64_t iters = (row_blocks + per_slice - 1) / per_slice;
  dim3 grid(unsigned((row_blocks + iters - 1) / iters), unsigned(ksplit));
  Epilogue ep = ep_final;
  int64_t slice_stride = 0;
  if (ksplit > 1) {
    TRY(ensure(ctx->part, size_t(ksplit) * size_t(M) * size_t(w->N) * 8));
    ep.mode = EPI_ACC_I64;
    ep.y = ctx->part.p;
    ep.ldy = w->N;
    ep.xs_world = 0;  // slice partials stay local; the final pass exchanges
    ep.xg_world = 0;
    ep.xb_world = 0;
    slice_stride = M * w->N;
  }
  const int8_t* dW = w->d_W;
  int64_t ldw = w->ldp, N = w->N;
  void* args[] = {(void*)&dW, (void*)&ldw, (void*)&N, (void*)&x, (void*)&ldx,
                  (void*)&K, (void*)&k_slice, (void*)&ep, (void*)&slice_stride};
  LaunchCfg lc(ctx, grid, dim3(GEMV_THREADS), smem, st);
  CUDA_TRY(cudaLaunchKernelExC(&lc.cfg, v.fn, args));
  ctx->launches++;
  if (ksplit > 1) {
    const int64_t total = M * w->N;
    unsigned blocks = unsigned(std::min<int64_t>((total + 255) / 256, int64_t(ctx->num_sms) * 8));
    LaunchCfg lr(ctx, dim3(blocks), dim3(256), 0, st);
    CUDA_TRY(cudaLaunchKernelEx(&lr.cfg, reduce_requant_kernel,
                                static_cast<const int64_t*>(ctx->part.p), ksplit, slice_stride, M,
                                w->N, ep_final));
    ctx->launches++;
  }
  return MYL_OK;
}

// Box height of the activation tensor maps for token tile BN (a power of two
// that divides BN); the kernel receives the same number in TcWork::xbox.
static int tc_xbox(const myl_ctx* ctx, int BN) { return std::min(ctx->xbox, BN); }

// Stage-ring depth per token tile: 192 KB of smem (one CTA per SM).
template <int BN>
struct TcStages;
template <> struct TcStages<32> { static constexpr int value = 8; };
template <> struct TcStages<64> { static constexpr int value = 6; };
template <> struct TcStages<128> { static constexpr int value = 4; };
// CTA pair: each SM holds the weight tile and one activation plane per stage.
constexpr int TC_PAIR_STAGES = 6;

// CTA pairs that can be resident at once for the pair kernel: SMs / 2, fewer
// when the GPCs' SM counts are odd (a pair shares a GPC).
template <typename Fn>
static int pair_slots(myl_ctx* ctx, Fn fn, size_t smem) {
  if (ctx->pair_slots > 0) return std::max(1, std::min(ctx->pair_slots, sms(ctx) / 2));
  TRY(kernel_smem_occupancy(ctx->device, reinterpret_cast<const void*>(fn), TC_THREADS, smem, nullptr));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(unsigned(2 * (ctx->num_sms / 2)));
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = ctx->num_sms / 2;
  }
  ctx->pair_slots = n;
  return std::max(1, std::min(n, sms(ctx) / 2));
}

template <int BN, int MODE, bool PAIR>
static int launch_tc_mode(myl_ctx* ctx, const myl_weight* w, const CUtensorMap& tm_xhi,
                          const CUtensorMap& tm_xlo, int64_t M, const TcWork& work,
                          const Epilogue& ep, int64_t slice_stride, cudaStream_t st) {
  constexpr int STAGES = PAIR ? TC_PAIR_STAGES : TcStages<BN>::value;
  using Cfg = TcCfg<BN, STAGES, PAIR>;
  auto fn = gemm_w8a16_tc_kernel<BN, STAGES, MODE, PAIR>;
  TRY(kernel_smem_occupancy(ctx->device, reinterpret_cast<const void*>(fn), TC_THREADS,
                            Cfg::SMEM_BYTES, nullptr));
  // Grouped work is sized on the device (the router's tile table): one CTA
  // (pair) per SM (pair of SMs); those without a unit exit after setup.
  const int64_t slots = PAIR ? pair_slots(ctx, fn, Cfg::SMEM_BYTES) : sms(ctx);
  const int64_t units = work.groups > 0 ? slots
                        : work.tail_tiles > 0
                            ? int64_t(work.full_units) + int64_t(work.tail_tiles) * work.tail_ks
                            : int64_t(work.tiles_n) * work.tiles_m * work.ksplit;
  const int64_t N = work.groups > 0 ? work.group_w_rows : w->N;  // channels per group
  TcWork wk = work;
  wk.wsum = w->d_wsum;
  wk.wsum_ld = w->wsum_ld;
  wk.xbox = tc_xbox(ctx, BN);
  const unsigned grid = unsigned(std::max<int64_t>(1, std::min<int64_t>(units, slots)));
  LaunchCfg lc(ctx, dim3(PAIR ? 2 * grid : grid), dim3(TC_THREADS), Cfg::SMEM_BYTES, st, PAIR ? 2u : 0u);
  CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, fn, w->tm128, tm_xhi, tm_xlo, M, N, wk, ep, slice_stride,
                              ctx->d_err, ctx->timeout_ns, ctx->inject_fault));
  ctx->launches++;
  return MYL_OK;
}

template <int BN, bool PAIR>
static int launch_tc_variant(myl_ctx* ctx, const myl_weight* w, const CUtensorMap& tm_xhi,
                             const CUtensorMap& tm_xlo, int64_t M, const TcWork& work,
                             const Epilogue& ep, int64_t slice_stride, cudaStream_t st) {
  switch (ep.mode) {
    case EPI_ACC_I64:
      return launch_tc_mode<BN, EPI_ACC_I64, PAIR>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
    case EPI_SHIFT:
      return launch_tc_mode<BN, EPI_SHIFT, PAIR>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
    case EPI_MULT:
      return launch_tc_mode<BN, EPI_MULT, PAIR>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
    case EPI_SILU:
      return launch_tc_mode<BN, EPI_SILU, PAIR>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
    case EPI_W16:
      return launch_tc_mode<BN, EPI_W16, PAIR>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
    default:
      return fail(MYL_ERR_ARG, "unknown epilogue mode %d", ep.mode);
  }
}

// The CTA-pair kernel runs 128-token tiles (the M = 256 MMA then reads one
// 16 KB activation plane per SM and stage instead of two).
static bool tc_pair(const myl_ctx* ctx, int BN) { return ctx->pair_mode != 0 && BN == 128; }

// Work slots of one wave: SMs, or co-resident CTA pairs.
static int tc_slots(myl_ctx* ctx, bool pair) {
  if (!pair) return sms(ctx);
  constexpr int S = TC_PAIR_STAGES;
  return pair_slots(ctx, gemm_w8a16_tc_kernel<128, S, EPI_SHIFT, true>,
                    size_t(TcCfg<128, S, true>::SMEM_BYTES));
}

static int tc_token_tile(const myl_ctx* ctx, int64_t M) {
  if (ctx->force_tile == 32 || ctx->force_tile == 64 || ctx->force_tile == 128) return ctx->force_tile;
  return M <= 32 ? 32 : (M <= 64 ? 64 : 128);
}

// pair: launch the CTA-pair kernel (BN = 128 only; work laid out in 256-channel units).
static int launch_tc_any(myl_ctx* ctx, const myl_weight* w, const CUtensorMap& tm_xhi,
                         const CUtensorMap& tm_xlo, int64_t M, int BN, bool pair,
                         const TcWork& work, const Epilogue& ep, int64_t slice_stride,
                         cudaStream_t st) {
  if (pair) {
    if (BN != 128) return fail(MYL_ERR_ARG, "CTA-pair GEMM needs 128-token tiles");
    return launch_tc_variant<128, true>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
  }
  if (BN == 32) return launch_tc_variant<32, false>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
  if (BN == 64) return launch_tc_variant<64, false>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
  return launch_tc_variant<128, false>(ctx, w, tm_xhi, tm_xlo, M, work, ep, slice_stride, st);
}

static int launch_split(myl_ctx* ctx, const int16_t* x, int64_t M, int64_t K, int64_t ldx,
                        uint8_t* xhi, uint8_t* xlo, int64_t ldp, cudaStream_t st) {
  const int64_t groups = M * (ldp / 8);
  unsigned blocks = unsigned(std::min<int64_t>((groups + 255) / 256, int64_t(ctx->num_sms) * 16));
  LaunchCfg lc(ctx, dim3(blocks), dim3(256), 0, st);
  CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, split_hilo_kernel, x, ldx, M, K, xhi, xlo, ldp));
  ctx->launches++;
  return MYL_OK;
}

// tcgen05 GEMM from hi/lo planes ([M][ldp] each, ldp a multiple of 16).
static int launch_tc_planes(myl_ctx* ctx, const myl_weight* w, const uint8_t* xhi, const uint8_t* xlo,
                            int64_t ldp, int64_t M, const Epilogue& ep_final, cudaStream_t st) {
  const int64_t K = w->K;
  const int BN = tc_token_tile(ctx, M);
  CUtensorMap tm_xhi, tm_xlo;
  TRY(encode_map(ctx, &tm_xhi, xhi, K, M, ldp, tc_xbox(ctx, BN)));
  TRY(encode_map(ctx, &tm_xlo, xlo, K, M, ldp, tc_xbox(ctx, BN)));
  // K split: enough work units for the SMs, and int32-exact slices (<= 65536).
  const bool pair = tc_pair(ctx, BN);
  const int ct = pair ? 256 : 128;  // channels per work unit
  const int64_t G = tc_slots(ctx, pair);
  const int k_tiles = int((K + TC_BK - 1) / TC_BK);
  const int64_t tiles = ((w->N + ct - 1) / ct) * ((M + BN - 1) / BN);
  int ksplit = 1;
  if (ctx->force_split_k > 0) {
    ksplit = ctx->force_split_k;
  } else if (tiles < G && k_tiles >= 8) {
    ksplit = int(std::min<int64_t>(G / tiles, k_tiles / 4));
  }
  ksplit = std::max(ksplit, int((K + 65535) / 65536));
  ksplit = std::max(1, std::min(ksplit, k_tiles));
  const int per = (k_tiles + ksplit - 1) / ksplit;
  ksplit = (k_tiles + per - 1) / per;  // no empty slice
  TcWork work{int((w->N + ct - 1) / ct), int((M + BN - 1) / BN), ksplit, k_tiles, per};
  // Tail split: when the tiles fill some waves and leave a small last wave,
  // that wave's tiles run as K slices on all SMs (int64 partials, then
  // tail_reduce_kernel), so the last wave costs a fraction of a full one.
  const int64_t R = tiles % G;
  if (ksplit == 1 && ctx->force_split_k == 0 && tiles >= G && R > 0) {
    const int ks = int(std::min<int64_t>({G / R, int64_t(k_tiles / 4), 16}));
    if (ks >= 2) {
      const int tper = (k_tiles + ks - 1) / ks;
      work.full_units = int(tiles - R);
      work.tail_tiles = int(R);
      work.tail_ks = (k_tiles + tper - 1) / tper;
      work.tail_per = tper;
      TRY(ensure(ctx->part, size_t(R) * size_t(work.tail_ks) * size_t(BN) * size_t(ct) * 8));
      work.tail_ws = static_cast<int64_t*>(ctx->part.p);
    }
  }
  if (work.tail_tiles > 0) {
    TRY(launch_tc_any(ctx, w, tm_xhi, tm_xlo, M, BN, pair, work, ep_final, 0, st));
    const int64_t total = int64_t(work.tail_tiles) * BN * (ct / 2);
    const unsigned blocks = unsigned(std::min<int64_t>((total + 255) / 256, int64_t(sms(ctx)) * 8));
    LaunchCfg lc(ctx, dim3(blocks), dim3(256), 0, st);
    CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, tail_reduce_kernel, work.tail_ws, work.tail_tiles,
                                work.tail_ks, work.full_units, work.tiles_n, BN, ct, M, w->N,
                                ep_final));
    ctx->launches++;
    return MYL_OK;
  }
  Epilogue ep = ep_final;
  int64_t slice_stride = 0;
  if (ksplit > 1) {
    TRY(ensure(ctx->part, size_t(ksplit) * size_t(M) * size_t(w->N) * 8));
    ep.mode = EPI_ACC_I64;
    ep.y = ctx->part.p;
    ep.ldy = w->N;
    ep.xs_world = 0;  // slice partials stay local; the final pass exchanges
    ep.xg_world = 0;
    ep.xb_world = 0;
    slice_stride = M * w->N;
  }
  TRY(launch_tc_any(ctx, w, tm_xhi, tm_xlo, M, BN, pair, work, ep, slice_stride, st));
  if (ksplit > 1) {
    const int64_t total = M * w->N;
    unsigned blocks = unsigned(std::min<int64_t>((total + 255) / 256, int64_t(ctx->num_sms) * 8));
    LaunchCfg lc(ctx, dim3(blocks), dim3(256), 0, st);
    CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, reduce_requant_kernel,
                                static_cast<const int64_t*>(ctx->part.p), ksplit, slice_stride, M,
                                w->N, ep_final));
    ctx->launches++;
  }
  return MYL_OK;
}

static int launch_tc(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M, int64_t ldx,
                     const Epilogue& ep_final, cudaStream_t st) {
  const int64_t ldp = w->ldp;
  TRY(ensure(ctx->planes, size_t(2) * size_t(M) * size_t(ldp)));
  uint8_t* xhi = static_cast<uint8_t*>(ctx->planes.p);
  uint8_t* xlo = xhi + M * ldp;
  TRY(launch_split(ctx, x, M, w->K, ldx, xhi, xlo, ldp, st));
  return launch_tc_planes(ctx, w, xhi, xlo, ldp, M, ep_final, st);
}

static int dispatch_linear(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                           int64_t ldx, const Epilogue& ep_in, cudaStream_t st) {
  Epilogue ep = ep_in;
  if (w->w16) {
    // int16 weights: the LM head's path A, i32 logits (model.rs:285-296).
    if (ep.mode != EPI_SHIFT || !ep.out_i32 || ep.bias)
      return fail(MYL_ERR_ARG, "int16 weights take the LM-head requant (MYL_RQ_SHIFT_I32) only");
    TRY(ensure(ctx->xsum, size_t(M) * 8));
    const unsigned blocks = unsigned(std::min<int64_t>((M + 7) / 8, int64_t(ctx->num_sms) * 8));
    LaunchCfg lc(ctx, dim3(blocks), dim3(256), 0, st);
    CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, x_row_sums_kernel, x, ldx, M, w->K,
                                static_cast<int64_t*>(ctx->xsum.p)));
    ctx->launches++;
    ep.mode = EPI_W16;
    ep.xsum = static_cast<const int64_t*>(ctx->xsum.p);
  }
  if (M <= ctx->gemv_max_m && M <= 4) return launch_gemv(ctx, w, x, M, ldx, ep, st);
  return launch_tc(ctx, w, x, M, ldx, ep, st);
}

static int run_linear(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M, int64_t ldx,
                      const Epilogue& ep, cudaStream_t st) {
  if (M == 0 || w->N == 0) return MYL_OK;
  CUDA_TRY(cudaSetDevice(ctx->device));
  TRY(ws_acquire(ctx, st));
  TRY(dispatch_linear(ctx, w, x, M, ldx, ep, st));
  return ws_release(ctx, st);
}

static int check_device_error(myl_ctx* ctx) {
  CUDA_TRY(cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  int e = *ctx->h_err;
  if (e != 0) {
    CUDA_TRY(cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream));
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    return fail(MYL_ERR_DEVICE, "kernel reported error 0x%x (%s)", e,
                e == DEV_BAD_EXPERT  ? "an expert id outside this object's experts"
                : e == DEV_BAD_TOKEN ? "a token id outside the vocabulary"
                                     : "a bounded wait ran out");
  }
  return MYL_OK;
}

static bool is_pinned(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// Host-pointer linear: upload x and the requant table, run, download y.
static int host_linear(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M, int mode,
                       int out_i32, const int8_t* shift, const int32_t* mult, void* y,
                       const int32_t* bias = nullptr) {
  if (!ctx || !w || (M > 0 && (!x || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (M < 0) return fail(MYL_ERR_SHAPE, "M = %lld is negative", (long long)M);
  if (M == 0 || w->N == 0) return MYL_OK;
  const int64_t N = out_features(w), K = w->K;
  const size_t osz = out_i32 ? 4 : 2;
  TRY(ensure(ctx->x, size_t(M) * size_t(K) * 2));
  TRY(ensure(ctx->y, size_t(M) * size_t(N) * osz));
  TRY(ensure(ctx->rq, size_t(N) * 9 + 64));
  int32_t* d_mult = reinterpret_cast<int32_t*>(ctx->rq.p);
  int32_t* d_bias = d_mult + N;
  int8_t* d_shift = reinterpret_cast<int8_t*>(d_bias + N);
  cudaStream_t st = ctx->stream;
  CUDA_TRY(cudaMemcpyAsync(d_shift, shift, size_t(N), cudaMemcpyHostToDevice, st));
  if (mult) CUDA_TRY(cudaMemcpyAsync(d_mult, mult, size_t(N) * 4, cudaMemcpyHostToDevice, st));
  if (bias) CUDA_TRY(cudaMemcpyAsync(d_bias, bias, size_t(N) * 4, cudaMemcpyHostToDevice, st));
  Epilogue ep{};
  ep.bias = bias ? d_bias : nullptr;
  ep.mode = mode;
  ep.out_i32 = out_i32;
  ep.shift = d_shift;
  ep.mult = mult ? d_mult : nullptr;
  ep.y = ctx->y.p;
  ep.ldy = N;
  // Page-locked x and y: the rows run in chunks on three streams, so the
  // upload of chunk i+1 and the download of chunk i-1 overlap the kernels of
  // chunk i (PCIe moves data both ways at once). Otherwise one pass.
  int64_t nch = (is_pinned(x) && is_pinned(y)) ? std::min<int64_t>(MYL_PIPE, M / 128) : 1;
  if (const char* env = std::getenv("MYL_HOST_CHUNKS"))  // tuning: chunk count, 1 = one pass
    nch = std::max<int64_t>(1, std::min<int64_t>({int64_t(std::atoi(env)), int64_t(MYL_PIPE), M}));
  if (nch < 2) {
    CUDA_TRY(cudaMemcpyAsync(ctx->x.p, x, size_t(M) * size_t(K) * 2, cudaMemcpyHostToDevice, st));
    TRY(run_linear(ctx, w, static_cast<const int16_t*>(ctx->x.p), M, K, ep, st));
    CUDA_TRY(cudaMemcpyAsync(y, ctx->y.p, size_t(M) * size_t(N) * osz, cudaMemcpyDeviceToHost, st));
    return check_device_error(ctx);
  }
  const int64_t rows = (M + nch - 1) / nch;
  CUDA_TRY(cudaSetDevice(ctx->device));
  TRY(ws_acquire(ctx, st));
  for (int64_t c = 0; c < nch; ++c) {
    const int64_t r0 = c * rows, rc = std::min(rows, M - r0);
    if (rc <= 0) break;
    const int16_t* dx = static_cast<const int16_t*>(ctx->x.p) + r0 * K;
    uint8_t* dy = static_cast<uint8_t*>(ctx->y.p) + size_t(r0) * size_t(N) * osz;
    CUDA_TRY(cudaMemcpyAsync(const_cast<int16_t*>(dx), x + r0 * K, size_t(rc) * size_t(K) * 2,
                             cudaMemcpyHostToDevice, ctx->s_in));
    CUDA_TRY(cudaEventRecord(ctx->ev_in[c], ctx->s_in));
    CUDA_TRY(cudaStreamWaitEvent(st, ctx->ev_in[c], 0));
    Epilogue epc = ep;
    epc.y = dy;
    TRY(dispatch_linear(ctx, w, dx, rc, K, epc, st));
    CUDA_TRY(cudaEventRecord(ctx->ev_comp[c], st));
    CUDA_TRY(cudaStreamWaitEvent(ctx->s_out, ctx->ev_comp[c], 0));
    CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(y) + size_t(r0) * size_t(N) * osz, dy,
                             size_t(rc) * size_t(N) * osz, cudaMemcpyDeviceToHost, ctx->s_out));
  }
  CUDA_TRY(cudaStreamSynchronize(ctx->s_out));
  TRY(ws_release(ctx, st));
  return check_device_error(ctx);
}

// ---------------------------------------------------------------------------------
// C ABI

extern "C" {

const char* myl_last_error(void) { return g_last_error.c_str(); }
int myl_abi_version(void) { return MYL_ABI_VERSION; }

int myl_init(int device, myl_ctx** out) {
  if (!out) return fail(MYL_ERR_ARG, "out is null");
  *out = nullptr;
  int n = 0;
  CUDA_TRY(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return fail(MYL_ERR_ARG, "device %d not present (%d devices)", device, n);
  CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(MYL_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only",
                device, prop.major, prop.minor);
  myl_ctx* c = new myl_ctx();
  c->device = device;
  c->sm = prop.major * 10 + prop.minor;
  c->num_sms = prop.multiProcessorCount;
  if (const char* env = std::getenv("MYL_TC_XBOX")) {  // tuning: 16, 32, 64 or 128 rows per box
    const int v = std::atoi(env);
    if (v == 16 || v == 32 || v == 64 || v == 128) c->xbox = v;
  }
  if (const char* env = std::getenv("MYL_TC_PAIR"))  // tuning: 0 = one CTA per tile only
    c->pair_mode = std::atoi(env) != 0 ? 1 : 0;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                   cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
    delete c;
    return fail(MYL_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
  }
  c->encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  bool ok = cudaStreamCreateWithFlags(&c->s_in, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&c->s_out, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; ok && i < MYL_PIPE; ++i)
    ok = cudaEventCreateWithFlags(&c->ev_in[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&c->ev_comp[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok || cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ws_event, cudaEventDisableTiming) != cudaSuccess ||
      cudaMalloc(&c->d_err, sizeof(int)) != cudaSuccess ||
      cudaMallocHost(&c->h_err, sizeof(int)) != cudaSuccess ||
      cudaMemset(c->d_err, 0, sizeof(int)) != cudaSuccess) {
    myl_destroy(c);
    return fail(MYL_ERR_CUDA, "context allocation failed");
  }
  *out = c;
  return MYL_OK;
}

int myl_destroy(myl_ctx* ctx) {
  if (!ctx) return MYL_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  for (auto& kv : ctx->backend_cache) myl_weight_release(ctx, kv.second);
  ctx->backend_cache.clear();
  for (DevBuf* b : {&ctx->x, &ctx->y, &ctx->rq, &ctx->planes, &ctx->part, &ctx->h, &ctx->hplanes,
                    &ctx->moe, &ctx->xsum, &ctx->crc})
    if (b->p) cudaFree(b->p);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->h_err) cudaFreeHost(ctx->h_err);
  if (ctx->ws_event) cudaEventDestroy(ctx->ws_event);
  for (int i = 0; i < MYL_PIPE; ++i) {
    if (ctx->ev_in[i]) cudaEventDestroy(ctx->ev_in[i]);
    if (ctx->ev_comp[i]) cudaEventDestroy(ctx->ev_comp[i]);
  }
  if (ctx->s_in) cudaStreamDestroy(ctx->s_in);
  if (ctx->s_out) cudaStreamDestroy(ctx->s_out);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return MYL_OK;
}

int myl_device_info(const myl_ctx* ctx, int* device, int* sm_version, int* num_sms) {
  if (!ctx) return fail(MYL_ERR_ARG, "ctx is null");
  if (device) *device = ctx->device;
  if (sm_version) *sm_version = ctx->sm;
  if (num_sms) *num_sms = ctx->num_sms;
  return MYL_OK;
}

int myl_weight_register(myl_ctx* ctx, const int8_t* W, int64_t out_features, int64_t in_features,
                        int64_t ldw, const uint8_t* w_shifts, myl_weight** out) {
  if (!ctx || !out || (out_features > 0 && (!W || !w_shifts))) return fail(MYL_ERR_ARG, "null argument");
  *out = nullptr;
  // linear.rs:61 W.chunks_exact(in_features) panics for 0; the row count must fit the TMA map.
  if (in_features <= 0 || out_features < 0 || ldw < in_features)
    return fail(MYL_ERR_SHAPE, "bad weight shape [%lld][%lld] ld %lld", (long long)out_features,
                (long long)in_features, (long long)ldw);
  if (out_features > (int64_t(1) << 31) || in_features > (int64_t(1) << 31))
    return fail(MYL_ERR_UNSUPPORTED, "weight dimension beyond 2^31");
  CUDA_TRY(cudaSetDevice(ctx->device));
  myl_weight* w = new myl_weight();
  w->N = out_features;
  w->K = in_features;
  w->ldp = (in_features + 15) & ~int64_t(15);
  w->w_shifts.assign(w_shifts, w_shifts + out_features);
  const size_t bytes = size_t(std::max<int64_t>(out_features, 1)) * size_t(w->ldp);
  if (cudaMalloc(&w->d_W, bytes) != cudaSuccess) {
    delete w;
    return fail(MYL_ERR_CUDA, "cudaMalloc of %zu weight bytes failed", bytes);
  }
  int rc = MYL_OK;
  if (cudaMemsetAsync(w->d_W, 0, bytes, ctx->stream) != cudaSuccess ||
      (out_features > 0 &&
       cudaMemcpy2DAsync(w->d_W, size_t(w->ldp), W, size_t(ldw), size_t(in_features),
                         size_t(out_features), cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess) ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess)
    rc = fail(MYL_ERR_CUDA, "weight upload failed: %s", cudaGetErrorString(cudaGetLastError()));
  if (rc == MYL_OK && out_features > 0) {
    rc = encode_map(ctx, &w->tm128, w->d_W, w->K, w->N, w->ldp, 128);
  }
  // Row sums per K tile for the tensor-core kernel's offset-binary correction.
  const int k_tiles = int((in_features + TC_BK - 1) / TC_BK);
  w->wsum_ld = k_tiles + 1;
  if (rc == MYL_OK) {
    const size_t wb = size_t(std::max<int64_t>(out_features, 1)) * size_t(w->wsum_ld) * 4;
    if (cudaMalloc(&w->d_wsum, wb) != cudaSuccess) {
      rc = fail(MYL_ERR_CUDA, "cudaMalloc of %zu row-sum bytes failed", wb);
    } else if (out_features > 0) {
      const unsigned blocks = unsigned(std::min<int64_t>(out_features, int64_t(ctx->num_sms) * 16));
      weight_tile_sums_kernel<<<blocks, 128, 0, ctx->stream>>>(w->d_W, w->ldp, out_features,
                                                                 in_features, k_tiles, w->d_wsum,
                                                                 w->wsum_ld);
      if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(ctx->stream) != cudaSuccess)
        rc = fail(MYL_ERR_CUDA, "row-sum kernel failed: %s", cudaGetErrorString(cudaGetLastError()));
    }
  }
  if (rc != MYL_OK) {
    if (w->d_wsum) cudaFree(w->d_wsum);
    cudaFree(w->d_W);
    delete w;
    return rc;
  }
  *out = w;
  return MYL_OK;
}

int myl_weight_release(myl_ctx* ctx, myl_weight* w) {
  if (!ctx || !w) return MYL_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (w->d_W) cudaFree(w->d_W);
  if (w->d_wsum) cudaFree(w->d_wsum);
  if (w->d_bwd_perm) cudaFree(w->d_bwd_perm);
  if (w->d_bwd_groups) cudaFree(w->d_bwd_groups);
  delete w;
  return MYL_OK;
}

int myl_linear_w8a16(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                     uint8_t act_frac_bits, uint8_t out_frac_bits, int16_t* y) {
  if (!ctx || !w) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: use myl_lm_head_w16a16_i32 or myl_linear_dev");
  std::vector<int8_t> s;
  TRY(shift_plan(w, act_frac_bits, &out_frac_bits, 0, s));
  return host_linear(ctx, w, x, M, EPI_SHIFT, 0, s.data(), nullptr, y);
}

int myl_linear_w8a16_pc(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                        uint8_t act_frac_bits, const uint8_t* out_frac_bits, int16_t* y) {
  if (!ctx || !w || (w->N > 0 && !out_frac_bits)) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: use myl_lm_head_w16a16_i32 or myl_linear_dev");
  std::vector<int8_t> s;
  TRY(shift_plan(w, act_frac_bits, out_frac_bits, 1, s));
  return host_linear(ctx, w, x, M, EPI_SHIFT, 0, s.data(), nullptr, y);
}

int myl_lm_head_w8a16_i32(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                          uint8_t final_norm_frac, uint8_t logit_frac, int32_t* logits) {
  if (!ctx || !w) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: use myl_lm_head_w16a16_i32 or myl_linear_dev");
  std::vector<int8_t> s;
  TRY(shift_plan(w, final_norm_frac, &logit_frac, 0, s));
  return host_linear(ctx, w, x, M, EPI_SHIFT, 1, s.data(), nullptr, logits);
}

int myl_weight16_register(myl_ctx* ctx, const int16_t* W, int64_t out_features_, int64_t in_features,
                          int64_t ldw, const uint8_t* w_shifts, myl_weight** out) {
  if (!ctx || !out || (out_features_ > 0 && (!W || !w_shifts))) return fail(MYL_ERR_ARG, "null argument");
  *out = nullptr;
  if (in_features <= 0 || out_features_ < 0 || ldw < in_features)
    return fail(MYL_ERR_SHAPE, "bad weight shape [%lld][%lld] ld %lld", (long long)out_features_,
                (long long)in_features, (long long)ldw);
  if (out_features_ > (int64_t(1) << 30))
    return fail(MYL_ERR_UNSUPPORTED, "int16 weight with more than 2^30 rows");
  // Row i of the int16 weight becomes int8 rows 2i (w >> 8) and 2i + 1
  // ((w & 255) - 128), so w = 256 * row_2i + row_2i+1 + 128.
  const int64_t N = out_features_, K = in_features;
  std::vector<int8_t> w8(size_t(2 * N) * size_t(K));
  for (int64_t i = 0; i < N; ++i) {
    const int16_t* src = W + i * ldw;
    int8_t* hi = &w8[size_t(2 * i) * size_t(K)];
    int8_t* lo = hi + K;
    for (int64_t k = 0; k < K; ++k) {
      hi[k] = int8_t(src[k] >> 8);
      lo[k] = int8_t(int(src[k] & 0xFF) - 128);
    }
  }
  std::vector<uint8_t> zero(size_t(std::max<int64_t>(2 * N, 1)), 0);
  myl_weight* w = nullptr;
  TRY(myl_weight_register(ctx, w8.data(), 2 * N, K, K, zero.data(), &w));
  w->w16 = true;
  w->n16 = N;
  w->w_shifts.assign(w_shifts, w_shifts + N);
  *out = w;
  return MYL_OK;
}

int myl_lm_head_w16a16_i32(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                           uint8_t final_norm_frac, uint8_t logit_frac, int32_t* logits) {
  if (!ctx || !w) return fail(MYL_ERR_ARG, "null argument");
  if (!w->w16) return fail(MYL_ERR_ARG, "weight is not int16 (myl_weight16_register)");
  std::vector<int8_t> s;
  TRY(shift_plan(w, final_norm_frac, &logit_frac, 0, s));
  return host_linear(ctx, w, x, M, EPI_SHIFT, 1, s.data(), nullptr, logits);
}

int myl_argmax_keys_dev(myl_ctx* ctx, const int32_t* logits, int64_t M, int64_t V, int64_t ld,
                        int64_t index_base, int64_t* keys, void* stream) {
  if (!ctx || (M > 0 && (!keys || (V > 0 && !logits)))) return fail(MYL_ERR_ARG, "null argument");
  if (M < 0 || V < 0 || (M > 0 && V > 0 && ld < V) || index_base < 0 ||
      index_base + V > (int64_t(1) << 32))
    return fail(MYL_ERR_SHAPE, "bad M/V/ld/index_base");
  if (M == 0) return MYL_OK;
  CUDA_TRY(cudaSetDevice(ctx->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  select_init_kernel<<<unsigned(std::min<int64_t>((M + 255) / 256, 1024)), 256, 0, st>>>(keys, M);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  if (V == 0) return MYL_OK;
  const dim3 grid(unsigned((V + SELECT_CHUNK - 1) / SELECT_CHUNK),
                  unsigned(std::min<int64_t>(M, 65535)));
  select_keys_kernel<<<grid, SELECT_THREADS, 0, st>>>(logits, M, V, ld, index_base, keys);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

int myl_linear_w8a16_mult(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                          const int32_t* mult, const uint8_t* shift, int16_t* y) {
  if (!ctx || !w || (w->N > 0 && (!mult || !shift))) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: use myl_lm_head_w16a16_i32 or myl_linear_dev");
  for (int64_t r = 0; r < w->N; ++r)
    if (shift[r] > 126) return fail(MYL_ERR_OVERFLOW, "multiplier shift %u > 126", unsigned(shift[r]));
  return host_linear(ctx, w, x, M, EPI_MULT, 0, reinterpret_cast<const int8_t*>(shift), mult, y);
}

// 64-bit digest of the weight bytes for the Backend cache: four interleaved
// multiply-xorshift lanes over 8-byte words (one pass at memory speed), then
// the tail bytes and the length. Not cryptographic: it tells a changed weight
// matrix from the cached one.
static uint64_t weight_digest(const int8_t* W, uint64_t bytes) {
  const uint64_t k = 0x9E3779B97F4A7C15ull;
  uint64_t h[4] = {1, 2, 3, 4};
  const uint8_t* p = reinterpret_cast<const uint8_t*>(W);
  uint64_t i = 0;
  for (; i + 32 <= bytes; i += 32) {
    for (int l = 0; l < 4; ++l) {
      uint64_t v;
      std::memcpy(&v, p + i + 8 * l, 8);
      h[l] = (h[l] ^ v) * k;
      h[l] ^= h[l] >> 29;
    }
  }
  uint64_t t = bytes;
  for (; i < bytes; ++i) t = (t ^ p[i]) * k;
  uint64_t d = t;
  for (int l = 0; l < 4; ++l) d = (d ^ h[l]) * k + uint64_t(l);
  return d ^ (d >> 31);
}

int myl_backend_linear_w8a16(myl_ctx* ctx, const int16_t* x, const int8_t* W, int16_t* out,
                             uint64_t in_features, uint64_t out_features, const uint8_t* w_shifts,
                             uint8_t act_frac, uint8_t out_frac) {
  if (!ctx || !W || !x || !out || !w_shifts) return fail(MYL_ERR_ARG, "null argument");
  myl_weight* w = nullptr;
  const uint64_t digest = weight_digest(W, in_features * out_features);
  auto it = ctx->backend_cache.find(W);
  if (it != ctx->backend_cache.end()) {
    myl_weight* c = it->second;
    if (uint64_t(c->K) == in_features && uint64_t(c->N) == out_features &&
        c->host_shifts == w_shifts && c->host_digest == digest &&
        std::memcmp(c->w_shifts.data(), w_shifts, size_t(out_features)) == 0) {
      w = c;
    } else {
      myl_weight_release(ctx, c);
      ctx->backend_cache.erase(it);
    }
  }
  if (!w) {
    TRY(myl_weight_register(ctx, W, int64_t(out_features), int64_t(in_features),
                            int64_t(in_features), w_shifts, &w));
    w->host_W = W;
    w->host_shifts = w_shifts;
    w->host_digest = digest;
    ctx->backend_cache[W] = w;
  }
  return myl_linear_w8a16(ctx, w, x, 1, act_frac, out_frac, out);
}

int myl_backend_forget(myl_ctx* ctx, const int8_t* W) {
  if (!ctx) return fail(MYL_ERR_ARG, "ctx is null");
  auto it = ctx->backend_cache.find(W);
  if (it != ctx->backend_cache.end()) {
    myl_weight_release(ctx, it->second);
    ctx->backend_cache.erase(it);
  }
  return MYL_OK;
}

int myl_requant_create(myl_ctx* ctx, const myl_weight* w, int mode, uint8_t act_frac,
                       const uint8_t* out_frac_pc, int per_channel, const int32_t* mult,
                       const uint8_t* shift, myl_requant** out) {
  if (!ctx || !w || !out) return fail(MYL_ERR_ARG, "null argument");
  *out = nullptr;
  const int64_t N = out_features(w);
  if (w->w16 && mode != MYL_RQ_SHIFT_I32)
    return fail(MYL_ERR_ARG, "int16 weights take the LM-head requant (MYL_RQ_SHIFT_I32) only");
  std::vector<int8_t> s;
  std::vector<int32_t> m;
  if (mode == MYL_RQ_SHIFT_I16 || mode == MYL_RQ_SHIFT_I32) {
    if (N > 0 && !out_frac_pc) return fail(MYL_ERR_ARG, "out_frac is null");
    if (N > 0) TRY(shift_plan(w, act_frac, out_frac_pc, per_channel, s));
  } else if (mode == MYL_RQ_MULT_I16) {
    if (N > 0 && (!mult || !shift)) return fail(MYL_ERR_ARG, "mult/shift is null");
    s.resize(size_t(N));
    m.assign(mult, mult + N);
    for (int64_t r = 0; r < N; ++r) {
      if (shift[r] > 126) return fail(MYL_ERR_OVERFLOW, "multiplier shift %u > 126", unsigned(shift[r]));
      s[size_t(r)] = int8_t(shift[r]);
    }
  } else {
    return fail(MYL_ERR_ARG, "unknown requant mode %d", mode);
  }
  CUDA_TRY(cudaSetDevice(ctx->device));
  myl_requant* rq = new myl_requant();
  rq->N = N;
  rq->mode = mode;
  const size_t nb = size_t(std::max<int64_t>(N, 1));
  if (cudaMalloc(&rq->d_shift, nb) != cudaSuccess ||
      (!m.empty() && cudaMalloc(&rq->d_mult, nb * 4) != cudaSuccess)) {
    myl_requant_release(ctx, rq);
    return fail(MYL_ERR_CUDA, "requant allocation failed");
  }
  if ((N > 0 && cudaMemcpy(rq->d_shift, s.data(), size_t(N), cudaMemcpyHostToDevice) != cudaSuccess) ||
      (!m.empty() && cudaMemcpy(rq->d_mult, m.data(), size_t(N) * 4, cudaMemcpyHostToDevice) != cudaSuccess)) {
    myl_requant_release(ctx, rq);
    return fail(MYL_ERR_CUDA, "requant upload failed");
  }
  *out = rq;
  return MYL_OK;
}

int myl_requant_release(myl_ctx* ctx, myl_requant* rq) {
  if (!rq) return MYL_OK;
  if (ctx) cudaSetDevice(ctx->device);
  if (rq->d_shift) cudaFree(rq->d_shift);
  if (rq->d_mult) cudaFree(rq->d_mult);
  if (rq->d_bias) cudaFree(rq->d_bias);
  delete rq;
  return MYL_OK;
}

static Epilogue make_ep(const myl_requant* rq, void* y, int64_t ldy) {
  Epilogue ep{};
  ep.mode = (rq->mode == MYL_RQ_MULT_I16) ? EPI_MULT : EPI_SHIFT;
  ep.out_i32 = (rq->mode == MYL_RQ_SHIFT_I32) ? 1 : 0;
  ep.shift = rq->d_shift;
  ep.mult = rq->d_mult;
  ep.bias = rq->d_bias;
  ep.y = y;
  ep.ldy = ldy;
  return ep;
}

int myl_linear_dev(myl_ctx* ctx, const myl_weight* w, const myl_requant* rq, const int16_t* x,
                   int64_t M, int64_t ldx, void* y, int64_t ldy, void* stream) {
  if (!ctx || !w || !rq || (M > 0 && (!x || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (rq->N != out_features(w))
    return fail(MYL_ERR_SHAPE, "requant has %lld channels, weight %lld", (long long)rq->N,
                (long long)out_features(w));
  if (M < 0 || ldx < w->K || ldy < out_features(w)) return fail(MYL_ERR_SHAPE, "bad M/ldx/ldy");
  return run_linear(ctx, w, x, M, ldx, make_ep(rq, y, ldy), static_cast<cudaStream_t>(stream));
}

int myl_linear_acc_dev(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M, int64_t ldx,
                       int64_t* acc, void* stream) {
  if (!ctx || !w || (M > 0 && (!x || !acc))) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: use myl_lm_head_w16a16_i32 or myl_linear_dev");
  if (M < 0 || ldx < w->K) return fail(MYL_ERR_SHAPE, "bad M/ldx");
  Epilogue ep{};
  ep.mode = EPI_ACC_I64;
  ep.y = acc;
  ep.ldy = w->N;
  return run_linear(ctx, w, x, M, ldx, ep, static_cast<cudaStream_t>(stream));
}

int myl_linear_acc_exchange_dev(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                                int64_t ldx, int64_t* const* dst, int world, int rank,
                                int64_t rows_per_rank, void* stream) {
  if (!ctx || !w || !dst || (M > 0 && !x)) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: the exchange carries int8-weight partials");
  if (world < 1 || world > MYL_XCHG_MAX || rank < 0 || rank >= world)
    return fail(MYL_ERR_ARG, "world %d / rank %d (at most %d ranks)", world, rank, MYL_XCHG_MAX);
  if (M < 0 || ldx < w->K || rows_per_rank <= 0 || rows_per_rank % 16 != 0 ||
      M > int64_t(world) * rows_per_rank)
    return fail(MYL_ERR_SHAPE, "bad M/ldx/rows_per_rank (a multiple of 16 covering M over the ranks)");
  for (int o = 0; o < world; ++o)
    if (!dst[o]) return fail(MYL_ERR_ARG, "null receive buffer of rank %d", o);
  Epilogue ep{};
  ep.mode = EPI_ACC_I64;
  ep.y = dst[rank];
  ep.ldy = w->N;
  for (int o = 0; o < world; ++o) ep.xs_dst[o] = dst[o];
  ep.xs_rows = rows_per_rank;
  ep.xs_rank = rank;
  ep.xs_world = world;
  return run_linear(ctx, w, x, M, ldx, ep, static_cast<cudaStream_t>(stream));
}

int myl_exchange_reduce_dev(myl_ctx* ctx, const myl_requant* rq, const int64_t* recv, int world,
                            int rank, int64_t rows_per_rank, int64_t M, void* const* out, int64_t ldo,
                            void* stream) {
  if (!ctx || !rq || !recv || !out) return fail(MYL_ERR_ARG, "null argument");
  if (world < 1 || world > MYL_XCHG_MAX || rank < 0 || rank >= world)
    return fail(MYL_ERR_ARG, "world %d / rank %d (at most %d ranks)", world, rank, MYL_XCHG_MAX);
  if (M < 0 || rows_per_rank <= 0 || M > int64_t(world) * rows_per_rank || ldo < rq->N)
    return fail(MYL_ERR_SHAPE, "bad M/rows_per_rank/ldo");
  for (int o = 0; o < world; ++o)
    if (!out[o]) return fail(MYL_ERR_ARG, "null output buffer of rank %d", o);
  // this rank's rows: [rank * R, min((rank + 1) * R, M))
  const int64_t own = std::max<int64_t>(0, std::min(rows_per_rank, M - int64_t(rank) * rows_per_rank));
  if (own == 0 || rq->N == 0) return MYL_OK;
  CUDA_TRY(cudaSetDevice(ctx->device));
  Epilogue ep = make_ep(rq, out[rank], ldo);
  for (int o = 0; o < world; ++o) ep.xg_dst[o] = out[o];
  ep.xg_row0 = int64_t(rank) * rows_per_rank;
  ep.xg_world = world;
  bool vec = rq->N % 8 == 0 && ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(recv) & 15) == 0;
  for (int o = 0; o < world; ++o) vec = vec && (reinterpret_cast<uintptr_t>(out[o]) & 15) == 0;
  const int64_t total = vec ? own * (rq->N / 8) : own * rq->N;
  unsigned blocks = unsigned(std::min<int64_t>((total + 255) / 256, int64_t(ctx->num_sms) * 8));
  // recv holds world slabs of rows_per_rank rows: the sender index is the K-slice index
  if (vec)
    xchg_reduce_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        recv, world, rows_per_rank * rq->N, own, rq->N, ep);
  else
    reduce_requant_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        recv, world, rows_per_rank * rq->N, own, rq->N, ep);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

int myl_exchange_barrier_dev(myl_ctx* ctx, unsigned long long* const* flags, int world, int rank,
                             unsigned long long epoch, void* stream) {
  if (!ctx || !flags) return fail(MYL_ERR_ARG, "null argument");
  if (world < 1 || world > MYL_XCHG_MAX || rank < 0 || rank >= world)
    return fail(MYL_ERR_ARG, "world %d / rank %d (at most %d ranks)", world, rank, MYL_XCHG_MAX);
  for (int o = 0; o < world; ++o)
    if (!flags[o]) return fail(MYL_ERR_ARG, "null flag array of rank %d", o);
  CUDA_TRY(cudaSetDevice(ctx->device));
  XchgFlags fp{};  // the pointers travel by value in the kernel's arguments
  for (int o = 0; o < world; ++o) fp.p[o] = flags[o];
  xchg_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(fp, world, rank, epoch,
                                                                       ctx->d_err, ctx->timeout_ns);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

int myl_ep_dispatch_dev(myl_ctx* ctx, const int16_t* x, int64_t T, int64_t ldx, int64_t H,
                        const int32_t* idx, int k, int E, int world, int rank, int16_t* const* rows,
                        int32_t* const* ids, int32_t* const* src, int32_t* const* counters,
                        int64_t capacity, void* stream) {
  if (!ctx || !rows || !ids || !src || !counters || (T > 0 && (!x || !idx)))
    return fail(MYL_ERR_ARG, "null argument");
  if (world < 1 || world > MYL_XCHG_MAX || rank < 0 || rank >= world)
    return fail(MYL_ERR_ARG, "world %d / rank %d (at most %d ranks)", world, rank, MYL_XCHG_MAX);
  if (T < 0 || H <= 0 || ldx < H || k < 1 || E < world || capacity < 0 || T * k >= (int64_t(1) << 24))
    return fail(MYL_ERR_SHAPE, "bad T/H/ldx/k/E/capacity");
  EpPeers pe{};
  for (int o = 0; o < world; ++o) {
    if (!rows[o] || !ids[o] || !src[o] || !counters[o])
      return fail(MYL_ERR_ARG, "null buffer of rank %d", o);
    pe.rows[o] = rows[o];
    pe.ids[o] = ids[o];
    pe.src[o] = src[o];
    pe.count[o] = counters[o];
  }
  if (T == 0) return MYL_OK;
  CUDA_TRY(cudaSetDevice(ctx->device));
  const unsigned blocks = unsigned(std::min<int64_t>((T * k + 7) / 8, int64_t(ctx->num_sms) * 8));
  ep_dispatch_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, T, ldx, H, idx, k, E, world, rank, pe, capacity, ctx->d_err);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

int myl_ep_return_dev(myl_ctx* ctx, const int16_t* y, int64_t count, int64_t H, const int32_t* src,
                      int16_t* const* back, int world, void* stream) {
  if (!ctx || !back || (count > 0 && (!y || !src))) return fail(MYL_ERR_ARG, "null argument");
  if (world < 1 || world > MYL_XCHG_MAX) return fail(MYL_ERR_ARG, "world %d", world);
  if (count < 0 || H <= 0) return fail(MYL_ERR_SHAPE, "bad count/H");
  EpPeers pe{};
  for (int o = 0; o < world; ++o) {
    if (!back[o]) return fail(MYL_ERR_ARG, "null return buffer of rank %d", o);
    pe.back[o] = back[o];
  }
  if (count == 0) return MYL_OK;
  CUDA_TRY(cudaSetDevice(ctx->device));
  const unsigned blocks = unsigned(std::min<int64_t>((count + 7) / 8, int64_t(ctx->num_sms) * 8));
  ep_return_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, count, H, src, pe);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

int myl_ipc_alloc(myl_ctx* ctx, size_t bytes, void** ptr, void* handle) {
  if (!ctx || !ptr || !handle || bytes == 0) return fail(MYL_ERR_ARG, "bad argument");
  CUDA_TRY(cudaSetDevice(ctx->device));
  CUDA_TRY(cudaMalloc(ptr, bytes));
  CUDA_TRY(cudaMemset(*ptr, 0, bytes));  // flag words start at epoch 0
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return fail(MYL_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == MYL_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return MYL_OK;
}

int myl_ipc_open(myl_ctx* ctx, const void* handle, void** ptr) {
  if (!ctx || !ptr || !handle) return fail(MYL_ERR_ARG, "null argument");
  CUDA_TRY(cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MYL_OK;
}

int myl_ipc_close(myl_ctx* ctx, void* ptr) {
  if (!ctx || !ptr) return fail(MYL_ERR_ARG, "null argument");
  CUDA_TRY(cudaSetDevice(ctx->device));
  CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return MYL_OK;
}

int myl_ipc_free(myl_ctx* ctx, void* ptr) {
  if (!ctx || !ptr) return fail(MYL_ERR_ARG, "null argument");
  CUDA_TRY(cudaSetDevice(ctx->device));
  CUDA_TRY(cudaFree(ptr));
  return MYL_OK;
}

int myl_requant_acc_dev(myl_ctx* ctx, const myl_requant* rq, const int64_t* acc, int64_t M, void* y,
                        int64_t ldy, void* stream) {
  if (!ctx || !rq || (M > 0 && (!acc || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (M < 0 || ldy < rq->N) return fail(MYL_ERR_SHAPE, "bad M/ldy");
  if (M == 0 || rq->N == 0) return MYL_OK;
  const int64_t total = M * rq->N;
  unsigned blocks = unsigned(std::min<int64_t>((total + 255) / 256, int64_t(ctx->num_sms) * 8));
  reduce_requant_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      acc, 1, 0, M, rq->N, make_ep(rq, y, ldy));
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

// linear.rs:142: rescale(b as i32, b_shift, out_frac) with the debug-build
// overflow checks of fixed_point.rs:173-180 (i32 width).
static int rescale_bias(const int16_t* bias, const uint8_t* bias_shifts, int64_t N, uint8_t out_frac,
                        std::vector<int32_t>& out) {
  out.resize(size_t(N));
  for (int64_t i = 0; i < N; ++i) {
    const int d = int(int8_t(bias_shifts[i])) - int(int8_t(out_frac));
    if (d < -128 || d > 127 || d > 30 || d < -31)
      return fail(MYL_ERR_OVERFLOW, "bias shift %u -> out_frac %u overflows i32 rescale",
                  unsigned(bias_shifts[i]), unsigned(out_frac));
    const int32_t b = bias[i];
    int32_t v;
    if (d > 0) {
      const int32_t q = b >> d, r = b & ((1 << d) - 1), h = 1 << (d - 1);
      v = q + ((r > h || (r == h && (q & 1))) ? 1 : 0);
    } else if (d == 0) {
      v = b;
    } else {
      v = int32_t(uint32_t(b) << (-d));
    }
    out[size_t(i)] = v;
  }
  return MYL_OK;
}

int myl_linear_w8a16_bias(myl_ctx* ctx, const myl_weight* w, const int16_t* x, int64_t M,
                          uint8_t act_frac_bits, uint8_t out_frac_bits, const int16_t* bias,
                          const uint8_t* bias_shifts, int16_t* y) {
  if (!ctx || !w || (w->N > 0 && (!bias || !bias_shifts))) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: use myl_lm_head_w16a16_i32 or myl_linear_dev");
  std::vector<int8_t> s;
  TRY(shift_plan(w, act_frac_bits, &out_frac_bits, 0, s));
  std::vector<int32_t> b;
  TRY(rescale_bias(bias, bias_shifts, w->N, out_frac_bits, b));
  return host_linear(ctx, w, x, M, EPI_SHIFT, 0, s.data(), nullptr, y, b.data());
}

int myl_requant_set_bias(myl_ctx* ctx, myl_requant* rq, const int16_t* bias,
                         const uint8_t* bias_shifts, uint8_t out_frac) {
  if (!ctx || !rq || (rq->N > 0 && (!bias || !bias_shifts))) return fail(MYL_ERR_ARG, "null argument");
  if (rq->mode == MYL_RQ_SHIFT_I32) return fail(MYL_ERR_ARG, "bias applies to int16 outputs only");
  std::vector<int32_t> b;
  TRY(rescale_bias(bias, bias_shifts, rq->N, out_frac, b));
  CUDA_TRY(cudaSetDevice(ctx->device));
  if (!rq->d_bias) CUDA_TRY(cudaMalloc(&rq->d_bias, size_t(std::max<int64_t>(rq->N, 1)) * 4));
  if (rq->N > 0) CUDA_TRY(cudaMemcpy(rq->d_bias, b.data(), size_t(rq->N) * 4, cudaMemcpyHostToDevice));
  return MYL_OK;
}

// ---- mlp_int (kernels/src/mlp.rs:28-74) -----------------------------------------

int myl_mlp_release(myl_ctx* ctx, myl_mlp* mlp) {
  if (!mlp) return MYL_OK;
  if (ctx) {
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (mlp->w_gu) myl_weight_release(ctx, mlp->w_gu);
    if (mlp->w_down) myl_weight_release(ctx, mlp->w_down);
  }
  if (mlp->d_shift_gu) cudaFree(mlp->d_shift_gu);
  if (mlp->d_shift_down) cudaFree(mlp->d_shift_down);
  if (mlp->d_lut) cudaFree(mlp->d_lut);
  delete mlp;
  return MYL_OK;
}

int myl_mlp_register(myl_ctx* ctx, const int8_t* W_gate, const int8_t* W_up, const int8_t* W_down,
                     int64_t hidden, int64_t intermediate, const uint8_t* gate_w_shifts,
                     const uint8_t* up_w_shifts, const uint8_t* down_w_shifts,
                     const int16_t* silu_lut, int64_t silu_lut_len, uint8_t in_frac,
                     uint8_t gate_out_frac, uint8_t up_out_frac, uint8_t down_in_frac,
                     uint8_t silu_in_frac, int16_t silu_lut_offset, uint8_t silu_out_frac,
                     const uint8_t* out_frac, myl_mlp** out) {
  if (!ctx || !out || !W_gate || !W_up || !W_down || !gate_w_shifts || !up_w_shifts ||
      !down_w_shifts || !silu_lut || !out_frac)
    return fail(MYL_ERR_ARG, "null argument");
  *out = nullptr;
  const int64_t H = hidden, I = intermediate;
  if (H <= 0 || I <= 0) return fail(MYL_ERR_SHAPE, "mlp_int: hidden %lld / intermediate %lld",
                                    (long long)H, (long long)I);
  // The table index is computed in i16 (integer_math.rs:166-170): lengths the
  // reference can index without a panic are 1 .. 32768.
  if (silu_lut_len < 1 || silu_lut_len > 32768)
    return fail(MYL_ERR_SHAPE, "silu_lut length %lld", (long long)silu_lut_len);
  // Every shift the reference computes, validated as its debug build would.
  std::vector<int8_t> sgu(static_cast<size_t>(2 * I));
  std::vector<int8_t> sdown(static_cast<size_t>(H));
  for (int64_t i = 0; i < I; ++i) {
    TRY(signed_total_shift(gate_w_shifts[i], in_frac, gate_out_frac, &sgu[size_t(2 * i)]));
    TRY(signed_total_shift(up_w_shifts[i], in_frac, up_out_frac, &sgu[size_t(2 * i + 1)]));
  }
  for (int64_t r = 0; r < H; ++r)
    TRY(signed_total_shift(down_w_shifts[r], down_in_frac, out_frac[r], &sdown[size_t(r)]));
  const int s1 = int(int8_t(gate_out_frac)) - int(int8_t(silu_in_frac));
  if (s1 > 30 || s1 < -31) return fail(MYL_ERR_OVERFLOW, "gate_out_frac -> silu_in_frac shift %d", s1);
  const unsigned prod_frac = unsigned(silu_out_frac) + unsigned(up_out_frac);
  if (prod_frac > 255u) return fail(MYL_ERR_OVERFLOW, "silu_out_frac + up_out_frac overflows u8");
  int8_t s2 = 0;
  TRY(signed_total_shift(uint8_t(prod_frac), 0, down_in_frac, &s2));
  // Interleave gate and up rows: row 2i = gate_i, row 2i + 1 = up_i.
  std::vector<int8_t> wgu(size_t(2 * I) * size_t(H));
  std::vector<uint8_t> gu_shifts(size_t(2 * I));
  for (int64_t i = 0; i < I; ++i) {
    std::memcpy(&wgu[size_t(2 * i) * size_t(H)], W_gate + i * H, size_t(H));
    std::memcpy(&wgu[size_t(2 * i + 1) * size_t(H)], W_up + i * H, size_t(H));
    gu_shifts[size_t(2 * i)] = gate_w_shifts[i];
    gu_shifts[size_t(2 * i + 1)] = up_w_shifts[i];
  }
  myl_mlp* m = new myl_mlp();
  m->H = H;
  m->I = I;
  m->lut_hi = int(int16_t(uint16_t(uint16_t(silu_lut_len) - 1u)));
  m->offset = silu_lut_offset;
  m->s1 = s1;
  m->s2 = s2;
  int rc = myl_weight_register(ctx, wgu.data(), 2 * I, H, H, gu_shifts.data(), &m->w_gu);
  if (rc == MYL_OK) rc = myl_weight_register(ctx, W_down, H, I, I, down_w_shifts, &m->w_down);
  if (rc == MYL_OK &&
      (cudaMalloc(&m->d_shift_gu, size_t(2 * I)) != cudaSuccess ||
       cudaMalloc(&m->d_shift_down, size_t(H)) != cudaSuccess ||
       cudaMalloc(&m->d_lut, size_t(silu_lut_len) * 2) != cudaSuccess ||
       cudaMemcpy(m->d_shift_gu, sgu.data(), size_t(2 * I), cudaMemcpyHostToDevice) != cudaSuccess ||
       cudaMemcpy(m->d_shift_down, sdown.data(), size_t(H), cudaMemcpyHostToDevice) != cudaSuccess ||
       cudaMemcpy(m->d_lut, silu_lut, size_t(silu_lut_len) * 2, cudaMemcpyHostToDevice) != cudaSuccess))
    rc = fail(MYL_ERR_CUDA, "mlp upload failed");
  if (rc != MYL_OK) {
    myl_mlp_release(ctx, m);
    return rc;
  }
  *out = m;
  return MYL_OK;
}

// y != nullptr: requantised output; otherwise acc receives the exact int64
// down-projection sums (tensor-parallel partials).
// Byte planes of an activation that several projections read (split once).
struct XPlanes {
  const uint8_t* hi = nullptr;
  const uint8_t* lo = nullptr;
  int64_t ldp = 0;
};

static int run_mlp(myl_ctx* ctx, const myl_mlp* mlp, const int16_t* x, int64_t M, int64_t ldx,
                   int16_t* y, int64_t ldy, cudaStream_t st, int64_t* acc = nullptr,
                   const XPlanes& xp = XPlanes(), const Epilogue* down_ep = nullptr) {
  if (M == 0) return MYL_OK;
  const int64_t I = mlp->I;
  Epilogue ep_gu{};
  ep_gu.mode = EPI_SILU;
  ep_gu.shift = mlp->d_shift_gu;
  ep_gu.silu.lut = mlp->d_lut;
  ep_gu.silu.lut_hi = mlp->lut_hi;
  ep_gu.silu.offset = mlp->offset;
  ep_gu.silu.s1 = mlp->s1;
  ep_gu.silu.s2 = mlp->s2;
  Epilogue ep_down{};
  ep_down.mode = acc ? EPI_ACC_I64 : EPI_SHIFT;
  ep_down.shift = mlp->d_shift_down;
  ep_down.y = acc ? static_cast<void*>(acc) : static_cast<void*>(y);
  ep_down.ldy = acc ? mlp->H : ldy;
  if (down_ep) ep_down = *down_ep;  // e.g. tensor-parallel partials broadcast to every rank
  CUDA_TRY(cudaSetDevice(ctx->device));
  TRY(ws_acquire(ctx, st));
  if (M <= ctx->gemv_max_m && M <= 4) {
    // Decode: GEMV with the SiLU pair epilogue writes h [M][I]; GEMV down.
    TRY(ensure(ctx->h, size_t(M) * size_t(I) * 2));
    ep_gu.y = ctx->h.p;
    ep_gu.ldy = I;
    TRY(launch_gemv(ctx, mlp->w_gu, x, M, ldx, ep_gu, st));
    TRY(launch_gemv(ctx, mlp->w_down, static_cast<const int16_t*>(ctx->h.p), M, I, ep_down, st));
  } else {
    // Prefill: the gate/up GEMM writes h straight into the byte planes the
    // down GEMM reads; h itself never goes to memory as int16.
    const int64_t ldp_h = mlp->w_down->ldp;
    TRY(ensure(ctx->hplanes, size_t(2) * size_t(M) * size_t(ldp_h)));
    uint8_t* hhi = static_cast<uint8_t*>(ctx->hplanes.p);
    uint8_t* hlo = hhi + M * ldp_h;
    ep_gu.y = nullptr;  // only the planes are needed
    ep_gu.ldy = I;
    ep_gu.silu.h_hi = hhi;
    ep_gu.silu.h_lo = hlo;
    ep_gu.silu.ldp = ldp_h;
    if (xp.hi) TRY(launch_tc_planes(ctx, mlp->w_gu, xp.hi, xp.lo, xp.ldp, M, ep_gu, st));
    else TRY(launch_tc(ctx, mlp->w_gu, x, M, ldx, ep_gu, st));
    TRY(launch_tc_planes(ctx, mlp->w_down, hhi, hlo, ldp_h, M, ep_down, st));
  }
  return ws_release(ctx, st);
}

int myl_mlp_dev(myl_ctx* ctx, const myl_mlp* mlp, const int16_t* x, int64_t M, int64_t ldx,
                int16_t* y, int64_t ldy, void* stream) {
  if (!ctx || !mlp || (M > 0 && (!x || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (M < 0 || ldx < mlp->H || ldy < mlp->H) return fail(MYL_ERR_SHAPE, "bad M/ldx/ldy");
  return run_mlp(ctx, mlp, x, M, ldx, y, ldy, static_cast<cudaStream_t>(stream));
}

int myl_mlp_partial_dev(myl_ctx* ctx, const myl_mlp* mlp, const int16_t* x, int64_t M, int64_t ldx,
                        int64_t* acc, void* stream) {
  if (!ctx || !mlp || (M > 0 && (!x || !acc))) return fail(MYL_ERR_ARG, "null argument");
  if (M < 0 || ldx < mlp->H) return fail(MYL_ERR_SHAPE, "bad M/ldx");
  return run_mlp(ctx, mlp, x, M, ldx, nullptr, 0, static_cast<cudaStream_t>(stream), acc);
}

int myl_mlp_requant_dev(myl_ctx* ctx, const myl_mlp* mlp, const int64_t* acc, int64_t M, int16_t* y,
                        int64_t ldy, void* stream) {
  if (!ctx || !mlp || (M > 0 && (!acc || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (M < 0 || ldy < mlp->H) return fail(MYL_ERR_SHAPE, "bad M/ldy");
  if (M == 0) return MYL_OK;
  Epilogue ep{};
  ep.mode = EPI_SHIFT;
  ep.shift = mlp->d_shift_down;
  ep.y = y;
  ep.ldy = ldy;
  CUDA_TRY(cudaSetDevice(ctx->device));
  const int64_t total = M * mlp->H;
  unsigned blocks = unsigned(std::min<int64_t>((total + 255) / 256, int64_t(ctx->num_sms) * 8));
  reduce_requant_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(acc, 1, 0, M, mlp->H, ep);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

int myl_mlp_int(myl_ctx* ctx, const myl_mlp* mlp, const int16_t* x, int64_t M, int16_t* y) {
  if (!ctx || !mlp || (M > 0 && (!x || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (M < 0) return fail(MYL_ERR_SHAPE, "M = %lld is negative", (long long)M);
  if (M == 0) return MYL_OK;
  const int64_t H = mlp->H;
  TRY(ensure(ctx->x, size_t(M) * size_t(H) * 2));
  TRY(ensure(ctx->y, size_t(M) * size_t(H) * 2));
  cudaStream_t st = ctx->stream;
  CUDA_TRY(cudaMemcpyAsync(ctx->x.p, x, size_t(M) * size_t(H) * 2, cudaMemcpyHostToDevice, st));
  TRY(run_mlp(ctx, mlp, static_cast<const int16_t*>(ctx->x.p), M, H, static_cast<int16_t*>(ctx->y.p),
              H, st));
  CUDA_TRY(cudaMemcpyAsync(y, ctx->y.p, size_t(M) * size_t(H) * 2, cudaMemcpyDeviceToHost, st));
  return check_device_error(ctx);
}

int myl_split_hilo_dev(myl_ctx* ctx, const int16_t* x, int64_t M, int64_t K, int64_t ldx,
                       uint8_t* xhi, uint8_t* xlo, int64_t ldp, void* stream) {
  if (!ctx || (M > 0 && (!x || !xhi || !xlo))) return fail(MYL_ERR_ARG, "null argument");
  if (M < 0 || K <= 0 || ldx < K || ldp < K || ldp % 16 != 0)
    return fail(MYL_ERR_SHAPE, "bad split shape (ldp must be a multiple of 16 and >= K)");
  if ((reinterpret_cast<uintptr_t>(xhi) | reinterpret_cast<uintptr_t>(xlo)) & 15)
    return fail(MYL_ERR_ARG, "plane pointers must be 16-byte aligned");
  if (M == 0) return MYL_OK;
  CUDA_TRY(cudaSetDevice(ctx->device));
  return launch_split(ctx, x, M, K, ldx, xhi, xlo, ldp, static_cast<cudaStream_t>(stream));
}

int myl_linear_planes_dev(myl_ctx* ctx, const myl_weight* w, const myl_requant* rq,
                          const uint8_t* xhi, const uint8_t* xlo, int64_t ldp, int64_t M, void* y,
                          int64_t ldy, void* stream) {
  if (!ctx || !w || (M > 0 && (!xhi || !xlo || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: use myl_lm_head_w16a16_i32 or myl_linear_dev");
  if (M < 0 || ldp < w->K || ldp % 16 != 0 || ldy < w->N)
    return fail(MYL_ERR_SHAPE, "bad M/ldp/ldy");
  if ((reinterpret_cast<uintptr_t>(xhi) | reinterpret_cast<uintptr_t>(xlo)) & 15)
    return fail(MYL_ERR_ARG, "plane pointers must be 16-byte aligned");
  if (rq && rq->N != w->N) return fail(MYL_ERR_SHAPE, "requant/weight channel mismatch");
  if (M == 0 || w->N == 0) return MYL_OK;
  Epilogue ep{};
  if (rq) {
    ep = make_ep(rq, y, ldy);
  } else {
    ep.mode = EPI_ACC_I64;
    ep.y = y;
    ep.ldy = ldy;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaSetDevice(ctx->device));
  TRY(ws_acquire(ctx, st));
  TRY(launch_tc_planes(ctx, w, xhi, xlo, ldp, M, ep, st));
  return ws_release(ctx, st);
}

int myl_synchronize(myl_ctx* ctx) {
  if (!ctx) return fail(MYL_ERR_ARG, "ctx is null");
  CUDA_TRY(cudaDeviceSynchronize());
  return check_device_error(ctx);
}

int myl_set_wait_timeout_ns(myl_ctx* ctx, uint64_t ns) {
  if (!ctx || ns == 0) return fail(MYL_ERR_ARG, "bad argument");
  ctx->timeout_ns = ns;
  return MYL_OK;
}

int myl_set_dispatch(myl_ctx* ctx, int gemv_max_m, int force_split_k, int force_token_tile) {
  if (!ctx) return fail(MYL_ERR_ARG, "ctx is null");
  ctx->gemv_max_m = gemv_max_m;
  ctx->force_split_k = force_split_k;
  ctx->force_tile = force_token_tile;
  return MYL_OK;
}

int myl_set_sm_limit(myl_ctx* ctx, int max_sms) {
  if (!ctx || max_sms < 0) return fail(MYL_ERR_ARG, "bad argument");
  ctx->sm_limit = max_sms;
  return MYL_OK;
}

int myl_set_tc_options(myl_ctx* ctx, int pair_mode, int xbox_rows) {
  if (!ctx) return fail(MYL_ERR_ARG, "ctx is null");
  if (pair_mode != 0 && pair_mode != 1) return fail(MYL_ERR_ARG, "pair_mode must be 0 or 1");
  if (xbox_rows != 0 && xbox_rows != 16 && xbox_rows != 32 && xbox_rows != 64 && xbox_rows != 128)
    return fail(MYL_ERR_ARG, "xbox_rows must be 0, 16, 32, 64 or 128");
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  ctx->pair_mode = pair_mode;
  if (xbox_rows) ctx->xbox = xbox_rows;
  return MYL_OK;
}

int myl_debug_inject_wait_fault(myl_ctx* ctx, int on) {
  if (!ctx) return fail(MYL_ERR_ARG, "ctx is null");
  ctx->inject_fault = on ? 1 : 0;
  return MYL_OK;
}

int64_t myl_launch_count(const myl_ctx* ctx) { return ctx ? ctx->launches : -1; }

}  // extern "C"

// ---------------------------------------------------------------------------------
// Allocation-free tensor-core linear.
//
// Some callers cannot let a library allocate device memory: a runtime that
// reserves its whole device budget in its own arena at start-up (so a long
// inference or mining job cannot fail half-way on a late cudaMalloc), or a
// loop that must not stall, since cudaMalloc/cudaFree synchronise the whole
// device and would hold up every other stream. The regular entry points grow
// a per-context workspace on demand; myl_linear_noalloc_dev instead keeps the
// activation byte planes in the fixed array below, which is part of this
// library's device image: every GPU that loads the library holds these
// MYL_NOALLOC_SCRATCH_BYTES until the process exits.
//
// The array is one per device and shared by every call: calls whose work
// overlaps on the GPU (other streams, other host threads) race on it. Nothing
// in it needs to start at zero: the split pass writes every plane byte the
// GEMM reads before the GEMM runs, on the same stream.

static __device__ __align__(256) uint8_t g_noalloc_scratch[MYL_NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {};

// Host code cannot use g_noalloc_scratch as an address (it names a host-side
// stand-in); the device address is looked up once per device, with that
// device current.
static int noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= 64) return fail(MYL_ERR_UNSUPPORTED, "device index %d", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(MYL_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch) failed: %s",
                  cudaGetErrorString(e));
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return MYL_OK;
}

extern "C" int myl_linear_noalloc_dev(myl_ctx* ctx, const myl_weight* w, const myl_requant* rq,
                                      const int16_t* x, int64_t M, int64_t ldx, void* y,
                                      int64_t ldy, void* stream) {
  if (!ctx || !w || !rq || (M > 0 && (!x || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (w->w16) return fail(MYL_ERR_ARG, "int16 weight: use myl_lm_head_w16a16_i32 or myl_linear_dev");
  if (rq->N != w->N) return fail(MYL_ERR_SHAPE, "requant/weight channel mismatch");
  if (M < 0 || ldx < w->K || ldy < w->N) return fail(MYL_ERR_SHAPE, "bad M/ldx/ldy");
  if (w->K > 65536)
    return fail(MYL_ERR_UNSUPPORTED,
                "myl_linear_noalloc_dev: in_features %lld > 65536 would need K-slice partial sums",
                (long long)w->K);
  const size_t need = size_t(2) * size_t(M) * size_t(w->ldp);
  if (need > size_t(MYL_NOALLOC_SCRATCH_BYTES))
    return fail(MYL_ERR_UNSUPPORTED,
                "myl_linear_noalloc_dev: 2 * M * round_up(K, 16) = %zu bytes exceeds the fixed "
                "scratch of %d bytes; use fewer rows per call",
                need, MYL_NOALLOC_SCRATCH_BYTES);
  if (M == 0 || w->N == 0) return MYL_OK;
  CUDA_TRY(cudaSetDevice(ctx->device));
  void* scratch = nullptr;
  TRY(noalloc_scratch(ctx->device, &scratch));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* xhi = static_cast<uint8_t*>(scratch);
  uint8_t* xlo = xhi + M * w->ldp;
  TRY(launch_split(ctx, x, M, w->K, ldx, xhi, xlo, w->ldp, st));
  // Same tile choice as the regular path, but always one K slice: no int64
  // partial buffer is needed.
  const int BN = tc_token_tile(ctx, M);
  CUtensorMap tm_xhi, tm_xlo;
  TRY(encode_map(ctx, &tm_xhi, xhi, w->K, M, w->ldp, tc_xbox(ctx, BN)));
  TRY(encode_map(ctx, &tm_xlo, xlo, w->K, M, w->ldp, tc_xbox(ctx, BN)));
  const int k_tiles = int((w->K + TC_BK - 1) / TC_BK);
  const bool pair = tc_pair(ctx, BN);
  const int ct = pair ? 256 : 128;
  const TcWork work{int((w->N + ct - 1) / ct), int((M + BN - 1) / BN), 1, k_tiles, k_tiles};
  return launch_tc_any(ctx, w, tm_xhi, tm_xlo, M, BN, pair, work, make_ep(rq, y, ldy), 0, st);
}

// ---------------------------------------------------------------------------------
// MoE layer (moe.cuh): router linear, integer top-k + softmax_int, counting
// sort of the (token, choice) pairs by expert, grouped tensor-core GEMMs over
// the experts' row segments, combine.

struct myl_moe {
  int64_t H = 0, I = 0, E = 0, k = 0, first = 0, L = 0;
  myl_weight* w_router = nullptr;  // [E][H]
  myl_requant* rq_router = nullptr;  // i32 logits
  myl_weight* w_gu = nullptr;      // [L * 2I][H], per expert rows 2i = gate_i, 2i + 1 = up_i
  myl_weight* w_down = nullptr;    // [L * H][I]
  int8_t* d_shift_gu = nullptr;    // [L * 2I]
  int8_t* d_shift_down = nullptr;  // [L * H]
  int16_t* d_silu_lut = nullptr;
  int lut_hi = 0, offset = 0, s1 = 0, s2 = 0;
  int16_t* d_exp_lut = nullptr;
  int exp_lut_len = 0, exp_lut_shift = 0, prob_frac = 0;
  const myl_mlp* shared = nullptr;
};

// Carves 256-byte aligned pieces out of ctx->moe.
struct MoeArena {
  size_t off = 0;
  template <typename T>
  size_t take(int64_t n) {
    const size_t at = off;
    off = (off + size_t(std::max<int64_t>(n, 1)) * sizeof(T) + 255) & ~size_t(255);
    return at;
  }
};

struct MoeExpertsWs {
  int *counts, *row_start, *rows, *tile_a, *tile_b, *cursor;
  int32_t *src, *pos;
  uint8_t* xhi;
  uint8_t* xlo;
  uint8_t* hhi;
  uint8_t* hlo;
  int16_t* y_perm;
};

struct MoeWs {
  MoeExpertsWs ex;
  int32_t *logits, *topk_idx, *topk_prob;
  int16_t* shared_out;
};

// Workspace for P pairs (and, with T > 0, the router and shared output of T
// tokens) inside ctx->moe.
static int moe_workspace(myl_ctx* ctx, const myl_moe* m, int64_t P, int64_t T, MoeWs* w) {
  const int64_t L = m->L, ldp_h = m->w_gu->ldp, ldp_i = m->w_down->ldp;
  MoeArena a;
  const size_t o_counts = a.take<int>(L), o_row_start = a.take<int>(L), o_rows = a.take<int>(L),
               o_tile_a = a.take<int>(L + 1), o_tile_b = a.take<int>(L + 1),
               o_cursor = a.take<int>(L), o_src = a.take<int32_t>(P), o_pos = a.take<int32_t>(P),
               o_xhi = a.take<int8_t>(P * ldp_h), o_xlo = a.take<uint8_t>(P * ldp_h),
               o_hhi = a.take<int8_t>(P * ldp_i), o_hlo = a.take<uint8_t>(P * ldp_i),
               o_y = a.take<int16_t>(P * m->H), o_logits = a.take<int32_t>(T * m->E),
               o_idx = a.take<int32_t>(T * m->k), o_prob = a.take<int32_t>(T * m->k),
               o_shared = a.take<int16_t>(T * m->H);
  TRY(ensure(ctx->moe, a.off));
  uint8_t* b = static_cast<uint8_t*>(ctx->moe.p);
  w->ex.counts = reinterpret_cast<int*>(b + o_counts);
  w->ex.row_start = reinterpret_cast<int*>(b + o_row_start);
  w->ex.rows = reinterpret_cast<int*>(b + o_rows);
  w->ex.tile_a = reinterpret_cast<int*>(b + o_tile_a);
  w->ex.tile_b = reinterpret_cast<int*>(b + o_tile_b);
  w->ex.cursor = reinterpret_cast<int*>(b + o_cursor);
  w->ex.src = reinterpret_cast<int32_t*>(b + o_src);
  w->ex.pos = reinterpret_cast<int32_t*>(b + o_pos);
  w->ex.xhi = b + o_xhi;
  w->ex.xlo = b + o_xlo;
  w->ex.hhi = b + o_hhi;
  w->ex.hlo = b + o_hlo;
  w->ex.y_perm = reinterpret_cast<int16_t*>(b + o_y);
  w->logits = reinterpret_cast<int32_t*>(b + o_logits);
  w->topk_idx = reinterpret_cast<int32_t*>(b + o_idx);
  w->topk_prob = reinterpret_cast<int32_t*>(b + o_prob);
  w->shared_out = reinterpret_cast<int16_t*>(b + o_shared);
  return MYL_OK;
}

static unsigned grid_for(const myl_ctx* ctx, int64_t items, int per_sm = 8) {
  return unsigned(std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256,
                                                         int64_t(ctx->num_sms) * per_sm)));
}

// Row-wise kernels: x covers a row with 8 elements per thread (256 threads),
// y walks the rows (grid-stride beyond 65535).
static dim3 rows_grid(int64_t cols, int64_t rows) {
  return dim3(unsigned((cols + 8 * 256 - 1) / (8 * 256)),
              unsigned(std::max<int64_t>(1, std::min<int64_t>(rows, 65535))));
}

// Token tile of the grouped GEMMs from the mean rows per expert.
static int moe_token_tile(const myl_ctx* ctx, int64_t P, int64_t L) {
  if (ctx->force_tile == 32 || ctx->force_tile == 64 || ctx->force_tile == 128) return ctx->force_tile;
  const int64_t mean = (P + L - 1) / std::max<int64_t>(L, 1);
  return mean <= 32 ? 32 : (mean <= 64 ? 64 : 128);
}

static int moe_route(myl_ctx* ctx, const myl_moe* m, const int16_t* x, int64_t T, int64_t ldx,
                     int32_t* logits, int32_t* idx, int32_t* prob, cudaStream_t st,
                     const XPlanes& xp = XPlanes()) {
  Epilogue ep{};
  ep.mode = EPI_SHIFT;
  ep.out_i32 = 1;
  ep.shift = m->rq_router->d_shift;
  ep.y = logits;
  ep.ldy = m->E;
  if (xp.hi) TRY(launch_tc_planes(ctx, m->w_router, xp.hi, xp.lo, xp.ldp, T, ep, st));
  else TRY(dispatch_linear(ctx, m->w_router, x, T, ldx, ep, st));
  MoeRouteParams rp{m->d_exp_lut, m->exp_lut_len, m->exp_lut_shift, m->prob_frac};
  moe_route_kernel<<<grid_for(ctx, T * 32), 256, 0, st>>>(logits, m->E, T, int(m->E), int(m->k), rp,
                                                           idx, prob);  // one warp per token
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

// Pairs q in [0, P) with expert ids[q] read source row q / div of x; y_perm
// row pos[q] receives mlp_int(x[q / div], expert ids[q]).
static int moe_experts(myl_ctx* ctx, const myl_moe* m, const int16_t* x, int64_t ldx,
                       const int32_t* ids, int64_t P, int div, const MoeExpertsWs& w,
                       cudaStream_t st) {
  const int L = int(m->L);
  const int BN = moe_token_tile(ctx, P, L);
  const bool pair = tc_pair(ctx, BN);
  const int ct = pair ? 256 : 128;  // channels per work unit
  const int tiles_gu = int((2 * m->I + ct - 1) / ct), tiles_down = int((m->H + ct - 1) / ct);
  CUDA_TRY(cudaMemsetAsync(w.counts, 0, size_t(L) * sizeof(int), st));
  moe_count_kernel<<<grid_for(ctx, P, 2), 256, 0, st>>>(ids, P, int(m->first), L, w.counts,
                                                        ctx->d_err);
  CUDA_TRY(cudaGetLastError());
  moe_plan_kernel<<<1, 1, 0, st>>>(w.counts, L, BN, tiles_gu, tiles_down, w.row_start, w.rows,
                                   w.tile_a, w.tile_b, w.cursor);
  CUDA_TRY(cudaGetLastError());
  // The scatter fills src[0, valid rows); with bad ids the tail up to P is
  // still read by the gather (and never stored), so it starts as row 0.
  CUDA_TRY(cudaMemsetAsync(w.src, 0, size_t(P) * sizeof(int32_t), st));
  moe_scatter_kernel<<<grid_for(ctx, P), 256, 0, st>>>(ids, P, int(m->first), L, div, w.cursor,
                                                        w.src, w.pos);
  CUDA_TRY(cudaGetLastError());
  const int64_t H = m->H, ldp_h = m->w_gu->ldp, ldp_i = m->w_down->ldp;
  moe_gather_split_kernel<<<rows_grid(ldp_h, P), 256, 0, st>>>(x, ldx, P, H, w.src, w.xhi, w.xlo,
                                                                ldp_h);
  CUDA_TRY(cudaGetLastError());
  ctx->launches += 4;
  // Gate/up: grouped GEMM with the SiLU pair epilogue into the down planes.
  CUtensorMap tm_xhi, tm_xlo, tm_hhi, tm_hlo;
  const int xb = tc_xbox(ctx, BN);
  TRY(encode_map(ctx, &tm_xhi, w.xhi, H, P, ldp_h, xb));
  TRY(encode_map(ctx, &tm_xlo, w.xlo, H, P, ldp_h, xb));
  TRY(encode_map(ctx, &tm_hhi, w.hhi, m->I, P, ldp_i, xb));
  TRY(encode_map(ctx, &tm_hlo, w.hlo, m->I, P, ldp_i, xb));
  TcWork wk{};
  wk.tiles_n = tiles_gu;
  wk.tiles_m = 1;
  wk.ksplit = 1;
  wk.k_tiles_total = int((H + TC_BK - 1) / TC_BK);
  wk.k_tiles_per_split = wk.k_tiles_total;
  wk.groups = L;
  wk.tile_start = w.tile_a;
  wk.row_start = w.row_start;
  wk.rows = w.rows;
  wk.group_w_rows = 2 * m->I;
  Epilogue ep_gu{};
  ep_gu.mode = EPI_SILU;
  ep_gu.shift = m->d_shift_gu;
  ep_gu.silu.lut = m->d_silu_lut;
  ep_gu.silu.lut_hi = m->lut_hi;
  ep_gu.silu.offset = m->offset;
  ep_gu.silu.s1 = m->s1;
  ep_gu.silu.s2 = m->s2;
  ep_gu.silu.h_hi = w.hhi;
  ep_gu.silu.h_lo = w.hlo;
  ep_gu.silu.ldp = ldp_i;
  ep_gu.ldy = m->I;
  TRY(launch_tc_any(ctx, m->w_gu, tm_xhi, tm_xlo, P, BN, pair, wk, ep_gu, 0, st));
  // Down: grouped GEMM, reference requant, rows in expert order.
  wk.tiles_n = tiles_down;
  wk.k_tiles_total = int((m->I + TC_BK - 1) / TC_BK);
  wk.k_tiles_per_split = wk.k_tiles_total;
  wk.tile_start = w.tile_b;
  wk.group_w_rows = H;
  Epilogue ep_down{};
  ep_down.mode = EPI_SHIFT;
  ep_down.shift = m->d_shift_down;
  ep_down.y = w.y_perm;
  ep_down.ldy = H;
  return launch_tc_any(ctx, m->w_down, tm_hhi, tm_hlo, P, BN, pair, wk, ep_down, 0, st);
}

extern "C" {

int myl_moe_release(myl_ctx* ctx, myl_moe* m) {
  if (!m) return MYL_OK;
  if (ctx) {
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (m->w_router) myl_weight_release(ctx, m->w_router);
    if (m->rq_router) myl_requant_release(ctx, m->rq_router);
    if (m->w_gu) myl_weight_release(ctx, m->w_gu);
    if (m->w_down) myl_weight_release(ctx, m->w_down);
  }
  for (void* p : {static_cast<void*>(m->d_shift_gu), static_cast<void*>(m->d_shift_down),
                  static_cast<void*>(m->d_silu_lut), static_cast<void*>(m->d_exp_lut)})
    if (p) cudaFree(p);
  delete m;
  return MYL_OK;
}

int myl_moe_register(myl_ctx* ctx, const myl_moe_spec* s, myl_moe** out) {
  if (!ctx || !s || !out) return fail(MYL_ERR_ARG, "null argument");
  *out = nullptr;
  const int64_t H = s->hidden, I = s->intermediate, E = s->num_experts, L = s->num_local;
  if (H <= 0 || I <= 0 || E <= 0 || L <= 0 || s->first_expert < 0 || s->first_expert + L > E)
    return fail(MYL_ERR_SHAPE, "moe: hidden %lld intermediate %lld experts %lld local [%lld, +%lld)",
                (long long)H, (long long)I, (long long)E, (long long)s->first_expert, (long long)L);
  if (E > MOE_MAX_EXPERTS || s->top_k < 1 || s->top_k > MOE_MAX_K || s->top_k > E)
    return fail(MYL_ERR_UNSUPPORTED, "moe: %lld experts, top-%lld (limits: 256 experts, top-8)",
                (long long)E, (long long)s->top_k);
  if (H > 65536 || I > 65536)
    return fail(MYL_ERR_UNSUPPORTED, "moe: hidden/intermediate beyond 65536");
  if (!s->W_router || !s->router_w_shifts || !s->W_gate || !s->W_up || !s->W_down ||
      !s->gate_w_shifts || !s->up_w_shifts || !s->down_w_shifts || !s->out_frac || !s->silu_lut ||
      (s->exp_lut_len > 0 && !s->exp_lut))
    return fail(MYL_ERR_ARG, "moe: null table or weight");
  if (s->silu_lut_len < 1 || s->silu_lut_len > 32768)
    return fail(MYL_ERR_SHAPE, "silu_lut length %lld", (long long)s->silu_lut_len);
  if (s->exp_lut_len < 0 || s->exp_lut_len > (int64_t(1) << 30) || s->exp_lut_shift > 31 ||
      s->prob_frac > 30)
    return fail(MYL_ERR_SHAPE, "exp_lut length %lld, shift %u, prob_frac %u",
                (long long)s->exp_lut_len, unsigned(s->exp_lut_shift), unsigned(s->prob_frac));
  // softmax_int multiplies e * 2^prob_frac in i32 (softmax.rs:52): every value
  // e can take (the table's entries, and 1 for an empty table) must keep it in
  // range, so the kernel never meets the overflow the reference would panic on.
  {
    const int64_t one = int64_t(1) << s->prob_frac;
    int64_t lo = s->exp_lut_len > 0 ? 0 : 1, hi = lo;
    for (int64_t i = 0; i < s->exp_lut_len; ++i) {
      lo = std::min<int64_t>(lo, s->exp_lut[i]);
      hi = std::max<int64_t>(hi, s->exp_lut[i]);
    }
    if (hi * one > INT32_MAX || lo * one < INT32_MIN)
      return fail(MYL_ERR_OVERFLOW, "exp_lut entry * 2^prob_frac overflows i32");
  }
  // Shifts, validated as the reference's debug build would (mlp.rs:28-74).
  std::vector<int8_t> sgu(size_t(L * 2 * I)), sdown(size_t(L * H));
  for (int64_t e = 0; e < L; ++e) {
    for (int64_t i = 0; i < I; ++i) {
      TRY(signed_total_shift(s->gate_w_shifts[e * I + i], s->in_frac, s->gate_out_frac,
                             &sgu[size_t(e * 2 * I + 2 * i)]));
      TRY(signed_total_shift(s->up_w_shifts[e * I + i], s->in_frac, s->up_out_frac,
                             &sgu[size_t(e * 2 * I + 2 * i + 1)]));
    }
    for (int64_t r = 0; r < H; ++r)
      TRY(signed_total_shift(s->down_w_shifts[e * H + r], s->down_in_frac, s->out_frac[e * H + r],
                             &sdown[size_t(e * H + r)]));
  }
  const int s1 = int(int8_t(s->gate_out_frac)) - int(int8_t(s->silu_in_frac));
  if (s1 > 30 || s1 < -31) return fail(MYL_ERR_OVERFLOW, "gate_out_frac -> silu_in_frac shift %d", s1);
  const unsigned prod_frac = unsigned(s->silu_out_frac) + unsigned(s->up_out_frac);
  if (prod_frac > 255u) return fail(MYL_ERR_OVERFLOW, "silu_out_frac + up_out_frac overflows u8");
  int8_t s2 = 0;
  TRY(signed_total_shift(uint8_t(prod_frac), 0, s->down_in_frac, &s2));
  // Stacked, interleaved gate/up rows per expert.
  std::vector<int8_t> wgu(size_t(L * 2 * I) * size_t(H));
  std::vector<uint8_t> gu_shifts(size_t(L * 2 * I));
  for (int64_t e = 0; e < L; ++e)
    for (int64_t i = 0; i < I; ++i) {
      const int64_t r = e * 2 * I + 2 * i;
      std::memcpy(&wgu[size_t(r) * size_t(H)], s->W_gate + (e * I + i) * H, size_t(H));
      std::memcpy(&wgu[size_t(r + 1) * size_t(H)], s->W_up + (e * I + i) * H, size_t(H));
      gu_shifts[size_t(r)] = s->gate_w_shifts[e * I + i];
      gu_shifts[size_t(r + 1)] = s->up_w_shifts[e * I + i];
    }
  CUDA_TRY(cudaSetDevice(ctx->device));
  myl_moe* m = new myl_moe();
  m->H = H;
  m->I = I;
  m->E = E;
  m->k = s->top_k;
  m->first = s->first_expert;
  m->L = L;
  m->lut_hi = int(int16_t(uint16_t(uint16_t(s->silu_lut_len) - 1u)));
  m->offset = s->silu_lut_offset;
  m->s1 = s1;
  m->s2 = s2;
  m->exp_lut_len = int(s->exp_lut_len);
  m->exp_lut_shift = s->exp_lut_shift;
  m->prob_frac = s->prob_frac;
  m->shared = s->shared;
  const uint8_t router_frac = s->router_frac;
  int rc = myl_weight_register(ctx, s->W_router, E, H, H, s->router_w_shifts, &m->w_router);
  if (rc == MYL_OK)
    rc = myl_requant_create(ctx, m->w_router, MYL_RQ_SHIFT_I32, s->router_in_frac, &router_frac, 0,
                            nullptr, nullptr, &m->rq_router);
  if (rc == MYL_OK) rc = myl_weight_register(ctx, wgu.data(), L * 2 * I, H, H, gu_shifts.data(), &m->w_gu);
  if (rc == MYL_OK)
    rc = myl_weight_register(ctx, s->W_down, L * H, I, I, s->down_w_shifts, &m->w_down);
  const size_t lut_bytes = size_t(std::max<int64_t>(s->exp_lut_len, 1)) * 2;
  if (rc == MYL_OK &&
      (cudaMalloc(&m->d_shift_gu, sgu.size()) != cudaSuccess ||
       cudaMalloc(&m->d_shift_down, sdown.size()) != cudaSuccess ||
       cudaMalloc(&m->d_silu_lut, size_t(s->silu_lut_len) * 2) != cudaSuccess ||
       cudaMalloc(&m->d_exp_lut, lut_bytes) != cudaSuccess ||
       cudaMemcpy(m->d_shift_gu, sgu.data(), sgu.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
       cudaMemcpy(m->d_shift_down, sdown.data(), sdown.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
       cudaMemcpy(m->d_silu_lut, s->silu_lut, size_t(s->silu_lut_len) * 2, cudaMemcpyHostToDevice) !=
           cudaSuccess ||
       (s->exp_lut_len > 0 && cudaMemcpy(m->d_exp_lut, s->exp_lut, size_t(s->exp_lut_len) * 2,
                                         cudaMemcpyHostToDevice) != cudaSuccess)))
    rc = fail(MYL_ERR_CUDA, "moe upload failed");
  if (rc != MYL_OK) {
    myl_moe_release(ctx, m);
    return rc;
  }
  *out = m;
  return MYL_OK;
}

int myl_moe_route_dev(myl_ctx* ctx, const myl_moe* m, const int16_t* x, int64_t T, int64_t ldx,
                      int32_t* topk_idx, int32_t* topk_prob, void* stream) {
  if (!ctx || !m || (T > 0 && (!x || !topk_idx || !topk_prob))) return fail(MYL_ERR_ARG, "null argument");
  if (T < 0 || ldx < m->H) return fail(MYL_ERR_SHAPE, "bad T/ldx");
  if (T == 0) return MYL_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaSetDevice(ctx->device));
  TRY(ws_acquire(ctx, st));
  MoeWs w;
  TRY(moe_workspace(ctx, m, 0, T, &w));
  TRY(moe_route(ctx, m, x, T, ldx, w.logits, topk_idx, topk_prob, st));
  return ws_release(ctx, st);
}

int myl_moe_experts_dev(myl_ctx* ctx, const myl_moe* m, const int16_t* x, int64_t P, int64_t ldx,
                        const int32_t* ids, int16_t* y, int64_t ldy, void* stream) {
  if (!ctx || !m || (P > 0 && (!x || !ids || !y))) return fail(MYL_ERR_ARG, "null argument");
  if (P < 0 || P > INT32_MAX || ldx < m->H || ldy < m->H) return fail(MYL_ERR_SHAPE, "bad P/ldx/ldy");
  if (P == 0) return MYL_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaSetDevice(ctx->device));
  TRY(ws_acquire(ctx, st));
  MoeWs w;
  TRY(moe_workspace(ctx, m, P, 0, &w));
  TRY(moe_experts(ctx, m, x, ldx, ids, P, 1, w.ex, st));
  moe_unpermute_kernel<<<grid_for(ctx, P * m->H), 256, 0, st>>>(w.ex.y_perm, m->H, w.ex.pos, P, m->H,
                                                                 y, ldy);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return ws_release(ctx, st);
}

int myl_moe_combine_dev(myl_ctx* ctx, const myl_moe* m, const int16_t* y, int64_t ldy,
                        const int32_t* prob, const int16_t* shared_out, int64_t ld_shared, int64_t T,
                        int16_t* out, int64_t ldo, void* stream) {
  if (!ctx || !m || (T > 0 && (!y || !prob || !out))) return fail(MYL_ERR_ARG, "null argument");
  if (T < 0 || ldy < m->H || ldo < m->H || (shared_out && ld_shared < m->H))
    return fail(MYL_ERR_SHAPE, "bad T/ldy/ldo/ld_shared");
  if (T == 0) return MYL_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaSetDevice(ctx->device));
  moe_combine_kernel<<<rows_grid(m->H, T), 256, 0, st>>>(y, ldy, nullptr, prob, shared_out,
                                                               ld_shared, T, int(m->k), m->H,
                                                               m->prob_frac, out, ldo);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return MYL_OK;
}

int myl_moe_dev(myl_ctx* ctx, const myl_moe* m, const int16_t* x, int64_t T, int64_t ldx,
                int16_t* out, int64_t ldo, int32_t* topk_idx, int32_t* topk_prob, void* stream) {
  if (!ctx || !m || (T > 0 && (!x || !out))) return fail(MYL_ERR_ARG, "null argument");
  if (m->L != m->E)
    return fail(MYL_ERR_ARG, "myl_moe_dev needs every expert (this object holds %lld of %lld)",
                (long long)m->L, (long long)m->E);
  if (T < 0 || T * m->k > INT32_MAX || ldx < m->H || ldo < m->H) return fail(MYL_ERR_SHAPE, "bad T/ldx/ldo");
  if (T == 0) return MYL_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaSetDevice(ctx->device));
  TRY(ws_acquire(ctx, st));
  const int64_t P = T * m->k;
  MoeWs w;
  TRY(moe_workspace(ctx, m, P, T, &w));
  int32_t* idx = topk_idx ? topk_idx : w.topk_idx;
  int32_t* prob = topk_prob ? topk_prob : w.topk_prob;
  // Prefill: the router and the shared expert read x from one split.
  XPlanes xp;
  if (!(T <= ctx->gemv_max_m && T <= 4)) {
    const int64_t ldp = m->w_router->ldp;
    TRY(ensure(ctx->planes, size_t(2) * size_t(T) * size_t(ldp)));
    uint8_t* hi = static_cast<uint8_t*>(ctx->planes.p);
    TRY(launch_split(ctx, x, T, m->H, ldx, hi, hi + T * ldp, ldp, st));
    xp.hi = hi;
    xp.lo = hi + T * ldp;
    xp.ldp = ldp;
  }
  TRY(moe_route(ctx, m, x, T, ldx, w.logits, idx, prob, st, xp));
  TRY(moe_experts(ctx, m, x, ldx, idx, P, int(m->k), w.ex, st));
  const int16_t* shared_out = nullptr;
  if (m->shared) {
    TRY(run_mlp(ctx, m->shared, x, T, ldx, w.shared_out, m->H, st, nullptr, xp));
    shared_out = w.shared_out;
  }
  moe_combine_kernel<<<rows_grid(m->H, T), 256, 0, st>>>(w.ex.y_perm, m->H, w.ex.pos, prob,
                                                               shared_out, m->H, T, int(m->k), m->H,
                                                               m->prob_frac, out, ldo);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  return ws_release(ctx, st);
}

int myl_moe_forward(myl_ctx* ctx, const myl_moe* m, const int16_t* x, int64_t T, int16_t* out) {
  if (!ctx || !m || (T > 0 && (!x || !out))) return fail(MYL_ERR_ARG, "null argument");
  if (T < 0) return fail(MYL_ERR_SHAPE, "T = %lld is negative", (long long)T);
  if (T == 0) return MYL_OK;
  const size_t bytes = size_t(T) * size_t(m->H) * 2;
  TRY(ensure(ctx->x, bytes));
  TRY(ensure(ctx->y, bytes));
  cudaStream_t st = ctx->stream;
  CUDA_TRY(cudaMemcpyAsync(ctx->x.p, x, bytes, cudaMemcpyHostToDevice, st));
  TRY(myl_moe_dev(ctx, m, static_cast<const int16_t*>(ctx->x.p), T, m->H,
                  static_cast<int16_t*>(ctx->y.p), m->H, nullptr, nullptr, st));
  CUDA_TRY(cudaMemcpyAsync(out, ctx->y.p, bytes, cudaMemcpyDeviceToHost, st));
  return check_device_error(ctx);
}

}  // extern "C"

// ---------------------------------------------------------------------------------
// linear_backward (kernels/src/backward.rs:147-211)

static int prepare_backward(myl_ctx* ctx, myl_weight* w) {
  if (w->bwd_ref >= 0) return MYL_OK;
  const int64_t N = w->N;
  int ref = 0;
  for (int64_t i = 0; i < N; ++i) ref = std::max(ref, int(w->w_shifts[size_t(i)]));
  // The alignment shifts of the i128 sum stay below 64 bits (the reference's
  // shifts are at most 20, quantize.py:15).
  if (ref > 64)
    return fail(MYL_ERR_UNSUPPORTED, "linear_backward: w_shift %d above 64", ref);
  std::vector<int32_t> perm(static_cast<size_t>(N));
  for (int64_t i = 0; i < N; ++i) perm[size_t(i)] = int32_t(i);
  std::stable_sort(perm.begin(), perm.end(), [&](int32_t a, int32_t b) {
    return w->w_shifts[size_t(a)] > w->w_shifts[size_t(b)];
  });
  std::vector<BwdGroup> groups;
  for (int64_t r = 0; r < N;) {
    const int sh = w->w_shifts[size_t(perm[size_t(r)])];
    int64_t e = r;
    while (e < N && w->w_shifts[size_t(perm[size_t(e)])] == sh) ++e;
    groups.push_back(BwdGroup{ref - sh, int(r), int(e)});
    r = e;
  }
  CUDA_TRY(cudaSetDevice(ctx->device));
  if (cudaMalloc(&w->d_bwd_perm, perm.size() * 4) != cudaSuccess ||
      cudaMalloc(&w->d_bwd_groups, groups.size() * sizeof(BwdGroup)) != cudaSuccess ||
      cudaMemcpy(w->d_bwd_perm, perm.data(), perm.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(w->d_bwd_groups, groups.data(), groups.size() * sizeof(BwdGroup),
                 cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(MYL_ERR_CUDA, "linear_backward: upload of the row groups failed");
  w->bwd_ngroups = int(groups.size());
  w->bwd_ref = ref;
  return MYL_OK;
}

static int run_backward(myl_ctx* ctx, myl_weight* w, const int32_t* g, int64_t ldg, const int16_t* x,
                        int64_t ldx, int64_t M, int frac_shift, int32_t* gx, int64_t ldgx, int64_t* gw,
                        cudaStream_t st) {
  constexpr int MT = 4;
  const int64_t K = w->K, N = w->N;
  const unsigned gx_blocks = unsigned((K + BWD_THREADS * BWD_COLS - 1) / (BWD_THREADS * BWD_COLS));
  for (int64_t m0 = 0; m0 < M; m0 += int64_t(MT) * 65535) {
    const int64_t mc = std::min<int64_t>(M - m0, int64_t(MT) * 65535);
    linear_backward_gx_kernel<MT><<<dim3(gx_blocks, unsigned((mc + MT - 1) / MT)), BWD_THREADS, 0, st>>>(
        w->d_W, w->ldp, K, w->d_bwd_perm, w->d_bwd_groups, w->bwd_ngroups, w->bwd_ref, g + m0 * ldg,
        ldg, mc, frac_shift, gx + m0 * ldgx, ldgx);
    CUDA_TRY(cudaGetLastError());
    ctx->launches++;
  }
  if (gw) {
    const unsigned blocks = unsigned(std::min<int64_t>(M * N, int64_t(ctx->num_sms) * 32));
    linear_backward_gw_kernel<<<blocks, 256, 0, st>>>(g, ldg, x, ldx, M, N, K, gw);
    CUDA_TRY(cudaGetLastError());
    ctx->launches++;
  }
  return MYL_OK;
}

static int check_backward(const myl_weight* w, uint8_t g_frac, uint8_t gx_frac, int* frac_shift) {
  if (w->w16) return fail(MYL_ERR_ARG, "linear_backward: int16 weights are not supported");
  if (w->N <= 0) return fail(MYL_ERR_SHAPE, "linear_backward: w_shifts is empty");
  if (w->N >= (int64_t(1) << 24))
    return fail(MYL_ERR_UNSUPPORTED, "linear_backward: 2^24 or more output rows");
  // rescale_i64(., g_frac, gx_frac) with the debug-build checks (fixed_point.rs:184-191).
  int8_t sh = 0;
  TRY(signed_total_shift(0, g_frac, gx_frac, &sh));
  *frac_shift = sh;
  return MYL_OK;
}

extern "C" {

int myl_linear_backward_dev(myl_ctx* ctx, const myl_weight* w, const int32_t* g, int64_t ldg,
                            const int16_t* x, int64_t ldx, int64_t M, uint8_t g_frac,
                            uint8_t gx_frac, int32_t* gx, int64_t ldgx, int64_t* gw, void* stream) {
  if (!ctx || !w || (M > 0 && (!g || !gx || (gw && !x)))) return fail(MYL_ERR_ARG, "null argument");
  int frac_shift = 0;
  TRY(check_backward(w, g_frac, gx_frac, &frac_shift));
  if (M < 0 || ldg < w->N || ldgx < w->K || (gw && ldx < w->K))
    return fail(MYL_ERR_SHAPE, "bad M/ldg/ldx/ldgx");
  if (M == 0) return MYL_OK;
  myl_weight* wm = const_cast<myl_weight*>(w);
  TRY(prepare_backward(ctx, wm));
  CUDA_TRY(cudaSetDevice(ctx->device));
  return run_backward(ctx, wm, g, ldg, x, ldx, M, frac_shift, gx, ldgx, gw,
                      static_cast<cudaStream_t>(stream));
}

int myl_linear_backward(myl_ctx* ctx, const myl_weight* w, const int32_t* g, const int16_t* x,
                        int64_t M, uint8_t g_frac, uint8_t gx_frac, int32_t* gx, int64_t* gw) {
  if (!ctx || !w || (M > 0 && (!g || !x || !gx))) return fail(MYL_ERR_ARG, "null argument");
  int frac_shift = 0;
  TRY(check_backward(w, g_frac, gx_frac, &frac_shift));
  if (M < 0) return fail(MYL_ERR_SHAPE, "M = %lld is negative", (long long)M);
  if (M == 0) return MYL_OK;
  myl_weight* wm = const_cast<myl_weight*>(w);
  TRY(prepare_backward(ctx, wm));
  const int64_t N = w->N, K = w->K;
  const size_t gb = size_t(M) * size_t(N) * 4, xb = size_t(M) * size_t(K) * 2,
               gxb = size_t(M) * size_t(K) * 4, gwb = gw ? size_t(M) * size_t(N) * size_t(K) * 8 : 0;
  // workspace: g | x | gx | gw (256-byte aligned pieces)
  MoeArena a;
  const size_t og = a.take<int32_t>(M * N), ox = a.take<int16_t>(M * K), ogx = a.take<int32_t>(M * K),
               ogw = gw ? a.take<int64_t>(M * N * K) : 0;
  TRY(ensure(ctx->moe, a.off));
  uint8_t* b = static_cast<uint8_t*>(ctx->moe.p);
  cudaStream_t st = ctx->stream;
  CUDA_TRY(cudaSetDevice(ctx->device));
  CUDA_TRY(cudaMemcpyAsync(b + og, g, gb, cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(b + ox, x, xb, cudaMemcpyHostToDevice, st));
  TRY(run_backward(ctx, wm, reinterpret_cast<const int32_t*>(b + og), N,
                   reinterpret_cast<const int16_t*>(b + ox), K, M, frac_shift,
                   reinterpret_cast<int32_t*>(b + ogx), K, gw ? reinterpret_cast<int64_t*>(b + ogw) : nullptr,
                   st));
  CUDA_TRY(cudaMemcpyAsync(gx, b + ogx, gxb, cudaMemcpyDeviceToHost, st));
  if (gw) CUDA_TRY(cudaMemcpyAsync(gw, b + ogw, gwb, cudaMemcpyDeviceToHost, st));
  return check_device_error(ctx);
}

}  // extern "C"

// ---------------------------------------------------------------------------------
// θ_v artifacts (runtime/src/loader.rs:322-560)

#include "artifact.hpp"

namespace {

using namespace myl_artifact_detail;

int load_weights_manifest(const std::string& dir, myl_artifact* a) {
  std::vector<uint8_t> raw;
  if (!read_file(dir + "/weights_manifest.json", raw))
    return fail(MYL_ERR_IO, "cannot read %s/weights_manifest.json", dir.c_str());
  const std::string text(raw.begin(), raw.end());
  Json root;
  JsonParser parser(text);
  if (!parser.parse(root) || root.kind != Json::OBJ)
    return fail(MYL_ERR_IO, "invalid weights_manifest.json: %s",
                parser.err.empty() ? "not an object" : parser.err.c_str());
  for (const auto& kv : root.obj) {
    const std::string& name = kv.first;
    const Json& e = kv.second;
    const Json *file = e.get("file"), *shape = e.get("shape"), *dtype = e.get("dtype"),
               *hash = e.get("hash"), *orig = e.get("original_name");
    if (e.kind != Json::OBJ || !file || file->kind != Json::STR || !shape || shape->kind != Json::ARR ||
        !dtype || dtype->kind != Json::STR || !hash || hash->kind != Json::STR)
      return fail(MYL_ERR_IO, "%s: manifest entry lacks file/shape/dtype/hash", name.c_str());
    ArtifactTensor t;
    t.key = name;
    t.original_name = (orig && orig->kind == Json::STR) ? orig->str : name;
    t.file = file->str;
    for (const Json& d : shape->arr) {
      int64_t v = 0;
      if (!as_int(&d, v) || v < 0) return fail(MYL_ERR_IO, "%s: bad shape", name.c_str());
      t.shape.push_back(v);
    }
    int64_t numel = 1;
    for (int64_t v : t.shape) numel *= v;
    const Json* sf = e.get("shifts_file");
    const Json* sh = e.get("shifts_hash");
    if (dtype->str == "int16") {
      // int16 only for the LM head and the attention biases (loader.rs:335-350).
      const bool bias = name.size() >= 5 && name.compare(name.size() - 5, 5, "_bias") == 0;
      if (name != "lm_head" && !bias)
        return fail(MYL_ERR_CORRUPT, "%s: int16 is allowed for the LM head and attention biases only",
                    name.c_str());
      if (!sf || sf->kind != Json::STR)
        return fail(MYL_ERR_CORRUPT, "%s: int16 entry without shifts_file", name.c_str());
      if ((!bias && t.shape.size() != 2) || (bias && t.shape.size() != 1))
        return fail(MYL_ERR_CORRUPT, "%s: %s expects a %s shape", name.c_str(),
                    bias ? "bias" : "LM head", bias ? "one-dimensional" : "[vocab, hidden]");
      t.dtype = 2;
    } else if (dtype->str == "int8") {
      if (t.shape.empty()) return fail(MYL_ERR_CORRUPT, "%s: empty shape in the manifest", name.c_str());
      t.dtype = 1;
    } else {
      return fail(MYL_ERR_CORRUPT, "%s: unsupported dtype '%s' (int8 or int16)", name.c_str(),
                  dtype->str.c_str());
    }
    if (!read_file(dir + "/" + t.file, t.bytes))
      return fail(MYL_ERR_IO, "cannot read %s", t.file.c_str());
    const int64_t want = numel * t.dtype;
    if (int64_t(t.bytes.size()) != want)
      return fail(MYL_ERR_CORRUPT, "%s: %zu bytes in '%s', shape expects %lld bytes", name.c_str(),
                  t.bytes.size(), t.file.c_str(), (long long)want);
    const std::string digest = sha256_hex(t.bytes);
    if (digest != hash->str)
      return fail(MYL_ERR_CORRUPT, "%s: SHA-256 %s does not match the manifest hash %s", name.c_str(),
                  digest.c_str(), hash->str.c_str());
    const int64_t rows = t.shape[0];
    if (sf && sf->kind == Json::STR) {
      if (!read_file(dir + "/" + sf->str, t.shifts))
        return fail(MYL_ERR_IO, "cannot read %s", sf->str.c_str());
      if (int64_t(t.shifts.size()) != rows)
        return fail(MYL_ERR_CORRUPT, "%s: %zu shifts in '%s', %lld rows expected", name.c_str(),
                    t.shifts.size(), sf->str.c_str(), (long long)rows);
      if (sh && sh->kind == Json::STR && sha256_hex(t.shifts) != sh->str)
        return fail(MYL_ERR_CORRUPT, "%s: SHA-256 of the shifts file does not match the manifest",
                    name.c_str());
    } else {
      // Older artifacts: one uniform shift for every row (loader.rs:452-462).
      int64_t shift = 0;
      if (!as_int(e.get("shift"), shift) || shift < 0 || shift > 255)
        return fail(MYL_ERR_CORRUPT, "%s: shift outside 0..=255 and no shifts_file", name.c_str());
      t.shifts.assign(size_t(rows), uint8_t(shift));
    }
    a->tensors.push_back(std::move(t));
  }
  return MYL_OK;
}

int load_luts_manifest(const std::string& dir, myl_artifact* a) {
  std::vector<uint8_t> raw;
  if (!read_file(dir + "/luts.json", raw)) return MYL_OK;  // an artifact without tables
  const std::string text(raw.begin(), raw.end());
  Json root;
  JsonParser parser(text);
  if (!parser.parse(root) || root.kind != Json::OBJ)
    return fail(MYL_ERR_IO, "invalid luts.json: %s", parser.err.empty() ? "not an object" : parser.err.c_str());
  for (const auto& kv : root.obj) {
    const std::string& name = kv.first;
    const Json& e = kv.second;
    const Json *file = e.get("file"), *dtype = e.get("dtype"), *hash = e.get("hash");
    int64_t length = 0;
    if (e.kind != Json::OBJ || !file || file->kind != Json::STR || !dtype || dtype->kind != Json::STR ||
        !hash || hash->kind != Json::STR || !as_int(e.get("length"), length) || length < 0)
      return fail(MYL_ERR_IO, "%s: luts.json entry lacks file/hash/length/dtype", name.c_str());
    if (dtype->str != "int16")
      return fail(MYL_ERR_CORRUPT, "%s: unsupported dtype '%s' (int16 expected)", name.c_str(),
                  dtype->str.c_str());
    std::vector<uint8_t> bytes;
    if (!read_file(dir + "/" + file->str, bytes)) return fail(MYL_ERR_IO, "cannot read %s", file->str.c_str());
    if (int64_t(bytes.size()) != 2 * length)
      return fail(MYL_ERR_CORRUPT, "%s: %zu bytes in '%s', length %lld expects %lld bytes", name.c_str(),
                  bytes.size(), file->str.c_str(), (long long)length, (long long)(2 * length));
    if (sha256_hex(bytes) != hash->str)
      return fail(MYL_ERR_CORRUPT, "%s: SHA-256 does not match the manifest hash", name.c_str());
    std::vector<int16_t> table(static_cast<size_t>(length));
    for (int64_t i = 0; i < length; ++i)
      table[size_t(i)] = int16_t(uint16_t(bytes[size_t(2 * i)]) | (uint16_t(bytes[size_t(2 * i + 1)]) << 8));
    a->luts[name] = std::move(table);
  }
  return MYL_OK;
}

}  // namespace

extern "C" {

int myl_sha256(const void* data, size_t len, uint8_t* out) {
  if ((!data && len) || !out) return fail(MYL_ERR_ARG, "null argument");
  sha256(static_cast<const uint8_t*>(data), len, out);
  return MYL_OK;
}

int myl_artifact_open(const char* dir, myl_artifact** out) {
  if (!dir || !out) return fail(MYL_ERR_ARG, "null argument");
  *out = nullptr;
  myl_artifact* a = new myl_artifact();
  int rc = load_weights_manifest(dir, a);
  if (rc == MYL_OK) rc = load_luts_manifest(dir, a);
  if (rc != MYL_OK) {
    delete a;
    return rc;
  }
  *out = a;
  return MYL_OK;
}

int myl_artifact_close(myl_artifact* a) {
  delete a;
  return MYL_OK;
}

int64_t myl_artifact_count(const myl_artifact* a) { return a ? int64_t(a->tensors.size()) : -1; }

int myl_artifact_find(const myl_artifact* a, const char* name, int64_t* index) {
  if (!a || !name || !index) return fail(MYL_ERR_ARG, "null argument");
  // Manifest keys are original names with '.' replaced by '_' (loader.rs:167-170).
  std::string key(name);
  for (char& c : key)
    if (c == '.') c = '_';
  for (size_t i = 0; i < a->tensors.size(); ++i)
    if (a->tensors[i].key == name || a->tensors[i].key == key || a->tensors[i].original_name == name) {
      *index = int64_t(i);
      return MYL_OK;
    }
  return fail(MYL_ERR_ARG, "no tensor '%s' in the artifact", name);
}

int myl_artifact_tensor(const myl_artifact* a, int64_t index, const char** key,
                        const char** original_name, int* dtype, int* ndim, int64_t* shape,
                        const void** data, const uint8_t** shifts) {
  if (!a || index < 0 || index >= int64_t(a->tensors.size())) return fail(MYL_ERR_ARG, "bad tensor index");
  const ArtifactTensor& t = a->tensors[size_t(index)];
  if (key) *key = t.key.c_str();
  if (original_name) *original_name = t.original_name.c_str();
  if (dtype) *dtype = t.dtype;
  if (ndim) *ndim = int(t.shape.size());
  if (shape)
    for (size_t i = 0; i < t.shape.size() && i < 4; ++i) shape[i] = t.shape[i];
  if (data) *data = t.bytes.data();
  if (shifts) *shifts = t.shifts.data();
  return MYL_OK;
}

int myl_artifact_register(myl_ctx* ctx, const myl_artifact* a, int64_t index, myl_weight** out) {
  if (!ctx || !a || !out || index < 0 || index >= int64_t(a->tensors.size()))
    return fail(MYL_ERR_ARG, "bad argument");
  const ArtifactTensor& t = a->tensors[size_t(index)];
  if (t.shape.size() != 2)
    return fail(MYL_ERR_SHAPE, "%s: only 2-D tensors are registered as weights", t.key.c_str());
  const int64_t N = t.shape[0], K = t.shape[1];
  if (t.dtype == 2) {
    std::vector<int16_t> w(static_cast<size_t>(N * K));
    for (size_t i = 0; i < w.size(); ++i)
      w[i] = int16_t(uint16_t(t.bytes[2 * i]) | (uint16_t(t.bytes[2 * i + 1]) << 8));
    return myl_weight16_register(ctx, w.data(), N, K, K, t.shifts.data(), out);
  }
  return myl_weight_register(ctx, reinterpret_cast<const int8_t*>(t.bytes.data()), N, K, K,
                             t.shifts.data(), out);
}

int myl_artifact_lut(const myl_artifact* a, const char* name, const int16_t** data, int64_t* len) {
  if (!a || !name || !data || !len) return fail(MYL_ERR_ARG, "null argument");
  auto it = a->luts.find(name);
  if (it == a->luts.end()) return fail(MYL_ERR_ARG, "no table '%s' in luts.json", name);
  *data = it->second.data();
  *len = int64_t(it->second.size());
  return MYL_OK;
}

}  // extern "C"

// ---- pipeline wire format (codec.rs) ------------------------------------------
namespace {

const CrcTables& crc_tables() {
  static const CrcTables t = [] {
    CrcTables v;
    crc_tables_host(&v);
    return v;
  }();
  return t;
}

bool host_little_endian() {
  const uint16_t one = 1;
  uint8_t b;
  std::memcpy(&b, &one, 1);
  return b == 1;
}

// decode_message's checks up to the payload bounds (codec.rs:113-157).
int wire_header(const uint8_t* buf, uint64_t len, myl_wire_meta* m) {
  if (len < WIRE_HEADER)
    return fail(MYL_ERR_CORRUPT, "buffer too small: %llu < %llu", (unsigned long long)len,
                (unsigned long long)WIRE_HEADER);
  if (std::memcmp(buf, "IINTPIPE", 8) != 0) return fail(MYL_ERR_CORRUPT, "bad magic");
  uint64_t f[9];
  for (int i = 0; i < 9; ++i) f[i] = wire_get_u64(buf + 8 + 8 * i);
  m->version = f[0];
  m->theta_v_hash = f[1];
  m->request_id = f[2];
  m->sequence_id = f[3];
  m->stage_id = f[4];
  m->token_position = f[5];
  m->payload_len = f[6];
  m->flags = f[7];
  m->reserved = f[8];
  m->crc = uint32_t(buf[80]) | (uint32_t(buf[81]) << 8) | (uint32_t(buf[82]) << 16) |
           (uint32_t(buf[83]) << 24);
  if (m->payload_len > len - WIRE_HEADER)  // also catches offsets that would overflow
    return fail(MYL_ERR_CORRUPT, "payload of %llu bytes runs past the buffer (%llu bytes)",
                (unsigned long long)m->payload_len, (unsigned long long)len);
  return MYL_OK;
}

void wire_write_header(const myl_wire_meta* meta, uint64_t payload_len, uint32_t crc, uint8_t* out) {
  std::memcpy(out, "IINTPIPE", 8);
  const uint64_t f[9] = {meta->version, meta->theta_v_hash, meta->request_id, meta->sequence_id,
                         meta->stage_id, meta->token_position, payload_len, meta->flags,
                         meta->reserved};
  for (int i = 0; i < 9; ++i) wire_put_u64(out + 8 + 8 * i, f[i]);
  for (int i = 0; i < 4; ++i) out[80 + i] = uint8_t(crc >> (8 * i));
}

void wire_values_to_bytes(const int16_t* v, uint64_t n, uint8_t* out) {
  if (host_little_endian()) {
    std::memcpy(out, v, size_t(n) * 2);
    return;
  }
  for (uint64_t i = 0; i < n; ++i) {
    out[2 * i] = uint8_t(uint16_t(v[i]) & 0xFF);
    out[2 * i + 1] = uint8_t(uint16_t(v[i]) >> 8);
  }
}

void wire_bytes_to_values(const uint8_t* p, uint64_t n, int16_t* v) {
  if (host_little_endian()) {
    std::memcpy(v, p, size_t(n) * 2);
    return;
  }
  for (uint64_t i = 0; i < n; ++i) v[i] = int16_t(uint16_t(p[2 * i]) | (uint16_t(p[2 * i + 1]) << 8));
}

// CRC-32 of len device bytes (enqueued on st; synchronises st).
int crc32_device(myl_ctx* ctx, const uint8_t* data, uint64_t len, cudaStream_t st, uint32_t* out) {
  if (len == 0) {
    *out = 0;
    return MYL_OK;
  }
  TRY(ensure(ctx->crc, 4));
  uint32_t* acc = static_cast<uint32_t*>(ctx->crc.p);
  CUDA_TRY(cudaMemsetAsync(acc, 0, 4, st));
  const uint64_t pad = (uint64_t(CRC_BLOCK) - len % uint64_t(CRC_BLOCK)) % uint64_t(CRC_BLOCK);
  const uint64_t nblocks = (len + pad) / uint64_t(CRC_BLOCK);
  const unsigned grid = unsigned(std::min<uint64_t>(nblocks, uint64_t(ctx->num_sms) * 8));
  crc32_blocks_kernel<<<grid, CRC_THREADS, 0, st>>>(data, len, pad, nblocks, crc_tables(), acc);
  CUDA_TRY(cudaGetLastError());
  ctx->launches++;
  uint32_t raw = 0;
  CUDA_TRY(cudaMemcpyAsync(&raw, acc, 4, cudaMemcpyDeviceToHost, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  *out = raw ^ gf2_mulmod(0xFFFFFFFFu, gf2_x8n(len)) ^ 0xFFFFFFFFu;
  return MYL_OK;
}

}  // namespace

extern "C" {

uint64_t myl_wire_frame_bytes(uint64_t n_values) { return wire_frame_bytes(n_values); }

uint32_t myl_crc32(const void* data, uint64_t len) {
  if (!data) return 0u;
  return crc32_host(static_cast<const uint8_t*>(data), len);
}

int myl_wire_encode(const myl_wire_meta* meta, const int16_t* values, uint64_t n, uint8_t* out,
                    uint64_t cap, uint64_t* out_len) {
  if (!meta || (n && !values) || !out_len) return fail(MYL_ERR_ARG, "null argument");
  if (n > (uint64_t(1) << 60)) return fail(MYL_ERR_SHAPE, "payload too large");
  const uint64_t need = wire_frame_bytes(n);
  *out_len = need;
  if (cap < need || !out)
    return fail(MYL_ERR_SHAPE, "frame needs %llu bytes, buffer holds %llu",
                (unsigned long long)need, (unsigned long long)cap);
  wire_values_to_bytes(values, n, out + WIRE_HEADER);
  const uint32_t crc = crc32_host(out + WIRE_HEADER, 2 * n);
  wire_write_header(meta, 2 * n, crc, out);
  std::memset(out + WIRE_HEADER + 2 * n, 0, size_t(need - WIRE_HEADER - 2 * n));
  return MYL_OK;
}

int myl_wire_decode(const uint8_t* buf, uint64_t len, myl_wire_meta* meta, int16_t* values,
                    uint64_t cap, uint64_t* n) {
  if ((!buf && len) || !meta || !n) return fail(MYL_ERR_ARG, "null argument");
  myl_wire_meta m{};
  TRY(wire_header(buf, len, &m));
  const uint8_t* payload = buf + WIRE_HEADER;
  const uint32_t crc = crc32_host(payload, m.payload_len);
  if (crc != m.crc)
    return fail(MYL_ERR_CORRUPT, "CRC mismatch: %08x != %08x", unsigned(m.crc), unsigned(crc));
  if (m.payload_len % 2) return fail(MYL_ERR_CORRUPT, "odd payload length %llu",
                                     (unsigned long long)m.payload_len);
  *meta = m;
  *n = m.payload_len / 2;
  if (!values && cap == 0) return MYL_OK;
  if (!values || cap < *n)
    return fail(MYL_ERR_SHAPE, "payload has %llu values, buffer holds %llu",
                (unsigned long long)*n, (unsigned long long)cap);
  wire_bytes_to_values(payload, *n, values);
  return MYL_OK;
}

int myl_crc32_dev(myl_ctx* ctx, const void* data, uint64_t len, uint32_t* crc, void* stream) {
  if (!ctx || (len && !data) || !crc) return fail(MYL_ERR_ARG, "null argument");
  CUDA_TRY(cudaSetDevice(ctx->device));
  return crc32_device(ctx, static_cast<const uint8_t*>(data), len,
                      static_cast<cudaStream_t>(stream), crc);
}

int myl_wire_decode_dev(myl_ctx* ctx, const uint8_t* buf, uint64_t len, myl_wire_meta* meta,
                        int16_t* dev_values, uint64_t cap, uint64_t* n, void* stream) {
  if (!ctx || (!buf && len) || !meta || !n) return fail(MYL_ERR_ARG, "null argument");
  if (!host_little_endian()) return fail(MYL_ERR_UNSUPPORTED, "big-endian host");
  myl_wire_meta m{};
  TRY(wire_header(buf, len, &m));
  const uint64_t nv = (m.payload_len + 1) / 2;
  if (nv > cap || (nv && !dev_values))
    return fail(MYL_ERR_SHAPE, "payload has %llu values, buffer holds %llu",
                (unsigned long long)nv, (unsigned long long)cap);
  CUDA_TRY(cudaSetDevice(ctx->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (m.payload_len)
    CUDA_TRY(cudaMemcpyAsync(dev_values, buf + WIRE_HEADER, size_t(m.payload_len),
                             cudaMemcpyHostToDevice, st));
  uint32_t crc = 0;
  TRY(crc32_device(ctx, reinterpret_cast<const uint8_t*>(dev_values), m.payload_len, st, &crc));
  if (crc != m.crc)
    return fail(MYL_ERR_CORRUPT, "CRC mismatch: %08x != %08x", unsigned(m.crc), unsigned(crc));
  if (m.payload_len % 2) return fail(MYL_ERR_CORRUPT, "odd payload length %llu",
                                     (unsigned long long)m.payload_len);
  *meta = m;
  *n = m.payload_len / 2;
  return MYL_OK;
}

int myl_wire_encode_dev(myl_ctx* ctx, const myl_wire_meta* meta, const int16_t* dev_values,
                        uint64_t n, uint8_t* out, uint64_t cap, uint64_t* out_len, void* stream) {
  if (!ctx || !meta || (n && !dev_values) || !out_len) return fail(MYL_ERR_ARG, "null argument");
  if (!host_little_endian()) return fail(MYL_ERR_UNSUPPORTED, "big-endian host");
  if (n > (uint64_t(1) << 60)) return fail(MYL_ERR_SHAPE, "payload too large");
  const uint64_t need = wire_frame_bytes(n);
  *out_len = need;
  if (cap < need || !out)
    return fail(MYL_ERR_SHAPE, "frame needs %llu bytes, buffer holds %llu",
                (unsigned long long)need, (unsigned long long)cap);
  CUDA_TRY(cudaSetDevice(ctx->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n)
    CUDA_TRY(cudaMemcpyAsync(out + WIRE_HEADER, dev_values, size_t(2 * n), cudaMemcpyDeviceToHost, st));
  uint32_t crc = 0;
  TRY(crc32_device(ctx, reinterpret_cast<const uint8_t*>(dev_values), 2 * n, st, &crc));
  wire_write_header(meta, 2 * n, crc, out);
  std::memset(out + WIRE_HEADER + 2 * n, 0, size_t(need - WIRE_HEADER - 2 * n));
  return MYL_OK;
}

int myl_wire_pack_tokens(const uint32_t* tokens, uint64_t n, int16_t* out) {
  if ((n && (!tokens || !out))) return fail(MYL_ERR_ARG, "null argument");
  for (uint64_t i = 0; i < n; ++i) {
    out[2 * i] = int16_t(uint16_t(tokens[i] & 0xFFFFu));
    out[2 * i + 1] = int16_t(uint16_t(tokens[i] >> 16));
  }
  return MYL_OK;
}

int myl_wire_unpack_tokens(const int16_t* values, uint64_t n_values, uint32_t* tokens) {
  if (n_values % 2) return fail(MYL_ERR_SHAPE, "token payload needs an even number of int16");
  if (n_values && (!values || !tokens)) return fail(MYL_ERR_ARG, "null argument");
  for (uint64_t i = 0; i < n_values / 2; ++i)
    tokens[i] = uint32_t(uint16_t(values[2 * i])) | (uint32_t(uint16_t(values[2 * i + 1])) << 16);
  return MYL_OK;
}

}  // extern "C"

#include "model.cuh"
