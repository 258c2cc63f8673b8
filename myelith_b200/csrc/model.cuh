// model.cuh — host driver of the integer decoder forward (myl_model_*,
// myl_session_*, myl_forward, myl_generate), included by myl_w8a16.cu after
// the linear, MLP and artifact code it composes.
//
// One layer of forward_layer (runtime/src/model.rs:401-674) is, per call of
// B sequences x T tokens (rows r = b * T + t):
//   [residual add of the previous layer's MLP +] input RMSNorm   resid_rmsnorm_kernel
//   q/k/v: one W8A16 GEMV/GEMM over the rows [wq; wk; wv] with the
//          per-segment out_frac and the rescaled int16 biases fused  run_linear
//   RoPE of q and k, k and v into the cache                        rope_kv_kernel
//          (decode: inside attn_scores_kernel)
//   scores, softmax_int + probability-weighted values + rescale     attn_scores/pv_kernel
//   o_proj onto min(residual_in, residual_mid) per channel          run_linear
//   residual add + post-attention RMSNorm                          resid_rmsnorm_kernel
//   mlp_int onto min(residual_mid, next residual_in)                run_mlp
// then the last residual add + final RMSNorm of each sequence's last token,
// the LM head (i32 logits) and, when generating, the greedy selection.
//
// Host validation restates every debug-build panic of the reference on these
// shifts (u8 additions, i8 differences, shift widths); invalid models fail in
// myl_model_create with MYL_ERR_OVERFLOW, bad shapes with MYL_ERR_SHAPE.

#include "forward.cuh"

namespace {

struct NormDev {
  uint8_t* align2 = nullptr;
  int8_t* gamma = nullptr;
  int16_t* sbase = nullptr;
  int32_t frac0 = 0;
  int64_t inv_n = 0;
};

struct ResidDev {
  int8_t* s1 = nullptr;
  int8_t* s2 = nullptr;
};

struct ModelLayer {
  myl_weight* w_qkv = nullptr;
  myl_requant* rq_qkv = nullptr;
  myl_weight* w_o = nullptr;
  myl_requant* rq_o = nullptr;
  myl_mlp* mlp = nullptr;
  NormDev norm1, norm2;
  ResidDev add_attn;  // hidden (residual_in) + o  ->  mid (residual_mid)
  ResidDev add_mlp;   // mid (residual_mid) + mlp  ->  next residual_in
  int score_shift = 0, out_shift = 0;
};

}  // namespace

struct myl_model {
  // V, nq, nkv, I (and QD, KD) are this rank's shares under tensor parallelism
  int64_t V = 0, H = 0, L = 0, nq = 0, nkv = 0, hd = 0, I = 0, QD = 0, KD = 0, ldq = 0;
  int world = 1, rank = 0;
  // global index of this rank's first query head, KV head, intermediate
  // channel and vocabulary row; global query heads per KV head
  int64_t q0 = 0, kv0 = 0, i0 = 0, v0 = 0, G = 1;
  int64_t V_global = 0;
  uint8_t final_norm_frac = 0, logit_frac = 0, prob_frac = 0, rope_frac = 0;
  int8_t* d_embed = nullptr;  // own table when the LM head is not the embedding
  const int8_t* embed_rows = nullptr;
  int64_t lde = 0;
  uint8_t* d_embed_shifts = nullptr;
  uint8_t* d_rin0 = nullptr;
  myl_weight* head = nullptr;
  myl_requant* rq_head = nullptr;
  std::vector<ModelLayer> layers;
  NormDev final_norm;
  int16_t *d_cos = nullptr, *d_sin = nullptr, *d_exp = nullptr, *d_rsqrt = nullptr;
  int64_t n_pos = 0, exp_len = 0, rsqrt_len = 0;
  int32_t exp_max = 0;
  int64_t score_mult = 0;
  int lut_shift = 0;
  std::vector<void*> allocs;
};

struct myl_session {
  const myl_model* m = nullptr;
  int64_t B = 0, max_pos = 0, rows_cap = 0, part_rows = 0;
  int16_t *kc = nullptr, *vc = nullptr;
  KvCache cache{};
  int64_t* d_pos = nullptr;   // position of the next token (device)
  int64_t* d_step = nullptr;  // decode step counter (device)
  int64_t* h_pos = nullptr;   // pinned staging
  int64_t pos = 0;            // host mirror of d_pos
  int16_t *hid = nullptr, *mid = nullptr, *xn = nullptr, *qkv = nullptr, *attn = nullptr,
          *o = nullptr, *mlp_out = nullptr, *xf = nullptr;
  int32_t* scores = nullptr;
  int64_t* part = nullptr;
  unsigned* counters = nullptr;
  unsigned* rowmax = nullptr;  // [rows_cap * nq] attention row maxima, zero between calls
  int max_chunks = 0;
  int32_t* logits = nullptr;
  int64_t* keys = nullptr;
  int32_t* tok_in = nullptr;
  int32_t* next_tok = nullptr;
  int64_t* last_rows = nullptr;
  int64_t last_rows_T = -1;
  int32_t* out_tokens = nullptr;  // [B][max_pos]
  int32_t* h_tokens = nullptr;    // pinned [B * rows_cap]
  int32_t* h_logits = nullptr;    // pinned [B][V]
  cudaGraphExec_t graph = nullptr;
  uint64_t graph_epoch = 0;
  // device time of the last prefill (myl_forward) and decode loop, CUDA
  // events on the launching stream
  cudaEvent_t ev[4] = {};
  float prefill_ms = 0.f, decode_ms = 0.f;
  // tensor parallelism: one peer-memory region per rank (myl_session_set_tp)
  // holding two receive regions [world][rows_cap][H] int64 (o_proj and down
  // projection partials), key slots [world][B] int64 and flag words [world].
  bool tp_ready = false;
  int64_t* recv[2] = {nullptr, nullptr};
  void* peer_recv[2][MYL_XCHG_MAX] = {};
  int64_t* key_slots = nullptr;
  TpPeers peers{};
  unsigned long long* d_epoch = nullptr;
  std::vector<void*> allocs;
};

namespace {

template <typename T>
int dev_alloc(std::vector<void*>& list, T** p, size_t count) {
  void* q = nullptr;
  if (cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess)
    return fail(MYL_ERR_CUDA, "cudaMalloc of %zu bytes failed", count * sizeof(T));
  list.push_back(q);
  *p = static_cast<T*>(q);
  return MYL_OK;
}

template <typename T>
int dev_upload(std::vector<void*>& list, T** p, const T* host, size_t count) {
  TRY(dev_alloc(list, p, count));
  if (count) CUDA_TRY(cudaMemcpy(*p, host, count * sizeof(T), cudaMemcpyHostToDevice));
  return MYL_OK;
}

// i8 difference and width checks of rescale (width 32) / rescale_i64 (64),
// fixed_point.rs:173-191: the signed shift in_frac - out_frac.
int rescale_shift(uint8_t in_frac, uint8_t out_frac, int width, int* s, const char* what) {
  const int d = int(int8_t(in_frac)) - int(int8_t(out_frac));
  if (d < -128 || d > 127 || (d >= 0 && d > width - 2) || (d < 0 && -d > width - 1))
    return fail(MYL_ERR_OVERFLOW, "%s: rescale from frac %u to %u overflows", what, unsigned(in_frac),
                unsigned(out_frac));
  *s = d;
  return MYL_OK;
}

// rmsnorm_i16 parameters of one norm (rmsnorm.rs:61-153), see NormParams.
int make_norm(myl_model* m, const uint8_t* x_shifts, const int8_t* gamma, const uint8_t* gamma_shifts,
              uint8_t lut_input_shift, uint8_t lut_output_frac, uint8_t out_frac, NormDev* nd) {
  const int64_t H = m->H;
  if (lut_input_shift & 1) return fail(MYL_ERR_SHAPE, "rmsnorm: lut_input_shift must be even");
  uint8_t ref = 0;
  for (int64_t i = 0; i < H; ++i) ref = std::max(ref, x_shifts[i]);
  std::vector<uint8_t> align2(static_cast<size_t>(H));
  std::vector<int16_t> sbase(static_cast<size_t>(H));
  const int frac0 = int(lut_output_frac) + int(lut_input_shift) / 2;
  for (int64_t i = 0; i < H; ++i) {
    const int a = 2 * (int(ref) - int(x_shifts[i]));
    // sum_i r_i^2 << a stays inside i128, and so does its product with inv_n
    if (a > 76) return fail(MYL_ERR_OVERFLOW, "rmsnorm: channel shift span %d too wide", a / 2);
    align2[size_t(i)] = uint8_t(a);
    const int sb = int(gamma_shifts[i]) + (int(x_shifts[i]) - int(ref)) - int(out_frac);
    // the smallest shift (q = 0) must stay a valid i128 left shift
    if (frac0 + sb < -127) return fail(MYL_ERR_OVERFLOW, "rmsnorm: left shift beyond i128");
    sbase[size_t(i)] = int16_t(sb);
  }
  TRY(dev_upload(m->allocs, &nd->align2, align2.data(), size_t(H)));
  TRY(dev_upload(m->allocs, &nd->gamma, gamma, size_t(H)));
  TRY(dev_upload(m->allocs, &nd->sbase, sbase.data(), size_t(H)));
  nd->frac0 = frac0;
  nd->inv_n = ((int64_t(1) << 20) + H / 2) / H;  // rmsnorm.rs:20-24
  return MYL_OK;
}

// Residual add: seg_in + add (on acc = min(seg_in, seg_out)) -> seg_out.
int make_resid(myl_model* m, const uint8_t* seg_in, const uint8_t* seg_out, ResidDev* rd,
               std::vector<uint8_t>* acc_out) {
  const int64_t H = m->H;
  std::vector<int8_t> s1(static_cast<size_t>(H)), s2(static_cast<size_t>(H));
  acc_out->resize(size_t(H));
  for (int64_t i = 0; i < H; ++i) {
    const uint8_t acc = std::min(seg_in[i], seg_out[i]);
    (*acc_out)[size_t(i)] = acc;
    int a = 0, b = 0;
    TRY(rescale_shift(seg_in[i], acc, 64, &a, "residual add"));
    TRY(rescale_shift(acc, seg_out[i], 64, &b, "residual add"));
    s1[size_t(i)] = int8_t(a);
    s2[size_t(i)] = int8_t(b);
  }
  TRY(dev_upload(m->allocs, &rd->s1, s1.data(), size_t(H)));
  TRY(dev_upload(m->allocs, &rd->s2, s2.data(), size_t(H)));
  return MYL_OK;
}

NormParams norm_params(const myl_model* m, const NormDev& nd) {
  NormParams np{};
  np.align2 = nd.align2;
  np.gamma = nd.gamma;
  np.sbase = nd.sbase;
  np.lut = m->d_rsqrt;
  np.lut_len = int32_t(m->rsqrt_len);
  np.frac0 = nd.frac0;
  np.inv_n = nd.inv_n;
  np.H = m->H;
  return np;
}

void release_model(myl_ctx* ctx, myl_model* m) {
  for (auto& L : m->layers) {
    myl_weight_release(ctx, L.w_qkv);
    myl_requant_release(ctx, L.rq_qkv);
    myl_weight_release(ctx, L.w_o);
    myl_requant_release(ctx, L.rq_o);
    myl_mlp_release(ctx, L.mlp);
  }
  myl_weight_release(ctx, m->head);
  myl_requant_release(ctx, m->rq_head);
  for (void* p : m->allocs) cudaFree(p);
  delete m;
}

int build_layer(myl_ctx* ctx, myl_model* m, const myl_model_spec* sp, int64_t l) {
  const myl_layer_spec& ls = sp->layers[l];
  ModelLayer& L = m->layers[size_t(l)];
  const int64_t H = m->H, QD = m->QD, KD = m->KD, I = m->I, hd = m->hd;
  // this rank's rows of q/k/v, columns of o_proj, channels of the MLP
  const int64_t qr0 = m->q0 * hd, kr0 = m->kv0 * hd, QDg = sp->num_heads * hd,
                Ig = sp->intermediate;
  const uint8_t* out_res = l + 1 < m->L ? sp->layers[l + 1].residual_in_frac : sp->final_residual_frac;
  if (!ls.ln1_gamma || !ls.ln1_gamma_shifts || !ls.ln2_gamma || !ls.ln2_gamma_shifts || !ls.wq ||
      !ls.wk || !ls.wv || !ls.wo || !ls.wg || !ls.wu || !ls.wd || !ls.sq || !ls.sk || !ls.sv ||
      !ls.so || !ls.sg || !ls.su || !ls.sd || !ls.residual_in_frac || !ls.residual_mid_frac ||
      !out_res)
    return fail(MYL_ERR_ARG, "layer %lld: null tensor", (long long)l);
  const bool bias = ls.bq || ls.bk || ls.bv;
  if (bias && (!ls.bq || !ls.bk || !ls.bv || !ls.bq_shifts || !ls.bk_shifts || !ls.bv_shifts))
    return fail(MYL_ERR_ARG, "layer %lld: q/k/v biases come together", (long long)l);
  // q/k/v as one weight [wq; wk; wv] with per-segment out_frac (model.rs:438-440)
  const int64_t NQKV = QD + 2 * KD;
  std::vector<int8_t> w(size_t(NQKV) * size_t(H));
  std::vector<uint8_t> ws(static_cast<size_t>(NQKV)), of(static_cast<size_t>(NQKV));
  std::memcpy(w.data(), ls.wq + qr0 * H, size_t(QD * H));
  std::memcpy(w.data() + QD * H, ls.wk + kr0 * H, size_t(KD * H));
  std::memcpy(w.data() + (QD + KD) * H, ls.wv + kr0 * H, size_t(KD * H));
  std::memcpy(ws.data(), ls.sq + qr0, size_t(QD));
  std::memcpy(ws.data() + QD, ls.sk + kr0, size_t(KD));
  std::memcpy(ws.data() + QD + KD, ls.sv + kr0, size_t(KD));
  std::fill(of.begin(), of.begin() + QD, ls.q_frac);
  std::fill(of.begin() + QD, of.begin() + QD + KD, ls.k_frac);
  std::fill(of.begin() + QD + KD, of.end(), ls.v_frac);
  TRY(myl_weight_register(ctx, w.data(), NQKV, H, H, ws.data(), &L.w_qkv));
  TRY(myl_requant_create(ctx, L.w_qkv, MYL_RQ_SHIFT_I16, ls.norm_attn_frac, of.data(), 1, nullptr,
                         nullptr, &L.rq_qkv));
  if (bias) {
    // add_bias_i16 (linear.rs:132-145) per segment, rescaled to its out_frac
    std::vector<int32_t> b(static_cast<size_t>(NQKV)), seg;
    TRY(rescale_bias(ls.bq + qr0, ls.bq_shifts + qr0, QD, ls.q_frac, seg));
    std::copy(seg.begin(), seg.end(), b.begin());
    TRY(rescale_bias(ls.bk + kr0, ls.bk_shifts + kr0, KD, ls.k_frac, seg));
    std::copy(seg.begin(), seg.end(), b.begin() + QD);
    TRY(rescale_bias(ls.bv + kr0, ls.bv_shifts + kr0, KD, ls.v_frac, seg));
    std::copy(seg.begin(), seg.end(), b.begin() + QD + KD);
    CUDA_TRY(cudaMalloc(&L.rq_qkv->d_bias, size_t(NQKV) * 4));
    CUDA_TRY(cudaMemcpy(L.rq_qkv->d_bias, b.data(), size_t(NQKV) * 4, cudaMemcpyHostToDevice));
  }
  // attention scaling (model.rs:543-546)
  const unsigned ss = unsigned(ls.q_frac) + unsigned(ls.k_frac) + 15u;
  const unsigned score_shift = ss > sp->score_frac_bits ? ss - sp->score_frac_bits : 0u;
  L.score_shift = int(uint8_t(score_shift));  // `as u8`
  if (L.score_shift > 62) return fail(MYL_ERR_OVERFLOW, "score shift %d", L.score_shift);
  TRY(rescale_shift(ls.v_frac, ls.attn_out_frac, 32, &L.out_shift, "attention output"));
  // o_proj onto min(residual_in, residual_mid) (model.rs:576-582)
  std::vector<uint8_t> acc_attn, acc_mlp;
  TRY(make_resid(m, ls.residual_in_frac, ls.residual_mid_frac, &L.add_attn, &acc_attn));
  TRY(make_resid(m, ls.residual_mid_frac, out_res, &L.add_mlp, &acc_mlp));
  TRY(myl_weight_register(ctx, ls.wo + qr0, H, QD, QDg, ls.so, &L.w_o));
  TRY(myl_requant_create(ctx, L.w_o, MYL_RQ_SHIFT_I16, ls.attn_out_frac, acc_attn.data(), 1, nullptr,
                         nullptr, &L.rq_o));
  // the down projection's columns of this rank's channels, contiguous
  std::vector<int8_t> wd_local;
  const int8_t* wd = ls.wd;
  if (I != Ig) {
    wd_local.resize(size_t(H) * size_t(I));
    for (int64_t r = 0; r < H; ++r)
      std::memcpy(wd_local.data() + r * I, ls.wd + r * Ig + m->i0, size_t(I));
    wd = wd_local.data();
  }
  TRY(myl_mlp_register(ctx, ls.wg + m->i0 * H, ls.wu + m->i0 * H, wd, H, I, ls.sg + m->i0,
                       ls.su + m->i0, ls.sd, sp->silu_lut, sp->silu_len, ls.norm_mlp_frac,
                       ls.gate_frac, ls.up_frac, ls.down_in_frac, sp->silu_in_frac,
                       sp->silu_lut_offset, sp->silu_out_frac, acc_mlp.data(), &L.mlp));
  TRY(make_norm(m, ls.residual_in_frac, ls.ln1_gamma, ls.ln1_gamma_shifts, sp->rsqrt_input_shift,
                sp->rsqrt_output_frac, ls.norm_attn_frac, &L.norm1));
  TRY(make_norm(m, ls.residual_mid_frac, ls.ln2_gamma, ls.ln2_gamma_shifts, sp->rsqrt_input_shift,
                sp->rsqrt_output_frac, ls.norm_mlp_frac, &L.norm2));
  return MYL_OK;
}

int session_alloc(myl_ctx* ctx, myl_session* s) {
  const myl_model* m = s->m;
  auto& A = s->allocs;
  const int64_t B = s->B, R = s->rows_cap, H = m->H;
  s->cache.head_stride = s->max_pos * m->hd;
  s->cache.layer_stride = m->nkv * s->cache.head_stride;
  s->cache.seq_stride = m->L * s->cache.layer_stride;
  const size_t cache_elems = size_t(B) * size_t(s->cache.seq_stride);
  TRY(dev_alloc(A, &s->kc, cache_elems));
  TRY(dev_alloc(A, &s->vc, cache_elems));
  CUDA_TRY(cudaMemset(s->kc, 0, cache_elems * 2));
  CUDA_TRY(cudaMemset(s->vc, 0, cache_elems * 2));
  s->cache.k = s->kc;
  s->cache.v = s->vc;
  TRY(dev_alloc(A, &s->d_pos, 1));
  TRY(dev_alloc(A, &s->d_step, 1));
  TRY(dev_alloc(A, &s->hid, size_t(R * H)));
  TRY(dev_alloc(A, &s->mid, size_t(R * H)));
  TRY(dev_alloc(A, &s->xn, size_t(R * H)));
  TRY(dev_alloc(A, &s->o, size_t(R * H)));
  TRY(dev_alloc(A, &s->mlp_out, size_t(R * H)));
  TRY(dev_alloc(A, &s->qkv, size_t(R * m->ldq)));
  TRY(dev_alloc(A, &s->attn, size_t(R * m->QD)));
  TRY(dev_alloc(A, &s->xf, size_t(B * H)));
  TRY(dev_alloc(A, &s->scores, size_t(R * m->nq) * size_t(s->max_pos)));
  s->max_chunks = int((s->max_pos + ATT_CHUNK - 1) / ATT_CHUNK);
  TRY(dev_alloc(A, &s->part, size_t(s->part_rows * m->nq) * size_t(s->max_chunks) * size_t(m->hd)));
  TRY(dev_alloc(A, &s->counters, size_t(s->part_rows * m->nq)));
  CUDA_TRY(cudaMemset(s->counters, 0, size_t(s->part_rows * m->nq) * sizeof(unsigned)));
  TRY(dev_alloc(A, &s->rowmax, size_t(R * m->nq)));
  CUDA_TRY(cudaMemset(s->rowmax, 0, size_t(R * m->nq) * sizeof(unsigned)));
  TRY(dev_alloc(A, &s->logits, size_t(B * m->V)));
  TRY(dev_alloc(A, &s->keys, size_t(B)));
  TRY(dev_alloc(A, &s->tok_in, size_t(R)));
  TRY(dev_alloc(A, &s->next_tok, size_t(B)));
  TRY(dev_alloc(A, &s->last_rows, size_t(B)));
  TRY(dev_alloc(A, &s->out_tokens, size_t(B * s->max_pos)));
  for (auto& e : s->ev) CUDA_TRY(cudaEventCreate(&e));
  CUDA_TRY(cudaMallocHost(&s->h_pos, sizeof(int64_t)));
  CUDA_TRY(cudaMallocHost(&s->h_tokens, size_t(R) * 4));
  CUDA_TRY(cudaMallocHost(&s->h_logits, size_t(B * m->V) * 4));
  (void)ctx;
  return MYL_OK;
}

void release_session(myl_ctx* ctx, myl_session* s) {
  if (ctx) cudaSetDevice(ctx->device);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  for (auto& e : s->ev)
    if (e) cudaEventDestroy(e);
  for (void* p : s->allocs) cudaFree(p);
  if (s->h_pos) cudaFreeHost(s->h_pos);
  if (s->h_tokens) cudaFreeHost(s->h_tokens);
  if (s->h_logits) cudaFreeHost(s->h_logits);
  delete s;
}

int set_pos(myl_session* s, int64_t pos, cudaStream_t st) {
  // the pinned staging word is only rewritten after the stream has used it
  CUDA_TRY(cudaStreamSynchronize(st));
  *s->h_pos = pos;
  CUDA_TRY(cudaMemcpyAsync(s->d_pos, s->h_pos, sizeof(int64_t), cudaMemcpyHostToDevice, st));
  s->pos = pos;
  return MYL_OK;
}

__global__ void advance_kernel(int64_t* pos, int64_t n) {
  pdl_wait();
  pdl_launch();
  if (threadIdx.x == 0 && blockIdx.x == 0) pos[0] += n;
}

// Attention of one layer over `rows` token rows (T tokens per sequence).
int run_attention(myl_ctx* ctx, const myl_model* m, myl_session* s, const ModelLayer& L, int layer,
                  int64_t rows, int64_t T, int64_t lds_len, cudaStream_t st) {
  AttnParams p{};
  p.qkv = s->qkv;
  p.ldq = m->ldq;
  p.T = T;
  p.rows = rows;
  p.pos0 = s->d_pos;
  p.nq = int(m->nq);
  p.nkv = int(m->nkv);
  p.hd = int(m->hd);
  p.q_head0 = int(m->q0);
  p.kv_head0 = int(m->kv0);
  p.G = int(m->G);
  p.kc = s->cache;
  p.layer = layer;
  p.score_mult = m->score_mult;
  p.score_shift = L.score_shift;
  p.scores = s->scores;
  p.lds = s->max_pos;
  p.mask = nullptr;
  p.exp_lut = m->d_exp;
  p.exp_len = int32_t(m->exp_len);
  p.lut_shift = m->lut_shift;
  p.prob_frac = m->prob_frac;
  p.out_shift = L.out_shift;
  p.part = s->part;
  p.max_chunks = s->max_chunks;
  p.counters = s->counters;
  p.rowmax = s->rowmax;
  p.rope = T == 1;
  p.rope_cos = m->d_cos;
  p.rope_sin = m->d_sin;
  p.n_pos = m->n_pos;
  p.rope_frac = m->rope_frac;
  p.out = s->attn;
  p.ldo = m->QD;
  // few rows (decode): chunks of ATT_DCHUNK keys, so that the keys of a long
  // context spread over many SMs; many rows: one block per row for pass 2
  const bool split = rows <= s->part_rows && rows * m->nq < 4 * int64_t(ctx->num_sms);
  // prefill of enough rows: both passes in 64-row tiles
  const int64_t tile_blocks = (rows / T) * ((T + ATT_TQ - 1) / ATT_TQ) * m->nq;
  const bool tiled = !split && T >= 64 && tile_blocks >= 2 * int64_t(ctx->num_sms) &&
                     (m->hd == 32 || m->hd == 64 || m->hd == 128);
  if (tiled && (m->hd == 64 || m->hd == 128)) {
    const dim3 g1 = dim3(unsigned((rows / T) * ((T + ATT_TQ - 1) / ATT_TQ)), unsigned(m->nq));
    LaunchCfg l1(ctx, g1, dim3(ATT_THREADS), 0, st);
    if (m->hd == 128) CUDA_TRY(cudaLaunchKernelEx(&l1.cfg, attn_scores_mma_kernel<128>, p));
    else CUDA_TRY(cudaLaunchKernelEx(&l1.cfg, attn_scores_mma_kernel<64>, p));
  } else {
    const int gsub = int((m->G + ATT_MAXG - 1) / ATT_MAXG);
    const dim3 g1 = dim3(unsigned(rows * m->nkv * gsub), unsigned((lds_len + ATT_SKEYS - 1) / ATT_SKEYS));
    LaunchCfg l1(ctx, g1, dim3(ATT_THREADS), att_scores_smem(int(m->hd)), st);
    CUDA_TRY(cudaLaunchKernelEx(&l1.cfg, attn_scores_kernel, p, gsub));
  }
  if (split && m->hd % 8 == 0 && m->hd <= 128 && s->max_pos <= ATT_RSHORT && T == 1) {
    // short rows (decode of a session of at most ATT_RSHORT positions): one
    // block per query row. Measured: 0.5B shape at ~600 positions 6 % less
    // decode time than the chunked kernel; 7B shape at ~2100 positions 21 % more.
    LaunchCfg l2(ctx, dim3(unsigned(rows * m->nq)), dim3(ATT_DTHREADS), 0, st);
    CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_row_kernel, p));
    ctx->launches += 2;
    return MYL_OK;
  }
  if (split && m->hd % 8 == 0 && m->hd <= 128) {
    const dim3 g2 = dim3(unsigned(rows * m->nq), unsigned((lds_len + ATT_DCHUNK - 1) / ATT_DCHUNK));
    LaunchCfg l2(ctx, g2, dim3(ATT_DTHREADS), 0, st);
    CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_dec_kernel, p));
    ctx->launches += 2;
    return MYL_OK;
  }
  if (tiled) {
    // prefill: 64-row x 64-key tiles, value rows and probabilities staged once per tile
    const int64_t B = rows / T;
    const dim3 g2 = dim3(unsigned(B * ((T + ATT_TQ - 1) / ATT_TQ)), unsigned(m->nq));
    LaunchCfg l2(ctx, g2, dim3(ATT_THREADS), 0, st);
    const bool mma = m->prob_frac <= 15;  // p <= 32768: two unsigned bytes
    if (mma && m->hd == 128) CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_mma_kernel<128>, p));
    else if (mma && m->hd == 64) CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_mma_kernel<64>, p));
    else if (m->hd == 128) CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_tile_kernel<4>, p));
    else if (m->hd == 64) CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_tile_kernel<2>, p));
    else CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_tile_kernel<1>, p));
    ctx->launches += 2;
    return MYL_OK;
  }
  const int64_t chunk = split ? ATT_CHUNK : ((lds_len + ATT_CHUNK - 1) / ATT_CHUNK) * ATT_CHUNK;
  const dim3 g2 = dim3(unsigned(rows * m->nq), unsigned((lds_len + chunk - 1) / chunk));
  if (m->hd % 8 == 0) {
    LaunchCfg l2(ctx, g2, dim3(ATT_THREADS), size_t(ATT_THREADS) * 8 * 8, st);
    CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_vec_kernel, p, chunk));
  } else {
    LaunchCfg l2(ctx, g2, dim3(ATT_THREADS), size_t(ATT_THREADS / 32) * size_t(m->hd) * 8, st);
    CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, attn_pv_kernel, p, chunk));
  }
  ctx->launches += 2;
  return MYL_OK;
}

int launch_norm(myl_ctx* ctx, const myl_model* m, const int16_t* x, int64_t rows, ResidParams rp,
                const NormDev& nd, int16_t* out, const int64_t* out_rows, int64_t n_out, cudaStream_t st) {
  const int64_t n = out_rows ? n_out : rows;
  if (n == 0) return MYL_OK;
  const unsigned blocks = unsigned(std::min<int64_t>(n, 65535));
  if (m->H % 8 == 0 && m->H <= 8 * NORM_CL * NORM_CL_THREADS && n <= 64) {
    // few rows (decode): each row over a cluster of SMs
    LaunchCfg lc(ctx, dim3(unsigned(n) * NORM_CL), dim3(NORM_CL_THREADS), 0, st, NORM_CL);
    CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, resid_rmsnorm_cluster_kernel, x, m->H, rows, rp,
                                norm_params(m, nd), out, m->H, out_rows, n_out));
  } else if (m->H % 8 == 0 && m->H <= 8 * NORM_THREADS * NORM_NV) {
    LaunchCfg lc(ctx, dim3(blocks), dim3(NORM_THREADS), 0, st);
    CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, resid_rmsnorm_vec_kernel, x, m->H, rows, rp,
                                norm_params(m, nd), out, m->H, out_rows, n_out));
  } else {
    LaunchCfg lc(ctx, dim3(blocks), dim3(NORM_THREADS), size_t(m->H) * 2, st);
    CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, resid_rmsnorm_kernel, x, m->H, rows, rp, norm_params(m, nd),
                                out, m->H, out_rows, n_out));
  }
  ctx->launches++;
  return MYL_OK;
}

// Tensor parallelism: the bounded barrier of all ranks (optionally carrying
// the B greedy keys of this rank into every rank's key slots).
int tp_barrier(myl_ctx* ctx, myl_session* s, const int64_t* keys, int64_t n, cudaStream_t st) {
  const myl_model* m = s->m;
  LaunchCfg lc(ctx, dim3(1), dim3(32), 0, st);
  CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, tp_barrier_kernel, s->peers, m->world, m->rank, s->d_epoch,
                              keys, n, ctx->d_err, ctx->timeout_ns));
  ctx->launches++;
  return MYL_OK;
}

// The epilogue of a row-parallel projection under tensor parallelism: exact
// int64 partials broadcast into slab `rank` of receive region `which` on
// every rank (rows of H).
Epilogue tp_partial_ep(const myl_session* s, int which) {
  Epilogue e{};
  e.mode = EPI_ACC_I64;
  e.ldy = s->m->H;
  e.xb_world = s->m->world;
  e.xb_rank = s->m->rank;
  e.xb_slab = s->rows_cap * s->m->H;
  for (int o = 0; o < s->m->world; ++o) e.xb_dst[o] = s->peer_recv[which][o];
  return e;
}

// The residual add of a row-parallel projection under tensor parallelism:
// the ranks' partial slabs of receive region `which`, requantised with shift.
void tp_parts(const myl_session* s, int which, const int8_t* shift, ResidParams* rp) {
  rp->add = nullptr;
  rp->parts = s->recv[which];
  rp->nparts = s->m->world;
  rp->part_slab = s->rows_cap * s->m->H;
  rp->part_shift = shift;
}

// The forward of T tokens per sequence (rows = B * T, tokens on the device,
// positions from s->d_pos). want_logits: the last token's logits into
// s->logits. lds_len bounds the keys any row reads (the attention grids cover
// it; a decode step captured once for all positions passes max_pos).
int model_forward(myl_ctx* ctx, const myl_model* m, myl_session* s, const int32_t* tokens, int64_t T,
                  bool want_logits, int64_t lds_len, cudaStream_t st) {
  const int64_t rows = s->B * T, H = m->H;
  {
    LaunchCfg lc(ctx, dim3(unsigned(std::min<int64_t>(rows, 65535))), dim3(256), 0, st);
    CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, embed_kernel, tokens, rows, m->embed_rows, m->lde,
                                static_cast<const uint8_t*>(m->d_embed_shifts),
                                static_cast<const uint8_t*>(m->d_rin0), H, m->V_global, s->hid, H,
                                ctx->d_err));
  }
  ctx->launches++;
  const bool tp = m->world > 1;
  for (int64_t l = 0; l < m->L; ++l) {
    const ModelLayer& L = m->layers[size_t(l)];
    ResidParams rp{};
    const int16_t* x1 = s->hid;
    if (l > 0) {
      const ModelLayer& P = m->layers[size_t(l - 1)];
      rp.add = s->mlp_out;
      rp.ld_add = H;
      rp.s1 = P.add_mlp.s1;
      rp.s2 = P.add_mlp.s2;
      rp.resid_out = s->hid;
      rp.ld_res = H;
      if (tp) tp_parts(s, 1, P.mlp->d_shift_down, &rp);
      x1 = s->mid;
    }
    TRY(launch_norm(ctx, m, x1, rows, rp, L.norm1, s->xn, nullptr, 0, st));
    TRY(dispatch_linear(ctx, L.w_qkv, s->xn, rows, H, make_ep(L.rq_qkv, s->qkv, m->ldq), st));
    if (T > 1) {  // decode (T == 1): the RoPE runs inside the scores kernel
      const int64_t items = (m->nq + m->nkv) * (m->hd / 2) + m->nkv * m->hd / ((m->hd % 8) ? 1 : 8);
      LaunchCfg lc(ctx, dim3(unsigned(std::min<int64_t>(rows, 65535)), unsigned((items + 255) / 256)),
                   dim3(256), 0, st);
      CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, rope_kv_kernel, s->qkv, m->ldq, rows, T,
                                  static_cast<const int64_t*>(s->d_pos), int(m->nq), int(m->nkv),
                                  int(m->hd), static_cast<const int16_t*>(m->d_cos),
                                  static_cast<const int16_t*>(m->d_sin), m->n_pos, int(m->rope_frac),
                                  s->cache, int(l)));
      ctx->launches++;
    }
    TRY(run_attention(ctx, m, s, L, int(l), rows, T, lds_len, st));
    ResidParams ra{};
    ra.ld_add = H;
    ra.s1 = L.add_attn.s1;
    ra.s2 = L.add_attn.s2;
    ra.resid_out = s->mid;
    ra.ld_res = H;
    if (tp) {
      // row-parallel o_proj: partials to every rank, barrier, sum + requant in the norm
      TRY(dispatch_linear(ctx, L.w_o, s->attn, rows, m->QD, tp_partial_ep(s, 0), st));
      TRY(tp_barrier(ctx, s, nullptr, 0, st));
      tp_parts(s, 0, L.rq_o->d_shift, &ra);
    } else {
      TRY(dispatch_linear(ctx, L.w_o, s->attn, rows, m->QD, make_ep(L.rq_o, s->o, H), st));
      ra.add = s->o;
    }
    TRY(launch_norm(ctx, m, s->hid, rows, ra, L.norm2, s->xn, nullptr, 0, st));
    if (tp) {
      const Epilogue down = tp_partial_ep(s, 1);
      TRY(run_mlp(ctx, L.mlp, s->xn, rows, H, nullptr, H, st, nullptr, XPlanes(), &down));
      TRY(tp_barrier(ctx, s, nullptr, 0, st));
    } else {
      TRY(run_mlp(ctx, L.mlp, s->xn, rows, H, s->mlp_out, H, st));
    }
  }
  if (want_logits) {
    const ModelLayer& P = m->layers[size_t(m->L - 1)];
    ResidParams rp{};
    rp.add = s->mlp_out;
    rp.ld_add = H;
    rp.s1 = P.add_mlp.s1;
    rp.s2 = P.add_mlp.s2;
    if (tp) tp_parts(s, 1, P.mlp->d_shift_down, &rp);
    const int64_t* sel = nullptr;
    if (T > 1) {
      if (s->last_rows_T != T) {
        std::vector<int64_t> lr(static_cast<size_t>(s->B));
        for (int64_t b = 0; b < s->B; ++b) lr[size_t(b)] = b * T + T - 1;
        CUDA_TRY(cudaMemcpyAsync(s->last_rows, lr.data(), size_t(s->B) * 8, cudaMemcpyHostToDevice, st));
        CUDA_TRY(cudaStreamSynchronize(st));
        s->last_rows_T = T;
      }
      sel = s->last_rows;
    }
    TRY(launch_norm(ctx, m, s->mid, rows, rp, m->final_norm, s->xf, sel, s->B, st));
    TRY(dispatch_linear(ctx, m->head, s->xf, s->B, H, make_ep(m->rq_head, s->logits, m->V), st));
  }
  return MYL_OK;
}

// Greedy selection of s->logits into s->next_tok and out_tokens[:, step].
int launch_select(myl_ctx* ctx, const myl_model* m, myl_session* s, cudaStream_t st) {
  LaunchCfg l0(ctx, dim3(1), dim3(64), 0, st);
  CUDA_TRY(cudaLaunchKernelEx(&l0.cfg, select_init_kernel, s->keys, s->B));
  const dim3 grid = dim3(unsigned((m->V + SELECT_CHUNK - 1) / SELECT_CHUNK), unsigned(std::min<int64_t>(s->B, 65535)));
  LaunchCfg l1(ctx, grid, dim3(SELECT_THREADS), 0, st);
  CUDA_TRY(cudaLaunchKernelEx(&l1.cfg, select_keys_kernel, static_cast<const int32_t*>(s->logits),
                              s->B, m->V, m->V, m->v0, s->keys));
  const int64_t* keys = s->keys;
  if (m->world > 1) {  // every rank's best key of its vocabulary rows, then the largest
    TRY(tp_barrier(ctx, s, s->keys, s->B, st));
    keys = s->key_slots;
  }
  LaunchCfg l2(ctx, dim3(1), dim3(256), 0, st);
  CUDA_TRY(cudaLaunchKernelEx(&l2.cfg, greedy_commit_kernel, keys, s->B, s->next_tok, s->out_tokens,
                              s->max_pos, s->d_step, s->d_pos, int64_t(0), m->world));
  ctx->launches += 3;
  return MYL_OK;
}

// ctx->pdl for the lifetime of a scope (the forward's kernel chains);
// MYL_PDL=0 turns it off.
struct PdlScope {
  myl_ctx* ctx;
  int saved;
  explicit PdlScope(myl_ctx* c) : ctx(c), saved(c->pdl) {
    const char* e = std::getenv("MYL_PDL");
    ctx->pdl = (e && e[0] == '0') ? 0 : 1;
  }
  ~PdlScope() { ctx->pdl = saved; }
};

// One decode step: select, forward of the chosen tokens, position + 1.
int decode_step(myl_ctx* ctx, const myl_model* m, myl_session* s, cudaStream_t st) {
  PdlScope pdl(ctx);
  TRY(launch_select(ctx, m, s, st));
  TRY(model_forward(ctx, m, s, s->next_tok, 1, true, s->max_pos, st));
  LaunchCfg lc(ctx, dim3(1), dim3(32), 0, st);
  CUDA_TRY(cudaLaunchKernelEx(&lc.cfg, advance_kernel, s->d_pos, int64_t(1)));
  ctx->launches++;
  return MYL_OK;
}

// Prefill of prompt [B][P] host tokens, in chunks of rows_cap rows; the last
// chunk computes the logits.
int prefill(myl_ctx* ctx, const myl_model* m, myl_session* s, const int32_t* prompt, int64_t P,
            bool want_logits, cudaStream_t st) {
  const int64_t Tc = std::max<int64_t>(1, s->rows_cap / s->B);
  for (int64_t t0 = 0; t0 < P; t0 += Tc) {
    const int64_t T = std::min(Tc, P - t0);
    CUDA_TRY(cudaStreamSynchronize(st));  // h_tokens is free again
    for (int64_t b = 0; b < s->B; ++b)
      std::memcpy(s->h_tokens + b * T, prompt + b * P + t0, size_t(T) * 4);
    CUDA_TRY(cudaMemcpyAsync(s->tok_in, s->h_tokens, size_t(s->B * T) * 4, cudaMemcpyHostToDevice, st));
    TRY(set_pos(s, s->pos, st));
    PdlScope pdl(ctx);
    TRY(model_forward(ctx, m, s, s->tok_in, T, want_logits && t0 + T == P, s->pos + T, st));
    s->pos += T;
  }
  return set_pos(s, s->pos, st);
}

}  // namespace

extern "C" {

int myl_model_create(myl_ctx* ctx, const myl_model_spec* sp, myl_model** out) {
  return myl_model_create_tp(ctx, sp, 1, 0, out);
}

// The share of rank r of n items split as evenly as possible (the first
// n % world ranks take one more): [begin, end).
static void even_share(int64_t n, int world, int rank, int64_t* b, int64_t* e) {
  const int64_t base = n / world, extra = n % world;
  *b = rank * base + std::min<int64_t>(rank, extra);
  *e = *b + base + (rank < extra ? 1 : 0);
}

int myl_model_create_tp(myl_ctx* ctx, const myl_model_spec* sp, int world, int rank, myl_model** out) {
  if (!ctx || !sp || !out) return fail(MYL_ERR_ARG, "null argument");
  *out = nullptr;
  if (world < 1 || world > MYL_XCHG_MAX || rank < 0 || rank >= world)
    return fail(MYL_ERR_ARG, "rank %d of world %d (at most %d ranks)", rank, world, MYL_XCHG_MAX);
  if (sp->vocab <= 0 || sp->hidden <= 0 || sp->num_layers <= 0 || sp->num_heads <= 0 ||
      sp->num_kv_heads <= 0 || sp->head_dim <= 0 || sp->intermediate <= 0)
    return fail(MYL_ERR_SHAPE, "model dimensions must be positive");
  if (sp->num_heads % sp->num_kv_heads)
    return fail(MYL_ERR_SHAPE, "num_heads %lld is not a multiple of num_kv_heads %lld",
                (long long)sp->num_heads, (long long)sp->num_kv_heads);
  if ((sp->head_dim & 1) || sp->head_dim > 254)
    return fail(MYL_ERR_UNSUPPORTED, "head_dim %lld: even and at most 254 supported",
                (long long)sp->head_dim);
  const int64_t half = sp->head_dim / 2;
  if (!sp->layers || !sp->embed || !sp->embed_shifts || !sp->final_gamma || !sp->final_gamma_shifts ||
      !sp->final_residual_frac || !sp->cos_lut || !sp->sin_lut || !sp->exp_lut || !sp->silu_lut ||
      !sp->rsqrt_lut)
    return fail(MYL_ERR_ARG, "null tensor");
  if (sp->rope_len < half || sp->rope_len % half || sp->exp_len < 1 || sp->rsqrt_len < 1 ||
      sp->silu_len < 1 || sp->exp_len > (int64_t(1) << 31))
    return fail(MYL_ERR_SHAPE, "lookup table lengths");
  if (sp->prob_frac_bits > 30 || sp->rope_frac_bits > 30)
    return fail(MYL_ERR_OVERFLOW, "prob_frac_bits / rope_frac_bits beyond i32 shifts");
  int32_t exp_max = 0;
  for (int64_t i = 0; i < sp->exp_len; ++i) exp_max = std::max<int32_t>(exp_max, sp->exp_lut[i]);
  // softmax.rs:53: e * one in i32
  if ((int64_t(exp_max) << sp->prob_frac_bits) > INT32_MAX)
    return fail(MYL_ERR_OVERFLOW, "exp LUT values times 2^prob_frac_bits overflow i32");
  CUDA_TRY(cudaSetDevice(ctx->device));
  if (world > 1) {
    if (sp->num_heads < world || sp->intermediate < world || sp->vocab < world)
      return fail(MYL_ERR_SHAPE, "%d ranks for %lld heads", world, (long long)sp->num_heads);
    if (sp->hidden % 8 || sp->hidden > 8 * NORM_THREADS * NORM_NV)
      return fail(MYL_ERR_UNSUPPORTED, "tensor parallelism needs hidden %% 8 == 0, <= %d",
                  8 * NORM_THREADS * NORM_NV);
  }
  myl_model* m = new myl_model();
  m->world = world;
  m->rank = rank;
  m->V_global = sp->vocab;
  m->G = sp->num_heads / sp->num_kv_heads;
  int64_t q1, i1, v1;
  even_share(sp->num_heads, world, rank, &m->q0, &q1);
  even_share(sp->intermediate, world, rank, &m->i0, &i1);
  even_share(sp->vocab, world, rank, &m->v0, &v1);
  m->kv0 = m->q0 / m->G;  // the KV heads this rank's query heads read
  const int64_t kv1 = (q1 - 1) / m->G + 1;
  m->V = v1 - m->v0;
  m->H = sp->hidden;
  m->L = sp->num_layers;
  m->nq = q1 - m->q0;
  m->nkv = kv1 - m->kv0;
  m->hd = sp->head_dim;
  m->I = i1 - m->i0;
  m->QD = m->nq * m->hd;
  m->KD = m->nkv * m->hd;
  m->ldq = m->QD + 2 * m->KD;
  m->final_norm_frac = sp->final_norm_frac;
  m->logit_frac = sp->logit_frac_bits;
  m->prob_frac = sp->prob_frac_bits;
  m->rope_frac = sp->rope_frac_bits;
  m->n_pos = sp->rope_len / half;
  m->exp_len = sp->exp_len;
  m->rsqrt_len = sp->rsqrt_len;
  m->exp_max = exp_max;
  // inv_sqrt_q15 (fixed_point.rs:102-107) and the exp LUT shift (model.rs:543-546)
  {
    const uint64_t n = (uint64_t(1) << 30) / uint64_t(m->hd);
    uint64_t r = n, next = n / 2 + (n & 1);
    while (next < r) {
      r = next;
      next = (r + n / r) / 2;
    }
    while (r > 0 && r > n / r) r -= 1;
    while ((r + 1) <= n / (r + 1)) r += 1;
    m->score_mult = int64_t((r + 1) * (r + 1) - n < n - r * r ? r + 1 : r);
  }
  m->lut_shift = sp->score_frac_bits > sp->exp_input_frac ? sp->score_frac_bits - sp->exp_input_frac : 0;
  m->layers.resize(size_t(m->L));
  int rc = MYL_OK;
  // embedding rescale (model.rs:241-248): every (row shift, channel shift) pair
  {
    bool es_seen[256] = {}, rs_seen[256] = {};
    for (int64_t v = 0; v < sp->vocab; ++v) es_seen[sp->embed_shifts[v]] = true;
    for (int64_t i = 0; i < m->H; ++i) rs_seen[sp->layers[0].residual_in_frac[i]] = true;
    for (int a = 0; a < 256 && rc == MYL_OK; ++a)
      for (int b = 0; b < 256 && rc == MYL_OK; ++b)
        if (es_seen[a] && rs_seen[b]) {
          int s;
          rc = rescale_shift(uint8_t(a), uint8_t(b), 32, &s, "embedding");
        }
  }
  for (int64_t l = 0; l < m->L && rc == MYL_OK; ++l) rc = build_layer(ctx, m, sp, l);
  if (rc == MYL_OK)
    rc = make_norm(m, sp->final_residual_frac, sp->final_gamma, sp->final_gamma_shifts,
                   sp->rsqrt_input_shift, sp->rsqrt_output_frac, sp->final_norm_frac, &m->final_norm);
  // LM head (model.rs:284-308): path A (int16) if present, else path B (int8,
  // the embedding when tied); i32 logits at logit_frac_bits.
  if (rc == MYL_OK) {
    const int64_t v0 = m->v0, H = m->H;
    if (sp->lm_head16) {
      if (!sp->lm_head16_shifts) rc = fail(MYL_ERR_ARG, "lm_head16 shifts");
      else rc = myl_weight16_register(ctx, sp->lm_head16 + v0 * H, m->V, H, H, sp->lm_head16_shifts + v0,
                                      &m->head);
    } else if (sp->lm_head) {
      if (!sp->lm_head_shifts) rc = fail(MYL_ERR_ARG, "lm_head shifts");
      else rc = myl_weight_register(ctx, sp->lm_head + v0 * H, m->V, H, H, sp->lm_head_shifts + v0,
                                    &m->head);
    } else {
      rc = myl_weight_register(ctx, sp->embed + v0 * H, m->V, H, H, sp->embed_shifts + v0, &m->head);
    }
  }
  if (rc == MYL_OK) {
    uint8_t lf = sp->logit_frac_bits;
    rc = myl_requant_create(ctx, m->head, MYL_RQ_SHIFT_I32, sp->final_norm_frac, &lf, 0, nullptr,
                            nullptr, &m->rq_head);
  }
  // embedding rows (every rank holds the whole table): the LM head's device
  // rows when it is the embedding itself, else an own table
  if (rc == MYL_OK) {
    if (!sp->lm_head16 && !sp->lm_head && world == 1) {
      m->embed_rows = m->head->d_W;
      m->lde = m->head->ldp;
    } else {
      rc = dev_upload(m->allocs, &m->d_embed, sp->embed, size_t(sp->vocab * m->H));
      m->embed_rows = m->d_embed;
      m->lde = m->H;
    }
  }
  if (rc == MYL_OK) rc = dev_upload(m->allocs, &m->d_embed_shifts, sp->embed_shifts, size_t(sp->vocab));
  if (rc == MYL_OK)
    rc = dev_upload(m->allocs, &m->d_rin0, sp->layers[0].residual_in_frac, size_t(m->H));
  if (rc == MYL_OK) rc = dev_upload(m->allocs, &m->d_cos, sp->cos_lut, size_t(sp->rope_len));
  if (rc == MYL_OK) rc = dev_upload(m->allocs, &m->d_sin, sp->sin_lut, size_t(sp->rope_len));
  if (rc == MYL_OK) rc = dev_upload(m->allocs, &m->d_exp, sp->exp_lut, size_t(sp->exp_len));
  if (rc == MYL_OK) rc = dev_upload(m->allocs, &m->d_rsqrt, sp->rsqrt_lut, size_t(sp->rsqrt_len));
  if (rc != MYL_OK) {
    release_model(ctx, m);
    return rc;
  }
  *out = m;
  return MYL_OK;
}

int myl_model_release(myl_ctx* ctx, myl_model* m) {
  if (!m) return MYL_OK;
  if (ctx) {
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
  }
  release_model(ctx, m);
  return MYL_OK;
}

int myl_session_create(myl_ctx* ctx, const myl_model* m, int64_t batch, int64_t max_positions,
                       myl_session** out) {
  if (!ctx || !m || !out) return fail(MYL_ERR_ARG, "null argument");
  *out = nullptr;
  if (batch <= 0 || max_positions <= 0) return fail(MYL_ERR_SHAPE, "batch and max_positions must be positive");
  // softmax.rs:46: the i32 sum of up to max_positions exponentials
  if (int64_t(m->exp_max) * max_positions > INT32_MAX)
    return fail(MYL_ERR_OVERFLOW, "%lld positions overflow the softmax's i32 sum", (long long)max_positions);
  CUDA_TRY(cudaSetDevice(ctx->device));
  myl_session* s = new myl_session();
  s->m = m;
  s->B = batch;
  s->max_pos = max_positions;
  // rows of one prefill call: bounded so the score rows stay near 1 GiB
  const int64_t score_row_bytes = m->nq * max_positions * 4;
  const int64_t cap = std::max<int64_t>(1, (int64_t(1) << 30) / score_row_bytes);
  s->rows_cap = std::max<int64_t>(batch, std::min<int64_t>(4096, cap));
  s->part_rows = std::max<int64_t>(batch, (4 * int64_t(ctx->num_sms) + m->nq - 1) / m->nq);
  const int rc = session_alloc(ctx, s);
  if (rc != MYL_OK) {
    release_session(ctx, s);
    return rc;
  }
  *out = s;
  return MYL_OK;
}

int myl_session_release(myl_ctx* ctx, myl_session* s) {
  if (!s) return MYL_OK;
  if (ctx) cudaStreamSynchronize(ctx->stream);
  release_session(ctx, s);
  return MYL_OK;
}

int myl_session_reset(myl_ctx* ctx, myl_session* s) {
  if (!ctx || !s) return fail(MYL_ERR_ARG, "null argument");
  CUDA_TRY(cudaSetDevice(ctx->device));
  return set_pos(s, 0, ctx->stream);
}

int64_t myl_session_position(const myl_session* s) { return s ? s->pos : -1; }

// Layout of a rank's tensor-parallel region: two receive regions, key slots,
// flag words; each part 256-byte aligned.
static void tp_layout(const myl_session* s, size_t off[4], size_t* total) {
  const size_t w = size_t(s->m->world);
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t recv = up(w * size_t(s->rows_cap) * size_t(s->m->H) * 8);
  off[0] = 0;
  off[1] = recv;
  off[2] = 2 * recv;
  off[3] = off[2] + up(w * size_t(s->B) * 8);
  *total = off[3] + up(w * 8);
}

int64_t myl_session_tp_bytes(const myl_session* s) {
  if (!s) return -1;
  size_t off[4], total;
  tp_layout(s, off, &total);
  return int64_t(total);
}

int myl_session_set_tp(myl_ctx* ctx, myl_session* s, void* const* bases) {
  if (!ctx || !s || !bases) return fail(MYL_ERR_ARG, "null argument");
  const myl_model* m = s->m;
  if (m->world < 2) return fail(MYL_ERR_ARG, "the session's model is not tensor-parallel");
  for (int o = 0; o < m->world; ++o)
    if (!bases[o]) return fail(MYL_ERR_ARG, "null region of rank %d", o);
  size_t off[4], total;
  tp_layout(s, off, &total);
  CUDA_TRY(cudaSetDevice(ctx->device));
  auto at = [&](int o, int part) { return static_cast<uint8_t*>(bases[o]) + off[part]; };
  for (int w = 0; w < 2; ++w) {
    s->recv[w] = reinterpret_cast<int64_t*>(at(m->rank, w));
    for (int o = 0; o < m->world; ++o) s->peer_recv[w][o] = at(o, w);
  }
  s->key_slots = reinterpret_cast<int64_t*>(at(m->rank, 2));
  for (int o = 0; o < m->world; ++o) {
    s->peers.keys[o] = reinterpret_cast<int64_t*>(at(o, 2));
    s->peers.flags[o] = reinterpret_cast<unsigned long long*>(at(o, 3));
  }
  // this rank's flag words and epoch start at zero; the caller synchronises
  // the ranks (on the host) before the first forward
  CUDA_TRY(cudaMemset(at(m->rank, 3), 0, size_t(m->world) * 8));
  if (!s->d_epoch) TRY(dev_alloc(s->allocs, &s->d_epoch, 1));
  CUDA_TRY(cudaMemset(s->d_epoch, 0, 8));
  CUDA_TRY(cudaDeviceSynchronize());
  s->tp_ready = true;
  return MYL_OK;
}

int myl_model_shard(const myl_model* m, int64_t* info) {
  if (!m || !info) return fail(MYL_ERR_ARG, "null argument");
  const int64_t v[10] = {m->world, m->rank, m->q0, m->q0 + m->nq, m->kv0, m->kv0 + m->nkv,
                         m->i0, m->i0 + m->I, m->v0, m->v0 + m->V};
  std::memcpy(info, v, sizeof(v));
  return MYL_OK;
}

int myl_forward(myl_ctx* ctx, const myl_model* m, myl_session* s, const int32_t* tokens, int64_t T,
                int32_t* logits) {
  if (!ctx || !m || !s || s->m != m || (T > 0 && !tokens)) return fail(MYL_ERR_ARG, "null argument");
  if (m->world > 1 && !s->tp_ready) return fail(MYL_ERR_ARG, "tensor-parallel session without myl_session_set_tp");
  if (T <= 0) return fail(MYL_ERR_SHAPE, "T = %lld", (long long)T);
  if (s->pos + T > s->max_pos)
    return fail(MYL_ERR_SHAPE, "position %lld beyond the session's %lld", (long long)(s->pos + T),
                (long long)s->max_pos);
  for (int64_t i = 0; i < s->B * T; ++i)
    if (tokens[i] < 0 || tokens[i] >= m->V_global)
      return fail(MYL_ERR_SHAPE, "token id %d outside the vocabulary", tokens[i]);
  CUDA_TRY(cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  TRY(ws_acquire(ctx, st));
  CUDA_TRY(cudaEventRecord(s->ev[0], st));
  TRY(prefill(ctx, m, s, tokens, T, true, st));
  CUDA_TRY(cudaEventRecord(s->ev[1], st));
  TRY(ws_release(ctx, st));
  if (logits)
    CUDA_TRY(cudaMemcpyAsync(logits, s->logits, size_t(s->B * m->V) * 4, cudaMemcpyDeviceToHost, st));
  TRY(check_device_error(ctx));
  CUDA_TRY(cudaEventElapsedTime(&s->prefill_ms, s->ev[0], s->ev[1]));
  return MYL_OK;
}

// The greedy decode loop from the session's current logits (after a prefill).
static int decode_loop(myl_ctx* ctx, const myl_model* m, myl_session* s, int64_t max_new,
                       int32_t* out_tokens, uint8_t* digests, int32_t* step_logits) {
  cudaStream_t st = ctx->stream;
  if (m->world > 1 && (digests || step_logits))
    return fail(MYL_ERR_UNSUPPORTED, "digests and step logits need the whole vocabulary (world 1)");
  const int64_t P = s->pos;
  CUDA_TRY(cudaMemsetAsync(s->d_step, 0, 8, st));
  const bool host_steps = digests || step_logits;
  std::vector<Sha256Stream> sha(digests ? size_t(s->B) : 0);
  const size_t lbytes = size_t(m->V) * 4;
  CUDA_TRY(cudaEventRecord(s->ev[2], st));
  for (int64_t k = 0; k < max_new; ++k) {
    if (host_steps) {
      // the logits this step selects from (generate.rs:182-184), then the token
      CUDA_TRY(cudaMemcpyAsync(s->h_logits, s->logits, size_t(s->B) * lbytes, cudaMemcpyDeviceToHost, st));
      TRY(decode_step(ctx, m, s, st));
      CUDA_TRY(cudaStreamSynchronize(st));
      std::vector<int32_t> tok(static_cast<size_t>(s->B));
      CUDA_TRY(cudaMemcpy(tok.data(), s->next_tok, size_t(s->B) * 4, cudaMemcpyDeviceToHost));
      for (int64_t b = 0; b < s->B; ++b) {
        const int32_t* lg = s->h_logits + b * m->V;
        if (step_logits) std::memcpy(step_logits + (b * max_new + k) * m->V, lg, lbytes);
        if (digests) {
          sha[size_t(b)].update(reinterpret_cast<const uint8_t*>(lg), lbytes);  // i32 LE
          const uint32_t t = uint32_t(tok[size_t(b)]);
          const uint8_t tb[4] = {uint8_t(t), uint8_t(t >> 8), uint8_t(t >> 16), uint8_t(t >> 24)};
          sha[size_t(b)].update(tb, 4);
        }
      }
    } else if (k == 0) {
      // the first step runs eagerly: it sizes every workspace the step uses
      TRY(decode_step(ctx, m, s, st));
    } else {
      if (!s->graph || s->graph_epoch != g_ws_epoch) {
        // capture the step once (again only if a workspace moved since)
        if (s->graph) {
          cudaGraphExecDestroy(s->graph);
          s->graph = nullptr;
        }
        cudaGraph_t g = nullptr;
        CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        const int crc = decode_step(ctx, m, s, st);
        const cudaError_t ce = cudaStreamEndCapture(st, &g);
        if (crc != MYL_OK) {
          if (g) cudaGraphDestroy(g);
          return crc;
        }
        if (ce != cudaSuccess) return fail(MYL_ERR_CUDA, "decode capture: %s", cudaGetErrorString(ce));
        const cudaError_t ie = cudaGraphInstantiate(&s->graph, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) {
          s->graph = nullptr;
          return fail(MYL_ERR_CUDA, "decode graph: %s", cudaGetErrorString(ie));
        }
        s->graph_epoch = g_ws_epoch;
      }
      CUDA_TRY(cudaGraphLaunch(s->graph, st));
    }
  }
  CUDA_TRY(cudaEventRecord(s->ev[3], st));
  s->pos = P + max_new;
  if (max_new > 0) {
    CUDA_TRY(cudaMemcpy2DAsync(out_tokens, size_t(max_new) * 4, s->out_tokens, size_t(s->max_pos) * 4,
                               size_t(max_new) * 4, size_t(s->B), cudaMemcpyDeviceToHost, st));
  }
  TRY(check_device_error(ctx));
  CUDA_TRY(cudaEventElapsedTime(&s->decode_ms, s->ev[2], s->ev[3]));
  for (int64_t b = 0; b < (digests ? s->B : 0); ++b) sha[size_t(b)].finish(digests + 32 * b);
  return MYL_OK;
}

int myl_generate(myl_ctx* ctx, const myl_model* m, myl_session* s, const int32_t* prompt, int64_t P,
                 int64_t max_new, int32_t* out_tokens, uint8_t* digests, int32_t* step_logits) {
  if (!ctx || !m || !s || s->m != m || !prompt || (max_new > 0 && !out_tokens))
    return fail(MYL_ERR_ARG, "null argument");
  if (P <= 0 || max_new < 0) return fail(MYL_ERR_SHAPE, "P = %lld, max_new = %lld", (long long)P,
                                         (long long)max_new);
  if (P + max_new > s->max_pos)
    return fail(MYL_ERR_SHAPE, "%lld positions beyond the session's %lld", (long long)(P + max_new),
                (long long)s->max_pos);
  if (m->world > 1 && !s->tp_ready) return fail(MYL_ERR_ARG, "tensor-parallel session without myl_session_set_tp");
  for (int64_t i = 0; i < s->B * P; ++i)
    if (prompt[i] < 0 || prompt[i] >= m->V_global)
      return fail(MYL_ERR_SHAPE, "token id %d outside the vocabulary", prompt[i]);
  CUDA_TRY(cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  TRY(ws_acquire(ctx, st));
  TRY(set_pos(s, 0, st));
  CUDA_TRY(cudaEventRecord(s->ev[0], st));
  TRY(prefill(ctx, m, s, prompt, P, true, st));
  CUDA_TRY(cudaEventRecord(s->ev[1], st));
  const int rc = decode_loop(ctx, m, s, max_new, out_tokens, digests, step_logits);
  CUDA_TRY(cudaEventElapsedTime(&s->prefill_ms, s->ev[0], s->ev[1]));
  TRY(ws_release(ctx, st));
  return rc;
}

int myl_decode_greedy(myl_ctx* ctx, const myl_model* m, myl_session* s, int64_t max_new,
                      int32_t* out_tokens, uint8_t* digests, int32_t* step_logits) {
  if (!ctx || !m || !s || s->m != m || (max_new > 0 && !out_tokens))
    return fail(MYL_ERR_ARG, "null argument");
  if (s->pos <= 0) return fail(MYL_ERR_ARG, "the session holds no prompt (run myl_forward first)");
  if (max_new < 0 || s->pos + max_new > s->max_pos)
    return fail(MYL_ERR_SHAPE, "%lld positions beyond the session's %lld", (long long)(s->pos + max_new),
                (long long)s->max_pos);
  CUDA_TRY(cudaSetDevice(ctx->device));
  TRY(ws_acquire(ctx, ctx->stream));
  TRY(set_pos(s, s->pos, ctx->stream));
  const int rc = decode_loop(ctx, m, s, max_new, out_tokens, digests, step_logits);
  TRY(ws_release(ctx, ctx->stream));
  return rc;
}

int myl_session_timing(const myl_session* s, float* prefill_ms, float* decode_ms) {
  if (!s) return fail(MYL_ERR_ARG, "null argument");
  if (prefill_ms) *prefill_ms = s->prefill_ms;
  if (decode_ms) *decode_ms = s->decode_ms;
  return MYL_OK;
}

int myl_rmsnorm_i16(myl_ctx* ctx, const int16_t* x, int64_t M, int64_t n, const uint8_t* x_shifts,
                    const int8_t* gamma, const uint8_t* gamma_shifts, const int16_t* rsqrt_lut,
                    int64_t lut_len, uint8_t lut_input_shift, uint8_t lut_output_frac,
                    int64_t inv_n_q20, uint8_t out_frac_bits, int16_t* out) {
  if (!ctx || (M > 0 && (!x || !out)) || !x_shifts || !gamma || !gamma_shifts || !rsqrt_lut)
    return fail(MYL_ERR_ARG, "null argument");
  if (n <= 0 || M < 0 || lut_len <= 0) return fail(MYL_ERR_SHAPE, "rmsnorm_i16 shape");
  if (M == 0) return MYL_OK;
  CUDA_TRY(cudaSetDevice(ctx->device));
  myl_model tmp;  // carries the norm's device arrays
  tmp.H = n;
  int rc = make_norm(&tmp, x_shifts, gamma, gamma_shifts, lut_input_shift, lut_output_frac,
                     out_frac_bits, &tmp.final_norm);
  tmp.final_norm.inv_n = inv_n_q20;
  int16_t *dx = nullptr, *dy = nullptr;
  if (rc == MYL_OK) rc = dev_upload(tmp.allocs, &tmp.d_rsqrt, rsqrt_lut, size_t(lut_len));
  tmp.rsqrt_len = lut_len;
  if (rc == MYL_OK) rc = dev_upload(tmp.allocs, &dx, x, size_t(M * n));
  if (rc == MYL_OK) rc = dev_alloc(tmp.allocs, &dy, size_t(M * n));
  if (rc == MYL_OK) rc = launch_norm(ctx, &tmp, dx, M, ResidParams{}, tmp.final_norm, dy, nullptr, 0, ctx->stream);
  if (rc == MYL_OK && cudaMemcpyAsync(out, dy, size_t(M * n) * 2, cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess)
    rc = fail(MYL_ERR_CUDA, "rmsnorm download");
  if (rc == MYL_OK) rc = check_device_error(ctx);
  for (void* p : tmp.allocs) cudaFree(p);
  tmp.allocs.clear();
  return rc;
}

int myl_attention_int(myl_ctx* ctx, const int16_t* q, int64_t q_len, const int16_t* k,
                      const int16_t* v, int64_t kv_len, int64_t head_dim, const uint8_t* mask,
                      int64_t score_mult, uint8_t score_shift, const int16_t* exp_lut,
                      int64_t exp_len, uint8_t lut_shift, uint8_t prob_frac_bits, int16_t* out) {
  if (!ctx || !q || !k || !v || !exp_lut || !out) return fail(MYL_ERR_ARG, "null argument");
  if (q_len <= 0 || kv_len <= 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 254 || exp_len <= 0)
    return fail(MYL_ERR_SHAPE, "attention_int shape");
  if (score_shift > 62 || prob_frac_bits > 30 || lut_shift > 31)
    return fail(MYL_ERR_OVERFLOW, "attention_int shifts");
  int32_t exp_max = 0;
  for (int64_t i = 0; i < exp_len; ++i) exp_max = std::max<int32_t>(exp_max, exp_lut[i]);
  if ((int64_t(exp_max) << prob_frac_bits) > INT32_MAX || int64_t(exp_max) * kv_len > INT32_MAX)
    return fail(MYL_ERR_OVERFLOW, "softmax_int i32 range");
  CUDA_TRY(cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  std::vector<void*> A;
  int16_t *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr, *dlut = nullptr;
  uint8_t* dmask = nullptr;
  int32_t* dsc = nullptr;
  int64_t *dpart = nullptr, *dpos = nullptr;
  unsigned *dcnt = nullptr, *dmax = nullptr;
  const int64_t zero = 0;
  const int max_chunks = int((kv_len + ATT_CHUNK - 1) / ATT_CHUNK);
  int rc = dev_upload(A, &dq, q, size_t(q_len * head_dim));
  if (rc == MYL_OK) rc = dev_upload(A, &dk, k, size_t(kv_len * head_dim));
  if (rc == MYL_OK) rc = dev_upload(A, &dv, v, size_t(kv_len * head_dim));
  if (rc == MYL_OK) rc = dev_upload(A, &dlut, exp_lut, size_t(exp_len));
  if (rc == MYL_OK) rc = dev_upload(A, &dpos, &zero, 1);
  if (rc == MYL_OK && mask) rc = dev_upload(A, &dmask, mask, size_t(q_len * kv_len));
  if (rc == MYL_OK) rc = dev_alloc(A, &dout, size_t(q_len * head_dim));
  if (rc == MYL_OK) rc = dev_alloc(A, &dsc, size_t(q_len * kv_len));
  if (rc == MYL_OK) rc = dev_alloc(A, &dpart, size_t(q_len * max_chunks * head_dim));
  if (rc == MYL_OK) rc = dev_alloc(A, &dcnt, size_t(q_len));
  if (rc == MYL_OK) rc = dev_alloc(A, &dmax, size_t(q_len));
  if (rc == MYL_OK && (cudaMemset(dcnt, 0, size_t(q_len) * 4) != cudaSuccess ||
                       cudaMemset(dmax, 0, size_t(q_len) * 4) != cudaSuccess))
    rc = fail(MYL_ERR_CUDA, "memset");
  if (rc == MYL_OK) {
    // one "sequence" of q_len query rows, one head; the K/V arrays are the cache
    AttnParams p{};
    p.qkv = dq;
    p.ldq = head_dim;
    p.T = q_len;
    p.rows = q_len;
    p.pos0 = dpos;
    p.nq = 1;
    p.nkv = 1;
    p.q_head0 = 0;
    p.kv_head0 = 0;
    p.G = 1;
    p.hd = int(head_dim);
    p.kc.k = dk;
    p.kc.v = dv;
    p.kc.head_stride = kv_len * head_dim;
    p.kc.layer_stride = p.kc.head_stride;
    p.kc.seq_stride = p.kc.head_stride;
    p.score_mult = score_mult;
    p.score_shift = score_shift;
    p.scores = dsc;
    p.lds = kv_len;
    p.mask = dmask;
    p.exp_lut = dlut;
    p.exp_len = int32_t(exp_len);
    p.lut_shift = lut_shift;
    p.prob_frac = prob_frac_bits;
    p.out_shift = 0;
    p.part = dpart;
    p.max_chunks = max_chunks;
    p.counters = dcnt;
    p.rowmax = dmax;
    p.out = dout;
    p.ldo = head_dim;
    // every query sees all kv_len keys: a pseudo-position with pos + 1 = kv_len
    // comes from the mask form (len = lds) in both passes
    if (!mask) {
      std::vector<uint8_t> ones(size_t(q_len * kv_len), 1);
      rc = dev_upload(A, &dmask, ones.data(), ones.size());
      p.mask = dmask;
    }
    if (rc == MYL_OK) {
      const dim3 g1 = dim3(unsigned(q_len), unsigned((kv_len + ATT_SKEYS - 1) / ATT_SKEYS));
      attn_scores_kernel<<<g1, ATT_THREADS, att_scores_smem(int(head_dim)), st>>>(p, 1);
      const dim3 g2 = dim3(unsigned(q_len), unsigned(max_chunks));
      if (head_dim % 8 == 0)
        attn_pv_vec_kernel<<<g2, ATT_THREADS, size_t(ATT_THREADS) * 8 * 8, st>>>(p, ATT_CHUNK);
      else
        attn_pv_kernel<<<g2, ATT_THREADS, size_t(ATT_THREADS / 32) * size_t(head_dim) * 8, st>>>(p, ATT_CHUNK);
      if (cudaGetLastError() != cudaSuccess) rc = fail(MYL_ERR_CUDA, "attention launch");
      ctx->launches += 2;
    }
    if (rc == MYL_OK && cudaMemcpyAsync(out, dout, size_t(q_len * head_dim) * 2, cudaMemcpyDeviceToHost, st) != cudaSuccess)
      rc = fail(MYL_ERR_CUDA, "attention download");
    if (rc == MYL_OK) rc = check_device_error(ctx);
  }
  cudaStreamSynchronize(st);
  for (void* ptr : A) cudaFree(ptr);
  return rc;
}

}  // extern "C"
