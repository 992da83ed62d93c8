// The whole drafter pass and extend_context as a fixed launch sequence over
// caller-owned memory (fm_plan_* / fm_draft / fm_extend_context).
//
// One draft (modeling_flashmap.py:422-479, batch B, block K, T = B*K rows):
//   draft_prep                         anchor embedding rows, positions
//   anchor_proj GEMM -> anchor_norm    (:453)
//   cross k|v GEMM of every layer for the anchor row, k-norm + RoPE fused,
//     written into the cache at position lengths[b]            (:456-457)
//   one step:  z (Philox) -> z L^T GEMM -> mix_state           (:462-466)
//   multi-step: state rows -> E_S^T GEMM -> mix_state          (:473, :378-399)
//   x_embed GEMM, then per layer:                               (:309-311)
//     adaln -> qkv GEMM (q/k norm + RoPE fused) -> self-attention
//       -> o GEMM (gated residual fused)
//     adaln -> q GEMM (norm + RoPE fused) -> cross-attention
//       -> o GEMM (gated residual fused)
//     adaln -> fc1/gate_up GEMM (GELU/SwiGLU fused) -> fc2/down GEMM (gated residual)
//   final adaln -> head GEMM -> LM-head GEMM (logits + argmax fused)  (:312-313, :475)
//   multi-step: state update between jumps                     (:476-478)
// Every kernel is launched with programmatic dependent launch on one stream.
//
// A batch-1, one-jump draft may instead run as the streamed single-launch
// pass (stream.cuh) over the same weights and buffers: build_stream lays out
// its stage list.
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "attention.cuh"
#include "gemm_plan.cuh"
#include "ops.cuh"
#include "stream.cuh"

namespace fm {
fm_status launch_self_attn(const SelfAttnArgs& a, int batch, cudaStream_t stream, bool pdl);
fm_status launch_cross_attn(const CrossAttnArgs& a, const CUtensorMap& tm, cudaStream_t stream, bool pdl);
}  // namespace fm

using namespace fm;

struct fm_plan {
  fm_model_desc m;
  std::vector<fm_layer_weights> layers;
  fm_plan_config cfg;
  std::vector<fm_jump> jumps;
  int B, K, T, D, H, hd, I, L, Ht, S, ctxw;
  // workspace carve-out
  int* err;
  int* gemm_counters;
  int* xattn_counters;
  float* gemm_ws;
  float* xattn_part;
  int nsplit;
  __nv_bfloat16 *anchor_rows, *anchor_h, *anchor_ctx;
  int *anchor_pos, *anchor_seq, *slot_pos;
  float *tok_cos, *tok_sin;  // [T][hd/2] rotary factors of the slots' positions
  unsigned long long* keys;
  __nv_bfloat16 *z, *zl, *inputs, *x, *h, *qkv, *attn, *qc, *mlp, *hidden, *logits_s;
  float* state;
  __nv_bfloat16 *srows, *semb;
  __nv_bfloat16 *ext_fc, *ext_ctx;
  int *ext_seq, *ext_pos;
  // launch plans
  GemmPlan g_anchor_proj, g_anchor_kv, g_zl, g_xembed, g_head, g_lm;
  GemmPlan g_nfold;   // eigen-folded noise: z times the folded weight (one-jump drafts)
  bool noise_folded;
  GemmPlan g_state_first, g_state_next;
  std::vector<GemmPlan> g_layer;  // 6 per layer: qkv, o, q, cross_o, mlp1, mlp2
  CUtensorMap cache_map;
  bool has_target;
  long long last_launches;
  // streamed single-launch pass (batch 1, one jump)
  bool stream_on;
  int stream_grid;
  stream::Params* sp;  // launch parameters (host), per-call fields filled by fm_draft
  unsigned long long *st_words, *st_done, *st_tickets;
  long long st_n_tickets;
  int* st_zero;
  float* st_ws;
  float* st_stats;
  stream::Stage* st_stages;
  ~fm_plan() { delete sp; }
};

namespace {

struct Carver {
  char* base;
  size_t off = 0;
  template <typename Tp>
  Tp* take(size_t count) {
    off = (off + 255) / 256 * 256;
    Tp* p = base ? reinterpret_cast<Tp*>(base + off) : nullptr;
    off += count * sizeof(Tp);
    return p;
  }
};

size_t max_gemm_partials(const fm_model_desc* m, const fm_plan_config* c) {
  const int64_t T = (int64_t)c->batch * m->block, B = c->batch, D = m->hidden, Ht = m->target_hidden;
  const int64_t I = m->inter, L = m->layers, S = m->state_vocab, R = c->max_extend_rows;
  const int64_t mlp1 = m->swiglu ? 2 * I : I;
  size_t mx = 0;
  auto upd = [&](int64_t M, int64_t N, int64_t K) {
    if (N <= 0) return;
    const size_t b = gemm_partials_bytes(M, N, K);
    if (b > mx) mx = b;
  };
  upd(D, B, Ht);
  upd(L * 2 * D, B, D);
  upd(Ht, T, Ht);
  upd(D, T, Ht);
  upd(3 * D, T, D);
  upd(D, T, D);
  upd(mlp1, T, D);
  upd(D, T, I);
  upd(Ht, T, D);
  upd(S, T, Ht);
  if (c->num_steps > 1) {
    upd(Ht, T, S);
    upd(Ht, 2 * T, S);
  }
  upd(D, R, (int64_t)m->n_target_layers * Ht);
  upd(L * 2 * D, R, D);
  return mx;
}

size_t max_gemm_tiles(const fm_model_desc* m, const fm_plan_config* c) {
  const int64_t T = (int64_t)c->batch * m->block, D = m->hidden, Ht = m->target_hidden;
  const int64_t S = m->state_vocab, L = m->layers, R = c->max_extend_rows, I = m->inter;
  int64_t mx = 0;
  auto upd = [&](int64_t M, int64_t N) {
    if (N <= 0) return;
    const int64_t t = gemm_counter_slots(M, N);
    if (t > mx) mx = t;
  };
  upd(S, T);
  upd(L * 2 * D, R);
  upd(L * 2 * D, c->batch);
  upd(2 * I, T);
  upd(Ht, 2 * T);
  upd(D, R);
  return (size_t)mx;
}

// splits of every (sequence, head)'s keys: at most one CTA per SM in total,
// so the cross-attention is one wave
int pick_nsplit(int B, int H, int cache_len) {
  const int sms = num_sms();
  int ns = sms / (B * H);
  const int maxs = (cache_len + 63) / 64;
  if (ns > maxs) ns = maxs;
  if (ns < 1) ns = 1;
  return ns;
}

// The streamed pass's shape: batch 1, one jump, the target attached, the
// HF-path arithmetic (no folds), head_dim 64 or 128, and not a plan that asks
// for the kernel sequence.
bool stream_shape(const fm_model_desc* m, const fm_plan_config* c) {
  if (c->batch != 1 || c->num_steps != 1 || c->launch_mode == FM_LAUNCH_KERNELS) return false;
  if (c->launch_mode == FM_LAUNCH_AUTO) {
    const char* e = getenv("FM_STREAM");
    if (!e || e[0] != '1') return false;
  }
  if (!m->embed || !m->lm_w || !m->chol || !m->uniform_embeds || m->lm_fold_w) return false;
  if (m->noise_fold_w && m->noise_fold_var && m->noise_fold_x0) return false;
  return m->head_dim == 64 || m->head_dim == 128;
}
int stream_stage_cap(const fm_model_desc* m) { return 16 + 7 * (int)m->layers; }
int64_t tiles128(int64_t rows) { return (rows + 127) / 128; }
// every ticket of the pass: per GEMM stage one per 128-row tile, then the
// self-attention groups and the cross-attention heads of every layer
int64_t stream_tickets(const fm_model_desc* m) {
  const int64_t D = m->hidden, Ht = m->target_hidden, L = m->layers, S = m->state_vocab;
  const int64_t mlp1 = m->swiglu ? 2 * (int64_t)m->inter : m->inter;
  int64_t n = tiles128(Ht) + tiles128(D) + tiles128(L * 2 * D) + tiles128(D);
  n += L * (tiles128(3 * D) + 3 * tiles128(D) + tiles128(mlp1) + tiles128(D));
  n += tiles128(Ht) + tiles128(S);
  n += L * (D / 128) + L * m->heads;
  return n;
}
constexpr int STREAM_WS_SLOTS = 4;
int64_t stream_stat_tiles(const fm_model_desc* m) {
  const int64_t a = tiles128(m->target_hidden), b = tiles128(m->hidden);
  return a > b ? a : b;
}

// Lay out every buffer; with base == nullptr only the size is computed.
size_t carve(fm_plan* p, const fm_model_desc* m, const fm_plan_config* c, void* base) {
  Carver cv{static_cast<char*>(base)};
  const int64_t B = c->batch, K = m->block, T = B * K, D = m->hidden, Ht = m->target_hidden;
  const int64_t I = m->inter, S = m->state_vocab, R = c->max_extend_rows > 0 ? c->max_extend_rows : 1;
  const int64_t H = m->heads, hd = m->head_dim;
  const int ns = pick_nsplit((int)B, (int)H, c->cache_len);
  // zero-initialised region first (counters and the error word)
  int* err = cv.take<int>(64);
  int* gc = cv.take<int>(max_gemm_tiles(m, c) + 64);
  int* xc = cv.take<int>((size_t)B * H + 64);
  // the streamed pass: counters, tickets and a zero token index (zero-initialised too)
  const bool sw = stream_shape(m, c);
  const int scap = sw ? stream_stage_cap(m) : 0;
  const int64_t n_tickets = sw ? stream_tickets(m) : 0;
  unsigned long long* st_words = cv.take<unsigned long long>(sw ? 4 : 0);
  unsigned long long* st_done = cv.take<unsigned long long>((size_t)scap);
  unsigned long long* st_tickets = cv.take<unsigned long long>((size_t)n_tickets);
  int* st_zero = cv.take<int>(sw ? 4 : 0);
  float* st_ws = cv.take<float>(sw ? (size_t)STREAM_WS_SLOTS * num_sms() * 2 * 16 * 128 : 0);
  float* st_stats = cv.take<float>(sw ? (size_t)(3 * m->layers + 3) * stream_stat_tiles(m) * 32 : 0);
  stream::Stage* st_stages = cv.take<stream::Stage>((size_t)scap);
  float* gws = cv.take<float>(max_gemm_partials(m, c) / sizeof(float) + 64);
  float* xp = cv.take<float>((size_t)B * H * ns * (16 * hd + 32));
  __nv_bfloat16* anchor_rows = cv.take<__nv_bfloat16>(B * Ht);
  __nv_bfloat16* anchor_h = cv.take<__nv_bfloat16>(B * D);
  __nv_bfloat16* anchor_ctx = cv.take<__nv_bfloat16>(B * D);
  int* anchor_pos = cv.take<int>(B);
  int* anchor_seq = cv.take<int>(B);
  int* slot_pos = cv.take<int>(T);
  float* tok_cos = cv.take<float>(T * (hd / 2));
  float* tok_sin = cv.take<float>(T * (hd / 2));
  unsigned long long* keys = cv.take<unsigned long long>(T);
  __nv_bfloat16* z = cv.take<__nv_bfloat16>(T * Ht);
  __nv_bfloat16* zl = cv.take<__nv_bfloat16>(T * Ht);
  __nv_bfloat16* inputs = cv.take<__nv_bfloat16>(T * Ht);
  __nv_bfloat16* x = cv.take<__nv_bfloat16>(T * D);
  __nv_bfloat16* h = cv.take<__nv_bfloat16>(T * D);
  __nv_bfloat16* qkv = cv.take<__nv_bfloat16>(T * 3 * D);
  __nv_bfloat16* attn = cv.take<__nv_bfloat16>(T * D);
  __nv_bfloat16* qc = cv.take<__nv_bfloat16>(T * D);
  __nv_bfloat16* mlp = cv.take<__nv_bfloat16>(T * I);
  __nv_bfloat16* hidden = cv.take<__nv_bfloat16>(T * Ht);
  __nv_bfloat16* logits_s = cv.take<__nv_bfloat16>(T * S);
  float* state = nullptr;
  __nv_bfloat16 *srows = nullptr, *semb = nullptr;
  if (c->num_steps > 1) {
    state = cv.take<float>(T * S);
    srows = cv.take<__nv_bfloat16>(2 * T * S);
    semb = cv.take<__nv_bfloat16>(2 * T * Ht);
  }
  __nv_bfloat16* ext_fc = cv.take<__nv_bfloat16>(R * D);
  __nv_bfloat16* ext_ctx = cv.take<__nv_bfloat16>(R * D);
  int* ext_seq = cv.take<int>(R);
  int* ext_pos = cv.take<int>(R);
  if (p) {
    p->st_words = st_words;
    p->st_done = st_done;
    p->st_tickets = st_tickets;
    p->st_n_tickets = n_tickets;
    p->st_zero = st_zero;
    p->st_ws = st_ws;
    p->st_stats = st_stats;
    p->st_stages = st_stages;
    p->err = err;
    p->gemm_counters = gc;
    p->xattn_counters = xc;
    p->gemm_ws = gws;
    p->xattn_part = xp;
    p->nsplit = ns;
    p->anchor_rows = anchor_rows;
    p->anchor_h = anchor_h;
    p->anchor_ctx = anchor_ctx;
    p->anchor_pos = anchor_pos;
    p->anchor_seq = anchor_seq;
    p->slot_pos = slot_pos;
    p->tok_cos = tok_cos;
    p->tok_sin = tok_sin;
    p->keys = keys;
    p->z = z;
    p->zl = zl;
    p->inputs = inputs;
    p->x = x;
    p->h = h;
    p->qkv = qkv;
    p->attn = attn;
    p->qc = qc;
    p->mlp = mlp;
    p->hidden = hidden;
    p->logits_s = logits_s;
    p->state = state;
    p->srows = srows;
    p->semb = semb;
    p->ext_fc = ext_fc;
    p->ext_ctx = ext_ctx;
    p->ext_seq = ext_seq;
    p->ext_pos = ext_pos;
  }
  return cv.off + 256;
}

fm_status validate(const fm_model_desc* m, const fm_plan_config* c) {
  if (!m || !c) return set_error(FM_ERR_INVALID, "plan: null model or config");
  if (m->hidden <= 0 || m->heads <= 0 || m->head_dim * m->heads != m->hidden)
    return set_error(FM_ERR_SHAPE, "plan: hidden must equal heads * head_dim");
  if (m->head_dim != 64 && m->head_dim != 128) return set_error(FM_ERR_UNSUPPORTED, "plan: head_dim must be 64 or 128");
  if (m->hidden % 128 != 0) return set_error(FM_ERR_UNSUPPORTED, "plan: hidden must be a multiple of 128");
  if (m->block != 16) return set_error(FM_ERR_UNSUPPORTED, "plan: the kernels serve block_size 16");
  if (m->swiglu && m->inter % 64 != 0) return set_error(FM_ERR_UNSUPPORTED, "plan: swiglu width must be a multiple of 64");
  if (m->target_hidden % 8 || m->inter % 8 || m->state_vocab % 8)
    return set_error(FM_ERR_ALIGN, "plan: widths must be multiples of 8");
  if (c->batch <= 0 || c->num_steps <= 0 || !c->jumps || !c->cache)
    return set_error(FM_ERR_INVALID, "plan: bad config");
  if (c->num_steps > 1 && m->embed && !m->embed_state_t)
    return set_error(FM_ERR_INVALID, "plan: multi-step drafts need embed_state_t");
  if (c->cache_batch < c->batch) return set_error(FM_ERR_SHAPE, "plan: cache batch smaller than plan batch");
  if (c->launch_mode != FM_LAUNCH_AUTO && c->launch_mode != FM_LAUNCH_KERNELS &&
      c->launch_mode != FM_LAUNCH_PERSISTENT)
    return set_error(FM_ERR_INVALID, "plan: unknown launch_mode %d", c->launch_mode);
  if (!m->layer || !m->rope_cos || !m->rope_sin) return set_error(FM_ERR_INVALID, "plan: missing weights");
  return FM_OK;
}


// ------------------------------------------------------------------ the streamed pass
//
// Stage list of one batch-1, one-jump draft (modeling_flashmap.py:422-479):
//   prep | z L^T (the noise built in the operand) | anchor_proj (the anchor's
//   embedding row) | every layer's cross k|v of the anchor row (anchor_norm
//   in the operand; k-norm + RoPE, into the cache) | x_embed (mix_state in
//   the operand) | per layer: q|k|v (AdaLN operand; q/k norm + RoPE, then the
//   block self-attention per head group), o (gated residual), cross q (AdaLN;
//   q norm + RoPE), cross-attention, cross o (gated residual), fc1 / gate_up
//   (AdaLN; GELU / SwiGLU), fc2 / down (gated residual) | head (final AdaLN) |
//   LM head (logits + argmax) | tokens.
// The residual stages and x_embed publish LayerNorm statistics per tile;
// z L^T and anchor_proj publish sums of squares (mix_state's and
// anchor_norm's RMS).
fm_status build_stream(fm_plan* p) {
  using namespace stream;
  const fm_model_desc& m = p->m;
  const int G = grid_size();
  if (G <= 0) return set_error(FM_ERR_UNSUPPORTED, "streamed pass: the kernel cannot be resident on every SM");
  if (G > num_sms()) return set_error(FM_ERR_UNSUPPORTED, "streamed pass: grid beyond the carved partials");
  using bf = __nv_bfloat16;
  const int D = p->D, Ht = p->Ht, L = p->L, hd = p->hd;
  const bf* mods = static_cast<const bf*>(p->jumps[0].mods);
  if (!mods) return set_error(FM_ERR_INVALID, "streamed pass: jump without modulations");
  std::vector<Stage> st;
  Params* P = new (std::nothrow) Params();
  if (!P) return set_error(FM_ERR_INVALID, "streamed pass: host allocation failed");
  int n_maps = 0;
  unsigned long long* tk = p->st_tickets;
  long long tk_used = 0;
  float* stats = p->st_stats;
  const int64_t stat_tiles = stream_stat_tiles(&m);
  auto take_tickets = [&](int64_t n) {
    unsigned long long* r = tk + tk_used;
    tk_used += n;
    return r;
  };
  auto take_stats = [&]() {
    float* r = stats;
    stats += stat_tiles * 32;
    return r;
  };
  int rot = 0;
  auto gemm = [&](const GemmPlan& g, int dep, int bkind, int ekind, int stat, int ntok) -> int {
    Stage S{};
    S.kind = K_GEMM;
    S.dep = dep;
    S.dep2 = -1;
    S.pieces = g.args.m_tiles;
    // the CTAs the stage's units are split over: at most 4 per 128-row tile (so a
    // tile's partials are few), more when a CTA would otherwise stream over 256 KB
    const int64_t units = g.args.units, bytes = (int64_t)g.args.M * g.args.K * 2;
    int64_t vg = std::min<int64_t>(G, (int64_t)g.args.m_tiles * 4);
    vg = std::max<int64_t>(vg, std::min<int64_t>(G, (bytes + (256 << 10) - 1) >> 18));
    vg = std::min<int64_t>(vg, units);
    // a transform stage builds every operand block of its units on its CTA's two
    // operand warps: spread it over the whole grid (and its constant rows, staged
    // at once, must fit)
    if (bkind != B_COPY) vg = std::min<int64_t>(G, units);
    S.vg = (int)vg;
    S.rot = rot;
    rot = (int)((rot + vg) % G);
    S.map = n_maps;
    P->maps[n_maps++] = g.tmA;
    S.bmap = -1;
    if (bkind == B_COPY) {
      S.bmap = n_maps;
      P->maps[n_maps++] = g.tmB;
    }
    S.bkind = bkind;
    S.ekind = ekind;
    S.stats = stat;
    S.ntok = ntok;
    S.ep = g.args;
    S.ep.N = ntok;
    S.tickets = take_tickets(g.args.m_tiles);
    S.stats_out = stat != S_NONE ? take_stats() : nullptr;
    S.eps = m.rms_eps;
    st.push_back(S);
    return (int)st.size() - 1;
  };
  auto tiles_of = [&](int stage) { return st[stage].ep.m_tiles; };
  auto aux_stage = [&](int kind, int dep, const bf* src, bf* dst, long long count) -> int {
    Stage S{};
    S.kind = kind;
    S.dep = dep;
    S.dep2 = -1;
    S.pieces = kind == K_NOISE ? G : 1;
    S.src = src;
    S.dst = dst;
    S.count = count;
    S.eps = m.rms_eps;
    st.push_back(S);
    return (int)st.size() - 1;
  };
  // the anchor's embedding row (and keys reset, index checks); the one-step noise
  const int s_prep = aux_stage(K_PREP, -1, nullptr, p->anchor_rows, Ht);
  st[s_prep].aux = static_cast<const bf*>(m.embed);
  const int s_noise = aux_stage(K_NOISE, -1, nullptr, p->z, (long long)p->T * Ht);
  const int s_zl = gemm(p->g_zl, s_noise, B_COPY, E_STORE, S_SQ, 16);
  const int s_ap = gemm(p->g_anchor_proj, s_prep, B_COPY, E_STORE, S_NONE, 1);
  const int s_an = aux_stage(K_ANORM, s_ap, p->anchor_h, p->anchor_ctx, D);
  st[s_an].w0 = static_cast<const bf*>(m.anchor_norm_w);
  const int s_akv = gemm(p->g_anchor_kv, s_an, B_COPY, E_KVCACHE, S_NONE, 1);
  st[s_akv].ep.token_seq = p->st_zero;
  const int s_xe = gemm(p->g_xembed, s_zl, B_MIX, E_STORE, S_LN, 16);
  st[s_xe].src = p->zl;
  st[s_xe].ld = Ht;
  st[s_xe].aux = static_cast<const bf*>(m.uniform_embeds);
  st[s_xe].w0 = static_cast<const bf*>(m.state_norm_w);
  st[s_xe].w1 = static_cast<const bf*>(m.noise_norm_w);
  st[s_xe].gate = p->jumps[0].noise_gate;
  st[s_xe].stats_in = st[s_zl].stats_out;
  st[s_xe].stats_tiles = tiles_of(s_zl);
  int s_x = s_xe;  // the stage that last wrote x (its LayerNorm statistics)
  auto adaln = [&](int stage, const bf* mod) {
    Stage& S = st[stage];
    S.src = p->x;
    S.ld = D;
    S.mod = mod;
    S.eps = m.ln_eps;
    S.stats_in = st[s_x].stats_out;
    S.stats_tiles = tiles_of(s_x);
  };
  for (int l = 0; l < L; ++l) {
    const GemmPlan* g = &p->g_layer[(size_t)l * 6];
    const bf* ms = mods + (size_t)(l * 3 + 0) * 3 * D;
    const bf* mc = mods + (size_t)(l * 3 + 1) * 3 * D;
    const bf* mm = mods + (size_t)(l * 3 + 2) * 3 * D;
    const int s_qkv = gemm(g[0], s_x, B_ADALN, E_QKV, S_NONE, 16);
    adaln(s_qkv, ms);
    st[s_qkv].pieces = D / 128;  // head groups whose self-attention is done
    st[s_qkv].groups = take_tickets(D / 128);
    st[s_qkv].attn = p->attn;
    const int s_o = gemm(g[1], s_qkv, B_COPY, E_RESID, S_LN, 16);
    st[s_o].src = p->attn;
    st[s_o].ld = D;
    st[s_o].ep.gate = ms + 2 * D;
    s_x = s_o;
    const int s_q = gemm(g[2], s_o, B_ADALN, E_QNORM, S_NONE, 16);
    adaln(s_q, mc);
    {
      Stage S{};
      S.kind = K_XATTN;
      S.dep = s_q;
      S.dep2 = s_akv;
      S.pieces = p->H;
      S.layer = l;
      S.nsplit = p->nsplit;
      S.q = p->qc;
      S.out = p->attn;
      S.part = p->xattn_part;
      S.xtickets = take_tickets(p->H);
      st.push_back(S);
    }
    const int s_xa = (int)st.size() - 1;
    const int s_co = gemm(g[3], s_xa, B_COPY, E_RESID, S_LN, 16);
    st[s_co].src = p->attn;
    st[s_co].ld = D;
    st[s_co].ep.gate = mc + 2 * D;
    s_x = s_co;
    const int s_f1 = gemm(g[4], s_co, B_ADALN, m.swiglu ? E_SWIGLU : E_GELU, S_NONE, 16);
    adaln(s_f1, mm);
    const int s_f2 = gemm(g[5], s_f1, B_COPY, E_RESID, S_LN, 16);
    st[s_f2].src = p->mlp;
    st[s_f2].ld = p->I;
    st[s_f2].ep.gate = mm + 2 * D;
    s_x = s_f2;
  }
  const int s_head = gemm(p->g_head, s_x, B_ADALN, E_STORE, S_NONE, 16);
  adaln(s_head, mods + (size_t)(L * 3) * 3 * D);
  const int s_lm = gemm(p->g_lm, s_head, B_COPY, E_LOGITS, S_NONE, 16);
  st[s_lm].src = p->hidden;
  st[s_lm].ld = Ht;
  st[s_lm].dep2 = s_prep;
  st[s_lm].ep.col_ids = reinterpret_cast<const long long*>(m.draft_ids);
  {
    Stage S{};
    S.kind = K_FINAL;
    S.dep = s_lm;
    S.dep2 = -1;
    S.pieces = 1;
    st.push_back(S);
  }
  const int n = (int)st.size();
  auto fail = [&](const char* why) {
    delete P;
    return set_error(FM_ERR_UNSUPPORTED, "streamed pass: %s", why);
  };
  if (n > stream_stage_cap(&m)) return fail("stage list longer than its carve-out");
  if (tk_used > p->st_n_tickets) return fail("tickets beyond their carve-out");
  if (n_maps + 1 > MAX_MAPS) return fail("more weight matrices than tensor-map slots");
  // split-K partial buffers: a stage may reuse a buffer once every earlier user
  // of it is among its ancestors (their finishers have read their partials
  // before the completion this stage waits for)
  std::vector<std::vector<char>> anc(n, std::vector<char>(n, 0));
  for (int i = 0; i < n; ++i)
    for (int d : {st[i].dep, st[i].dep2})
      if (d >= 0) {
        anc[i][d] = 1;
        for (int k = 0; k < n; ++k)
          if (anc[d][k]) anc[i][k] = 1;
      }
  std::vector<std::vector<int>> users(STREAM_WS_SLOTS);
  const size_t slot_floats = (size_t)num_sms() * 2 * 16 * 128;
  for (int i = 0; i < n; ++i) {
    if (st[i].kind != K_GEMM) continue;
    int pick = -1;
    for (int k = 0; k < STREAM_WS_SLOTS && pick < 0; ++k) {
      bool okk = true;
      for (int u : users[k]) okk = okk && anc[i][u];
      if (okk) pick = k;
    }
    if (pick < 0) return fail("no split-K partial buffer is free of a concurrent stage");
    users[pick].push_back(i);
    st[i].ws = p->st_ws + pick * slot_floats;
  }
  // checks the kernel relies on
  for (int i = 0; i < n; ++i) {
    const Stage& S = st[i];
    if (S.kind != K_GEMM) continue;
    if (S.ep.n_tiles != 1 || S.ep.N > 16) return fail("a stage with more than 16 tokens");
    if (S.ep.K % 8) return fail("a stage's width is not a multiple of 8");
    auto misaligned = [](const void* q) { return q != nullptr && (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
    if (misaligned(S.src) || misaligned(S.mod) || misaligned(S.w0) || misaligned(S.w1) || misaligned(S.aux) ||
        (S.ld % 8) != 0)
      return fail("a stage's operand sources are not 16-byte aligned");
    if (S.stats != S_NONE && S.ep.M > stat_tiles * 128) return fail("statistics beyond their carve-out");
    if (S.bkind == B_ADALN && (S.ep.K % 128 || S.stats_tiles * 128 != S.ep.K))
      return fail("AdaLN rows must be whole 128-feature tiles");
    if (S.bkind != B_COPY && S.stats_tiles > 40) return fail("source rows wider than 40 tiles of 128");
    if (S.kind == K_GEMM && S.ep.units * (int64_t)G >= (int64_t(1) << 31))
      return fail("a GEMM stage of more units than the 32-bit split arithmetic holds");
    if (S.bkind != B_COPY && (S.vg > G || (S.ep.units + S.vg - 1) / S.vg > MAX_TRANSFORM_UNITS))
      return fail("a transform stage with more units per CTA than its constant staging holds");
    if (S.bkind == B_COPY && S.bmap < 0) return fail("a copied operand without its tensor map");
  }
  if (D % 128) return fail("hidden must be a multiple of 128");
  if (cudaMemcpy(p->st_stages, st.data(), st.size() * sizeof(Stage), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    return fail("could not copy the stage list to the device");
  }
  P->maps[n_maps] = p->cache_map;
  P->cache_map = n_maps;
  P->stages = p->st_stages;
  P->n_stages = n;
  P->done = p->st_done;
  P->words = p->st_words;
  P->all_tickets = p->st_tickets;
  P->n_tickets = tk_used;
  P->err = p->err;
  P->keys = p->keys;
  P->lm_stage = s_lm;
  P->rope_cos = m.rope_cos;
  P->rope_sin = m.rope_sin;
  P->rope_len = m.rope_len;
  P->half = hd / 2;
  P->cache_len = p->cfg.cache_len;
  P->cache_batch = p->cfg.cache_batch;
  P->heads = p->H;
  P->head_dim = hd;
  P->hidden = D;
  P->target_hidden = Ht;
  P->vocab = m.vocab;
  P->block = p->K;
  P->scale = (float)(1.0 / std::sqrt((double)hd));
  p->sp = P;
  p->stream_grid = G;
  p->stream_on = true;
  return FM_OK;
}

fm_status run_stream(fm_plan* p, const fm_draft_io* io, cudaStream_t s) {
  stream::Params& P = *p->sp;
  P.anchor_ids = io->anchor_ids;
  P.lengths = io->lengths;
  P.z = static_cast<const __nv_bfloat16*>(io->z);
  P.seed = io->seed;
  P.offset = io->offset;
  P.offset_ptr = io->offset_ptr;
  P.tokens = io->tokens;
  if (io->logits) {
    P.logits = static_cast<__nv_bfloat16*>(io->logits);
    P.ldl = io->ldl;
    P.scatter = (io->scatter && p->m.draft_ids) ? 1 : 0;
  } else {
    P.logits = p->logits_s;
    P.ldl = p->S;
    P.scatter = 0;
  }
  fm_status st = stream::launch(&P, p->stream_grid, s);
  if (st) return st;
  if (io->hidden)
    return check_cuda(cudaMemcpyAsync(io->hidden, p->hidden, (size_t)p->T * p->Ht * 2, cudaMemcpyDeviceToDevice, s),
                      "draft: copy hidden");
  return FM_OK;
}

}  // namespace

extern "C" fm_status fm_plan_workspace_size(const fm_model_desc* m, const fm_plan_config* c, size_t* bytes) {
  fm_status st = validate(m, c);
  if (st) return st;
  if (!bytes) return set_error(FM_ERR_INVALID, "plan: null size pointer");
  *bytes = carve(nullptr, m, c, nullptr);
  return FM_OK;
}

extern "C" fm_status fm_plan_create(const fm_model_desc* m, const fm_plan_config* c, void* workspace,
                                    size_t workspace_bytes, fm_plan** out) {
  fm_status st = validate(m, c);
  if (st) return st;
  if (!out) return set_error(FM_ERR_INVALID, "plan: null output");
  const size_t need = carve(nullptr, m, c, nullptr);
  if (!workspace || workspace_bytes < need) return set_error(FM_ERR_WORKSPACE, "plan: workspace of %zu bytes needed", need);
  fm_plan* p = new (std::nothrow) fm_plan();
  if (!p) return set_error(FM_ERR_INVALID, "plan: host allocation failed");
  p->m = *m;
  p->layers.assign(m->layer, m->layer + m->layers);
  p->m.layer = p->layers.data();
  p->cfg = *c;
  p->jumps.assign(c->jumps, c->jumps + c->num_steps);
  p->cfg.jumps = p->jumps.data();
  p->B = c->batch;
  p->K = m->block;
  p->T = p->B * p->K;
  p->D = m->hidden;
  p->H = m->heads;
  p->hd = m->head_dim;
  p->I = m->inter;
  p->L = m->layers;
  p->Ht = m->target_hidden;
  p->S = m->state_vocab;
  p->ctxw = m->n_target_layers * m->target_hidden;
  carve(p, m, c, workspace);
  const int T = p->T, B = p->B, D = p->D, Ht = p->Ht, L = p->L, S = p->S;
  int* gc = p->gemm_counters;
  float* ws = p->gemm_ws;
  int* err = p->err;
  auto fail = [&](fm_status s) {
    delete p;
    return s;
  };
  // anchor path
  if ((st = gemm_prepare(&p->g_anchor_proj, m->anchor_proj_w, D, Ht, Ht, p->anchor_rows, B, Ht, EPI_STORE, ws, gc, err)))
    return fail(st);
  p->g_anchor_proj.args.out = p->anchor_h;
  p->g_anchor_proj.args.ldo = D;
  p->g_anchor_proj.args.bias = static_cast<const __nv_bfloat16*>(m->anchor_proj_b);
  if ((st = gemm_prepare(&p->g_anchor_kv, m->cross_kv_w, (int64_t)L * 2 * D, D, D, p->anchor_ctx, B, D, EPI_KVCACHE, ws,
                         gc, err)))
    return fail(st);
  {
    GemmArgs& a = p->g_anchor_kv.args;
    a.norm_w0 = static_cast<const __nv_bfloat16*>(m->cross_k_norm);
    a.norm_layer_stride = p->hd;
    a.part_rows = D;
    a.head_dim = p->hd;
    a.eps = m->qk_eps;
    a.rope_cos = m->rope_cos;
    a.rope_sin = m->rope_sin;
    a.rope_len = m->rope_len;
    a.positions = p->anchor_pos;
    a.token_seq = p->anchor_seq;
    a.cache = static_cast<__nv_bfloat16*>(c->cache);
    a.cache_batch = c->cache_batch;
    a.cache_heads = p->H;
    a.cache_len = c->cache_len;
  }
  p->has_target = m->embed && m->lm_w && m->chol && m->uniform_embeds;
  // noise path
  if (p->has_target &&
      (st = gemm_prepare(&p->g_zl, m->chol, Ht, Ht, Ht, p->z, T, Ht, EPI_STORE, ws, gc, err)))
    return fail(st);
  p->g_zl.args.out = p->zl;
  p->g_zl.args.ldo = Ht;
  if (c->num_steps > 1 && p->has_target) {
    if ((st = gemm_prepare(&p->g_state_first, m->embed_state_t, Ht, S, S, p->srows, T, S, EPI_STORE, ws, gc, err)))
      return fail(st);
    p->g_state_first.args.out = p->semb;
    p->g_state_first.args.ldo = Ht;
    if ((st = gemm_prepare(&p->g_state_next, m->embed_state_t, Ht, S, S, p->srows, 2 * T, S, EPI_STORE, ws, gc, err)))
      return fail(st);
    p->g_state_next.args.out = p->semb;
    p->g_state_next.args.ldo = Ht;
  }
  if ((st = gemm_prepare(&p->g_xembed, m->x_embed_w, D, Ht, Ht, p->inputs, T, Ht, EPI_STORE, ws, gc, err)))
    return fail(st);
  p->g_xembed.args.out = p->x;
  p->g_xembed.args.ldo = D;
  p->g_xembed.args.bias = static_cast<const __nv_bfloat16*>(m->x_embed_b);
  p->noise_folded = p->has_target && c->num_steps == 1 && m->noise_fold_w && m->noise_fold_var && m->noise_fold_x0;
  if (p->noise_folded) {
    if ((st = gemm_prepare(&p->g_nfold, m->noise_fold_w, D, Ht, Ht, p->z, T, Ht, EPI_STORE, ws, gc, err)))
      return fail(st);
    p->g_nfold.args.out = p->attn;  // free until layer 0's attention
    p->g_nfold.args.ldo = D;
  }
  // layers
  p->g_layer.resize((size_t)L * 6);
  const int64_t mlp1_rows = m->swiglu ? 2 * (int64_t)p->I : p->I;
  for (int l = 0; l < L; ++l) {
    const fm_layer_weights& w = p->layers[l];
    GemmPlan* g = &p->g_layer[(size_t)l * 6];
    if ((st = gemm_prepare(&g[0], w.self_qkv_w, 3 * D, D, D, p->h, T, D, EPI_QKNORM, ws, gc, err))) return fail(st);
    if ((st = gemm_prepare(&g[1], w.self_o_w, D, D, D, p->attn, T, D, EPI_RESID, ws, gc, err))) return fail(st);
    if ((st = gemm_prepare(&g[2], w.cross_q_w, D, D, D, p->h, T, D, EPI_QKNORM, ws, gc, err))) return fail(st);
    if ((st = gemm_prepare(&g[3], w.cross_o_w, D, D, D, p->attn, T, D, EPI_RESID, ws, gc, err))) return fail(st);
    if ((st = gemm_prepare(&g[4], w.mlp_w1, mlp1_rows, D, D, p->h, T, D, m->swiglu ? EPI_SWIGLU : EPI_GELU, ws, gc,
                           err)))
      return fail(st);
    if ((st = gemm_prepare(&g[5], w.mlp_w2, D, p->I, p->I, p->mlp, T, p->I, EPI_RESID, ws, gc, err))) return fail(st);
    for (int q = 0; q < 3; q += 2) {
      GemmArgs& a = g[q].args;
      a.out = q == 0 ? p->qkv : p->qc;
      a.ldo = q == 0 ? 3 * D : D;
      a.norm_w0 = static_cast<const __nv_bfloat16*>(q == 0 ? w.self_q_norm : w.cross_q_norm);
      a.norm_w1 = static_cast<const __nv_bfloat16*>(q == 0 ? w.self_k_norm : nullptr);
      a.part_rows = D;
      a.head_dim = p->hd;
      a.eps = m->qk_eps;
      a.rope_cos = m->rope_cos;
      a.rope_sin = m->rope_sin;
      a.rope_len = m->rope_len;
      a.positions = p->slot_pos;
      a.tok_cos = p->tok_cos;  // filled per draft by draft_prep, per forward by rope_gather
      a.tok_sin = p->tok_sin;
    }
    g[1].args.out = p->x;
    g[1].args.ldo = D;
    g[3].args.out = p->x;
    g[3].args.ldo = D;
    g[4].args.out = p->mlp;
    g[4].args.ldo = p->I;
    g[4].args.bias = static_cast<const __nv_bfloat16*>(w.mlp_b1);
    g[5].args.out = p->x;
    g[5].args.ldo = D;
    g[5].args.bias = static_cast<const __nv_bfloat16*>(w.mlp_b2);
  }
  if ((st = gemm_prepare(&p->g_head, m->head_w, Ht, D, D, p->h, T, D, EPI_STORE, ws, gc, err))) return fail(st);
  p->g_head.args.out = p->hidden;
  p->g_head.args.ldo = Ht;
  p->g_head.args.bias = static_cast<const __nv_bfloat16*>(m->head_b);
  if (p->has_target) {
    if (m->lm_fold_w) {
      // the folded head: final AdaLN output [T, D] times lm_w·head_w [S, D]
      if ((st = gemm_prepare(&p->g_lm, m->lm_fold_w, S, D, D, p->h, T, D, EPI_LOGITS, ws, gc, err)))
        return fail(st);
      p->g_lm.args.bias = static_cast<const __nv_bfloat16*>(m->lm_fold_b);
    } else {
      if ((st = gemm_prepare(&p->g_lm, m->lm_w, S, Ht, Ht, p->hidden, T, Ht, EPI_LOGITS, ws, gc, err)))
        return fail(st);
      p->g_lm.args.bias = static_cast<const __nv_bfloat16*>(m->lm_b);
    }
    p->g_lm.args.argmax_keys = p->keys;
  }
  // the cache as one [rows, head_dim] matrix for the cross-attention TMA
  const uint64_t rows = (uint64_t)L * 2 * c->cache_batch * p->H * c->cache_len;
  if ((st = make_tmap_bf16(&p->cache_map, c->cache, rows, (uint64_t)p->hd, (uint64_t)p->hd, 64))) return fail(st);
  // the streamed pass: asked for (FM_LAUNCH_PERSISTENT), or chosen by FM_LAUNCH_AUTO when its shape fits
  if (stream_shape(m, c) && !p->noise_folded) {
    st = build_stream(p);
    if (st && c->launch_mode == FM_LAUNCH_PERSISTENT) return fail(st);
    if (st) p->stream_on = false;
  } else if (c->launch_mode == FM_LAUNCH_PERSISTENT) {
    return fail(set_error(FM_ERR_UNSUPPORTED, "plan: the streamed pass serves batch-1, one-jump drafts of the "
                                              "unfolded head with head_dim 64 or 128"));
  }
  *out = p;
  return FM_OK;
}

extern "C" fm_status fm_plan_destroy(fm_plan* p) {
  delete p;
  return FM_OK;
}

extern "C" int32_t* fm_plan_error_word(fm_plan* p) { return p ? p->err : nullptr; }

extern "C" int64_t fm_plan_last_launches(const fm_plan* p) { return p ? p->last_launches : -1; }

extern "C" fm_status fm_plan_lm_head(fm_plan* p, void* logits, int64_t ldl, fm_stream stream) {
  if (!p || !p->has_target) return set_error(FM_ERR_INVALID, "lm_head: plan without target");
  GemmPlan lm = p->g_lm;
  lm.args.out = logits ? static_cast<__nv_bfloat16*>(logits) : p->logits_s;
  lm.args.ldo = logits ? ldl : p->S;
  lm.args.scatter = 0;
  lm.args.col_ids = reinterpret_cast<const long long*>(p->m.draft_ids);
  return gemm_launch(lm, static_cast<cudaStream_t>(stream), false);
}

namespace {

// embed: the first layer's input is x_embed(p->inputs) (else p->x is already it)
fm_status run_dit(fm_plan* p, const fm_jump& j, cudaStream_t s, bool with_head = true, bool embed = true) {
  const fm_model_desc& m = p->m;
  const int T = p->T, D = p->D, L = p->L;
  const __nv_bfloat16* mods = static_cast<const __nv_bfloat16*>(j.mods);
  fm_status st;
  if (embed && (st = gemm_launch(p->g_xembed, s, true))) return st;
  for (int l = 0; l < L; ++l) {
    GemmPlan* g = &p->g_layer[(size_t)l * 6];
    const __nv_bfloat16* ms = mods + (size_t)(l * 3 + 0) * 3 * D;
    const __nv_bfloat16* mc = mods + (size_t)(l * 3 + 1) * 3 * D;
    const __nv_bfloat16* mm = mods + (size_t)(l * 3 + 2) * 3 * D;
    if ((st = launch_adaln(p->x, ms, p->h, T, D, m.ln_eps, s, true))) return st;
    if ((st = gemm_launch(g[0], s, true))) return st;
    SelfAttnArgs sa{};
    sa.qkv = p->qkv;
    sa.out = p->attn;
    sa.block = p->K;
    sa.heads = p->H;
    sa.head_dim = p->hd;
    sa.hidden = D;
    sa.scale = (float)(1.0 / std::sqrt((double)p->hd));
    if ((st = launch_self_attn(sa, p->B, s, true))) return st;
    GemmPlan go = g[1];
    go.args.gate = ms + 2 * D;
    if ((st = gemm_launch(go, s, true))) return st;
    if ((st = launch_adaln(p->x, mc, p->h, T, D, m.ln_eps, s, true))) return st;
    if ((st = gemm_launch(g[2], s, true))) return st;
    CrossAttnArgs ca{};
    ca.q = p->qc;
    ca.out = p->attn;
    ca.batch = p->B;
    ca.heads = p->H;
    ca.head_dim = p->hd;
    ca.hidden = D;
    ca.layer = l;
    ca.cache_batch = p->cfg.cache_batch;
    ca.cache_len = p->cfg.cache_len;
    ca.nsplit = p->nsplit;
    ca.scale = sa.scale;
    ca.part = p->xattn_part;
    ca.counters = p->xattn_counters;
    ca.err = p->err;
    ca.lengths = p->anchor_pos;  // lengths[b], as copied by draft_prep
    if ((st = launch_cross_attn(ca, p->cache_map, s, true))) return st;
    GemmPlan gc = g[3];
    gc.args.gate = mc + 2 * D;
    if ((st = gemm_launch(gc, s, true))) return st;
    if ((st = launch_adaln(p->x, mm, p->h, T, D, m.ln_eps, s, true))) return st;
    if ((st = gemm_launch(g[4], s, true))) return st;
    GemmPlan gm = g[5];
    gm.args.gate = mm + 2 * D;
    if ((st = gemm_launch(gm, s, true))) return st;
  }
  const __nv_bfloat16* mf = mods + (size_t)(L * 3) * 3 * D;
  if ((st = launch_adaln(p->x, mf, p->h, T, D, m.ln_eps, s, true))) return st;
  return with_head ? gemm_launch(p->g_head, s, true) : FM_OK;
}

}  // namespace

extern "C" fm_status fm_forward(fm_plan* p, const fm_forward_io* io, fm_stream stream) {
  if (!p || !io || !io->inputs || !io->positions || !io->ctx_last || !io->mods || !io->hidden)
    return set_error(FM_ERR_INVALID, "forward: null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t T = (size_t)p->T;
  fm_status st;
  if ((st = check_cuda(cudaMemcpyAsync(p->inputs, io->inputs, T * p->Ht * 2, cudaMemcpyDeviceToDevice, s),
                       "forward: inputs")) ||
      (st = check_cuda(cudaMemcpyAsync(p->slot_pos, io->positions, T * 4, cudaMemcpyDeviceToDevice, s),
                       "forward: positions")) ||
      (st = check_cuda(cudaMemcpyAsync(p->anchor_pos, io->ctx_last, (size_t)p->B * 4, cudaMemcpyDeviceToDevice, s),
                       "forward: context")))
    return st;
  if ((st = launch_rope_gather(p->slot_pos, (int)T, static_cast<const float*>(p->m.rope_cos),
                               static_cast<const float*>(p->m.rope_sin), p->m.rope_len, p->hd / 2, p->tok_cos,
                               p->tok_sin, p->err, s)))
    return st;
  fm_jump j{};
  j.mods = io->mods;
  if ((st = run_dit(p, j, s))) return st;
  return check_cuda(cudaMemcpyAsync(io->hidden, p->hidden, T * p->Ht * 2, cudaMemcpyDeviceToDevice, s),
                    "forward: hidden");
}

extern "C" fm_status fm_draft(fm_plan* p, const fm_draft_io* io, fm_stream stream) {
  if (!p || !io || !io->anchor_ids || !io->lengths) return set_error(FM_ERR_INVALID, "draft: null argument");
  if (!p->has_target) return set_error(FM_ERR_INVALID, "draft: the plan was built without the target's weights");
  const long long launches0 = launch_counter();
  struct Count {
    fm_plan* p;
    long long l0;
    ~Count() { p->last_launches = launch_counter() - l0; }
  } count{p, launches0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->stream_on) return run_stream(p, io, s);
  const fm_model_desc& m = p->m;
  const int T = p->T, Ht = p->Ht, S = p->S;
  fm_status st;
  DraftPrepArgs pa{};
  pa.anchor_ids = io->anchor_ids;
  pa.lengths = io->lengths;
  pa.embed = static_cast<const __nv_bfloat16*>(m.embed);
  pa.anchor_rows = p->anchor_rows;
  pa.anchor_pos = p->anchor_pos;
  pa.anchor_seq = p->anchor_seq;
  pa.slot_pos = p->slot_pos;
  pa.tok_cos = p->tok_cos;
  pa.tok_sin = p->tok_sin;
  pa.rope_cos = static_cast<const float*>(m.rope_cos);
  pa.rope_sin = static_cast<const float*>(m.rope_sin);
  pa.rope_half = p->hd / 2;
  pa.keys = p->keys;
  pa.B = p->B;
  pa.K = p->K;
  pa.Ht = Ht;
  pa.V = m.vocab;
  pa.rope_len = m.rope_len;
  pa.cache_len = p->cfg.cache_len;
  pa.offset_bump = io->offset_ptr;
  pa.err = p->err;
  if ((st = launch_draft_prep(pa, s, true))) return st;
  if ((st = gemm_launch(p->g_anchor_proj, s, true))) return st;
  if ((st = launch_rmsnorm(p->anchor_h, static_cast<const __nv_bfloat16*>(m.anchor_norm_w), p->anchor_ctx, p->B,
                           p->D, m.rms_eps, s, true)))
    return st;
  if ((st = gemm_launch(p->g_anchor_kv, s, true))) return st;

  const int n = p->cfg.num_steps;
  for (int ji = 0; ji < n; ++ji) {
    const fm_jump& j = p->jumps[ji];
    MixArgs mx{};
    mx.state_norm_w = static_cast<const __nv_bfloat16*>(m.state_norm_w);
    mx.noise_norm_w = static_cast<const __nv_bfloat16*>(m.noise_norm_w);
    mx.out = p->inputs;
    mx.gate = j.noise_gate;
    mx.eps = m.rms_eps;
    mx.T = T;
    mx.Ht = Ht;
    if (n == 1) {
      if (io->z) {
        if ((st = check_cuda(cudaMemcpyAsync(p->z, io->z, (size_t)T * Ht * 2, cudaMemcpyDeviceToDevice, s),
                             "draft: copy z")))
          return st;
      } else if ((st = launch_philox_normal_bf16(p->z, (long long)T * Ht, io->seed, io->offset, io->offset_ptr, s, true))) {
        return st;
      }
      if (p->noise_folded) {
        if ((st = gemm_launch(p->g_nfold, s, true))) return st;
        NoiseFoldArgs nf{};
        nf.proj = p->attn;
        nf.z = p->z;
        nf.var = m.noise_fold_var;
        nf.x0 = static_cast<const __nv_bfloat16*>(m.noise_fold_x0);
        nf.out = p->x;
        nf.gate = j.noise_gate;
        nf.eps = m.rms_eps;
        nf.T = T;
        nf.D = p->D;
        nf.Ht = Ht;
        if ((st = launch_noise_fold(nf, s, true))) return st;
      } else if ((st = gemm_launch(p->g_zl, s, true))) {
        return st;
      }
      mx.post = static_cast<const __nv_bfloat16*>(m.uniform_embeds);
      mx.post_stride = 0;
      mx.state = p->zl;
    } else {
      if (ji == 0) {
        if (io->noise) {
          if ((st = check_cuda(cudaMemcpyAsync(p->state, io->noise, (size_t)T * S * 4, cudaMemcpyDeviceToDevice, s),
                               "draft: copy noise")))
            return st;
        } else if ((st = launch_philox_normal_f32(p->state, (long long)T * S, io->seed, io->offset, io->offset_ptr, s, true))) {
          return st;
        }
      }
      const int with_post = j.s != 0.0f;
      const float c = with_post ? (float)((double)j.s / std::pow(std::fmax(1.0 - (double)j.s, 1e-3), 2.0)) : 0.0f;
      if ((st = launch_state_rows(p->state, p->srows, T, S, c, with_post, s, true))) return st;
      if ((st = gemm_launch(with_post ? p->g_state_next : p->g_state_first, s, true))) return st;
      if (with_post) {
        mx.post = p->semb;
        mx.post_stride = Ht;
        mx.state = p->semb + (size_t)T * Ht;
      } else {
        mx.post = static_cast<const __nv_bfloat16*>(m.uniform_embeds);
        mx.post_stride = 0;
        mx.state = p->semb;
      }
    }
    const bool nfold = n == 1 && p->noise_folded;  // the folded noise wrote layer 0's input
    if (!nfold && (st = launch_mix_state(mx, s, true))) return st;
    const bool last = ji == n - 1;
    // the folded head reads the final AdaLN output; the DiT head then runs only for io->hidden
    const bool folded = m.lm_fold_w != nullptr;
    if ((st = run_dit(p, j, s, !folded || (last && io->hidden), !nfold))) return st;
    GemmPlan lm = p->g_lm;
    lm.args.col_ids = reinterpret_cast<const long long*>(m.draft_ids);  // token ids of the argmax
    if (last && io->logits) {
      lm.args.out = static_cast<__nv_bfloat16*>(io->logits);
      lm.args.ldo = io->ldl;
      lm.args.scatter = (io->scatter && m.draft_ids) ? 1 : 0;
    } else {
      lm.args.out = p->logits_s;
      lm.args.ldo = S;
      lm.args.scatter = 0;
    }
    lm.args.argmax_keys = last ? p->keys : nullptr;
    if ((st = gemm_launch(lm, s, true))) return st;
    if (!last) {
      const double sd = j.s, nd = j.next;
      if ((st = launch_state_update(p->state, p->logits_s, S, T, S, (float)(1.0 - nd), (float)(nd - sd),
                                    (float)(1.0 - sd), s, true)))
        return st;
    }
  }
  if (io->hidden &&
      (st = check_cuda(cudaMemcpyAsync(io->hidden, p->hidden, (size_t)T * Ht * 2, cudaMemcpyDeviceToDevice, s),
                       "draft: copy hidden")))
    return st;
  if (io->tokens && (st = launch_argmax_tokens(p->keys, io->tokens, T, s, true))) return st;
  return FM_OK;
}

extern "C" fm_status fm_extend_context(fm_plan* p, const fm_extend_io* io, fm_stream stream) {
  if (!p || !io || !io->target_hidden || !io->cu_rows || !io->lengths)
    return set_error(FM_ERR_INVALID, "extend_context: null argument");
  if (io->rows <= 0) return FM_OK;
  if (io->rows > p->cfg.max_extend_rows)
    return set_error(FM_ERR_SHAPE, "extend_context: %d rows exceed the plan's %d", io->rows, p->cfg.max_extend_rows);
  if (io->batch <= 0 || io->batch > p->cfg.cache_batch) return set_error(FM_ERR_SHAPE, "extend_context: bad batch");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const fm_model_desc& m = p->m;
  const int D = p->D, L = p->L, R = io->rows;
  fm_status st;
  ExtendPrepArgs ea{};
  ea.cu_rows = io->cu_rows;
  ea.lengths = io->lengths;
  ea.token_seq = p->ext_seq;
  ea.positions = p->ext_pos;
  ea.rows = R;
  ea.B = io->batch;
  ea.rope_len = m.rope_len;
  ea.cache_len = p->cfg.cache_len;
  ea.err = p->err;
  if ((st = launch_extend_prep(ea, s, true))) return st;
  GemmPlan g_fc, g_kv;
  if ((st = gemm_prepare(&g_fc, m.fc_w, D, p->ctxw, p->ctxw, io->target_hidden, R, p->ctxw, EPI_STORE, p->gemm_ws,
                         p->gemm_counters, p->err)))
    return st;
  g_fc.args.out = p->ext_fc;
  g_fc.args.ldo = D;
  if ((st = gemm_launch(g_fc, s, true))) return st;
  if ((st = launch_rmsnorm(p->ext_fc, static_cast<const __nv_bfloat16*>(m.hidden_norm_w), p->ext_ctx, R, D, m.rms_eps,
                           s, true)))
    return st;
  if ((st = gemm_prepare(&g_kv, m.cross_kv_w, (int64_t)L * 2 * D, D, D, p->ext_ctx, R, D, EPI_KVCACHE, p->gemm_ws,
                         p->gemm_counters, p->err)))
    return st;
  {
    GemmArgs& a = g_kv.args;
    a.norm_w0 = static_cast<const __nv_bfloat16*>(m.cross_k_norm);
    a.norm_layer_stride = p->hd;
    a.part_rows = D;
    a.head_dim = p->hd;
    a.eps = m.qk_eps;
    a.rope_cos = m.rope_cos;
    a.rope_sin = m.rope_sin;
    a.rope_len = m.rope_len;
    a.positions = p->ext_pos;
    a.token_seq = p->ext_seq;
    a.cache = static_cast<__nv_bfloat16*>(p->cfg.cache);
    a.cache_batch = p->cfg.cache_batch;
    a.cache_heads = p->H;
    a.cache_len = p->cfg.cache_len;
  }
  if ((st = gemm_launch(g_kv, s, true))) return st;
  return launch_extend_commit(io->cu_rows, io->lengths, io->batch, s, true);
}
