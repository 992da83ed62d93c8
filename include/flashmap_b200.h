/*
 * flashmap_b200 — C ABI of the B200 (sm_100a) FlashMap drafter hot path.
 *
 * The reference (al-jshen/flashmap v0.2.1) is pure Python; its hot path is
 * FlashMapDraftModel.draft()/forward()/extend_context() and the acceptance
 * block of spec_generate() in flashmap/modeling_flashmap.py, plus the
 * torch.library operators of its serving plugins.  Each entry point below
 * names the reference interface it replaces.
 *
 * Conventions
 *   - Every function returns fm_status (0 = FM_OK).  fm_last_error() gives a
 *     thread-local message for the last failure.  Nothing aborts or traps;
 *     device-side problems (an index out of range, a wait that ran out) are
 *     written to the caller's int32 error word, read back with the stream
 *     synchronised.
 *   - The caller owns all memory: weights, caches, workspaces and outputs
 *     are device pointers it allocated.  No entry point allocates device
 *     memory; plans hold host memory only (TMA descriptors, sizes).
 *   - All kernels run on the given CUDA stream (0 = legacy default) with no
 *     host synchronisation, so sequences of calls can be captured in a CUDA
 *     graph.  Per-step values that change between replays (anchor ids,
 *     cache lengths) are read from device memory.
 *   - Tensors are row-major and contiguous unless a leading dimension is
 *     given.  bf16 = 16-bit bfloat16 stored as uint16_t.
 */
#ifndef FLASHMAP_B200_H_
#define FLASHMAP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FM_API __attribute__((visibility("default")))
#else
#define FM_API
#endif

typedef int fm_status;
enum {
  FM_OK = 0,
  FM_ERR_INVALID = 1,     /* null pointer / bad argument */
  FM_ERR_SHAPE = 2,       /* unsupported or inconsistent shape */
  FM_ERR_ALIGN = 3,       /* pointer or stride misaligned for TMA (16 bytes) */
  FM_ERR_ARCH = 4,        /* device is not sm_100 */
  FM_ERR_LAUNCH = 5,      /* kernel launch failed */
  FM_ERR_CUDA = 6,        /* other CUDA runtime error */
  FM_ERR_UNSUPPORTED = 7, /* configuration outside what the kernels serve */
  FM_ERR_WORKSPACE = 8    /* workspace too small */
};

typedef void* fm_stream; /* cudaStream_t */

FM_API const char* fm_last_error(void);
FM_API int fm_version(void);
/* 0 when the current device is an sm_100 part this library was built for. */
FM_API fm_status fm_check_device(void);

/* ------------------------------------------------------------------------
 * Primitive operators (unit-test entry points and building blocks).
 * ------------------------------------------------------------------------ */

/* Epilogue selectors of fm_gemm_bf16. */
enum {
  FM_EPI_STORE = 0, /* out = bf16(X W^T + bias) */
  FM_EPI_GELU = 1,  /* out = bf16(gelu(bf16(X W^T + bias))) */
  FM_EPI_SWIGLU = 2,/* W rows interleaved per 128 (64 gate, 64 up): out = bf16(bf16(silu(g)) * u) */
  FM_EPI_RESID = 3, /* out += bf16(gate * bf16(X W^T + bias)) (in place, bf16 rounding per op) */
  FM_EPI_F32 = 7    /* out (fp32) = X W^T */
};

/* Y = X W^T with a fused epilogue, on tcgen05 tensor cores.
 * Replaces the nn.Linear calls of modeling_flashmap.py (:89-90, 105,
 * 129-132, 159-163, 250-264) and F.linear of the LM head (:475).
 *   W   [M, K] bf16 (nn.Linear layout), X [N, K] bf16 (tokens), K % 8 == 0
 *   out [N, ldo] bf16 (fp32 for FM_EPI_F32); bias/gate [M] bf16 or NULL
 *   workspace: fm_gemm_workspace_size() bytes, laid out as 256 reserved
 *   bytes, then one int32 counter per output tile of 128 rows (zero before the
 *   first call, left zero by every call that completes), then the split-K
 *   partials.  A split tile's head CTA waits for its contributors' count
 *   for at most 2 s; if the count never arrives it records a timeout in
 *   *err (when non-NULL), leaves the tile unwritten and returns. */
FM_API size_t fm_gemm_workspace_size(int64_t M, int64_t N, int64_t K);
FM_API fm_status fm_gemm_bf16(const void* W, const void* X, void* out, int64_t M, int64_t N, int64_t K, int64_t ldo,
                       const void* bias, const void* gate, int epilogue, void* workspace, size_t workspace_bytes,
                       int32_t* err, fm_stream stream);

/* The CTAs fm_gemm_bf16 launches for a shape (one per SM at most): a
 * caller sizing its own split-K workspace per launch reads it here. */
FM_API int32_t fm_gemm_grid(int64_t M, int64_t N, int64_t K);

/* RMSNorm of modeling_flashmap.py:69-80: y = x * bf16(w * rsqrt(mean(x^2) + eps)). */
FM_API fm_status fm_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t cols, float eps,
                     fm_stream stream);

/* AdaLN of modeling_flashmap.py:112-115 (LayerNorm without affine, then
 * * (1 + scale) + shift, each op rounded to bf16). mod = [scale|shift|gate] x D. */
FM_API fm_status fm_adaln(const void* x, const void* mod, void* y, int64_t rows, int64_t cols, float eps,
                   fm_stream stream);

/* RoPE tables of modeling_flashmap.py:53-58: cos/sin[pos][i] of the fp32 angle pos * inv_freq[i],
 * inv_freq [head_dim/2] = 1 / theta^(2i/head_dim) as the reference computes it (fp32). */
FM_API fm_status fm_rope_table(float* cos_out, float* sin_out, int64_t max_pos, int64_t head_dim,
                               const float* inv_freq, fm_stream stream);

/* Philox4x32-10 standard normals (Box-Muller) rounded to bf16: the draft noise z
 * of modeling_flashmap.py:465.  Elements 2p and 2p+1 use counter (p, 0, offset, 4). */
FM_API fm_status fm_philox_normal(void* out, int64_t count, uint64_t seed, uint32_t offset, fm_stream stream);

/* Seeded draft noise of the serving plugins (vllm/kernels.py:367-414): row r holds n_cols
 * bf16 standard normals times scale, keyed by seed seeds[rows[r]] (0 when rows[r] < 0) and
 * Philox counter offset positions[r], so a seeded request draws the same noise whatever is
 * batched with it.  rows, seeds and positions are int64. */
FM_API fm_status fm_philox_normal_rows(void* out, int64_t n_rows, int64_t n_cols, const int64_t* seeds,
                                       const int64_t* rows, const int64_t* positions, float scale, fm_stream stream);

/* fp32 form of fm_philox_normal_rows (the vocabulary-sized starting state of a
 * multi-jump draft, vllm/model.py:968-975). */
FM_API fm_status fm_philox_normal_rows_f32(float* out, int64_t n_rows, int64_t n_cols, const int64_t* seeds,
                                           const int64_t* rows, const int64_t* positions, float scale,
                                           fm_stream stream);

/* Multi-jump state featurisation rows (modeling_flashmap.py:378-391,
 * vllm/model.py:944-956): for rows t of the fp32 state [rows, cols], out gets
 * bf16(state) at row rows + t and, with with_posterior, bf16(softmax(evidence *
 * state)) at row t (fixed-order max and sum); without, bf16(state) at row t.
 * out [rows or 2*rows, cols] is the GEMM operand against E_S^T. */
FM_API fm_status fm_state_rows(const float* state, void* out, int64_t rows, int64_t cols, float evidence,
                               int32_t with_posterior, fm_stream stream);

/* Jump update (modeling_flashmap.py:470-472): state = (keep * state + step *
 * softmax(logits)) / denom per row, logits bf16 [rows, ldl] (first cols used). */
FM_API fm_status fm_state_update(float* state, const void* logits, int64_t ldl, int64_t rows, int64_t cols,
                                 float keep, float step, float denom, fm_stream stream);

/* ---------------------------------------------------------------- banked jumps
 * The sglang plugin's multi-jump draft without vocabulary-sized states
 * (flashmap/sglang/jump_bank.py).  A bank row holds, for one draw z of the
 * starting noise, z @ E and per later jump n softmax(a_n z) @ E and
 * logsumexp(a_n z); a draft reads only the embedding rows of the earlier
 * predictions' top-k support. */

/* One chunk of bank draws (jump_bank.py:124-150): z [rows, cols] fp32 (the
 * temperature applied) -> z_bf16 [rows, cols], and per slope a_j (n_slopes <= 8,
 * host array) probs[j] = bf16(softmax(a_j z)) [n_slopes, rows, cols] and
 * log_mass[j] = logsumexp(a_j z) [n_slopes, rows] fp32. */
FM_API fm_status fm_bank_rows(const float* z, void* z_bf16, void* probs, float* log_mass, int64_t rows,
                              int64_t cols, const float* slopes, int32_t n_slopes, fm_stream stream);

/* A jump's prediction (jump_bank.py:89-92): per row of bf16 logits [rows, ld],
 * the top k (1..32; larger value first, then smaller index) as ids (the
 * column, or row_map[column] when row_map [map_len] is given) and their
 * probabilities under the row's full fp32 softmax. ids [rows, k] int64,
 * probs [rows, k] fp32; err (optional) records an out-of-range map index. */
FM_API fm_status fm_topk_rows(const void* logits, int64_t ld, int64_t rows, int64_t cols, int32_t k,
                              const int64_t* row_map, int64_t map_len, int64_t* ids, float* probs, int32_t* err,
                              fm_stream stream);

/* out[i] = table[rows[i]] (bf16 rows of cols); an out-of-range row is
 * recorded in err (optional) and gives zeros. */
FM_API fm_status fm_bank_gather(const void* table, int64_t table_rows, int64_t cols, const int64_t* rows,
                                int64_t n, void* out, int32_t* err, fm_stream stream);

/* A later jump n's state rows per slot (jump_bank.py:171-205), before the
 * norms: out rows [0, slots) the posterior (mean_embed[row] + sum_v
 * bf16(r_v) E_v) / (1 + sum_v r_v), rows [slots, 2 slots) the noise term
 * alpha noise_embed[row] + sum_v bf16(beta delta_v) E_v, both bf16; with
 * r_v = exp(slope z_v - log_mass[row]) expm1(evidence c_v) on each distinct
 * support token (c_v its summed prediction weight, z_v = temperature *
 * normal(seed, v)).  The support is the earlier predictions' top-k
 * concatenated: ids [slots, support] state rows, probs [slots, support],
 * betas [support / topk]. */
typedef struct fm_bank_jump {
  const void* noise_embed;  /* [bank_rows, hidden] bf16 */
  const void* mean_embed;   /* [bank_rows, hidden] bf16, this jump's */
  const float* log_mass;    /* [bank_rows] fp32, this jump's */
  const void* embed;        /* embedding rows [*, hidden] bf16 */
  const int64_t* state_map; /* [state_rows] state row -> embed row, or NULL (identity) */
  int64_t bank_rows, state_rows, hidden, slots;
  const int64_t* rows;      /* [slots] bank rows */
  const int64_t* seeds;     /* [slots] slot seeds */
  const int64_t* ids;       /* [slots, support] */
  const float* probs;       /* [slots, support] */
  const float* betas;       /* [support / topk] */
  int32_t support, topk;
  float alpha, evidence, slope, temperature;
  void* out;                /* [2 slots, hidden] bf16 */
  int32_t* err;             /* optional: out-of-range rows / ids */
} fm_bank_jump;
FM_API fm_status fm_bank_jump_rows(const fm_bank_jump* args, fm_stream stream);

/* The per-(seed, token) standard normals of the support (jump_bank.py:62-73):
 * out[r, l] = normal(seeds[r], ids[r, l]), fp32 [rows, cols]. */
FM_API fm_status fm_token_normals(const int64_t* seeds, const int64_t* ids, int64_t rows, int64_t cols,
                                  float* out, fm_stream stream);

/* out[i] = floor(u_i * high), u_i a Philox4x32-10 uniform of counter
 * (i, offset, purpose) under seed; 1 <= high <= 2^32 - 1 (bank rows, slot seeds). */
FM_API fm_status fm_philox_randint(int64_t* out, int64_t n, int64_t high, uint64_t seed, uint32_t offset,
                                   uint32_t purpose, fm_stream stream);

/* ---------------------------------------------------------------- tree drafting
 * The verify tree of N candidate blocks per request (flashmap/sglang/tree.py:9-78,
 * build_tree_abi): per request, the trie of candidates [bs, N, K] int64 (a
 * node per distinct prefix, voted by the candidates through it), its
 * width - 1 best-voted nodes (ties: shallower, then lower candidate) listed by
 * depth then candidate: tokens [bs, width - 1], ids [bs, width - 1] = parent *
 * width + index (root 0; a trie with fewer nodes is padded with copies of the
 * first node under the root), stats [bs, 2] = (trie nodes, distinct
 * candidates), all int64.  N <= 64, K <= 64, N * K <= 1024. */
FM_API fm_status fm_tree_build(const int64_t* candidates, int64_t bs, int64_t n, int64_t k, int64_t width,
                               int64_t* tokens, int64_t* ids, int64_t* stats, fm_stream stream);

/* Commit of the accepted tree paths (flashmap/sglang/kernels.py:363-454,
 * tree_commit): accept [bs, depth1] int32 global node ids of the path (root
 * first, -1 past it), num_correct [bs] int32, window [bs, width] int64 KV slots,
 * predict [bs * width] int32 (the target's token after each node), req_pool /
 * prefix [bs] int64; req_to_token [req_rows, row_stride] int32 gets the path's
 * slots first, then the other nodes' in index order, from column prefix.
 * Returns out_tokens [bs, depth1] int64, bonus [bs] int64, commit [bs] int32 =
 * n + 1, new_seq_lens [bs] int64 = prefix + n + 1, inject_locs [bs * width]
 * int64 (the path's slots, 0 elsewhere); err (optional) records an index out
 * of range (the write is skipped). */
FM_API fm_status fm_tree_commit(const int32_t* accept, const int32_t* num_correct, const int64_t* window,
                                const int32_t* predict, const int64_t* req_pool, const int64_t* prefix,
                                int32_t* req_to_token, int64_t row_stride, int64_t req_rows, int64_t bs,
                                int64_t width, int64_t depth1, int64_t* out_tokens, int64_t* bonus, int32_t* commit,
                                int64_t* new_seq_lens, int64_t* inject_locs, int32_t* err, fm_stream stream);

/* One-jump input mix (modeling_flashmap.py:393-399): out = bf16(state_norm(post) +
 * bf16(gate * noise_norm(state))), post rows post_stride apart (0: one shared row). */
FM_API fm_status fm_mix_state(const void* post, int64_t post_stride, const void* state, const void* state_norm_w,
                              const void* noise_norm_w, void* out, float gate, float eps, int64_t rows, int64_t cols,
                              fm_stream stream);

/* Eigen-folded noise, first layer input (sglang/model.py:945-958): per row t,
 * scale = gate * rsqrt(sum_i var_i z[t,i]^2 + eps) and out[t] = bf16(x0 +
 * bf16(scale * proj[t])); proj [rows, cols] = z [rows, noise_cols] times the
 * fold weight (fm_model_desc.noise_fold_w), var [noise_cols] fp32, x0 [cols]. */
FM_API fm_status fm_noise_fold(const void* proj, const void* z, const float* var, const void* x0, void* out,
                               float gate, float eps, int64_t rows, int64_t cols, int64_t noise_cols,
                               fm_stream stream);

/* Self-attention over the block slots (modeling_flashmap.py:188 with :144-147);
 * qkv [B*K, 3*D] with q, k already normed and rotated. Replaces the
 * flashmap_vllm::block_self_attention / flashmap_sglang::block_self_attention ops. */
FM_API fm_status fm_block_self_attn(const void* qkv, void* out, int64_t batch, int64_t block, int64_t heads,
                             int64_t head_dim, fm_stream stream);

/* Cross-attention of the 16 block slots of each sequence over its context cache
 * positions 0..lengths[b] (modeling_flashmap.py:190, :218-219).  Replaces
 * flashmap_vllm::paged_cross_attention (vllm/model.py:93) for a dense cache.
 *   cache (L, 2, cache_batch, heads, cache_len, head_dim) bf16; q/out [B*16, heads*head_dim]
 *   workspace: fm_cross_attn_workspace_size() bytes (counters zero). */
FM_API size_t fm_cross_attn_workspace_size(int64_t batch, int64_t heads, int64_t head_dim, int64_t nsplit);
FM_API fm_status fm_cross_attn(const void* q, const void* cache, void* out, const int32_t* lengths, int64_t batch,
                        int64_t heads, int64_t head_dim, int64_t layers, int64_t layer, int64_t cache_batch,
                        int64_t cache_len, int64_t nsplit, void* workspace, size_t workspace_bytes, int32_t* err,
                        fm_stream stream);

/* ------------------------------------------------------------------------
 * Operators of the serving plugins (flashmap/vllm/kernels.py,
 * flashmap/vllm/model.py:93, flashmap/sglang/kernels.py,
 * flashmap/sglang/model.py:127-178, :728-766): q/k RMSNorm + interleaved
 * RoPE, block self-attention from raw qkv, cross-attention over paged KV
 * caches (bf16 or e4m3), and the writers of context keys/values into paged
 * caches.  The torch.library ops of flashmap_b200.serving_ops call these.
 * ------------------------------------------------------------------------ */

/* Element types of operator arguments. */
enum { FM_DT_BF16 = 0, FM_DT_F32 = 1, FM_DT_E4M3 = 2, FM_DT_I32 = 3, FM_DT_I64 = 4 };

/* RMSNorm rounding: FM_NORM_DIT is the DiT's x * bf16(w * rsqrt(mean(x^2) + eps))
 * (modeling_flashmap.py:69-80, vllm/kernels.py:38-46); FM_NORM_FUSED is
 * bf16(x * rsqrt(mean(x^2) + eps) * w), the context writer of an e4m3 pool
 * (sglang/kernels.py:309-311). */
enum { FM_NORM_DIT = 0, FM_NORM_FUSED = 1 };

/* A rotary table: cos(p, i) = cos[p * row_stride + i * pair_stride] (fp32), sin
 * likewise, for positions p < rows and pairs i < head_dim / 2.  The vLLM table
 * (positions, hd/2, [cos, sin]) is {t, t + 1, hd, 2}; sglang's per-token freqs
 * are the same with the token index as position; sglang's writer table
 * (positions, [cos | sin]) is {t, t + hd/2, hd, 1}. */
typedef struct fm_rope_view {
  const float* cos;
  const float* sin;
  int64_t row_stride;
  int64_t pair_stride;
  int64_t rows;
} fm_rope_view;

/* RMSNorm then interleaved RoPE of rows x[t, h, :] (rows of head_dim bf16,
 * heads contiguous, tokens x_token_stride apart) into out (out_token_stride).
 * The rotary row of token t is positions[t] (int32 or int64), or t when
 * positions is NULL.  Replaces flashmap_vllm::rms_norm_rope (vllm/kernels.py:100)
 * and flashmap_sglang::rms_norm_rope (sglang/kernels.py:170).  weight is
 * head_dim values, bf16 or fp32. */
FM_API fm_status fm_qk_norm_rope(const void* x, int64_t x_token_stride, void* out, int64_t out_token_stride,
                                 int64_t tokens, int64_t heads, int64_t head_dim, const void* weight,
                                 int32_t weight_dtype, fm_rope_view rope, const void* positions,
                                 int32_t positions_dtype, float eps, int32_t norm_mode, int32_t* err,
                                 fm_stream stream);

/* Block self-attention from projected qkv (blocks, block, 3, heads, head_dim):
 * q and k RMSNorm (FM_NORM_DIT) and RoPE at positions[blocks * block] (or the
 * token index when NULL), unmasked softmax attention with the given scale,
 * out (blocks * block, heads * head_dim).  One kernel; block == 16 and
 * head_dim 64 or 128 (FM_ERR_UNSUPPORTED otherwise: compose fm_qk_norm_rope
 * and fm_block_self_attn).  Replaces flashmap_vllm::block_self_attention
 * (vllm/kernels.py:193) and flashmap_sglang::block_self_attention
 * (sglang/kernels.py:84). */
FM_API fm_status fm_block_self_attn_qknorm(const void* qkv, void* out, int64_t blocks, int64_t block, int64_t heads,
                                           int64_t head_dim, const void* q_norm, const void* k_norm,
                                           int32_t weight_dtype, fm_rope_view rope, const void* positions,
                                           int32_t positions_dtype, float eps, float scale, int32_t* err,
                                           fm_stream stream);

/* Non-causal attention of each request's query rows onto the first
 * seqused_k[r] positions of its paged context.  Position p of request r is
 * row (p % page_size) of page page_table[r * page_table_stride + p / page_size];
 * its key is k + page * kv_page_stride + head * kv_head_stride +
 * (p % page_size) * kv_token_stride (elements), its value the same offset from
 * v.  The vLLM FlashAttention cache (pages, heads, page, 2 * hd) is k = cache,
 * v = cache + hd; sglang's pools (rows, heads, hd) are page_size 1.
 * Query rows of request r: cu_seqlens_q[r] .. cu_seqlens_q[r + 1] - 1, or
 * q_per_request rows from r * q_per_request when cu_seqlens_q is NULL.
 * e4m3 caches: scores and outputs are descaled by descales (3, requests, heads)
 * (query, key, value), or, with quantize_q, the bf16 query is quantised to
 * e4m3 per (request, head) with scale amax / 448 (sglang/model.py:164-170).
 * A request with no positions gets zero output rows.
 * Replaces flashmap_vllm::paged_cross_attention (vllm/model.py:93-132),
 * flashmap_sglang::paged_cross_attention[_fp8] (sglang/model.py:127-175). */
typedef struct fm_paged_attn {
  const void* q;
  int32_t q_dtype; /* FM_DT_BF16 or FM_DT_E4M3 */
  int64_t q_token_stride, q_head_stride;
  const int32_t* cu_seqlens_q;
  int64_t q_per_request;
  int64_t max_q; /* the most query rows of one request */
  const void* k;
  const void* v;
  int32_t kv_dtype; /* FM_DT_BF16 or FM_DT_E4M3 */
  int64_t kv_page_stride, kv_head_stride, kv_token_stride;
  int64_t page_size, num_pages;
  const int32_t* page_table;
  int64_t page_table_stride, page_table_cols;
  const int32_t* seqused_k;
  int64_t max_seqlen_k;
  int64_t requests, heads, head_dim;
  float softmax_scale;
  const float* descales; /* (3, requests, heads) or NULL */
  int32_t quantize_q;
  void* out; /* bf16 */
  int64_t out_token_stride, out_head_stride;
  void* workspace; /* fm_paged_attn_workspace_size() bytes, zero on first use */
  size_t workspace_bytes;
  int32_t nsplit; /* key splits per (request, head, 16 query rows); 0 = choose */
  int32_t* err;
} fm_paged_attn;
FM_API int32_t fm_paged_attn_nsplit(int64_t requests, int64_t heads, int64_t max_q, int64_t max_seqlen_k,
                                    int32_t nsplit);
FM_API size_t fm_paged_attn_workspace_size(int64_t requests, int64_t heads, int64_t head_dim, int64_t max_q,
                                           int32_t nsplit);
FM_API fm_status fm_paged_cross_attn(const fm_paged_attn* args, fm_stream stream);

/* Every layer's context keys (k-normed FM_NORM_DIT, rotated at positions[t])
 * and values of kv (tokens, layers, 2, heads, head_dim) bf16 into paged caches
 * at slots[t] (negative: skipped).  Head g = layer * heads + h goes to cache
 * g / heads_per_cache, head slot g % heads_per_cache; element strides (block,
 * head, token) and the value offset are those of the vLLM FlashAttention cache,
 * the same for every cache; cache_ptrs is a device array of num_caches data
 * pointers.  With scales (layers, 2) fp32 the caches are e4m3 and hold key /
 * k_scale and value / v_scale.  Replaces write_context_kv (vllm/kernels.py:311). */
FM_API fm_status fm_write_context_kv_paged(const void* kv, int64_t tokens, int64_t layers, int64_t heads,
                                           int64_t head_dim, const int64_t* positions, const int64_t* slots,
                                           const void* k_norm, int32_t k_norm_dtype, fm_rope_view rope,
                                           const int64_t* cache_ptrs, int64_t num_caches, int64_t heads_per_cache,
                                           int64_t stride_block, int64_t stride_head, int64_t stride_token,
                                           int64_t v_offset, int64_t block_size, float eps, const float* scales,
                                           int32_t* err, fm_stream stream);

/* sglang's context writer: kv (tokens, layers, 2, kv_size) bf16 with kv_size =
 * heads * head_dim; per layer meta (layers, 4) int64 = (key pool pointer, value
 * pool pointer, key row stride, value row stride) in elements; keys
 * k-normed (norm_mode: FM_NORM_FUSED is the reference's e4m3 writer,
 * FM_NORM_DIT the HF path's k_norm) and rotated at positions[t], written with values
 * at pool row locs[t] (negative: skipped).  With commit_lens (rows of
 * locs_row_width tokens), token t is written only when t % locs_row_width <
 * commit_lens[t / locs_row_width].  pool_dtype FM_DT_E4M3 divides keys by
 * k_scale and values by v_scale.  Replaces kv_norm_rope_write_fp8
 * (sglang/kernels.py:284-331) and, for bf16 pools, the fused writer sglang/model.py:746-766 calls. */
FM_API fm_status fm_kv_norm_rope_write_pool(const void* kv, int64_t tokens, int64_t layers, int64_t kv_size,
                                            int64_t head_dim, const int64_t* meta, const void* k_norm,
                                            int32_t k_norm_dtype, fm_rope_view rope, const int64_t* positions,
                                            const int64_t* locs, const int32_t* commit_lens, int64_t locs_row_width,
                                            int32_t pool_dtype, int32_t norm_mode, float k_scale, float v_scale,
                                            float eps, int32_t* err, fm_stream stream);

/* ------------------------------------------------------------------------
 * Sampling and acceptance (modeling_flashmap.py:553-557, :579-594).
 * Randomness: Philox4x32-10 keyed by seed; counters documented per call.
 * ------------------------------------------------------------------------ */

/* Logit rows may be bf16 (logits_dtype 0) or fp32 (logits_dtype 1). */

/* Per-row max m and sum of exp(x/T - m) (fixed reduction order) and the first
 * argmax of logit rows. stats [rows][2] fp32, argmax [rows] int64 (either may be NULL).
 * V < 2^31 (else FM_ERR_SHAPE). */
FM_API fm_status fm_row_stats(const void* logits, int32_t logits_dtype, int64_t rows, int64_t V, float temperature,
                              float* stats, int64_t* argmax, fm_stream stream);

/* probs = softmax(logits / T) in fp32, rows of V < 2^31 (draft_probs of :556). */
FM_API fm_status fm_softmax_rows(const void* logits, int32_t logits_dtype, int64_t rows, int64_t V,
                                 float temperature, float* probs, fm_stream stream);

/* Draft tokens: T <= 0 argmax of logits; else a categorical draw from probs (row r = b*K + k
 * uses uniform counter (k, b, offset, 3)). tokens [B*K] int64. */
FM_API fm_status fm_sample_rows(const void* logits, int32_t logits_dtype, const float* probs, int64_t B, int64_t K,
                                int64_t V, float temperature, uint64_t seed, uint32_t offset, int64_t* tokens,
                                fm_stream stream);

/* Greedy acceptance (:579-582). target_logits [B, K+1, V], draft [B, K] int64
 * -> accepted [B], bonus [B] (int64). */
FM_API size_t fm_accept_workspace_size(int64_t B, int64_t K);
FM_API fm_status fm_accept_greedy(const void* target_logits, int32_t logits_dtype, const int64_t* draft, int64_t B,
                                  int64_t K, int64_t V, int64_t* accepted, int64_t* bonus, void* workspace,
                                  size_t workspace_bytes, fm_stream stream);

/* Greedy acceptance like fm_accept_greedy, for callers that cannot allocate
 * device memory at this point (an engine that plans all buffers before
 * capturing its decode step in a CUDA graph; host code in another language
 * that only holds the tensors it was given).  No counterpart in the reference:
 * its per-row argmax scratch is a fixed array inside the library, so
 * B*(K+1) may not exceed FM_ACCEPT_NOALLOC_MAX_ROWS (larger calls return
 * FM_ERR_WORKSPACE).  The array is shared by all calls on a device and keeps
 * the last call's contents; calls that overlap on the GPU race on it.  The
 * first call on each device looks the array's address up (make it before any
 * stream capture); no call allocates or frees memory. */
#define FM_ACCEPT_NOALLOC_MAX_ROWS 16384
FM_API fm_status fm_accept_greedy_noalloc(const void* target_logits, int32_t logits_dtype, const int64_t* draft,
                                          int64_t B, int64_t K, int64_t V, int64_t* accepted, int64_t* bonus,
                                          fm_stream stream);

/* Rejection acceptance (:583-594). q [B, K, V] fp32 draft probabilities.
 * u[b,k] = uniform (k, b, offset, 1); bonus draw uniform (0, b, offset, 2),
 * a sliced categorical draw (slices of 256 ranges of 32 weights, their totals
 * summed in slice order; V <= 256 * 8192). */
FM_API fm_status fm_accept_rejection(const void* target_logits, int32_t logits_dtype, const int64_t* draft,
                                     const float* q, int64_t B, int64_t K, int64_t V, float temperature,
                                     uint64_t seed, uint32_t offset, int64_t* accepted, int64_t* bonus,
                                     void* workspace, size_t workspace_bytes, fm_stream stream);

/* Helpers of the one-time constants (time conditioning, embedding transpose). */
FM_API fm_status fm_transpose_bf16(const void* in, void* out, int64_t rows, int64_t cols, fm_stream stream);
/* rows 0 and 1: bf16 [cos | sin] of the fp32 arguments (s resp. t) * scale * freqs[i], i < dim/2,
 * with freqs = exp(-ln(10000) i / (dim/2)) as the reference computes it (modeling_flashmap.py:92-96). */
FM_API fm_status fm_time_sinusoid(void* out, int64_t dim, float s, float t, float scale, const float* freqs,
                                  fm_stream stream);
FM_API fm_status fm_silu(const void* x, void* y, int64_t n, fm_stream stream);
FM_API fm_status fm_add(const void* a, const void* b, void* y, int64_t n, fm_stream stream);

/* ------------------------------------------------------------------------
 * The whole drafter: a plan over caller-owned weights and buffers.
 * ------------------------------------------------------------------------ */

typedef struct fm_layer_weights {
  const void* self_qkv_w;  /* [3D, D]: q_proj; k_proj; v_proj rows */
  const void* self_o_w;    /* [D, D] */
  const void* self_q_norm; /* [hd] */
  const void* self_k_norm; /* [hd] */
  const void* cross_q_w;   /* [D, D] */
  const void* cross_o_w;   /* [D, D] */
  const void* cross_q_norm;/* [hd] */
  const void* mlp_w1;      /* gelu: fc1 [I, D]; swiglu: gate_up [2I, D] interleaved per 64 rows */
  const void* mlp_b1;      /* gelu: fc1 bias [I]; swiglu: NULL */
  const void* mlp_w2;      /* fc2 / down_proj [D, I] */
  const void* mlp_b2;      /* fc2 bias [D] or NULL */
} fm_layer_weights;

typedef struct fm_model_desc {
  int32_t hidden, heads, head_dim, inter, layers, target_hidden, n_target_layers, block;
  int32_t vocab;       /* target vocabulary V */
  int32_t state_vocab; /* S: rows of lm_head/embedding the state lives on (= V without draft_ids) */
  int32_t swiglu;      /* 0 gelu, 1 swiglu */
  float rms_eps, qk_eps, ln_eps;
  const void* fc_w;          /* [D, n_target_layers*Ht] */
  const void* hidden_norm_w; /* [D] */
  const void* anchor_proj_w; /* [D, Ht] */
  const void* anchor_proj_b; /* [D] */
  const void* anchor_norm_w; /* [D] */
  const void* noise_norm_w;  /* [Ht] */
  const void* x_embed_w;     /* [D, Ht] */
  const void* x_embed_b;     /* [D] */
  const void* head_w;        /* [Ht, D] */
  const void* head_b;        /* [Ht] */
  const void* cross_kv_w;    /* [L*2*D, D]: per layer cross k_proj then v_proj */
  const void* cross_k_norm;  /* [L, hd] */
  const fm_layer_weights* layer; /* host array of L entries */
  /* the target's side; all NULL for a plan that only runs extend_context / forward */
  const void* embed;         /* target embedding [V, Ht] */
  const void* lm_w;          /* state-vocab rows of the target lm_head [S, Ht] */
  const void* lm_b;          /* [S] or NULL */
  const int64_t* draft_ids;  /* [S] ids into V, or NULL (S == V) */
  const void* embed_state_t; /* E_S^T [Ht, S] (multi-step drafts), or NULL */
  const void* chol;          /* L with L L^T = E_S^T E_S, [Ht, Ht] lower triangular */
  const void* uniform_embeds;/* bf16(1/S) summed over E_S rows: the s = 0 posterior embedding [Ht] */
  const void* state_norm_w;  /* [Ht] */
  const float* rope_cos;     /* [rope_len, hd/2] */
  const float* rope_sin;
  int32_t rope_len;
  /* Optional fast mode (the serving plugins' folded head, vllm/fold.py:76-100,
   * sglang/model.py:515-531): lm_w rows x head_w as one [S, D] weight and its
   * [S] bias (bf16 of the fp32 products).  When set, fm_draft's logits are
   * the final AdaLN output times this weight — the DiT head is skipped (it
   * still runs when fm_draft_io.hidden asks for the head output).  It changes
   * rounding, so it sits outside parity with the reference's HF path. */
  const void* lm_fold_w;
  const void* lm_fold_b;
  /* Optional fast mode (the serving plugins' eigen-folded noise,
   * vllm/fold.py:44-73, sglang/model.py:576-595), one-jump drafts only.
   * With E_S^T E_S = Q diag(lam) Q^T: noise_fold_w = W_x diag(w_noise) Q
   * diag(sqrt lam) [D, Ht] (bf16), noise_fold_var = lam / Ht [Ht] (fp32),
   * noise_fold_x0 = x_embed(state_norm(uniform_embeds)) [D] (bf16).  When all
   * three are set, a one-jump fm_draft forms the first layer's input as
   * x0 + bf16(gate * rsqrt(sum(var z^2) + rms_eps) * bf16(z noise_fold_w^T))
   * in place of x_embed(state_norm(u) + gate * noise_norm(z chol^T)): the
   * same distribution from other draws, so outside parity with the HF path.
   * Multi-jump drafts ignore these. */
  const void* noise_fold_w;
  const float* noise_fold_var;
  const void* noise_fold_x0;
} fm_model_desc;

/* One jump of a draft: its modulations and noise-gate value. */
typedef struct fm_jump {
  const void* mods;  /* [(3L+1), 3, D] bf16: per layer (self, cross, mlp), then final; each scale|shift|gate */
  float noise_gate;  /* bf16-rounded noise_gate * (t - s) (or noise_gate for "constant") */
  float s, next;     /* start time and the time the state moves to (next == 1: last jump) */
} fm_jump;

/* How fm_draft launches its work. */
enum {
  FM_LAUNCH_AUTO = 0,       /* the kernel sequence */
  FM_LAUNCH_KERNELS = 1,    /* the kernel sequence: one launch per operation, chained by programmatic
                               dependent launch */
  FM_LAUNCH_PERSISTENT = 2  /* the streamed single-launch pass: one cooperative kernel (one CTA per SM)
                               streams every weight tile through shared memory while the dependent
                               steps follow one another across the grid; batch 1, one jump, the
                               unfolded head, head_dim 64 or 128 (else fm_plan_create returns
                               FM_ERR_UNSUPPORTED) */
};

typedef struct fm_plan_config {
  int32_t batch;        /* sequences drafted together */
  int32_t num_steps;    /* jumps per draft */
  const fm_jump* jumps; /* host array of num_steps entries */
  void* cache;          /* (L, 2, cache_batch, heads, cache_len, hd) bf16 */
  int32_t cache_batch, cache_len;
  int32_t max_extend_rows; /* largest extend_context call (rows over all sequences) */
  int32_t launch_mode;     /* FM_LAUNCH_* */
} fm_plan_config;

typedef struct fm_plan fm_plan;

/* Device workspace the plan needs (bytes). */
FM_API fm_status fm_plan_workspace_size(const fm_model_desc* model, const fm_plan_config* cfg, size_t* bytes);
/* Build a plan over caller-owned memory (host allocation only). The workspace
 * must stay valid for the plan's lifetime; its first bytes must be zero. */
FM_API fm_status fm_plan_create(const fm_model_desc* model, const fm_plan_config* cfg, void* workspace,
                         size_t workspace_bytes, fm_plan** plan);
FM_API fm_status fm_plan_destroy(fm_plan* plan);
/* Device error word of the plan (int32, 0 = none). */
FM_API int32_t* fm_plan_error_word(fm_plan* plan);
/* Kernels launched by the plan's last fm_draft call. */
FM_API int64_t fm_plan_last_launches(const fm_plan* plan);
/* The plan's LM-head GEMM alone (logits + argmax of the plan's current DiT
 * output; state-vocabulary columns), for timing the pass's largest kernel. */
FM_API fm_status fm_plan_lm_head(fm_plan* plan, void* logits, int64_t ldl, fm_stream stream);

typedef struct fm_draft_io {
  const int64_t* anchor_ids; /* [B] device */
  const int32_t* lengths;    /* [B] device: verified positions per sequence */
  const void* z;             /* [B*K, Ht] bf16 one-step noise, or NULL (drawn by Philox) */
  const float* noise;        /* [B*K, S] fp32 multi-step start state, or NULL (drawn) */
  uint64_t seed;
  uint32_t offset;           /* Philox counter word 2 for this draft ... */
  uint32_t* offset_ptr;      /* ... plus this device word when non-NULL; every draft first increments it,
                                so replays of a captured draft draw fresh noise */
  void* logits;              /* [B*K, ldl] bf16 output or NULL */
  int64_t ldl;               /* logits row stride (V, or S when not scattering) */
  int32_t scatter;           /* 1: write at draft_ids columns of a V-wide row */
  int64_t* tokens;           /* [B*K] argmax tokens (target ids) or NULL */
  void* hidden;              /* [B*K, Ht] bf16 DiT output of the last jump, or NULL */
} fm_draft_io;

/* One draft of the whole block (modeling_flashmap.py:422-479): the anchor row
 * of every layer's context, the noise, all jumps of the DiT, the LM head and
 * the argmax.  Replaces FlashMapDraftModel.draft/forward and the plugins'
 * forward + compute_draft_logits (vllm/model.py:991-1045). */
FM_API fm_status fm_draft(fm_plan* plan, const fm_draft_io* io, fm_stream stream);

typedef struct fm_forward_io {
  const void* inputs;        /* [B*K, Ht] bf16 featurised block state */
  const int32_t* positions;  /* [B*K] rotary positions of the slots */
  const int32_t* ctx_last;   /* [B] cross-attention keys are cache positions 0..ctx_last[b] */
  const void* mods;          /* [(3L+1), 3, D] bf16 modulations of the jump */
  void* hidden;              /* [B*K, Ht] bf16 output */
} fm_forward_io;

/* One jump of the DiT on featurised inputs (modeling_flashmap.py:302-313,
 * FlashMapDraftModel.forward): x_embed, the L blocks and the head. */
FM_API fm_status fm_forward(fm_plan* plan, const fm_forward_io* io, fm_stream stream);

typedef struct fm_extend_io {
  const void* target_hidden; /* [rows, n_target_layers*Ht] bf16 */
  int32_t rows;
  const int32_t* cu_rows;    /* [B+1] device: rows of sequence b are cu_rows[b]..cu_rows[b+1] */
  int32_t* lengths;          /* [B] device: rows are written at lengths[b].., then lengths += n_b */
  int32_t batch;
} fm_extend_io;

/* extend_context (modeling_flashmap.py:342-351): fc, hidden_norm, then every
 * layer's cross k (k_norm + RoPE) and v written into the cache. */
FM_API fm_status fm_extend_context(fm_plan* plan, const fm_extend_io* io, fm_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHMAP_B200_H_ */
