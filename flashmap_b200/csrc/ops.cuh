// Launchers of the row-wise, sampling and acceptance kernels (ops.cu).
#pragma once

#include "launch.cuh"

namespace fm {

fm_status launch_rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int64_t rows,
                         int64_t cols, float eps, cudaStream_t s, bool pdl);
fm_status launch_adaln(const __nv_bfloat16* x, const __nv_bfloat16* mod, __nv_bfloat16* y, int64_t rows,
                       int64_t cols, float eps, cudaStream_t s, bool pdl);

struct DraftPrepArgs {
  const int64_t* anchor_ids;  // [B]
  const int32_t* lengths;     // [B]
  const __nv_bfloat16* embed; // [V, Ht]
  __nv_bfloat16* anchor_rows; // [B, Ht]
  int* anchor_pos;            // [B]
  int* anchor_seq;            // [B]
  int* slot_pos;              // [B*K]
  float *tok_cos, *tok_sin;   // [B*K][rope_half] rotary factors of the slots' positions
  const float *rope_cos, *rope_sin;  // [rope_len][rope_half]
  int rope_half;
  unsigned long long* keys;   // [B*K]
  int B, K, Ht;
  long long V;
  int rope_len, cache_len;
  uint32_t* offset_bump;  // incremented once per draft when non-null
  int* err;
};
fm_status launch_draft_prep(const DraftPrepArgs& a, cudaStream_t s, bool pdl);

// tok_cos/tok_sin[t] = rotary factors of positions[t] (out-of-range positions
// record DEV_BAD_INDEX and read position 0)
fm_status launch_rope_gather(const int* positions, int T, const float* rope_cos, const float* rope_sin, int rope_len,
                             int half, float* tok_cos, float* tok_sin, int* err, cudaStream_t s);

// inputs = bf16(state_norm(post) + bf16(gate * noise_norm(state)))  (modeling_flashmap.py:393-399)
struct MixArgs {
  const __nv_bfloat16* post;  // posterior embeddings; row stride post_stride (0: one shared row)
  long long post_stride;
  const __nv_bfloat16* state;  // [T, Ht] state embeddings
  const __nv_bfloat16* state_norm_w;
  const __nv_bfloat16* noise_norm_w;
  __nv_bfloat16* out;  // [T, Ht]
  float gate;          // bf16-representable
  float eps;
  int T, Ht;
};
fm_status launch_mix_state(const MixArgs& a, cudaStream_t s, bool pdl);

// The eigen-folded noise's first-layer input (sglang/model.py:945-958): per
// token t, scale = gate * rsqrt(sum_i var_i z_ti^2 + eps) and
// out[t] = x0 + bf16(scale * proj[t]), proj = bf16(z W_fold^T) from the GEMM.
struct NoiseFoldArgs {
  const __nv_bfloat16* proj;  // [T, D]
  const __nv_bfloat16* z;     // [T, Ht]
  const float* var;           // [Ht] lam / Ht
  const __nv_bfloat16* x0;    // [D] x_embed(state_norm(uniform))
  __nv_bfloat16* out;         // [T, D]
  float gate;                 // bf16-representable
  float eps;
  int T, D, Ht;
};
fm_status launch_noise_fold(const NoiseFoldArgs& a, cudaStream_t s, bool pdl);

// offset_ptr (device, optional): its value is added to `offset` when the kernel runs
fm_status launch_philox_normal_bf16(__nv_bfloat16* out, long long count, uint64_t seed, uint32_t offset,
                                    const uint32_t* offset_ptr, cudaStream_t s, bool pdl);
fm_status launch_philox_normal_f32(float* out, long long count, uint64_t seed, uint32_t offset,
                                   const uint32_t* offset_ptr, cudaStream_t s, bool pdl);
fm_status launch_argmax_tokens(const unsigned long long* keys, int64_t* tokens, int n, cudaStream_t s, bool pdl);

// multi-step state featurisation inputs: rows [0, T) = bf16(softmax(state * c)) (when with_posterior),
// rows [T*with_posterior, ...) = bf16(state)
fm_status launch_state_rows(const float* state, __nv_bfloat16* out, int T, int S, float c, int with_posterior,
                            cudaStream_t s, bool pdl);
// state = ((1 - next) * state + (next - s) * softmax(logits)) / (1 - s)
fm_status launch_state_update(float* state, const __nv_bfloat16* logits, long long ldl, int T, int S, float a,
                              float b, float d, cudaStream_t s, bool pdl);

struct ExtendPrepArgs {
  const int32_t* cu_rows;  // [B+1]
  const int32_t* lengths;  // [B]
  int* token_seq;          // [rows]
  int* positions;          // [rows]
  int rows, B, rope_len, cache_len;
  int* err;
};
fm_status launch_extend_prep(const ExtendPrepArgs& a, cudaStream_t s, bool pdl);
fm_status launch_extend_commit(const int32_t* cu_rows, int32_t* lengths, int B, cudaStream_t s, bool pdl);

}  // namespace fm
