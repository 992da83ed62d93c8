// Attention of the FlashMap DiT block (modeling_flashmap.py:144-147, SDPA
// without mask, scale 1/sqrt(head_dim)).
//
// Numerics follow the CPU flash-attention of the reference's SDPA on bf16
// inputs: scores in fp32, softmax numerators exp(s - m) in fp32 with their
// sum kept in fp32, the numerators rounded to bf16 for the P*V product,
// fp32 accumulation, and the division by the sum at the end.
//
// * self_attn_kernel: the K block slots attend to each other (K <= 32 keys);
//   one CTA per (sequence, head), plain FMA.
// * cross_attn_kernel: the slots attend to the context cache positions
//   0..len (len = verified length, the anchor at position len).  The keys of
//   one (sequence, head) are split over CTAs; each CTA streams 64-key K/V
//   tiles through a TMA (128-byte swizzled) pipeline and computes with
//   mma.sync m16n8k16 (16 query rows = the block); split results are merged
//   by the last CTA of the (sequence, head) to finish.
#pragma once

#include "common.cuh"

namespace fm {

struct SelfAttnArgs {
  const __nv_bfloat16* qkv;  // [T, 3*D] (q, k already normed + roped)
  __nv_bfloat16* out;        // [T, D]
  int block;                 // K (slots per sequence)
  int heads, head_dim, hidden;
  float scale;
};

struct CrossAttnArgs {
  const __nv_bfloat16* q;  // [B*16, D] normed + roped queries
  __nv_bfloat16* out;      // [B*16, D]
  const int* lengths;      // [B] verified length; keys are positions 0..lengths[b]
  int batch, heads, head_dim, hidden;
  int layer, cache_batch, cache_len;  // cache (L, 2, cache_batch, heads, cache_len, hd)
  int nsplit;
  float scale;
  float* part;     // [B*H*nsplit][16*hd + 32]
  int* counters;   // [B*H]
  int* err;
};

}  // namespace fm
