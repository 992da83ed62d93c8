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

// ---------------------------------------------------------------------------
// Self-attention of one head of a 16-slot block, by one warp on the tensor
// cores (mma.sync m16n8k16, bf16 in, fp32 accumulate).  q, k, v are staged in
// shared memory as [16 x HD] bf16 in 64-column boxes of 2 KB, rows of 128
// bytes with the 16-byte chunks swizzled by chunk ^ (row & 7) (the layout TMA
// writes with 128-byte swizzling).  Scores fp32, scaled; softmax numerators
// exp(s - m) in fp32 summed per lane then over the quad, rounded to bf16 for
// P V; out(i, d) = (P V)(i, d) / l(i).  store(i, d, lo, hi) receives columns
// d, d + 1 of row i.  The block self-attention and the serving operator share it.
__device__ __forceinline__ uint32_t blk_sw(int row, int chunk) {
  return (uint32_t)((chunk >> 3) * 2048 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}
__device__ __forceinline__ void sa_mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void sa_ldsm4(uint32_t addr, uint32_t* r, bool trans) {
  if (trans)
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
  else
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

template <int HD, class Store>
__device__ __forceinline__ void block_attn_head(uint32_t qs, uint32_t ks, uint32_t vs, float scale, Store store) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  // S = Q K^T: two n8 tiles of keys, HD / 16 k-steps
  float sc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
  for (int kst = 0; kst < HD / 16; kst += 2) {
    uint32_t qa0[4], qa1[4];
    // A fragments of k-steps kst and kst + 1 (rows 0-15)
    sa_ldsm4(qs + blk_sw((lane & 7) + ((lane >> 3) & 1) * 8, 2 * kst + (lane >> 4)), qa0, false);
    sa_ldsm4(qs + blk_sw((lane & 7) + ((lane >> 3) & 1) * 8, 2 * kst + 2 + (lane >> 4)), qa1, false);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      uint32_t kb[4];
      sa_ldsm4(ks + blk_sw(nt * 8 + (lane & 7), 2 * kst + (lane >> 3)), kb, false);
      sa_mma(sc[nt], qa0, kb[0], kb[1]);
      sa_mma(sc[nt], qa1, kb[2], kb[3]);
    }
  }
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sc[nt][e] = __fmul_rn(sc[nt][e], scale);
      sc[nt][2 + e] = __fmul_rn(sc[nt][2 + e], scale);
      m0 = fmaxf(m0, sc[nt][e]);
      m1 = fmaxf(m1, sc[nt][2 + e]);
    }
  m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
  m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
  float p[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    p[nt][0] = expf(__fsub_rn(sc[nt][0], m0));
    p[nt][1] = expf(__fsub_rn(sc[nt][1], m0));
    p[nt][2] = expf(__fsub_rn(sc[nt][2], m1));
    p[nt][3] = expf(__fsub_rn(sc[nt][3], m1));
  }
  float l0 = __fadd_rn(__fadd_rn(p[0][0], p[0][1]), __fadd_rn(p[1][0], p[1][1]));
  float l1 = __fadd_rn(__fadd_rn(p[0][2], p[0][3]), __fadd_rn(p[1][2], p[1][3]));
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 1));
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 2));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 1));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 2));
  uint32_t pa[4];
  {
    __nv_bfloat162 t;
    t = __floats2bfloat162_rn(p[0][0], p[0][1]);
    pa[0] = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(p[0][2], p[0][3]);
    pa[1] = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(p[1][0], p[1][1]);
    pa[2] = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(p[1][2], p[1][3]);
    pa[3] = *reinterpret_cast<uint32_t*>(&t);
  }
  // O = P V over the 16 keys, HD / 8 n8 tiles of dims
  const int vr = ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
  for (int dn = 0; dn < HD / 8; dn += 2) {
    uint32_t vb[4];
    sa_ldsm4(vs + blk_sw(vr, dn + (lane >> 4)), vb, true);
    float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
    sa_mma(o0, pa, vb[0], vb[1]);
    sa_mma(o1, pa, vb[2], vb[3]);
    const int c0 = dn * 8 + tig * 2, c1 = c0 + 8;
    store(gid, c0, __fdiv_rn(o0[0], l0), __fdiv_rn(o0[1], l0));
    store(gid + 8, c0, __fdiv_rn(o0[2], l1), __fdiv_rn(o0[3], l1));
    store(gid, c1, __fdiv_rn(o1[0], l0), __fdiv_rn(o1[1], l0));
    store(gid + 8, c1, __fdiv_rn(o1[2], l1), __fdiv_rn(o1[3], l1));
  }
}

}  // namespace fm
