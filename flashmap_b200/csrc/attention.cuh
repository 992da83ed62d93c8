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


// ---------------------------------------------------------------------------
// Cross-attention of the 16 block queries of one (sequence, head) over a
// range of context keys, shared by cross_attn_kernel and the streamed draft
// pass.  Four warps take 16 keys each of every 64-key tile (K and V staged
// as 128-byte-swizzled [64 x 64] boxes); every warp keeps its own online
// softmax; the warps are merged by the CTA at the end, and the key ranges
// ("splits") of one (sequence, head) are merged by the last split to finish.

constexpr int XA_TILE = 64;  // keys per tile

__device__ __forceinline__ void mma_bf16_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// byte offset of (row, 8-element chunk) inside a tile written by TMA with
// 128-byte swizzling as boxes of [64 rows x 64 bf16]
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
  const int box = chunk >> 3, cin = chunk & 7;
  return (uint32_t)(box * (XA_TILE * 128) + row * 128 + ((cin ^ (row & 7)) << 4));
}

// one key split's split boundaries: keys 0..ctx-1 cut into nsplit ranges of
// whole 64-key tiles
__device__ __forceinline__ int xa_split_keys(int ctx, int nsplit) {
  return ((((ctx + nsplit - 1) / nsplit) + XA_TILE - 1) / XA_TILE) * XA_TILE;
}

template <int HD>
struct XaAcc {
  float o[HD / 8][4];
  float m0, m1, l0, l1;
};

template <int HD>
__device__ __forceinline__ void xa_init(XaAcc<HD>& s) {
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) s.o[i][0] = s.o[i][1] = s.o[i][2] = s.o[i][3] = 0.0f;
  s.m0 = s.m1 = -INFINITY;
  s.l0 = s.l1 = 0.0f;
}

// the query fragments (A operand, HD/16 k-steps) of rows 0-15: ld32(row, col)
// returns the two bf16 at (row, col), (row, col + 1) as one word
template <int HD, class Ld32>
__device__ __forceinline__ void xa_load_q(uint32_t (&qa)[HD / 16][4], Ld32 ld32) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks) {
    const int c = ks * 16 + tig * 2;
    qa[ks][0] = ld32(gid, c);
    qa[ks][1] = ld32(gid + 8, c);
    qa[ks][2] = ld32(gid, c + 8);
    qa[ks][3] = ld32(gid + 8, c + 8);
  }
}

// One 64-key tile for this warp's 16 keys (key0 = 16 * warp within the
// tile): scores, mask past k_end, online softmax, O += P V.  kabs: absolute
// position of the warp's first key.
template <int HD>
__device__ __forceinline__ void xa_tile(XaAcc<HD>& s, const uint32_t (&qa)[HD / 16][4], uint32_t kbase, uint32_t vbase,
                                        int key0, int kabs, int k_end, float scale) {
  constexpr int NT = HD / 8;
  const int lane = threadIdx.x & 31, tig = lane & 3;
  float sc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
    const int kr = key0 + nt * 8 + (lane & 7);
#pragma unroll
    for (int ks = 0; ks < HD / 16; ks += 2) {
      uint32_t r0, r1, r2, r3;
      ldsm_x4(kbase + sw128_offset(kr, 2 * ks + (lane >> 3)), r0, r1, r2, r3);
      mma_bf16_16816(sc[nt], qa[ks], r0, r1);
      mma_bf16_16816(sc[nt], qa[ks + 1], r2, r3);
    }
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const bool valid = kabs + nt * 8 + tig * 2 + e < k_end;
      sc[nt][e] = valid ? __fmul_rn(sc[nt][e], scale) : -INFINITY;
      sc[nt][2 + e] = valid ? __fmul_rn(sc[nt][2 + e], scale) : -INFINITY;
      mx0 = fmaxf(mx0, sc[nt][e]);
      mx1 = fmaxf(mx1, sc[nt][2 + e]);
    }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float n0 = fmaxf(s.m0, mx0), n1 = fmaxf(s.m1, mx1);
  const float u0 = n0 == -INFINITY ? 0.0f : n0, u1 = n1 == -INFINITY ? 0.0f : n1;
  const float al0 = expf(__fsub_rn(s.m0, u0)), al1 = expf(__fsub_rn(s.m1, u1));
  s.m0 = n0;
  s.m1 = n1;
  float p[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    p[nt][0] = expf(__fsub_rn(sc[nt][0], u0));
    p[nt][1] = expf(__fsub_rn(sc[nt][1], u0));
    p[nt][2] = expf(__fsub_rn(sc[nt][2], u1));
    p[nt][3] = expf(__fsub_rn(sc[nt][3], u1));
  }
  s.l0 = __fadd_rn(__fmul_rn(s.l0, al0), __fadd_rn(__fadd_rn(p[0][0], p[0][1]), __fadd_rn(p[1][0], p[1][1])));
  s.l1 = __fadd_rn(__fmul_rn(s.l1, al1), __fadd_rn(__fadd_rn(p[0][2], p[0][3]), __fadd_rn(p[1][2], p[1][3])));
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    s.o[i][0] *= al0;
    s.o[i][1] *= al0;
    s.o[i][2] *= al1;
    s.o[i][3] *= al1;
  }
  uint32_t pa[4];
  pa[0] = pack_bf16(p[0][0], p[0][1]);
  pa[1] = pack_bf16(p[0][2], p[0][3]);
  pa[2] = pack_bf16(p[1][0], p[1][1]);
  pa[3] = pack_bf16(p[1][2], p[1][3]);
  const int vr = key0 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
  for (int dn = 0; dn < NT; dn += 2) {
    uint32_t r0, r1, r2, r3;
    ldsm_x4_t(vbase + sw128_offset(vr, dn + (lane >> 4)), r0, r1, r2, r3);
    mma_bf16_16816(s.o[dn], pa, r0, r1);
    mma_bf16_16816(s.o[dn + 1], pa, r2, r3);
  }
}

// Shared-memory floats the merge uses (xa_finish's `mrg`)
template <int HD>
__host__ __device__ constexpr int xa_merge_floats() {
  return 4 * 16 * HD + 64 * 4 + 32;
}

// After the tiles: merge the four warps' softmax states (CTA threads t =
// 0..127, `bar()` a barrier over them), then either write the attention of
// the 16 rows (when this is the only split with keys) or publish this
// split's partial (fp32 [16][HD] numerators, 16 maxima, 16 sums) at
// `mine` and take a ticket (`ticket()`, called by t == 0 between two barriers
// of the group, an atomic with acquire-release semantics at GPU scope, true
// for the last split to arrive); the last split merges every split's partial in split
// order from `base` (stride 16*HD + 32 floats) and writes the rows.
// store(i, d, lo, hi) writes columns d, d + 1 of row i.  Returns whether this
// CTA wrote the rows.
template <int HD, class Bar, class Ticket, class Store>
__device__ __forceinline__ bool xa_finish(XaAcc<HD>& s, float* mrg, int t, int n_active, float* mine,
                                          const float* base, int* flag, Bar bar, Ticket ticket, Store store) {
  constexpr int NT = HD / 8;
  const int lane = threadIdx.x & 31, warp = t >> 5, gid = lane >> 2, tig = lane & 3;
  s.l0 = __fadd_rn(s.l0, __shfl_xor_sync(0xffffffffu, s.l0, 1));
  s.l0 = __fadd_rn(s.l0, __shfl_xor_sync(0xffffffffu, s.l0, 2));
  s.l1 = __fadd_rn(s.l1, __shfl_xor_sync(0xffffffffu, s.l1, 1));
  s.l1 = __fadd_rn(s.l1, __shfl_xor_sync(0xffffffffu, s.l1, 2));
  bar();
  float* mO = mrg;
  float* mM = mrg + 4 * 16 * HD;
  float* mL = mM + 64;
  float* mF = mL + 64;  // [4][16] exp(m_w - m)
  float* mR = mF + 64;  // [16] merged m, [16] merged l
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int col = i * 8 + tig * 2;
    *reinterpret_cast<float2*>(&mO[(warp * 16 + gid) * HD + col]) = make_float2(s.o[i][0], s.o[i][1]);
    *reinterpret_cast<float2*>(&mO[(warp * 16 + gid + 8) * HD + col]) = make_float2(s.o[i][2], s.o[i][3]);
  }
  if (tig == 0) {
    mM[warp * 16 + gid] = s.m0;
    mM[warp * 16 + gid + 8] = s.m1;
    mL[warp * 16 + gid] = s.l0;
    mL[warp * 16 + gid + 8] = s.l1;
  }
  bar();
  if (t < 16) {
    const int i = t;
    float mm = -INFINITY;
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, mM[w * 16 + i]);
    float ll = 0.0f;
    for (int w = 0; w < 4; ++w) {
      const float f = mM[w * 16 + i] == -INFINITY ? 0.0f : expf(__fsub_rn(mM[w * 16 + i], mm));
      mF[w * 16 + i] = f;
      ll = __fadd_rn(ll, __fmul_rn(mL[w * 16 + i], f));
    }
    mR[i] = mm;
    mR[16 + i] = ll;
  }
  bar();
  for (int v4 = t; v4 < 16 * HD / 4; v4 += 128) {
    const int i = (v4 * 4) / HD, d = (v4 * 4) % HD;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = mF[w * 16 + i];
      const float4 ow = *reinterpret_cast<const float4*>(&mO[(w * 16 + i) * HD + d]);
      acc.x = __fadd_rn(acc.x, __fmul_rn(ow.x, f));
      acc.y = __fadd_rn(acc.y, __fmul_rn(ow.y, f));
      acc.z = __fadd_rn(acc.z, __fmul_rn(ow.z, f));
      acc.w = __fadd_rn(acc.w, __fmul_rn(ow.w, f));
    }
    if (n_active == 1) {
      const float ll = mR[16 + i];
      store(i, d, __fdiv_rn(acc.x, ll), __fdiv_rn(acc.y, ll));
      store(i, d + 2, __fdiv_rn(acc.z, ll), __fdiv_rn(acc.w, ll));
    } else {
      __stcg(reinterpret_cast<float4*>(mine + i * HD + d), acc);
    }
  }
  if (n_active == 1) return true;
  if (t < 16) {
    __stcg(mine + 16 * HD + t, mR[t]);
    __stcg(mine + 16 * HD + 16 + t, mR[16 + t]);
  }
  bar();
  if (t == 0) *flag = ticket() ? 1 : 0;  // an acquire-release ticket: orders the split's stores and the merge's loads
  bar();
  if (!*flag) return false;
  // the last split of this (sequence, head): every split in split order
  float* sF = mO;  // reuse: [n_active][16] weights, then [16] l
  bar();
  for (int r = t; r < 16; r += 128) {
    float mm = -INFINITY;
    for (int sp = 0; sp < n_active; ++sp) mm = fmaxf(mm, __ldcg(base + (long long)sp * (16 * HD + 32) + 16 * HD + r));
    float ll = 0.0f;
    for (int sp = 0; sp < n_active; ++sp) {
      const float* ps = base + (long long)sp * (16 * HD + 32);
      const float ms = __ldcg(ps + 16 * HD + r);
      const float f = ms == -INFINITY ? 0.0f : expf(__fsub_rn(ms, mm));
      sF[sp * 16 + r] = f;
      ll = __fadd_rn(ll, __fmul_rn(__ldcg(ps + 16 * HD + 16 + r), f));
    }
    sF[n_active * 16 + r] = ll;
  }
  bar();
  for (int v4 = t; v4 < 16 * HD / 4; v4 += 128) {
    const int i = (v4 * 4) / HD, d = (v4 * 4) % HD;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int sp = 0;
    for (; sp + 4 <= n_active; sp += 4) {
      float4 t4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        t4[u] = __ldcg(reinterpret_cast<const float4*>(base + (long long)(sp + u) * (16 * HD + 32) + i * HD + d));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float f = sF[(sp + u) * 16 + i];
        acc.x = __fadd_rn(acc.x, __fmul_rn(t4[u].x, f));
        acc.y = __fadd_rn(acc.y, __fmul_rn(t4[u].y, f));
        acc.z = __fadd_rn(acc.z, __fmul_rn(t4[u].z, f));
        acc.w = __fadd_rn(acc.w, __fmul_rn(t4[u].w, f));
      }
    }
    for (; sp < n_active; ++sp) {
      const float4 tt = __ldcg(reinterpret_cast<const float4*>(base + (long long)sp * (16 * HD + 32) + i * HD + d));
      const float f = sF[sp * 16 + i];
      acc.x = __fadd_rn(acc.x, __fmul_rn(tt.x, f));
      acc.y = __fadd_rn(acc.y, __fmul_rn(tt.y, f));
      acc.z = __fadd_rn(acc.z, __fmul_rn(tt.z, f));
      acc.w = __fadd_rn(acc.w, __fmul_rn(tt.w, f));
    }
    const float ll = sF[n_active * 16 + i];
    store(i, d, __fdiv_rn(acc.x, ll), __fdiv_rn(acc.y, ll));
    store(i, d + 2, __fdiv_rn(acc.z, ll), __fdiv_rn(acc.w, ll));
  }
  return true;
}

}  // namespace fm
