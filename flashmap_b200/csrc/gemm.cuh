// tcgen05 GEMM for the FlashMap drafter: Y[n, m] = sum_k X[n, k] * W[m, k].
//
// Orientation ("swap-AB"): the weight W (nn.Linear layout, out x in) is the
// 128-row A operand and the tokens X are the N = BN operand, so a batch-1
// draft (16 tokens) runs M=128 x N=16 UMMAs that stream W straight from HBM.
//
// Work decomposition: the (tile, k-block) units of the whole GEMM are split
// evenly over the grid (stream-K).  A tile whose k-range spans several CTAs
// is finished by its head CTA (the holder of its first k-block): the other
// contributors write their fp32 partials to the workspace and release-add a
// per-tile counter; the head waits (bounded, the contributors are resident:
// the grid never exceeds one CTA per SM) for the count, stages the partials
// into its idle pipeline buffers with bulk copies, sums them in contributor
// order (so the result does not depend on arrival order) and runs the
// epilogue.
//
// Roles (192 threads): warp 0 lane 0 issues TMA loads, warp 1 lane 0 issues
// tcgen05.mma and owns the TMEM allocation, warps 2-5 read the accumulators
// (TMEM lane quarter = warp % 4) and run the fused epilogue.
//
// Programmatic dependent launch: the producer loads the first pipeline
// stages of W (constant weights) before griddepcontrol.wait, so the weight
// stream of this GEMM overlaps the tail of the kernel before it.
#pragma once

#include "common.cuh"

namespace fm {

enum GemmEpilogue : int {
  EPI_STORE = 0,    // out = bf16(acc + bias)
  EPI_GELU = 1,     // out = bf16(gelu(bf16(acc + bias)))
  EPI_SWIGLU = 2,   // tiles hold 64 gate rows then 64 up rows: out = bf16(bf16(silu(g)) * u)
  EPI_RESID = 3,    // out (in place) = bf16(out + bf16(gate * bf16(acc + bias)))
  EPI_QKNORM = 4,   // parts q | k | v: q,k get per-head RMSNorm + interleaved RoPE
  EPI_KVCACHE = 5,  // rows (layer, k|v, head, dim): k gets norm + RoPE; written into the cache
  EPI_LOGITS = 6,   // out = bf16(acc + bias) at column col_ids[m]; per-token argmax key
  EPI_F32 = 7,      // out32 = acc (fp32, no rounding): one-time constants
  EPI_COUNT = 8,
};

struct GemmArgs {
  int M, N, K;  // output features (rows of W), tokens (rows of X), reduction
  int kb;       // k-blocks of 64
  int m_tiles, n_tiles;
  long long units;  // m_tiles * n_tiles * kb
  __nv_bfloat16* out;
  float* out32;
  long long ldo;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* gate;
  const __nv_bfloat16* norm_w0;  // q-norm (QKNORM) or per-layer k-norm base (KVCACHE)
  const __nv_bfloat16* norm_w1;  // k-norm (QKNORM)
  int part_rows;                 // rows per q/k/v part (the hidden size)
  int head_dim;
  float eps;
  const float* rope_cos;  // [rope_len][head_dim/2]
  const float* rope_sin;
  int rope_len;
  const int* positions;  // [N]
  const float* tok_cos;  // optional [N][head_dim/2]: rotary factors of the N tokens' positions
  const float* tok_sin;  //   (QKNORM reads these instead of positions + tables when set)
  const int* token_seq;  // [N] (KVCACHE)
  __nv_bfloat16* cache;  // (L, 2, cache_batch, heads, cache_len, head_dim)
  int cache_batch, cache_heads, cache_len;
  int norm_layer_stride;  // elements between layers' k-norm weights
  unsigned long long* argmax_keys;  // [N] or null (no argmax)
  const long long* col_ids;         // [M] target ids of the rows, or null (row = id)
  int scatter;                      // LOGITS: store row m at column col_ids[m] (else at m)
  float* ws;                        // split-K partials: grid * 2 slots * BN * 128 fp32
  int* counters;                    // [m_tiles * n_tiles], zero between launches
  int* err;
};

// Trace slots per CTA: 0 entry, 1 setup done, then per segment s < 3:
// 2+4s MMA issue done, 3+4s accumulator seen by the epilogue, 4+4s partial
// written / epilogue done, 5+4s split fix-up done; 14 exit; 15 the head's
// staged partials landed (first round).
constexpr int GEMM_TRACE = 16;
__device__ __forceinline__ void gemm_stamp(unsigned long long* trace, int slot) {
  if (trace) trace[(long long)blockIdx.x * GEMM_TRACE + slot] = global_ns();
}

// CG = 2: a CTA pair computes 256 x BN tiles with one M = 256 MMA; each CTA
// stages its 128 weight rows and BN / 2 token rows per k-block (32 KB for
// BN = 256 instead of 48 KB), so six stages fit where a single CTA held four.
template <int BN, int CG = 1>
struct GemmShape {
  static constexpr int A_BYTES = 128 * 64 * 2;
  static constexpr int B_BYTES = (BN / CG) * 64 * 2;
  static constexpr int STAGES =
      CG == 2 ? 6 : BN <= 16 ? 5 : BN <= 32 ? 4 : BN <= 64 ? 7 : BN <= 128 ? 5 : 4;
  static constexpr int ACC = 2;
  static constexpr uint32_t TMEM_COLS =
      ACC * BN <= 32 ? 32 : ACC * BN <= 64 ? 64 : ACC * BN <= 128 ? 128 : ACC * BN <= 256 ? 256 : 512;
  // epilogue exchange (union) + split flags, then for wide blocks a ring of
  // residual chunks ([16 tokens][128 features] bf16) loaded ahead
  static constexpr int RING = 4;
  static constexpr int RING_BYTES = BN >= 64 ? RING * 4096 : 0;
  static constexpr int SCRATCH = 4096 + 1024 + RING_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 /*alignment slack*/ + STAGES * (A_BYTES + B_BYTES) + BAR_BYTES + SCRATCH;
};

__device__ __forceinline__ long long cta_of_unit(long long u, long long U, int G) {
  return ((u + 1) * (long long)G - 1) / U;
}

__device__ __forceinline__ int gemm_ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void gemm_red_release(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Split tiles are finished by their head CTA (the one holding the tile's
// first k-block; the split segment is always its last segment, so its
// pipeline shared memory is idle by then): it waits (bounded) until the other
// contributors have published their fp32 partials, stages them into the idle
// pipeline buffers with bulk copies (one round trip for all of them, instead
// of a few serial ones), and sums them with its own accumulator in
// contributor order.

// ---------------------------------------------------------------------------------------------
// Epilogue on 16 accumulator columns (tokens n0 .. n0+15) of tile row r (feature m).
// Threads of the 4 epilogue warps call it together (it may use named barrier 1).
// Values an epilogue reads from global memory for 16 token columns, loaded
// ahead of the chunk that needs them (so that a wide tile's chunks overlap
// their round trips): the residual x (EPI_RESID), the rotary factors from the
// per-token tables (EPI_QKNORM with tok_cos).  Returns false when the
// epilogue has nothing to prefetch.
template <int EPI>
__device__ __forceinline__ bool epilogue_prefetch(const GemmArgs& a, int m, int n0, float* pre) {
  if constexpr (EPI == EPI_RESID) {
    const bool mvalid = m < a.M;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = n0 + j;
      pre[j] = (mvalid && n < a.N) ? bf2f(a.out[(long long)n * a.ldo + m]) : 0.0f;
    }
    return true;
  } else if constexpr (EPI == EPI_QKNORM) {
    // only q and k rows are rotated (the tile's part is uniform: rows m & ~127)
    if (a.tok_cos == nullptr || (m & ~127) / a.part_rows >= 2) return false;
    const int half = a.head_dim >> 1;
    const int d = (m % a.part_rows) % a.head_dim;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = (n0 + j < a.N) ? n0 + j : 0;
      pre[j] = a.tok_cos[n * half + (d >> 1)];
      pre[16 + j] = a.tok_sin[n * half + (d >> 1)];
    }
    return true;
  } else {
    return false;
  }
}

// ---------------------------------------------------------------------------------------------
// Wide blocks (BN >= 64) with the STORE / GELU / RESID epilogues run each
// 128 x 16 chunk through shared memory ([16 tokens][128 features] bf16, the
// 4 KB exchange area): the output (token-major) is then read and written as
// 16-byte vectors along the features, two per thread, instead of sixteen
// 2-byte accesses per thread.  Same arithmetic as epilogue16.
template <int BN, int EPI>
struct VecEpilogue {
  static constexpr bool ON = BN >= 64 && (EPI == EPI_STORE || EPI == EPI_GELU || EPI == EPI_RESID);
};

__device__ __forceinline__ bool vec_epilogue_ok(const GemmArgs& a) {
  return a.M % 8 == 0 && a.ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
}

__device__ __forceinline__ void gemm_cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16u : 0u)
               : "memory");
}
__device__ __forceinline__ void gemm_cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void gemm_cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Residual chunk (tokens n0 .. n0+15, features m0 .. m0+127) into a ring slot
// [16][128] with asynchronous 16-byte copies (zero-filled outside the output);
// one commit group per chunk, issued (or empty) by every epilogue thread.
__device__ __forceinline__ void vec_issue(const GemmArgs& a, int m0, int n0, __nv_bfloat16* slot, bool any) {
  if (any) {
    const int t = threadIdx.x - 64;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int idx = t + 128 * k, nl = idx >> 4, gi = idx & 15;
      const int n = n0 + nl, m = m0 + gi * 8;
      const bool ok = n < a.N && m < a.M;
      gemm_cp_async16(slot + nl * 128 + gi * 8, ok ? (const void*)(a.out + (long long)n * a.ldo + m) : (const void*)a.out,
                      ok);
    }
  }
  gemm_cp_commit();
}

// The residual epilogue of a chunk whose residuals sit in `slot` (landed and
// visible): out = bf16(x + bf16(gate * bf16(acc + bias))) computed in place,
// then written back as vectors.
__device__ __forceinline__ void vec_resid16(const GemmArgs& a, const float* v, int r, int m0, int n0,
                                            __nv_bfloat16* slot) {
  const int m = m0 + r;
  const bool mvalid = m < a.M;
  const float b = (a.bias && mvalid) ? bf2f(a.bias[m]) : 0.0f;
  const float g = mvalid ? bf2f(a.gate[m]) : 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float y = round_bf(__fadd_rn(v[j], b));
    const float gy = round_bf(__fmul_rn(g, y));
    slot[j * 128 + r] = f2bf(__fadd_rn(bf2f(slot[j * 128 + r]), gy));
  }
  named_bar_sync(1, 128);
  const int t = threadIdx.x - 64;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int idx = t + 128 * k, nl = idx >> 4, gi = idx & 15;
    const int n = n0 + nl, mm = m0 + gi * 8;
    if (n < a.N && mm < a.M)
      *reinterpret_cast<uint4*>(a.out + (long long)n * a.ldo + mm) =
          *reinterpret_cast<const uint4*>(slot + nl * 128 + gi * 8);
  }
  named_bar_sync(1, 128);  // the slot is refilled RING - 1 chunks later
}

// residual vectors of the chunk (tokens n0 .. n0+15, features m0 .. m0+127)
template <int EPI>
__device__ __forceinline__ void vec_prefetch(const GemmArgs& a, int m0, int n0, uint4* pre) {
  if constexpr (EPI == EPI_RESID) {
    const int t = threadIdx.x - 64;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int idx = t + 128 * k, nl = idx >> 4, gi = idx & 15;
      const int n = n0 + nl, m = m0 + gi * 8;
      pre[k] = (n < a.N && m < a.M) ? *reinterpret_cast<const uint4*>(a.out + (long long)n * a.ldo + m)
                                    : make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

template <int EPI>
__device__ __forceinline__ void vec_epilogue16(const GemmArgs& a, const float* v, int r, int m0, int n0,
                                               __nv_bfloat16* xt, const uint4* pre) {
  const int m = m0 + r;
  const bool mvalid = m < a.M;
  const float b = (a.bias && mvalid) ? bf2f(a.bias[m]) : 0.0f;
  const float g = (EPI == EPI_RESID && mvalid) ? bf2f(a.gate[m]) : 0.0f;
  const int t = threadIdx.x - 64;
  if constexpr (EPI == EPI_RESID) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int idx = t + 128 * k, nl = idx >> 4, gi = idx & 15;
      *reinterpret_cast<uint4*>(xt + nl * 128 + gi * 8) = pre[k];
    }
    named_bar_sync(1, 128);
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float y = round_bf(__fadd_rn(v[j], b));
    __nv_bfloat16 o;
    if constexpr (EPI == EPI_GELU) {
      y = __fmul_rn(__fmul_rn(y, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn(y, 0.70710678118654752f))));
      o = f2bf(y);
    } else if constexpr (EPI == EPI_RESID) {
      const float gy = round_bf(__fmul_rn(g, y));
      o = f2bf(__fadd_rn(bf2f(xt[j * 128 + r]), gy));
    } else {
      o = f2bf(y);
    }
    xt[j * 128 + r] = o;
  }
  named_bar_sync(1, 128);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int idx = t + 128 * k, nl = idx >> 4, gi = idx & 15;
    const int n = n0 + nl, mm = m0 + gi * 8;
    if (n < a.N && mm < a.M)
      *reinterpret_cast<uint4*>(a.out + (long long)n * a.ldo + mm) = *reinterpret_cast<const uint4*>(xt + nl * 128 + gi * 8);
  }
  named_bar_sync(1, 128);  // the exchange tile is refilled by the next chunk
}

// The [16 tokens][128 features] tile `xt` (bf16, shared) written to the
// token-major output as 16-byte vectors, two per epilogue thread; then (with
// refill_barrier) the tile may be refilled.
__device__ __forceinline__ void vec_store_tile(const GemmArgs& a, int m0, int n0, const __nv_bfloat16* xt,
                                               bool refill_barrier = true) {
  named_bar_sync(1, 128);
  const int t = threadIdx.x - 64;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int idx = t + 128 * k, nl = idx >> 4, gi = idx & 15;
    const int n = n0 + nl, mm = m0 + gi * 8;
    if (n < a.N && mm < a.M)
      *reinterpret_cast<uint4*>(a.out + (long long)n * a.ldo + mm) = *reinterpret_cast<const uint4*>(xt + nl * 128 + gi * 8);
  }
  if (refill_barrier) named_bar_sync(1, 128);
}

// The q/k-norm epilogue of a wide tile (vector path), over columns
// [c_begin, c_end) (chunks of 16), in three phases instead of three barriers
// per chunk: (1) every chunk's per-warp sums of squares of the rounded
// values (the transposing shuffle reduction, no barrier between chunks),
// (2) after one barrier every (head, token) 1/rms by the whole block, written
// back after a second barrier, (3) every chunk normalised, rotated and
// stored as vectors through two alternating store tiles.  `chunk(c0, v)`
// yields the 16 accumulator values of the chunk starting at column c0 (the
// same values both times it is asked).  Same arithmetic as epilogue16.
template <typename ChunkFn>
__device__ __forceinline__ void qknorm_wide(const GemmArgs& a, ChunkFn chunk, int r, int mt, int n_tile, int c_begin,
                                            int c_end, float* xch, __nv_bfloat16* vec_xt) {
  const int lane = threadIdx.x & 31;
  const int q = (threadIdx.x >> 5) & 3;
  const int m = mt * 128 + r;
  const int hd = a.head_dim, hq = hd >> 5, heads = 128 / hd;
  const int ncols = c_end - c_begin;
  const int part = (mt * 128) / a.part_rows;  // 0 q, 1 k, 2 v (uniform over the tile)
  const bool normed = part < 2;
  const int d = (m % a.part_rows) % hd;
  float wd = 0.0f;
  if (normed) {
    wd = bf2f((part == 0 ? a.norm_w0 : a.norm_w1)[d]);
    for (int c0 = c_begin; c0 < c_end; c0 += 16) {
      float v[16], sq[16];
      chunk(c0, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float y = round_bf(v[j]);
        sq[j] = __fmul_rn(y, y);
      }
#pragma unroll
      for (int width = 8; width >= 1; width >>= 1) {
        const bool up = (lane & (width * 2)) != 0;
#pragma unroll
        for (int i = 0; i < width; ++i) {
          const float send = up ? sq[i] : sq[i + width];
          const float keep = up ? sq[i + width] : sq[i];
          sq[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, width * 2));
        }
      }
      sq[0] = __fadd_rn(sq[0], __shfl_xor_sync(0xffffffffu, sq[0], 1));
      const int tl = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
      if ((lane & 1) == 0) xch[q * ncols + (c0 - c_begin) + tl] = sq[0];
    }
    named_bar_sync(1, 128);
    // the head's warp quarters in order, mean, 1 / sqrt(mean + eps); up to 8 per thread
    constexpr int MAXI = 8;
    float inv[MAXI];
    const int t = r;
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {
      const int idx = t + k * 128;
      inv[k] = 0.0f;
      if (idx < heads * ncols) {
        const int hh = idx / ncols, col = idx % ncols;
        float tot = 0.0f;
        for (int qq = hh * hq; qq < hh * hq + hq; ++qq) tot = __fadd_rn(tot, xch[qq * ncols + col]);
        const float mean = __fdiv_rn(tot, (float)hd);
        inv[k] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
      }
    }
    named_bar_sync(1, 128);
#pragma unroll
    for (int k = 0; k < MAXI; ++k)
      if (t + k * 128 < heads * ncols) xch[t + k * 128] = inv[k];
    named_bar_sync(1, 128);
  }
  const int half = hd >> 1;
  const float* xinv = xch + (q / hq) * ncols;  // this thread's head's 1/rms, by column
  for (int c0 = c_begin; c0 < c_end; c0 += 16) {
    const int n0 = n_tile + c0;
    float v[16], y[16];
    chunk(c0, v);
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = round_bf(v[j]);
    if (normed) {
      float rc[16], rs[16];
      if (a.tok_cos != nullptr) {
        // the tokens' rotary factors, gathered once per draft (positions checked there)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = (n0 + j < a.N) ? n0 + j : 0;
          rc[j] = a.tok_cos[n * half + (d >> 1)];
          rs[j] = a.tok_sin[n * half + (d >> 1)];
        }
      } else {
        int pos[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = n0 + j;
          int pj = (n < a.N) ? a.positions[n] : 0;
          if (pj < 0 || pj >= a.rope_len) {
            if (n < a.N) record_error(a.err, DEV_BAD_INDEX);
            pj = 0;
          }
          pos[j] = pj;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          rc[j] = a.rope_cos[(long long)pos[j] * half + (d >> 1)];
          rs[j] = a.rope_sin[(long long)pos[j] * half + (d >> 1)];
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float scale = round_bf(__fmul_rn(wd, xinv[(c0 - c_begin) + j]));
        const float xn = round_bf(__fmul_rn(y[j], scale));
        const float other = __shfl_xor_sync(0xffffffffu, xn, 1);
        float o;
        if ((d & 1) == 0)
          o = __fsub_rn(__fmul_rn(xn, rc[j]), __fmul_rn(other, rs[j]));
        else
          o = __fadd_rn(__fmul_rn(xn, rc[j]), __fmul_rn(other, rs[j]));
        y[j] = round_bf(o);
      }
    }
    // two store tiles used alternately; the store tile's barrier also comes
    // after every thread's reads of xch (1/rms) for this chunk, so after the
    // last chunk xch may be refilled
    __nv_bfloat16* tile = vec_xt + ((n0 >> 4) & 1) * 2048;
#pragma unroll
    for (int j = 0; j < 16; ++j) tile[j * 128 + r] = f2bf(y[j]);
    vec_store_tile(a, mt * 128, n0, tile, false);
  }
}

// vec_xt (wide blocks, aligned output): QKNORM and unscattered LOGITS store
// through [16][128] shared tiles as vectors instead of scalars (QKNORM: two
// tiles from vec_xt on, alternating by chunk; LOGITS: one).
template <int EPI>
__device__ __forceinline__ void epilogue16(const GemmArgs& a, const float* v, int r, int m, int mt, int n0,
                                           float* xch, unsigned long long* xch64, const float* pre = nullptr,
                                           __nv_bfloat16* vec_xt = nullptr) {
  const int lane = threadIdx.x & 31;
  const int q = (threadIdx.x >> 5) & 3;
  const bool mvalid = m < a.M;
  if constexpr (EPI == EPI_F32) {
    if (mvalid)
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (n0 + j < a.N) a.out32[(long long)(n0 + j) * a.ldo + m] = v[j];
  } else if constexpr (EPI == EPI_STORE || EPI == EPI_GELU || EPI == EPI_RESID) {
    if (!mvalid) return;
    const float b = a.bias ? bf2f(a.bias[m]) : 0.0f;
    const float g = (EPI == EPI_RESID) ? bf2f(a.gate[m]) : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = n0 + j;
      if (n >= a.N) continue;
      float y = round_bf(__fadd_rn(v[j], b));
      __nv_bfloat16* dst = a.out + (long long)n * a.ldo + m;
      if constexpr (EPI == EPI_GELU) {
        y = __fmul_rn(__fmul_rn(y, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn(y, 0.70710678118654752f))));
        *dst = f2bf(y);
      } else if constexpr (EPI == EPI_RESID) {
        const float gy = round_bf(__fmul_rn(g, y));
        *dst = f2bf(__fadd_rn(pre ? pre[j] : bf2f(*dst), gy));
      } else {
        *dst = f2bf(y);
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // rows 64..127 of the tile are the "up" halves of features mt*64 + (r - 64)
    if (vec_epilogue_ok(a)) {
      // every thread stages its 16 rounded values in a [16 tokens][128 rows]
      // bf16 tile, then computes 8 outputs (one token, 8 consecutive
      // features) and stores them as one 16-byte vector
      __nv_bfloat16* xt = reinterpret_cast<__nv_bfloat16*>(xch);
#pragma unroll
      for (int j = 0; j < 16; ++j) xt[j * 128 + r] = f2bf(v[j]);
      named_bar_sync(1, 128);
      const int t = threadIdx.x - 64, jj = t >> 3, f0 = (t & 7) * 8;
      const int n = n0 + jj, F = mt * 64 + f0;
      if (n < a.N && F < a.M / 2) {
        const uint4 gw = *reinterpret_cast<const uint4*>(xt + jj * 128 + f0);
        const uint4 uw = *reinterpret_cast<const uint4*>(xt + jj * 128 + 64 + f0);
        const uint32_t g4[4] = {gw.x, gw.y, gw.z, gw.w}, u4[4] = {uw.x, uw.y, uw.z, uw.w};
        uint32_t o4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float o[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float gt = __uint_as_float(h ? (g4[i] & 0xffff0000u) : (g4[i] << 16));
            const float ut = __uint_as_float(h ? (u4[i] & 0xffff0000u) : (u4[i] << 16));
            const float s = round_bf(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))));
            o[h] = __fmul_rn(s, ut);
          }
          const __nv_bfloat162 pr = __floats2bfloat162_rn(o[0], o[1]);
          o4[i] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        *reinterpret_cast<uint4*>(a.out + (long long)n * a.ldo + F) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
      named_bar_sync(1, 128);  // the exchange tile is refilled by the next chunk
      return;
    }
    if (r >= 64) {
#pragma unroll
      for (int j = 0; j < 16; ++j) xch[(r - 64) * 16 + j] = round_bf(v[j]);
    }
    named_bar_sync(1, 128);
    if (r < 64) {
      const int f = mt * 64 + r;
      if (f < a.M / 2) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = n0 + j;
          if (n >= a.N) continue;
          const float gt = round_bf(v[j]);
          const float s = round_bf(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))));
          a.out[(long long)n * a.ldo + f] = f2bf(__fmul_rn(s, xch[r * 16 + j]));
        }
      }
    }
    named_bar_sync(1, 128);
  } else if constexpr (EPI == EPI_QKNORM || EPI == EPI_KVCACHE) {
    const int hd = a.head_dim;
    int part, layer = 0;
    if constexpr (EPI == EPI_QKNORM) {
      part = (mt * 128) / a.part_rows;  // 0 q, 1 k, 2 v (uniform over the tile)
    } else {
      layer = (mt * 128) / (2 * a.part_rows);
      part = ((mt * 128) / a.part_rows) & 1;  // 0 k, 1 v
    }
    // (a pair's second half tile may lie wholly past M: no k-norm weight read for it)
    const bool normed = (EPI == EPI_QKNORM) ? (part < 2) : (part == 0 && mt * 128 < a.M);
    const int d = (m % a.part_rows) % hd;
    float y[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = round_bf(v[j]);
    if (normed) {  // uniform branch over the whole tile
      const __nv_bfloat16* w;
      if constexpr (EPI == EPI_QKNORM)
        w = part == 0 ? a.norm_w0 : a.norm_w1;
      else
        w = a.norm_w0 + (long long)layer * a.norm_layer_stride;
      const float wd = bf2f(w[d]);  // issued here: its latency hides under the reduction
      // per-head sum of squares over the warp's 32 rows, all 16 tokens at once:
      // each exchange step halves the tokens a lane holds (the half picked by
      // the lane bit), 8 + 4 + 2 + 1 + 1 shuffles; lanes 2i and 2i+1 end with
      // token tl's warp sum.  Then the head's warp quarters, in order.
      float sq[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) sq[j] = __fmul_rn(y[j], y[j]);
#pragma unroll
      for (int width = 8; width >= 1; width >>= 1) {
        const bool up = (lane & (width * 2)) != 0;
#pragma unroll
        for (int i = 0; i < width; ++i) {
          const float send = up ? sq[i] : sq[i + width];
          const float keep = up ? sq[i + width] : sq[i];
          sq[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, width * 2));
        }
      }
      sq[0] = __fadd_rn(sq[0], __shfl_xor_sync(0xffffffffu, sq[0], 1));
      const int tl = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
      if ((lane & 1) == 0) xch[q * 16 + tl] = sq[0];
      named_bar_sync(1, 128);
      const int hq = hd >> 5;  // warp quarters per head
      // one thread per (head of the tile, token) finishes the statistic: the
      // quarters' sums in order, mean, 1 / sqrt(mean + eps)
      float* xinv = xch + 64;
      {
        const int t = (int)threadIdx.x - 64;
        if (t < (128 / hd) * 16) {
          const int hh = t >> 4, jj = t & 15;
          float tot = 0.0f;
          for (int qq = hh * hq; qq < hh * hq + hq; ++qq) tot = __fadd_rn(tot, xch[qq * 16 + jj]);
          const float mean = __fdiv_rn(tot, (float)hd);
          xinv[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        }
      }
      named_bar_sync(1, 128);
      const int hrow = (q / hq) * 16;  // this thread's head's entries of xinv
      const int half = hd >> 1;
      float rc[16], rs[16];
      if (EPI == EPI_QKNORM && pre != nullptr) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          rc[j] = pre[j];
          rs[j] = pre[16 + j];
        }
      } else if (EPI == EPI_QKNORM && a.tok_cos != nullptr) {
        // the tokens' rotary factors, gathered once per draft (positions checked there)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = (n0 + j < a.N) ? n0 + j : 0;
          rc[j] = a.tok_cos[n * half + (d >> 1)];
          rs[j] = a.tok_sin[n * half + (d >> 1)];
        }
      } else {
        // all positions, then all rotary factors: independent loads issued together
        int pos[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = n0 + j;
          int pj = (n < a.N) ? a.positions[n] : 0;
          if (pj < 0 || pj >= a.rope_len) {
            if (n < a.N) record_error(a.err, DEV_BAD_INDEX);
            pj = 0;
          }
          pos[j] = pj;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          rc[j] = a.rope_cos[(long long)pos[j] * half + (d >> 1)];
          rs[j] = a.rope_sin[(long long)pos[j] * half + (d >> 1)];
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float inv = xinv[hrow + j];
        const float scale = round_bf(__fmul_rn(wd, inv));
        const float xn = round_bf(__fmul_rn(y[j], scale));
        const float other = __shfl_xor_sync(0xffffffffu, xn, 1);
        const float cs = rc[j];
        const float sn = rs[j];
        float o;
        if ((d & 1) == 0)
          o = __fsub_rn(__fmul_rn(xn, cs), __fmul_rn(other, sn));
        else
          o = __fadd_rn(__fmul_rn(xn, cs), __fmul_rn(other, sn));
        y[j] = round_bf(o);
      }
      // xch is reused by the next chunk; on the vector path the store tile's
      // barrier (after every thread's last xinv read) orders that instead
      if (EPI != EPI_QKNORM || vec_xt == nullptr) named_bar_sync(1, 128);
    }
    if (EPI == EPI_QKNORM && vec_xt != nullptr) {
      // two store tiles used alternately (chunk parity): a tile is rewritten
      // two chunks later, after barriers that every thread reaches only once
      // its vector stores from it are done
      __nv_bfloat16* t = vec_xt + ((n0 >> 4) & 1) * 2048;
#pragma unroll
      for (int j = 0; j < 16; ++j) t[j * 128 + r] = f2bf(y[j]);
      vec_store_tile(a, mt * 128, n0, t, false);
      return;
    }
    if (!mvalid) return;
    if constexpr (EPI == EPI_QKNORM) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (n0 + j < a.N) a.out[(long long)(n0 + j) * a.ldo + m] = f2bf(y[j]);
    } else {
      const int h = (m % a.part_rows) / hd;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = n0 + j;
        if (n >= a.N) continue;
        const int seq = a.token_seq[n];
        const int pos = a.positions[n];
        if (seq < 0 || seq >= a.cache_batch || pos < 0 || pos >= a.cache_len) {
          record_error(a.err, DEV_BAD_INDEX);
          continue;
        }
        const long long idx =
            ((((long long)(layer * 2 + part) * a.cache_batch + seq) * a.cache_heads + h) * a.cache_len + pos) * hd +
            d;
        a.cache[idx] = f2bf(y[j]);
      }
    }
  } else if constexpr (EPI == EPI_LOGITS) {
    const float b = (a.bias && mvalid) ? bf2f(a.bias[m]) : 0.0f;
    const long long id = mvalid ? (a.col_ids ? a.col_ids[m] : (long long)m) : 0;
    const long long col = a.scatter ? id : (long long)m;
    const bool want_argmax = a.argmax_keys != nullptr;  // uniform over the launch
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = n0 + j;
      const float y = round_bf(__fadd_rn(v[j], b));
      if (vec_xt != nullptr)
        vec_xt[j * 128 + r] = f2bf(y);
      else if (mvalid && n < a.N)
        a.out[(long long)n * a.ldo + col] = f2bf(y);
      if (!want_argmax) continue;
      // warp max of the 64-bit key (value bits, then complement index) as two
      // 32-bit reductions: the largest value, then among its holders the smallest index
      const unsigned long long key = mvalid ? argmax_key(y, (uint32_t)id) : 0ull;
      const uint32_t hi = (uint32_t)(key >> 32);
      const uint32_t mh = __reduce_max_sync(0xffffffffu, hi);
      const uint32_t ml = __reduce_max_sync(0xffffffffu, hi == mh ? (uint32_t)key : 0u);
      if (lane == j) xch64[q * 16 + j] = ((unsigned long long)mh << 32) | ml;
    }
    if (vec_xt != nullptr) vec_store_tile(a, mt * 128, n0, vec_xt);
    if (!want_argmax) return;
    named_bar_sync(1, 128);
    if (threadIdx.x >= 64 && threadIdx.x < 80) {
      const int j = threadIdx.x - 64;
      unsigned long long key = xch64[j];
      for (int qq = 1; qq < 4; ++qq) key = xch64[qq * 16 + j] > key ? xch64[qq * 16 + j] : key;
      if (n0 + j < a.N) atomicMax(a.argmax_keys + n0 + j, key);
    }
    named_bar_sync(1, 128);
  }
}

// The LM-head epilogue of a whole wide tile (vector path, unscattered
// output): the logits of each 16-column chunk go out through two [16][128]
// store tiles used alternately (no refill barrier), and each chunk's per-warp
// argmax keys stay in shared memory ([4 warp quarters][BN]), so the quarters
// meet once per tile instead of twice per chunk: after the last chunk every
// thread folds the four quarters' keys of BN / 128 columns and atomicMax-es
// them into the tokens' keys.  Same values and keys as epilogue16.
// `ring` holds the two store tiles then the keys (8 KB + 32 * BN bytes).
template <int BN, typename ChunkFn>
__device__ __forceinline__ void logits_wide(const GemmArgs& a, ChunkFn chunk, int r, int mt, int n_tile,
                                            __nv_bfloat16* ring) {
  const int lane = threadIdx.x & 31;
  const int q = (threadIdx.x >> 5) & 3;
  const int m = mt * 128 + r;
  const bool mvalid = m < a.M;
  const float b = (a.bias && mvalid) ? bf2f(a.bias[m]) : 0.0f;
  const uint32_t id = mvalid ? (uint32_t)(a.col_ids ? a.col_ids[m] : (long long)m) : 0u;
  const bool want_argmax = a.argmax_keys != nullptr;  // uniform over the launch
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(ring + 2 * 2048);
  for (int c0 = 0; c0 < BN; c0 += 16) {
    float v[16];
    chunk(c0, v);
    __nv_bfloat16* tile = ring + ((c0 >> 4) & 1) * 2048;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float y = round_bf(__fadd_rn(v[j], b));
      tile[j * 128 + r] = f2bf(y);
      if (!want_argmax) continue;
      const unsigned long long key = mvalid ? argmax_key(y, id) : 0ull;
      const uint32_t hi = (uint32_t)(key >> 32);
      const uint32_t mh = __reduce_max_sync(0xffffffffu, hi);
      const uint32_t ml = __reduce_max_sync(0xffffffffu, hi == mh ? (uint32_t)key : 0u);
      if (lane == j) keys[q * BN + c0 + j] = ((unsigned long long)mh << 32) | ml;
    }
    // the store tile's barrier also orders the reads of the tile two chunks back
    vec_store_tile(a, mt * 128, n_tile + c0, tile, false);
  }
  if (!want_argmax) return;
  named_bar_sync(1, 128);
  const int t = threadIdx.x - 64;
#pragma unroll
  for (int k = 0; k < BN / 128; ++k) {
    const int j = t + 128 * k;
    unsigned long long key = keys[j];
#pragma unroll
    for (int qq = 1; qq < 4; ++qq) key = keys[qq * BN + j] > key ? keys[qq * BN + j] : key;
    if (n_tile + j < a.N) atomicMax(a.argmax_keys + n_tile + j, key);
  }
  named_bar_sync(1, 128);  // the keys and store tiles are refilled by the next tile
}

// ---------------------------------------------------------------------------------------------
// CG = 1: one CTA per 128 x BN tile.  CG = 2 (launched as clusters of two):
// a CTA pair per 256 x BN tile, the units (pair tile, k-block) split over the
// pairs; each CTA finishes its own 128 rows (its own split-K counter and
// partial slots), so the epilogues are those of the single-CTA tile.
template <int BN, int EPI, int CG = 1>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const GemmArgs a, unsigned long long* trace) {
  using S = GemmShape<BN, CG>;
  constexpr int STAGES = S::STAGES;
  constexpr int ACC = S::ACC;
  constexpr bool PAIR = CG == 2;
  static_assert(CG == 1 || (CG == 2 && BN == 256), "CTA pairs run 256 x 256 tiles");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * S::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + ACC);
  int* flags = reinterpret_cast<int*>(tmem_slot + 2);  // [0] abort, [1] last-arriver, [2..3] segment ok
  uint64_t* fix_bar = reinterpret_cast<uint64_t*>(flags + 6);  // staged-partials barrier (8-byte aligned)
  uint8_t* scratch = smem + STAGES * (S::A_BYTES + S::B_BYTES) + S::BAR_BYTES;
  float* xch = reinterpret_cast<float*>(scratch);
  // the argmax keys sit past the 4 KB exchange tile, which the wide LOGITS path fills meanwhile
  unsigned long long* xch64 = reinterpret_cast<unsigned long long*>(scratch + 4096);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long U = a.units;
  // units are split over the CTAs (CG = 1) or the pairs (CG = 2)
  const int G = gridDim.x / CG;
  const int c = blockIdx.x / CG;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const long long u0 = (long long)c * U / G, u1 = (long long)(c + 1) * U / G;
  const int kb = a.kb;
  if (threadIdx.x == 0) gemm_stamp(trace, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < ACC; ++i) {
      mbar_init(&acc_full[i], 1);
      // a pair's accumulator is released by the epilogue warps of both CTAs
      mbar_init(&acc_empty[i], 4 * CG);
    }
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    flags[3] = 0;
    mbar_init(fix_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, S::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers initialised before either signals the other's
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) gemm_stamp(trace, 1);
  // every CTA now holds its TMEM: the next kernel may be scheduled
  pdl_launch_dependents();
  volatile int* abort_flag = flags;

  if (warp == 0) {
    if constexpr (!PAIR) {
      if (lane == 0 && u1 > u0) {
        const uint64_t pol = a.n_tiles == 1 ? policy_evict_first() : policy_evict_last();
        const long long n = u1 - u0;
        const int pre = (int)(n < STAGES ? n : STAGES);
        // weights of the first stages before the dependency wait
        for (int i = 0; i < pre; ++i) {
          const long long u = u0 + i;
          const int tile = (int)(u / kb), k = (int)(u % kb);
          mbar_arrive_expect_tx(&full[i], S::A_BYTES + S::B_BYTES);
          tma_load_2d_hint(sA + i * S::A_BYTES, &tmA, &full[i], k * 64, (tile / a.n_tiles) * 128, pol);
        }
        pdl_wait();
        for (int i = 0; i < pre; ++i) {
          const long long u = u0 + i;
          const int tile = (int)(u / kb), k = (int)(u % kb);
          tma_load_2d(sB + i * S::B_BYTES, &tmB, &full[i], k * 64, (tile % a.n_tiles) * BN);
        }
        bool ok = true;
        for (long long i = pre; i < n; ++i) {
          const int s = (int)(i % STAGES);
          const uint32_t r = (uint32_t)(i / STAGES);
          if (!mbar_wait(&empty[s], (r - 1) & 1u, abort_flag)) {
            record_error(a.err, DEV_TIMEOUT_EMPTY);
            *abort_flag = 1;
            ok = false;
            break;
          }
          const long long u = u0 + i;
          const int tile = (int)(u / kb), k = (int)(u % kb);
          mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
          tma_load_2d_hint(sA + s * S::A_BYTES, &tmA, &full[s], k * 64, (tile / a.n_tiles) * 128, pol);
          tma_load_2d(sB + s * S::B_BYTES, &tmB, &full[s], k * 64, (tile % a.n_tiles) * BN);
        }
        if (!ok) {
          // drain: every issued stage must land before the CTA's shared memory goes away
          const long long issued_end = n;
          for (long long i = (issued_end > STAGES ? issued_end - STAGES : 0); i < issued_end; ++i)
            mbar_wait(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u, nullptr);
        }
      }
    } else {
      if (lane == 0 && u1 > u0) {
        // pair producer (both CTAs): this CTA's 128 weight rows and BN / 2 token
        // rows of each k-block into its own stage buffers, the bytes counted on
        // rank 0's full barrier, which rank 0 arms for both CTAs' copies
        const uint64_t pol = a.n_tiles == 1 ? policy_evict_first() : policy_evict_last();
        const uint64_t pol_b = policy_evict_last();
        const long long n = u1 - u0;
        const int pre = (int)(n < STAGES ? n : STAGES);
        constexpr uint32_t STAGE_TX = CG * (S::A_BYTES + S::B_BYTES);
        auto a_row = [&](int tile) { return (tile / a.n_tiles) * 256 + (int)rank * 128; };
        auto b_row = [&](int tile) { return (tile % a.n_tiles) * BN + (int)rank * (BN / 2); };
        for (int i = 0; i < pre; ++i) {
          const long long u = u0 + i;
          const int tile = (int)(u / kb), k = (int)(u % kb);
          if (rank == 0) mbar_arrive_expect_tx(&full[i], STAGE_TX);
          tma_load_2d_pair(sA + i * S::A_BYTES, &tmA, mapa_shared(smem_u32(&full[i]), 0), k * 64, a_row(tile), pol);
        }
        pdl_wait();
        for (int i = 0; i < pre; ++i) {
          const long long u = u0 + i;
          const int tile = (int)(u / kb), k = (int)(u % kb);
          tma_load_2d_pair(sB + i * S::B_BYTES, &tmB, mapa_shared(smem_u32(&full[i]), 0), k * 64, b_row(tile), pol_b);
        }
        bool ok = true;
        long long issued = pre;
        for (long long i = pre; i < n; ++i) {
          const int s = (int)(i % STAGES);
          const uint32_t r = (uint32_t)(i / STAGES);
          if (!mbar_wait(&empty[s], (r - 1) & 1u, abort_flag)) {
            record_error(a.err, DEV_TIMEOUT_EMPTY);
            *abort_flag = 1;
            ok = false;
            break;
          }
          const long long u = u0 + i;
          const int tile = (int)(u / kb), k = (int)(u % kb);
          const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], STAGE_TX);
          tma_load_2d_pair(sA + s * S::A_BYTES, &tmA, fb, k * 64, a_row(tile), pol);
          tma_load_2d_pair(sB + s * S::B_BYTES, &tmB, fb, k * 64, b_row(tile), pol_b);
          issued = i + 1;
        }
        // Every stage this CTA filled is consumed (its empty barrier completed by
        // rank 0's commit) before the CTA may leave: no commit then arrives on a
        // barrier of a CTA that has exited.  After a failure rank 0 waits instead
        // (bounded) for the copies it armed to land.
        const long long from = issued > STAGES ? issued - STAGES : 0;
        for (long long i = from; i < issued; ++i) {
          if (rank == 0 && !ok) mbar_wait(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u, nullptr);
          if (ok && !mbar_wait(&empty[i % STAGES], (uint32_t)(i / STAGES) & 1u, abort_flag)) {
            record_error(a.err, DEV_TIMEOUT_EMPTY);
            *abort_flag = 1;
            ok = false;
          }
        }
      }
    }
  } else if (warp == 1) {
    // CG = 2: only rank 0 issues; its MMAs read both CTAs' stages and write
    // both CTAs' accumulators, and each commit is sent to both CTAs' barriers
    if (lane == 0 && u1 > u0 && rank == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128 * CG, BN);
      long long i = 0;
      int seg = 0;
      for (long long u = u0; u < u1; ++seg) {
        const int tile = (int)(u / kb);
        const long long seg_begin = u;
        const long long seg_end = (long long)(tile + 1) * kb < u1 ? (long long)(tile + 1) * kb : u1;
        const int acc = seg % ACC;
        const uint32_t ar = (uint32_t)(seg / ACC);
        if (ar > 0 && !mbar_wait(&acc_empty[acc], (ar - 1) & 1u, abort_flag)) {
          record_error(a.err, DEV_TIMEOUT_ACC);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (; u < seg_end; ++u, ++i) {
          const int s = (int)(i % STAGES);
          if (!mbar_wait(&full[s], (uint32_t)(i / STAGES) & 1u, abort_flag)) {
            record_error(a.err, DEV_TIMEOUT_FULL);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sdesc_k_sw128(smem_u32(sA + s * S::A_BYTES));
          const uint64_t bd = sdesc_k_sw128(smem_u32(sB + s * S::B_BYTES));
          if constexpr (PAIR) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16_pair(d_tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), IDESC,
                             (u > seg_begin || kk > 0) ? 1u : 0u);
            umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 0));
            umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16(d_tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), IDESC,
                        (u > seg_begin || kk > 0) ? 1u : 0u);
            umma_commit(&empty[s]);
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          umma_commit_pair(mapa_shared(smem_u32(&acc_full[acc]), 0));
          umma_commit_pair(mapa_shared(smem_u32(&acc_full[acc]), 1));
        } else {
          umma_commit(&acc_full[acc]);
        }
        if (seg < 3) gemm_stamp(trace, 2 + 4 * seg);
      }
    }
  } else {
    // epilogue warps
    const int q = warp & 3;
    const int r = q * 32 + lane;
    pdl_wait();
    int seg = 0;
    for (long long u = u0; u < u1; ++seg) {
      const int tile = (int)(u / kb);
      const long long seg_begin = u;
      const long long seg_end = (long long)(tile + 1) * kb < u1 ? (long long)(tile + 1) * kb : u1;
      u = seg_end;
      const int acc = seg % ACC;
      // one thread waits (bounded) and publishes the outcome, so that every
      // epilogue thread leaves the loop together if the wait gave up
      if (threadIdx.x == 64) {
        const bool ok = mbar_wait(&acc_full[acc], (uint32_t)(seg / ACC) & 1u, abort_flag);
        if (!ok) {
          record_error(a.err, DEV_TIMEOUT_ACC);
          *abort_flag = 1;
        }
        flags[2 + (seg & 1)] = ok ? 1 : 0;
      }
      named_bar_sync(1, 128);
      if (!flags[2 + (seg & 1)]) break;
      if (threadIdx.x == 64 && seg < 3) gemm_stamp(trace, 3 + 4 * seg);
      tc_fence_after();
      // this CTA's 128-row tile (its half of a pair tile) and its split-K counter
      const int mt = (tile / a.n_tiles) * CG + (int)rank, nt = tile % a.n_tiles;
      const int ctile = tile * CG + (int)rank;
      const int m = mt * 128 + r;
      const int n0 = nt * BN;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const bool whole = (seg_begin == (long long)tile * kb) && (seg_end == (long long)(tile + 1) * kb);
      const bool vec = VecEpilogue<BN, EPI>::ON && vec_epilogue_ok(a);
      __nv_bfloat16* xt = reinterpret_cast<__nv_bfloat16*>(xch);
      constexpr bool XT_EPI = BN >= 64 && (EPI == EPI_QKNORM || EPI == EPI_LOGITS);
      __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(scratch + 4096 + 1024);
      // QKNORM's two store tiles sit in the residual ring (idle for it)
      __nv_bfloat16* vxt = (XT_EPI && vec_epilogue_ok(a) && !(EPI == EPI_LOGITS && a.scatter))
                               ? (EPI == EPI_QKNORM ? ring : xt)
                               : nullptr;
      const bool qk_wide = EPI == EPI_QKNORM && vxt != nullptr;  // the three-phase q/k-norm epilogue
      if (whole && vec && EPI == EPI_RESID) {
        constexpr int NCH = BN / 16, RG = S::RING;
#pragma unroll
        for (int pc = 0; pc < RG - 1; ++pc) vec_issue(a, mt * 128, n0 + pc * 16, ring + (pc % RG) * 2048, pc < NCH);
        for (int ci = 0; ci < NCH; ++ci) {
          float v[16];
          tmem_ld_x16(taddr + ci * 16, v);
          const int pc = ci + RG - 1;
          vec_issue(a, mt * 128, n0 + pc * 16, ring + (pc % RG) * 2048, pc < NCH);
          gemm_cp_wait<S::RING - 1>();
          tmem_wait_ld();
          named_bar_sync(1, 128);  // every thread's copies of chunk ci have landed
          vec_resid16(a, v, r, mt * 128, n0 + ci * 16, ring + (ci % RG) * 2048);
        }
        gemm_cp_wait<0>();
      } else if (whole && vec) {
        uint4 vp[2];
        vec_prefetch<EPI>(a, mt * 128, n0, vp);
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          uint4 vn[2];
          tmem_ld_x16(taddr + c0, v);
          if (c0 + 16 < BN) vec_prefetch<EPI>(a, mt * 128, n0 + c0 + 16, vn);
          tmem_wait_ld();
          vec_epilogue16<EPI>(a, v, r, mt * 128, n0 + c0, xt, vp);
          vp[0] = vn[0];
          vp[1] = vn[1];
        }
      } else if (whole && qk_wide) {
        if constexpr (EPI == EPI_QKNORM)
          qknorm_wide(
              a,
              [&](int c0, float* v) {
                tmem_ld_x16(taddr + c0, v);
                tmem_wait_ld();
              },
              r, mt, n0, 0, BN, xch, vxt);
      } else if (whole && EPI == EPI_LOGITS && BN >= 128 && vxt != nullptr) {
        if constexpr (EPI == EPI_LOGITS && BN >= 128)
          logits_wide<BN>(
              a,
              [&](int c0, float* v) {
                tmem_ld_x16(taddr + c0, v);
                tmem_wait_ld();
              },
              r, mt, n0, ring);
      } else if (whole) {
        // chunks of 16 columns; each chunk's global reads issued one chunk ahead
        float pre[32];
        bool have = epilogue_prefetch<EPI>(a, m, n0, pre);
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16], nxt[32];
          tmem_ld_x16(taddr + c0, v);
          const bool more = have && c0 + 16 < BN && epilogue_prefetch<EPI>(a, m, n0 + c0 + 16, nxt);
          tmem_wait_ld();
          epilogue16<EPI>(a, v, r, m, mt, n0 + c0, xch, xch64, have ? pre : nullptr, vxt);
          if (more) {
#pragma unroll
            for (int j = 0; j < 32; ++j) pre[j] = nxt[j];
          }
        }
      } else {
        const long long c_first = cta_of_unit((long long)tile * kb, U, G);
        const long long c_last = cta_of_unit((long long)(tile + 1) * kb - 1, U, G);
        if (c != c_first) {
          // a later contributor: this tile is its first segment (partials slot 0)
          float* mine = a.ws + ((long long)((c * CG + (int)rank) * 2) * BN) * 128;
          for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            tmem_ld_x16(taddr + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) __stcg(mine + (long long)(c0 + j) * 128 + r, v[j]);
          }
          // the barrier orders every thread's partial stores before thread 64's
          // release, which publishes them (a per-thread fence would wait, on
          // every thread, for all of the SM's loads in flight)
          named_bar_sync(1, 128);
          if (threadIdx.x == 64) {
            if (seg < 3) gemm_stamp(trace, 4 + 4 * seg);
            gemm_red_release(a.counters + ctile, 1);
          }
        } else {
          // the head: wait for the others, stage their partials, finish the tile
          const int others = (int)(c_last - c_first);
          if (threadIdx.x == 64) {
            bool ok = gemm_ld_acquire(a.counters + ctile) >= others;
            if (!ok) {
              const uint64_t t0 = global_ns();
              for (uint32_t i = 1;; ++i) {
                if (gemm_ld_acquire(a.counters + ctile) >= others) {
                  ok = true;
                  break;
                }
                if ((i & 63u) == 0 && (*abort_flag || global_ns() - t0 > FM_WAIT_NS)) break;
                __nanosleep(64);
              }
            }
            if (!ok) {
              record_error(a.err, DEV_TIMEOUT_OTHER);
              *abort_flag = 1;
            } else {
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
            flags[1] = ok ? 1 : 0;
            if (seg < 3) gemm_stamp(trace, 4 + 4 * seg);
          }
          named_bar_sync(1, 128);
          if (flags[1]) {
            // the pipeline buffers are idle: every k-block of this CTA was consumed
            float* stage = reinterpret_cast<float*>(sA);
            constexpr int AREA = STAGES * (S::A_BYTES + S::B_BYTES);
            const int per_col = others * 128 * 4;
            int cols = (AREA / per_col) / 16 * 16;
            if (cols > BN) cols = BN;
            bool staged_ok = true;
            if (cols < 16) {
              // many contributors (narrow blocks, small M, long K): one 16-column
              // chunk at a time, the partials staged in groups
              constexpr int MAX_O = AREA / (16 * 512);
              int round = 0;
              for (int c0 = 0; c0 < BN && staged_ok; c0 += 16) {
                float v[16];
                tmem_ld_x16(taddr + c0, v);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(0.0f, v[j]);
                for (int og = 0; og < others; og += MAX_O, ++round) {
                  const int n = (others - og) < MAX_O ? (others - og) : MAX_O;
                  named_bar_sync(1, 128);  // the previous group was consumed
                  if (threadIdx.x == 64) {
                    mbar_arrive_expect_tx(fix_bar, (uint32_t)(n * 16 * 512));
                    for (int o = 0; o < n; ++o)
                      bulk_load(stage + (long long)o * 16 * 128,
                                a.ws + ((long long)(((c_first + 1 + og + o) * CG + rank) * 2) * BN + c0) * 128, 16u * 512u,
                                fix_bar);
                    flags[1] = mbar_wait(fix_bar, (uint32_t)round & 1u, nullptr) ? 1 : 0;
                    if (!flags[1]) {
                      record_error(a.err, DEV_TIMEOUT_OTHER);
                      *abort_flag = 1;
                    }
                  }
                  named_bar_sync(1, 128);
                  if (!flags[1]) {
                    staged_ok = false;
                    break;
                  }
                  for (int o = 0; o < n; ++o) {
                    const float* src = stage + (long long)o * 16 * 128 + r;
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], src[j * 128]);
                  }
                }
                if (!staged_ok) break;
                epilogue16<EPI>(a, v, r, m, mt, n0 + c0, xch, xch64, nullptr, vxt);
              }
              cols = BN + 1;  // the staged rounds below are skipped
            }
            float pre[32];
            bool have = false;
            uint4 vp[2];
            constexpr bool RESID_RING = EPI == EPI_RESID && S::RING_BYTES > 0;
            constexpr int NCH = BN / 16;
            // residual epilogue with every partial staged in one round: the
            // whole residual tile ([BN / 16 chunks][16][128] bf16) follows the
            // partials in the idle buffers, all of it requested at once
            const bool preload =
                vec && RESID_RING && cols == BN && (long long)others * BN * 512 + BN * 256 <= (long long)AREA;
            __nv_bfloat16* res_tile = reinterpret_cast<__nv_bfloat16*>(stage + (long long)others * BN * 128);
            for (int col0 = 0, round = 0; cols <= BN && col0 < BN; col0 += cols, ++round) {
              const int ncols = (BN - col0) < cols ? (BN - col0) : cols;
              if (threadIdx.x == 64) {
                mbar_arrive_expect_tx(fix_bar, (uint32_t)(others * ncols * 512));
                for (int o = 0; o < others; ++o)
                  bulk_load(stage + (long long)o * ncols * 128,
                            a.ws + ((long long)(((c_first + 1 + o) * CG + rank) * 2) * BN + col0) * 128, (uint32_t)(ncols * 512),
                            fix_bar);
              }
              if (round == 0) {
                // the epilogue's own global reads go out after the partials' bulk copies
                have = !vec && !qk_wide && epilogue_prefetch<EPI>(a, m, n0, pre);
                if (vec && !RESID_RING) vec_prefetch<EPI>(a, mt * 128, n0, vp);
                if (preload) {
                  for (int pc = 0; pc < NCH; ++pc) vec_issue(a, mt * 128, n0 + pc * 16, res_tile + pc * 2048, true);
                } else if (vec && RESID_RING) {
#pragma unroll
                  for (int pc = 0; pc < S::RING - 1; ++pc)
                    vec_issue(a, mt * 128, n0 + pc * 16, ring + (pc % S::RING) * 2048, pc < NCH);
                }
              }
              if (threadIdx.x == 64) {
                flags[1] = mbar_wait(fix_bar, (uint32_t)round & 1u, nullptr) ? 1 : 0;
                if (!flags[1]) {
                  record_error(a.err, DEV_TIMEOUT_OTHER);
                  *abort_flag = 1;
                }
                if (round == 0) gemm_stamp(trace, 15);
              }
              if (preload && round == 0) gemm_cp_wait<0>();  // this thread's residual copies
              named_bar_sync(1, 128);
              if (!flags[1]) {
                staged_ok = false;
                break;
              }
              if (qk_wide) {
                // the head's accumulator, then the later CTAs' staged partials, in contributor order
                if constexpr (EPI == EPI_QKNORM)
                  qknorm_wide(
                      a,
                      [&](int c0, float* v) {
                        tmem_ld_x16(taddr + c0, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(0.0f, v[j]);
                        for (int o = 0; o < others; ++o) {
                          const float* src = stage + ((long long)o * ncols + (c0 - col0)) * 128 + r;
#pragma unroll
                          for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], src[j * 128]);
                        }
                      },
                      r, mt, n0, col0, col0 + ncols, xch, vxt);
                named_bar_sync(1, 128);  // the staging area is refilled by the next round
                continue;
              }
              for (int c0 = col0; c0 < col0 + ncols; c0 += 16) {
                float v[16], nxt[32];
                uint4 vn[2];
                tmem_ld_x16(taddr + c0, v);
                const bool more =
                    have && c0 + 16 < BN && epilogue_prefetch<EPI>(a, m, n0 + c0 + 16, nxt);
                const int ci = c0 / 16;
                if (vec && !RESID_RING && c0 + 16 < BN) vec_prefetch<EPI>(a, mt * 128, n0 + c0 + 16, vn);
                if (vec && RESID_RING && !preload) {
                  const int pc = ci + S::RING - 1;
                  vec_issue(a, mt * 128, n0 + pc * 16, ring + (pc % S::RING) * 2048, pc < NCH);
                  gemm_cp_wait<S::RING - 1>();
                }
                tmem_wait_ld();
                // contributor order: the head's own accumulator first, then the later CTAs
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(0.0f, v[j]);
                for (int o = 0; o < others; ++o) {
                  const float* src = stage + ((long long)o * ncols + (c0 - col0)) * 128 + r;
#pragma unroll
                  for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], src[j * 128]);
                }
                if (preload) {
                  vec_resid16(a, v, r, mt * 128, n0 + c0, res_tile + ci * 2048);
                } else if (vec && RESID_RING) {
                  named_bar_sync(1, 128);  // every thread's copies of chunk ci have landed
                  vec_resid16(a, v, r, mt * 128, n0 + c0, ring + (ci % S::RING) * 2048);
                } else if (vec) {
                  vec_epilogue16<EPI>(a, v, r, mt * 128, n0 + c0, xt, vp);
                  vp[0] = vn[0];
                  vp[1] = vn[1];
                } else {
                  epilogue16<EPI>(a, v, r, m, mt, n0 + c0, xch, xch64, have ? pre : nullptr, vxt);
                }
                if (more) {
#pragma unroll
                  for (int j = 0; j < 32; ++j) pre[j] = nxt[j];
                }
              }
              named_bar_sync(1, 128);  // the staging area is refilled by the next round
            }
            if (vec && RESID_RING) gemm_cp_wait<0>();
            if (threadIdx.x == 64) {
              if (staged_ok) a.counters[ctile] = 0;
              if (seg < 3) gemm_stamp(trace, 5 + 4 * seg);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));  // rank 0 issues the MMAs
        else
          mbar_arrive(&acc_empty[acc]);
      }
    }
  }
  // a pair leaves together: no barrier or TMEM of one CTA is signalled or
  // read by the other after it exits
  if constexpr (PAIR)
    cluster_sync();
  else
    __syncthreads();
  if (threadIdx.x == 0) gemm_stamp(trace, 14);
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace fm
