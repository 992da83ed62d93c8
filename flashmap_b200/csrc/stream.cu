// The streamed single-launch draft pass (stream.cuh): kernel and launch.
#include <cstdio>

#include "philox.cuh"
#include "rows.cuh"
#include "stream.cuh"

namespace fm {
namespace stream {

namespace {

// ------------------------------------------------------------------ shared memory
constexpr int EPI_SCRATCH = 34 * 1024;  // epilogue / attention warps: exchange tiles, staging, merge buffers
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + NA * A_BYTES;
constexpr int OFF_STAGE = OFF_B + NB * B_BYTES;
constexpr int OFF_CONST = OFF_STAGE + BATCH * STAGE_SLOT;  // constant rows of a transform stage's units
constexpr int OFF_EPI = OFF_CONST + MAX_TRANSFORM_UNITS * CONST_SLOT;
constexpr int OFF_BSTAT = OFF_EPI + EPI_SCRATCH;       // operand warps: [16][2] row statistics, misc
constexpr int MAX_STAT_TILES = 40;                      // source rows of up to 40 * 128 features
constexpr int OFF_SSTAT = OFF_BSTAT + 256;              // the producing stage's per-tile statistics
constexpr int OFF_SDESC = OFF_SSTAT + MAX_STAT_TILES * 16 * 2 * 4;  // stage descriptors: 2 per warp group
constexpr int OFF_BAR = OFF_SDESC + 4 * (int)sizeof(Stage);
constexpr int N_BARS = 2 * NA + 2 * NB + 2 + 2 + 1;
constexpr int OFF_FLAGS = OFF_BAR + N_BARS * 8;
constexpr int SMEM_USED = OFF_FLAGS + 64;
constexpr int SMEM_TOTAL = SMEM_USED + 1024;  // alignment slack
static_assert(SMEM_TOTAL <= 232448, "streamed pass exceeds the shared memory of one SM");
static_assert(OFF_B % 1024 == 0 && OFF_A % 1024 == 0, "UMMA operand rings need 1024-byte alignment");
static_assert(sizeof(Stage) % 16 == 0 && OFF_SDESC % 16 == 0, "stage descriptors are copied as 16-byte vectors");

// flags: each written by one thread of one warp group and read by the group after a barrier
constexpr int F_ABORT = 0, F_DEP = 1, F_EPI = 2, F_TICKET = 3, F_XA = 4, F_XW = 5 /* 5, 6 */, F_BDEP = 7,
              F_BW = 8 /* 8, 9 */, F_BCOPY = 10;

// ------------------------------------------------------------------ cross-CTA counters
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// atomic add with acquire-release semantics at GPU scope: the caller's CTA
// barrier before it orders the group's stores, the one after it the group's loads
__device__ __forceinline__ unsigned long long atom_add_acqrel_u64(unsigned long long* p, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ bool aborted(const Params& P, volatile int* cta_abort) {
  return *cta_abort != 0 || *reinterpret_cast<volatile unsigned long long*>(P.words + 1) != 0ull;
}
__device__ __forceinline__ void raise_abort(const Params& P, volatile int* cta_abort, int code) {
  record_error(P.err, code);
  *cta_abort = 1;
  atomicExch(P.words + 1, 1ull);
}
// wait (bounded) until *p >= target
__device__ bool wait_count(const Params& P, const unsigned long long* p, unsigned long long target,
                           volatile int* cta_abort) {
  if (ld_acquire_u64(p) >= target) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(20);
    if (ld_acquire_u64(p) >= target) return true;
    if ((i & 15u) == 0) {
      if (aborted(P, cta_abort)) {
        *cta_abort = 1;  // the rest of this CTA gives up at its next ring wait
        return false;
      }
      if (global_ns() - t0 > FM_WAIT_NS) {
        raise_abort(P, cta_abort, DEV_TIMEOUT_OTHER);
        return false;
      }
    }
  }
}
// the inputs of stage S complete (its one or two dependencies)
__device__ bool wait_deps(const Params& P, const Stage& S, volatile int* cta_abort) {
  if (S.dep >= 0 && !wait_count(P, P.done + S.dep, (unsigned long long)P.stages[S.dep].pieces, cta_abort)) return false;
  if (S.dep2 >= 0 && !wait_count(P, P.done + S.dep2, (unsigned long long)P.stages[S.dep2].pieces, cta_abort))
    return false;
  return true;
}
// a ring wait that gives up on an abort of this CTA or after FM_WAIT_NS
__device__ __forceinline__ bool ring_wait(const Params& P, uint64_t* bar, uint32_t parity, volatile int* cta_abort) {
  if (mbar_wait(bar, parity, cta_abort)) return true;
  if (!*cta_abort) raise_abort(P, cta_abort, DEV_TIMEOUT_FULL);
  return false;
}

// A warp group's shared copy of stage s's descriptor (threads t < nthreads of
// the group copy it; the caller's barrier publishes it).  Threads then read
// the descriptor from shared memory instead of each holding a local copy.
__device__ __forceinline__ void load_stage(const Params& P, int s, Stage* dst, int t, int nthreads) {
  const uint4* src = reinterpret_cast<const uint4*>(P.stages + s);
  for (int i = t; i < (int)(sizeof(Stage) / 16); i += nthreads) reinterpret_cast<uint4*>(dst)[i] = __ldg(src + i);
}

// CTA c's units of a stream-K split of U units over G CTAs (32-bit: the host
// checks U * G < 2^31, so the products and quotients stay in range)
__device__ __forceinline__ int split_at(int U, int G, int c) { return (int)((uint32_t)c * (uint32_t)U / (uint32_t)G); }
__device__ __forceinline__ void unit_range(int U, int G, int c, int& u0, int& u1) {
  u0 = split_at(U, G, c);
  u1 = split_at(U, G, c + 1);
}
// the CTA of a split whose range holds unit u
__device__ __forceinline__ int cta_of(int u, int U, int G) {
  return (int)(((uint32_t)u * (uint32_t)G + (uint32_t)G - 1u) / (uint32_t)U);
}
// the virtual CTA of CTA c in a GEMM stage (-1: none) and its units
__device__ __forceinline__ int stage_vcta(const Stage& S, int c, int G) {
  const int v = (c - S.rot % G + G) % G;
  return v < S.vg ? v : -1;
}
__device__ __forceinline__ int stage_range(const Stage& S, int c, int G, int& u0, int& u1) {
  const int v = stage_vcta(S, c, G);
  if (v < 0) {
    u0 = u1 = 0;
    return -1;
  }
  unit_range((int)S.ep.units, S.vg, v, u0, u1);
  return v;
}

// Operand blocks and tiles of a cross-attention item (the split of cross_attn_kernel)
struct XaItem {
  int h, split, k_begin, k_end, ntiles, n_active;
};
__device__ __forceinline__ bool xa_item(const Params& P, const Stage& S, int it, XaItem& x) {
  int ctx = P.lengths[0] + 1;
  if (ctx > P.cache_len || ctx < 1) ctx = ctx < 1 ? 1 : P.cache_len;  // recorded by the prep stage
  const int per = xa_split_keys(ctx, S.nsplit);
  x.h = it / S.nsplit;
  x.split = it % S.nsplit;
  x.k_begin = x.split * per;
  x.k_end = min(ctx, x.k_begin + per);
  x.n_active = (ctx + per - 1) / per;
  if (x.k_begin >= ctx) return false;
  x.ntiles = (x.k_end - x.k_begin + XA_TILE - 1) / XA_TILE;
  return true;
}

// ring slots one 64-key tile of K and V takes
template <int HD>
__host__ __device__ constexpr int xa_slots() {
  return 2 * XA_TILE * HD * 2 > A_BYTES ? 2 : 1;
}

// slots this CTA takes from the weight ring in stage S
template <int HD>
__device__ int stage_slots(const Params& P, const Stage& S, int c, int G) {
  if (S.kind == K_GEMM) {
    int u0, u1;
    stage_range(S, c, G, u0, u1);
    return u1 - u0;
  }
  if (S.kind == K_XATTN) {
    int n = 0;
    XaItem x;
    for (int it = c; it < P.heads * S.nsplit; it += G)
      if (xa_item(P, S, it, x)) n += x.ntiles * xa_slots<HD>();
    return n;
  }
  return 0;
}

// ------------------------------------------------------------------ per-token sums over a tile's 128 rows
// Each of the 128 epilogue threads holds 16 token values of its row; the
// sum over rows of each token: a transposing shuffle reduction per warp
// (lanes 2i, 2i+1 end with token tl's warp sum), then the four warp
// quarters in order.  Result in out[0..15] (shared).
__device__ __forceinline__ void token_sums(float* val, float* xch, float* out, int q, int lane, int t) {
#pragma unroll
  for (int width = 8; width >= 1; width >>= 1) {
    const bool up = (lane & (width * 2)) != 0;
#pragma unroll
    for (int i = 0; i < width; ++i) {
      const float send = up ? val[i] : val[i + width];
      const float keep = up ? val[i + width] : val[i];
      val[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, width * 2));
    }
  }
  val[0] = __fadd_rn(val[0], __shfl_xor_sync(0xffffffffu, val[0], 1));
  const int tl = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
  if ((lane & 1) == 0) xch[q * 16 + tl] = val[0];
  named_bar_sync(1, 128);
  if (t < 16) out[t] = __fadd_rn(__fadd_rn(__fadd_rn(xch[t], xch[16 + t]), xch[32 + t]), xch[48 + t]);
  named_bar_sync(1, 128);
}

// ------------------------------------------------------------------ epilogue of one finished tile
// The inputs of a tile's epilogue that do not depend on its sums (bias,
// gate, the residual rows, the rotary factors), loaded before the tile's
// accumulator is ready so that finishing the tile takes no extra round trip.
struct EpiPre {
  float bias, gate, warm;
  float pre[32];
};
// the tile's constants: bias, gate, rotary factors, and a touch of the norm
// weight and column ids the fused epilogue reads (so they sit in L1)
__device__ __forceinline__ void epi_constants(const Params& P, const Stage& S, int mt, int r, EpiPre& e) {
  const GemmArgs& a = S.ep;
  const int m = mt * 128 + r;
  const bool mvalid = m < a.M;
  e.bias = (a.bias && mvalid) ? bf2f(a.bias[m]) : 0.0f;
  e.gate = (S.ekind == E_RESID && mvalid) ? bf2f(a.gate[m]) : 0.0f;
  e.warm = 0.0f;
  if (S.ekind == E_QKV || S.ekind == E_QNORM || S.ekind == E_KVCACHE) {
    const int part = (mt * 128) / a.part_rows;
    const int d = (m % a.part_rows) % a.head_dim;
    const __nv_bfloat16* w = S.ekind == E_KVCACHE ? a.norm_w0 + (long long)((mt * 128) / (2 * a.part_rows)) *
                                                                    a.norm_layer_stride
                                                  : (part == 0 ? a.norm_w0 : a.norm_w1);
    if (w != nullptr && part < 2) e.warm = bf2f(w[d]);
  } else if (S.ekind == E_LOGITS && a.col_ids && mvalid) {
    e.warm = (float)a.col_ids[m];
  }
  if (S.ekind == E_QKV || S.ekind == E_QNORM) {
    // rotary factors of the slots' positions lengths[0] + 1 + j
    const int d = (m % a.part_rows) % a.head_dim;
    const int base = P.lengths[0] + 1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      int pos = base + j;
      if (pos < 0 || pos >= P.rope_len) pos = 0;  // recorded by the prep stage
      e.pre[j] = P.rope_cos[(long long)pos * P.half + (d >> 1)];
      e.pre[16 + j] = P.rope_sin[(long long)pos * P.half + (d >> 1)];
    }
  }
}
// the residual rows (E_RESID), final once the stage's inputs are
__device__ __forceinline__ void epi_residual(const Stage& S, int mt, int r, EpiPre& e) {
  const GemmArgs& a = S.ep;
  const int m = mt * 128 + r;
  const bool mvalid = m < a.M;
#pragma unroll
  for (int j = 0; j < 16; ++j) e.pre[j] = (mvalid && j < a.N) ? bf2f(__ldcg(a.out + (long long)j * a.ldo + m)) : 0.0f;
}

// v: the tile's fp32 sums for tokens 0..15 of row r.  Stores the outputs
// (the arithmetic of gemm_bf16_tc's epilogues) and the tile's row statistics.
template <int HD>
__device__ void finish_tile(const Params& P, const Stage& S, float* v, int r, int mt, uint8_t* escr, EpiPre& e) {
  const int lane = threadIdx.x & 31, q = (threadIdx.x >> 5) & 3, t = (int)threadIdx.x - 64;
  float* xch = reinterpret_cast<float*>(escr);
  unsigned long long* xch64 = reinterpret_cast<unsigned long long*>(escr + 4096);
  float* sums = reinterpret_cast<float*>(escr + 4096 + 512);  // [2][16]
  GemmArgs a = S.ep;
  const int m = mt * 128 + r;
  const bool mvalid = m < a.M;
  float y[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) y[j] = 0.0f;
  if (S.ekind == E_STORE || S.ekind == E_GELU || S.ekind == E_RESID) {
    const float b = e.bias, g = e.gate;
    const float* pre = e.pre;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float o = round_bf(__fadd_rn(v[j], b));
      if (S.ekind == E_GELU) {
        o = round_bf(__fmul_rn(__fmul_rn(o, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn(o, 0.70710678118654752f)))));
      } else if (S.ekind == E_RESID) {
        const float gy = round_bf(__fmul_rn(g, o));
        o = round_bf(__fadd_rn(pre[j], gy));
      }
      if (mvalid) {
        y[j] = o;
        if (j < a.N) a.out[(long long)j * a.ldo + m] = f2bf(o);
      }
    }
  } else if (S.ekind == E_SWIGLU) {
    epilogue16<EPI_SWIGLU>(a, v, r, m, mt, 0, xch, xch64);
  } else if (S.ekind == E_QKV || S.ekind == E_QNORM) {
    epilogue16<EPI_QKNORM>(a, v, r, m, mt, 0, xch, xch64, e.pre);
  } else if (S.ekind == E_KVCACHE) {
    a.positions = P.lengths;  // the anchor row (token 0 of sequence 0) sits at position lengths[0]
    epilogue16<EPI_KVCACHE>(a, v, r, m, mt, 0, xch, xch64);
  } else if (S.ekind == E_LOGITS) {
    a.out = P.logits;
    a.ldo = P.ldl;
    a.scatter = P.scatter;
    a.argmax_keys = P.keys;
    epilogue16<EPI_LOGITS>(a, v, r, m, mt, 0, xch, xch64);
  }
  if (S.stats != S_NONE) {
    // per token over the tile's 128 rows: (sum, sum of squared deviations from
    // the tile mean) for a LayerNorm, (sum of squares, 0) for an RMSNorm
    float w[16];
    if (S.stats == S_LN) {
#pragma unroll
      for (int j = 0; j < 16; ++j) w[j] = y[j];
      token_sums(w, xch, sums, q, lane, t);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float dd = mvalid ? __fsub_rn(y[j], __fmul_rn(sums[j], 0.0078125f)) : 0.0f;  // mean over 128 rows
        w[j] = __fmul_rn(dd, dd);
      }
      token_sums(w, xch, sums + 16, q, lane, t);
      if (t < 16) {
        __stcg(S.stats_out + (mt * 16 + t) * 2, sums[t]);
        __stcg(S.stats_out + (mt * 16 + t) * 2 + 1, sums[16 + t]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) w[j] = __fmul_rn(y[j], y[j]);
      token_sums(w, xch, sums, q, lane, t);
      if (t < 16) {
        __stcg(S.stats_out + (mt * 16 + t) * 2, sums[t]);
        __stcg(S.stats_out + (mt * 16 + t) * 2 + 1, 0.0f);
      }
    }
  }
}

// The block self-attention of the head group of a finished q|k|v tile group
// (the three tiles of group g hold q, k, v of heads g*128/HD ...).
template <int HD>
__device__ void group_attention(const Params& P, const Stage& S, int g, uint8_t* escr) {
  constexpr int HPG = 128 / HD;  // heads per group
  constexpr int PART = 16 * HD * 2;
  const int t = (int)threadIdx.x - 64, w = t >> 5;
  const int D = P.hidden;
  uint8_t* st = escr + 5120;  // [HPG][q | k | v][16 x HD] swizzled
  const bf16* qkv = S.ep.out;  // [16, 3D]
  for (int idx = t; idx < HPG * 3 * 16 * (HD / 8); idx += 128) {
    const int hh = idx / (3 * 16 * (HD / 8));
    const int rem = idx % (3 * 16 * (HD / 8));
    const int part = rem / (16 * (HD / 8)), rr = rem % (16 * (HD / 8)), row = rr / (HD / 8), ch = rr % (HD / 8);
    const int h = g * HPG + hh;
    const uint4 val = __ldcg(reinterpret_cast<const uint4*>(qkv + (long long)row * 3 * D + part * D + h * HD + ch * 8));
    *reinterpret_cast<uint4*>(st + (hh * 3 + part) * PART + blk_sw(row, ch)) = val;
  }
  named_bar_sync(1, 128);
  if (w < HPG) {
    const int h = g * HPG + w;
    const uint32_t base = smem_u32(st + w * 3 * PART);
    bf16* out = S.attn + h * HD;
    block_attn_head<HD>(base, base + PART, base + 2 * PART, P.scale, [&](int i, int d, float lo, float hi) {
      *reinterpret_cast<__nv_bfloat162*>(out + (long long)i * D + d) = __floats2bfloat162_rn(lo, hi);
    });
  }
}

// ------------------------------------------------------------------ operand construction
// One 16 x 64 operand block in the UMMA K-major 128-byte-swizzled layout:
// row n's 16-byte chunk c at n * 128 + ((c ^ (n & 7)) << 4).
__device__ __forceinline__ uint32_t b_off(int n, int c) { return (uint32_t)(n * 128 + ((c ^ (n & 7)) << 4)); }

__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16u : 0u)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}


}  // namespace

// ------------------------------------------------------------------ the kernel
template <int HD>
__global__ void __launch_bounds__(THREADS, 1) stream_kernel(const __grid_constant__ Params P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + OFF_A;
  uint8_t* sB = smem + OFF_B;
  uint8_t* sStage = smem + OFF_STAGE;
  uint8_t* escr = smem + OFF_EPI;
  float* bstat = reinterpret_cast<float*>(smem + OFF_BSTAT);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty = full + NA;
  uint64_t* bfull = empty + NA;
  uint64_t* bempty = bfull + NB;
  uint64_t* acc_full = bempty + NB;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  int* flags = reinterpret_cast<int*>(smem + OFF_FLAGS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(flags + 12);
  volatile int* cta_abort = flags + F_ABORT;
  Stage* sdesc = reinterpret_cast<Stage*>(smem + OFF_SDESC);  // [0, 1] epilogue warps, [2, 3] operand warps

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int n_stages = P.n_stages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NA; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&bfull[i], 1);
      mbar_init(&bempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 12; ++i) flags[i] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t bump = P.offset_ptr ? *reinterpret_cast<volatile uint32_t*>(P.offset_ptr) + 1u : 0u;

  if (warp == 0) {
    // ---------------------------------------------------------- weight and K/V stream
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t ia = 0;
      bool ok = true;
      for (int s = 0; s < n_stages && ok; ++s) {
        const Stage S = P.stages[s];  // a local copy: its fields are read without a global round trip
        if (S.kind == K_GEMM) {
          int u0, u1;
          stage_range(S, c, G, u0, u1);
          const CUtensorMap* map = &P.maps[S.map];
          if (u1 > u0) tma_prefetch_desc(map);
          for (int u = u0; u < u1; ++u) {
            const int slot = ia % NA;
            if (ia >= NA && !ring_wait(P, &empty[slot], ((ia / NA) - 1) & 1u, cta_abort)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[slot], A_BYTES);
            tma_load_2d_hint(sA + slot * A_BYTES, map, &full[slot], (int)(u % S.ep.kb) * 64, (int)(u / S.ep.kb) * 128,
                             pol);
            ++ia;
          }
        } else if (S.kind == K_XATTN) {
          constexpr int TB = XA_TILE * HD * 2;  // bytes of K (or V) of one tile
          constexpr int SPT = xa_slots<HD>();
          const CUtensorMap* map = &P.maps[P.cache_map];
          const int anchor = P.lengths[0];
          XaItem x;
          for (int it = c; it < P.heads * S.nsplit && ok; it += G) {
            if (!xa_item(P, S, it, x)) continue;
            // rows of (layer, k | v, sequence 0, head) in the cache viewed as [rows, head_dim]
            const long long krow = (((long long)S.layer * 2 + 0) * P.cache_batch * P.heads + x.h) * P.cache_len;
            const long long vrow = (((long long)S.layer * 2 + 1) * P.cache_batch * P.heads + x.h) * P.cache_len;
            for (int tl = 0; tl < x.ntiles && ok; ++tl) {
              const int row = x.k_begin + tl * XA_TILE;
              if (anchor >= row && anchor < row + XA_TILE) {
                // the anchor's keys and values are written by this draft: wait, then read them through TMA
                if (!wait_count(P, P.done + S.dep2, (unsigned long long)P.stages[S.dep2].pieces, cta_abort)) {
                  ok = false;
                  break;
                }
                fence_proxy_async_global();
              }
              for (int sl = 0; sl < SPT; ++sl) {
                const int slot = ia % NA;
                if (ia >= NA && !ring_wait(P, &empty[slot], ((ia / NA) - 1) & 1u, cta_abort)) {
                  ok = false;
                  break;
                }
                uint8_t* dst = sA + slot * A_BYTES;
                if (SPT == 2) {
                  mbar_arrive_expect_tx(&full[slot], TB);
                  const long long rr = (sl == 0 ? krow : vrow) + row;
#pragma unroll
                  for (int bx = 0; bx < HD / 64; ++bx)
                    tma_load_2d(dst + bx * XA_TILE * 128, map, &full[slot], bx * 64, (int)rr);
                } else {
                  mbar_arrive_expect_tx(&full[slot], 2 * TB);
#pragma unroll
                  for (int bx = 0; bx < HD / 64; ++bx) {
                    tma_load_2d(dst + bx * XA_TILE * 128, map, &full[slot], bx * 64, (int)(krow + row));
                    tma_load_2d(dst + TB + bx * XA_TILE * 128, map, &full[slot], bx * 64, (int)(vrow + row));
                  }
                }
                ++ia;
              }
            }
          }
        }
      }
      if (!ok) {
        // every issued copy lands before the CTA's shared memory goes away
        for (uint32_t i = ia > NA ? ia - NA : 0; i < ia; ++i) mbar_wait(&full[i % NA], (i / NA) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- tensor-core MMA
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128, 16);
      uint32_t ia = 0, ib = 0, sg = 0;
      bool ok = true, any = false;
      for (int s = 0; s < n_stages && ok; ++s) {
        const Stage S = P.stages[s];  // a local copy: its fields are read without a global round trip
        if (S.kind != K_GEMM) {
          ia += (uint32_t)stage_slots<HD>(P, S, c, G);
          continue;
        }
        int u0, u1;
        stage_range(S, c, G, u0, u1);
        const int kb = S.ep.kb;
        for (int u = u0; u < u1 && ok;) {
          const int tile = u / kb;
          const int sb = u, se = min((tile + 1) * kb, u1);
          const int acc = sg & 1;
          if (sg >= 2 && !ring_wait(P, &acc_empty[acc], ((sg >> 1) - 1) & 1u, cta_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + (uint32_t)(acc * 16);
          for (; u < se; ++u) {
            const int sa = ia % NA, sbk = ib % NB;
            if (!ring_wait(P, &full[sa], (ia / NA) & 1u, cta_abort) ||
                !ring_wait(P, &bfull[sbk], (ib / NB) & 1u, cta_abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = sdesc_k_sw128(smem_u32(sA + sa * A_BYTES));
            const uint64_t bd = sdesc_k_sw128(smem_u32(sB + sbk * B_BYTES));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16(d_tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), IDESC, (u > sb || kk > 0) ? 1u : 0u);
            umma_commit(&empty[sa]);
            umma_commit(&bempty[sbk]);
            any = true;
            ++ia;
            ++ib;
          }
          if (!ok) break;
          umma_commit(&acc_full[acc]);
          ++sg;
        }
      }
      if (any) {
        // every MMA issued has completed before the accumulators are released
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr);
      }
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------- epilogues, attention, tokens
    const int q = warp & 3, r = q * 32 + lane, t = (int)threadIdx.x - 64;
    uint32_t ia = 0, sg = 0;
    bool ok = true;
    for (int s = 0; s < n_stages && ok; ++s) {
      // the group's shared copy of the descriptor (double-buffered: the barrier after
      // each copy orders it after every reader of the copy two stages back)
      load_stage(P, s, sdesc + (s & 1), t, 128);
      named_bar_sync(1, 128);
      const Stage& S = sdesc[s & 1];
      if (S.kind == K_GEMM) {
        int u0, u1;
        const int v = stage_range(S, c, G, u0, u1);
        const int kb = S.ep.kb;
        // the first segment's constants are loaded before any wait: their latency hides under it
        EpiPre pf;
        if (u1 > u0) epi_constants(P, S, u0 / kb, r, pf);
        if (u1 > u0 && S.ekind == E_RESID) {
          // the residual rows are final once the stage's inputs are (every earlier
          // writer of x is an ancestor of its dependency): wait before reading them
          if (t == 0) flags[F_DEP] = wait_deps(P, S, cta_abort) ? 1 : 0;
          named_bar_sync(1, 128);
          if (!flags[F_DEP]) {
            ok = false;
            break;
          }
        }
        for (int u = u0; u < u1;) {
          const int tile = u / kb;
          const int sb = u, se = min((tile + 1) * kb, u1);
          u = se;
          const int acc = sg & 1;
          if (sb != u0) epi_constants(P, S, tile, r, pf);
          if (S.ekind == E_RESID) epi_residual(S, tile, r, pf);
          if (t == 0) flags[F_EPI] = ring_wait(P, &acc_full[acc], (sg >> 1) & 1u, cta_abort) ? 1 : 0;
          named_bar_sync(1, 128);
          if (!flags[F_EPI]) {
            ok = false;
            break;
          }
          tc_fence_after();
          float v16[16];
          tmem_ld_x16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 16), v16);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
          ++sg;
          const bool whole = sb == tile * kb && se == (tile + 1) * kb;
          bool finisher = whole;
          if (!whole) {
            // publish this CTA's partial (row r's 16 tokens contiguous); the last
            // contributor to arrive finishes the tile
            const int U = (int)S.ep.units;
            const int vg = S.vg;
            const int c_first = cta_of(tile * kb, U, vg);
            const int c_last = cta_of((tile + 1) * kb - 1, U, vg);
            // virtual CTAs between c_first and c_last without units (a stage of fewer
            // units than virtual CTAs) contribute nothing
            int n_contrib = 0;
            for (int cc = c_first, a0 = split_at(U, vg, c_first); cc <= c_last; ++cc) {
              const int a1 = split_at(U, vg, cc + 1);
              n_contrib += a1 > a0 ? 1 : 0;
              a0 = a1;
            }
            const int slot = sb == u0 ? 0 : 1;
            float4* mine = reinterpret_cast<float4*>(S.ws + ((long long)(v * 2 + slot) * 128 + r) * 16);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              __stcg(mine + j, make_float4(v16[4 * j], v16[4 * j + 1], v16[4 * j + 2], v16[4 * j + 3]));
            named_bar_sync(1, 128);
            if (t == 0) {
              const unsigned long long old = atom_add_acqrel_u64(S.tickets + tile, 1ull);
              const bool last = old == (unsigned long long)(n_contrib - 1);
              if (last) S.tickets[tile] = 0ull;
              flags[F_TICKET] = last ? 1 : 0;
            }
            named_bar_sync(1, 128);
            finisher = flags[F_TICKET] != 0;
            if (finisher) {
              // the contributors' partials in contributor order (slot 0 when the tile holds
              // their first unit), read four contributors at a time
#pragma unroll
              for (int j = 0; j < 16; ++j) v16[j] = 0.0f;
              int cc = c_first;
              while (cc <= c_last) {
                float4 pv[4][4];
                int n = 0, who[4];
                for (; cc <= c_last && n < 4; ++cc) {
                  const int cu0 = split_at(U, vg, cc);
                  if (split_at(U, vg, cc + 1) <= cu0) continue;  // no units of this stage
                  const int cs = cu0 >= tile * kb ? 0 : 1;
                  who[n++] = cc * 2 + cs;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  if (i < n) {
                    const float4* pp = reinterpret_cast<const float4*>(S.ws + ((long long)who[i] * 128 + r) * 16);
#pragma unroll
                    for (int j = 0; j < 4; ++j) pv[i][j] = __ldcg(pp + j);
                  }
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  if (i < n) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                      v16[4 * j] = __fadd_rn(v16[4 * j], pv[i][j].x);
                      v16[4 * j + 1] = __fadd_rn(v16[4 * j + 1], pv[i][j].y);
                      v16[4 * j + 2] = __fadd_rn(v16[4 * j + 2], pv[i][j].z);
                      v16[4 * j + 3] = __fadd_rn(v16[4 * j + 3], pv[i][j].w);
                    }
                  }
              }
            }
          }
          if (!finisher) continue;
          finish_tile<HD>(P, S, v16, r, tile, escr, pf);
          named_bar_sync(1, 128);
          if (S.ekind == E_QKV) {
            // the last of the group's q, k, v tiles runs the group's self-attention
            const int g = tile % (P.hidden / 128);
            if (t == 0) {
              const unsigned long long old = atom_add_acqrel_u64(S.groups + g, 1ull);
              const bool last = old == 2ull;
              if (last) S.groups[g] = 0ull;
              flags[F_TICKET] = last ? 1 : 0;
            }
            named_bar_sync(1, 128);
            if (!flags[F_TICKET]) continue;
            group_attention<HD>(P, S, g, escr);
            named_bar_sync(1, 128);
          }
          if (t == 0) red_release_add_u64(P.done + s, 1ull);
        }
        ia += (uint32_t)(u1 - u0);
      } else if (S.kind == K_XATTN) {
        constexpr int TB = XA_TILE * HD * 2;
        constexpr int SPT = xa_slots<HD>();
        bool waited = false;
        XaItem x;
        for (int it = c; it < P.heads * S.nsplit && ok; it += G) {
          if (!xa_item(P, S, it, x)) continue;
          if (!waited) {
            if (t == 0) flags[F_DEP] = wait_deps(P, S, cta_abort) ? 1 : 0;
            named_bar_sync(1, 128);
            if (!flags[F_DEP]) {
              ok = false;
              break;
            }
            waited = true;
          }
          uint32_t qa[HD / 16][4];
          const bf16* qb = S.q + x.h * HD;
          xa_load_q<HD>(qa, [&](int row, int col) {
            return __ldcg(reinterpret_cast<const unsigned int*>(qb + (long long)row * P.hidden + col));
          });
          XaAcc<HD> acc;
          xa_init<HD>(acc);
          const int w = t >> 5;
          for (int tl = 0; tl < x.ntiles; ++tl) {
            const int s0 = ia % NA;
            const int s1 = (ia + 1) % NA;
            // one thread waits (bounded) for the tile and publishes the outcome (alternating
            // flags: a flag is rewritten only after a barrier every reader has passed)
            int* wflag = flags + F_XW + (tl & 1);
            if (t == 0) {
              bool good = ring_wait(P, &full[s0], (ia / NA) & 1u, cta_abort);
              if (good && SPT == 2) good = ring_wait(P, &full[s1], ((ia + 1) / NA) & 1u, cta_abort);
              *wflag = good ? 1 : 0;
            }
            named_bar_sync(1, 128);
            if (!*wflag) {
              ok = false;
              break;
            }
            const uint32_t kbase = smem_u32(sA + s0 * A_BYTES);
            const uint32_t vbase = SPT == 2 ? smem_u32(sA + s1 * A_BYTES) : kbase + TB;
            xa_tile<HD>(acc, qa, kbase, vbase, 16 * w, x.k_begin + tl * XA_TILE + 16 * w, x.k_end, P.scale);
            __syncwarp();
            named_bar_sync(1, 128);
            if (t == 0) {
              mbar_arrive(&empty[s0]);
              if (SPT == 2) mbar_arrive(&empty[s1]);
            }
            ia += SPT;
          }
          if (!ok) break;
          float* mine = S.part + (long long)(x.h * S.nsplit + x.split) * (16 * HD + 32);
          const float* base = S.part + (long long)x.h * S.nsplit * (16 * HD + 32);
          bf16* outp = S.out + x.h * HD;
          const int n_active = x.n_active;
          unsigned long long* xt = S.xtickets + x.h;
          const bool merged = xa_finish<HD>(
              acc, reinterpret_cast<float*>(escr), t, n_active, mine, base, flags + F_XA,
              [] { named_bar_sync(1, 128); },
              [&] {
                const unsigned long long old = atom_add_acqrel_u64(xt, 1ull);
                const bool last = old == (unsigned long long)(n_active - 1);
                if (last) *xt = 0ull;
                return last;
              },
              [&](int i, int d, float lo, float hi) {
                *reinterpret_cast<__nv_bfloat162*>(outp + (long long)i * P.hidden + d) = __floats2bfloat162_rn(lo, hi);
              });
          if (merged) {
            named_bar_sync(1, 128);
            if (t == 0) red_release_add_u64(P.done + s, 1ull);
          }
          named_bar_sync(1, 128);  // the merge buffers are reused by the next item
        }
        // slots of items this CTA skipped after an abort are not counted: the loop ends anyway
      } else if (S.kind == K_FINAL) {
        if (c == 0 && P.tokens) {
          if (t == 0) flags[F_DEP] = wait_deps(P, S, cta_abort) ? 1 : 0;
          named_bar_sync(1, 128);
          if (!flags[F_DEP]) {
            ok = false;
            break;
          }
          if (t < P.block) P.tokens[t] = (int64_t)argmax_key_index(__ldcg(P.keys + t));
        }
      }
    }
  } else {
    // ---------------------------------------------------------- operand builders (warps 6, 7)
    const int tb = (int)threadIdx.x - 192;
    uint32_t ib = 0;  // operand blocks issued into the ring
    bool ok = true;
    const uint32_t noise_off = P.offset + bump;
    float* sstat = reinterpret_cast<float*>(smem + OFF_SSTAT);
    uint8_t* sConst = smem + OFF_CONST;
    // the operand slot `slot` free again: one thread waits (bounded) and the group
    // reads the outcome (alternating flags, as for the attention tiles)
    uint32_t nwait = 0;
    auto slot_free = [&](int slot, uint32_t parity) -> bool {
      int* f = flags + F_BW + (nwait++ & 1);
      if (tb == 0) *f = ring_wait(P, &bempty[slot], parity, cta_abort) ? 1 : 0;
      named_bar_sync(2, 64);
      return *f != 0;
    };
    auto finish_piece = [&](int s) {
      named_bar_sync(2, 64);
      if (tb == 0) red_release_add_u64(P.done + s, 1ull);
    };
    for (int s = 0; s < n_stages && ok; ++s) {
      load_stage(P, s, sdesc + 2 + (s & 1), tb, 64);
      named_bar_sync(2, 64);
      const Stage& S = sdesc[2 + (s & 1)];
      if (S.kind == K_PREP) {
        // keys reset, index checks, the anchor's embedding row
        if (c == 0) {
          if (tb < P.block) P.keys[tb] = 0ull;
          long long id = P.anchor_ids[0];
          if (tb == 0) {
            const int len = P.lengths[0];
            if (id < 0 || id >= P.vocab) record_error(P.err, DEV_BAD_INDEX);
            if (len < 0 || len + P.block + 1 > P.rope_len || len >= P.cache_len) record_error(P.err, DEV_BAD_INDEX);
          }
          if (id < 0 || id >= P.vocab) id = 0;
          const uint4* src = reinterpret_cast<const uint4*>(S.aux + id * S.count);
          uint4* dst = reinterpret_cast<uint4*>(S.dst);
          for (long long k = tb; k < S.count / 8; k += 64) dst[k] = src[k];
          finish_piece(s);
        }
        continue;
      }
      if (S.kind == K_NOISE) {
        // this CTA's share of the one-step noise: Philox pairs, or the caller's z
        const long long pairs = S.count / 2;
        const long long p0 = (long long)c * pairs / G, p1 = (long long)(c + 1) * pairs / G;
        __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(S.dst);
        const __nv_bfloat162* zin = reinterpret_cast<const __nv_bfloat162*>(P.z);
        for (long long pp = p0 + tb; pp < p1; pp += 64) {
          if (zin) {
            dst[pp] = zin[pp];
          } else {
            float z0, z1;
            normal_pair(P.seed, noise_off, pp, z0, z1);
            dst[pp] = __floats2bfloat162_rn(z0, z1);
          }
        }
        finish_piece(s);
        continue;
      }
      if (S.kind == K_ANORM) {
        // anchor_norm of the projected anchor row (the rmsnorm kernel's arithmetic)
        if (c == 0) {
          if (tb == 0) flags[F_BDEP] = wait_deps(P, S, cta_abort) ? 1 : 0;
          named_bar_sync(2, 64);
          if (!flags[F_BDEP]) {
            ok = false;
            break;
          }
          if (tb < 32) {
            const float inv = inv_rms(warp_row_sumsq_batched(S.src, (int)S.count, lane), (int)S.count, S.eps);
            for (int ch = lane; ch < S.count / 8; ch += 32) {
              float x[8], w8[8], y[8];
              unpack_bf16x8(__ldcg(reinterpret_cast<const uint4*>(S.src) + ch), x);
              unpack_bf16x8(*(reinterpret_cast<const uint4*>(S.w0) + ch), w8);
#pragma unroll
              for (int e = 0; e < 8; ++e) y[e] = rms_value(x[e], w8[e], inv);
              *(reinterpret_cast<uint4*>(S.dst) + ch) = pack_bf16x8(y);
            }
          }
          finish_piece(s);
        }
        continue;
      }
      if (S.kind != K_GEMM) continue;
      int u0, u1;
      stage_range(S, c, G, u0, u1);
      if (u1 <= u0) continue;
      // the operand's tensor map fetched before the wait (its first use would otherwise
      // fetch the descriptor on the critical path)
      if (S.bkind == B_COPY && tb == 0) tma_prefetch_desc(&P.maps[S.bmap]);
      if (S.bkind != B_COPY) {
        // the constant rows of every unit ([scale, shift] of an AdaLN, [uniform posterior,
        // state_norm, noise_norm] of mix_state) staged before the wait: they do not depend
        // on the stage's inputs, and their HBM latency hides under the wait
        for (int k = tb; k < (u1 - u0) * 24; k += 64) {
          const int j = k / 24, row = (k % 24) >> 3, ch = k & 7;
          const int kk = (u0 + j) % S.ep.kb;
          const int k0 = kk * 64 + ch * 8;
          const bf16* src = S.bkind == B_ADALN ? (row == 0 ? S.mod : row == 1 ? S.mod + S.ep.K : nullptr)
                                               : (row == 0 ? S.aux : row == 1 ? S.w0 : S.w1);
          const bool valid = src != nullptr && k0 < S.ep.K;
          cp16(sConst + j * CONST_SLOT + row * 128 + ch * 16, valid ? (const void*)(src + k0) : (const void*)S.src,
               valid);
        }
        cp_commit();
        if (S.bkind == B_MIX && tb >= 32) {
          // the uniform posterior row's RMS (a constant row)
          const float ssu = warp_row_sumsq_batched(S.aux, S.ep.K, lane);
          if (lane == 0) bstat[32] = inv_rms(ssu, S.ep.K, S.eps);
        }
      }
      if (tb == 0) flags[F_BDEP] = wait_deps(P, S, cta_abort) ? 1 : 0;
      named_bar_sync(2, 64);
      if (!flags[F_BDEP]) {
        ok = false;
        break;
      }
      const int K = S.ep.K, kb = S.ep.kb;
      if (S.bkind == B_COPY) {
        // the source rows by TMA ([16 x 64] boxes, 128-byte swizzled: the UMMA
        // layout), one thread issuing up to the ring's depth ahead of the MMA
        if (tb == 0) {
          fence_proxy_async_global();  // rows written by other CTAs' epilogues, read by TMA
          const CUtensorMap* map = &P.maps[S.bmap];
          bool good = true;
          for (int u = u0; u < u1; ++u) {
            const int slot = ib % NB;
            if (ib >= NB && !ring_wait(P, &bempty[slot], ((ib / NB) - 1) & 1u, cta_abort)) {
              good = false;
              break;
            }
            mbar_arrive_expect_tx(&bfull[slot], B_BYTES);
            tma_load_2d(sB + slot * B_BYTES, map, &bfull[slot], (int)(u % kb) * 64, 0);
            ++ib;
          }
          flags[F_BCOPY] = good ? 1 : 0;
        }
        named_bar_sync(2, 64);
        if (tb != 0) ib += (uint32_t)(u1 - u0);  // thread 0 counted its copies as it issued them
        if (!flags[F_BCOPY]) {
          ok = false;
          break;
        }
        continue;
      }
      // transforms: the producing stage's per-tile statistics and the first batch's
      // source rows staged in one round trip (the constant rows were staged on entry,
      // before the dependency wait); the statistics combined per token in tile order
      auto stage_batch = [&](int ub, int nb) {
        for (int j = 0; j < nb; ++j) {
          const int kk = (ub + j) % kb;
          uint8_t* st = sStage + j * STAGE_SLOT;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int idx = tb + 64 * i, n = idx >> 3, ch = idx & 7;
            const int k0 = kk * 64 + ch * 8;
            const bool valid = k0 < K;
            cp16(st + n * 128 + ch * 16, valid ? (const void*)(S.src + (long long)n * S.ld + k0) : (const void*)S.src,
                 valid);
          }
        }
      };
      for (int k = tb; k < S.stats_tiles * 8; k += 64) cp16(sstat + k * 4, S.stats_in + k * 4, true);
      stage_batch(u0, min(BATCH, u1 - u0));
      cp_commit();
      cp_wait<0>();
      named_bar_sync(2, 64);
      if (tb < 16) {
        if (S.bkind == B_ADALN) {
          // Chan's combination of the tiles' (sum, sum of squared deviations), 128 rows each
          float tot = 0.0f;
          for (int i = 0; i < S.stats_tiles; ++i) tot = __fadd_rn(tot, sstat[(i * 16 + tb) * 2]);
          const float mean = __fdiv_rn(tot, (float)K);
          float m2 = 0.0f;
          for (int i = 0; i < S.stats_tiles; ++i) {
            const float dm = __fsub_rn(__fmul_rn(sstat[(i * 16 + tb) * 2], 0.0078125f), mean);  // tile mean - mean
            m2 = __fadd_rn(m2, __fadd_rn(sstat[(i * 16 + tb) * 2 + 1], __fmul_rn(128.0f, __fmul_rn(dm, dm))));
          }
          bstat[tb * 2] = mean;
          bstat[tb * 2 + 1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(m2, (float)K), S.eps)));
        } else {
          float ss = 0.0f;
          for (int i = 0; i < S.stats_tiles; ++i) ss = __fadd_rn(ss, sstat[(i * 16 + tb) * 2]);
          bstat[tb * 2] = inv_rms(ss, K, S.eps);
        }
      }
      named_bar_sync(2, 64);
      // per batch: the operand blocks computed from the staged rows, one proxy fence,
      // then the blocks handed to the MMA
      for (int ub = u0; ub < u1 && ok; ub += BATCH) {
        const int nb = min(BATCH, u1 - ub);
        if (ub != u0) {
          stage_batch(ub, nb);
          cp_commit();
          cp_wait<0>();
          named_bar_sync(2, 64);
        }
        // the batch's slots are free once the MMA has consumed the block NB before
        // its last one (the MMA consumes in order)
        const uint32_t last = ib + (uint32_t)nb - 1;
        if (last >= NB && !slot_free(last % NB, ((last / NB) - 1) & 1u)) {
          ok = false;
          break;
        }
        for (int j = 0; j < nb; ++j) {
          const int slot = (ib + j) % NB;
          const int kk = (int)((ub + j) % kb);
          const uint8_t* st = sStage + j * STAGE_SLOT;
          const uint8_t* cst = sConst + (int)(ub + j - u0) * CONST_SLOT;
          uint8_t* dst = sB + slot * B_BYTES;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int idx = tb + 64 * i, n = idx >> 3, ch = idx & 7;
            const int k0 = kk * 64 + ch * 8;
            uint4 o = make_uint4(0u, 0u, 0u, 0u);
            if (k0 < K) {
              float x[8], y[8];
              unpack_bf16x8(*reinterpret_cast<const uint4*>(st + n * 128 + ch * 16), x);
              if (S.bkind == B_ADALN) {
                float sc[8], sh[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(cst + ch * 16), sc);
                unpack_bf16x8(*reinterpret_cast<const uint4*>(cst + 128 + ch * 16), sh);
                const float mean = bstat[n * 2], rstd = bstat[n * 2 + 1];
#pragma unroll
                for (int e = 0; e < 8; ++e) y[e] = adaln_value(x[e], mean, rstd, sc[e], sh[e]);
              } else {
                float pu[8], sw[8], nw[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(cst + ch * 16), pu);
                unpack_bf16x8(*reinterpret_cast<const uint4*>(cst + 128 + ch * 16), sw);
                unpack_bf16x8(*reinterpret_cast<const uint4*>(cst + 256 + ch * 16), nw);
                const float ip = bstat[32], is = bstat[n * 2];
#pragma unroll
                for (int e = 0; e < 8; ++e) y[e] = mix_value(pu[e], x[e], sw[e], nw[e], ip, is, S.gate);
              }
              o = pack_bf16x8(y);
            }
            *reinterpret_cast<uint4*>(dst + b_off(n, ch)) = o;
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(2, 64);
        if (tb == 0)
          for (int j = 0; j < nb; ++j) mbar_arrive(&bfull[(ib + j) % NB]);
        ib += (uint32_t)nb;
        named_bar_sync(2, 64);  // the staging slots are refilled by the next round
      }
    }
    // operand copies issued by TMA land before the CTA's shared memory goes away
    if (tb == 0 && !ok)
      for (uint32_t i = ib > NB ? ib - NB : 0; i < ib; ++i) mbar_wait(&bfull[i % NB], (i / NB) & 1u, nullptr);
    cp_wait<0>();  // no copy into shared memory outlives the CTA
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned long long out = atomicAdd(P.words, 1ull);
    if (out == (unsigned long long)G - 1) {
      // every CTA is past its last wait: the counters return to zero for the next launch
      for (int s = 0; s < n_stages; ++s) P.done[s] = 0ull;
      if (P.words[1] != 0ull) {
        for (long long i = 0; i < P.n_tickets; ++i) P.all_tickets[i] = 0ull;
        P.words[1] = 0ull;
      }
      if (P.offset_ptr) *P.offset_ptr = bump;
      P.words[0] = 0ull;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------ host
size_t smem_bytes() { return (size_t)SMEM_TOTAL; }

int grid_size() {
  static thread_local int dev_cached = -1, grid = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev == dev_cached) return grid;
  dev_cached = dev;
  grid = 0;
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (!coop) return 0;
  for (auto k : {stream_kernel<64>, stream_kernel<128>})
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TOTAL) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stream_kernel<128>, THREADS, SMEM_TOTAL) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    return 0;
  }
  grid = num_sms();
  return grid;
}

fm_status launch(const Params* P, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_TOTAL;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (P->head_dim == 128)
    e = cudaLaunchKernelEx(&cfg, stream_kernel<128>, *P);
  else if (P->head_dim == 64)
    e = cudaLaunchKernelEx(&cfg, stream_kernel<64>, *P);
  else
    return set_error(FM_ERR_UNSUPPORTED, "streamed pass: head_dim %d", P->head_dim);
  if (e != cudaSuccess) return set_error(FM_ERR_LAUNCH, "streamed pass launch failed: %s", cudaGetErrorString(e));
  ++launch_counter();
  return FM_OK;
}

}  // namespace stream
}  // namespace fm
