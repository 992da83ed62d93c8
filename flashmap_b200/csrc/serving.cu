// Operators of the serving plugins (flashmap/vllm/kernels.py, flashmap/vllm/model.py:93,
// flashmap/sglang/kernels.py, flashmap/sglang/model.py:127-178 and :728-766), behind
// the C ABI:
//   * qk_norm_rope_kernel      RMSNorm + interleaved RoPE of (token, head) rows
//   * self_attn_qknorm_kernel  block self-attention from raw qkv (norms and RoPE
//                              applied while the rows are staged)
//   * paged_xattn_kernel       cross-attention over paged bf16 / e4m3 KV caches
//   * write_ctx_paged_kernel   context keys/values into vLLM-layout paged caches
//   * write_ctx_pool_kernel    context keys/values into sglang-layout pools
//
// Numerics follow the DiT (modeling_flashmap.py:53-80, 144-147): norms and RoPE
// in fp32 with the bf16 roundings of the reference, attention scores in fp32,
// softmax numerators exp(s - m) in fp32 rounded to bf16 for P V, the sum in fp32.
#include <cuda_fp8.h>

#include "attention.cuh"
#include "launch.cuh"

namespace fm {
namespace {

struct RopeRef {
  const float* cos;
  const float* sin;
  long long rs, ps, rows;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

RopeRef rope_ref(const fm_rope_view& v) { return RopeRef{v.cos, v.sin, v.row_stride, v.pair_stride, v.rows}; }

__device__ __forceinline__ float load_w(const void* w, int dt, long long i) {
  return dt == FM_DT_F32 ? static_cast<const float*>(w)[i] : bf2f(static_cast<const __nv_bfloat16*>(w)[i]);
}

__device__ __forceinline__ long long load_pos(const void* p, int dt, long long t) {
  if (p == nullptr) return t;
  return dt == FM_DT_I64 ? static_cast<const long long*>(p)[t] : (long long)static_cast<const int*>(p)[t];
}

__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float e4m3_to_f(uint8_t b) {
  const __half h = __half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3));
  return __half2float(h);
}

// One warp normalises and rotates a row of hd (<= 64 * NP) bf16 values: pair i
// = lane + 32 j (j < NP) holds elements 2i, 2i + 1.  Results are the rotated
// fp32 values (the caller rounds them to bf16 or scales them to e4m3).
//   FM_NORM_DIT:   x * bf16(w * inv), rounded to bf16   (modeling_flashmap.py:76-80)
//   FM_NORM_FUSED: bf16((x * inv) * w)                  (sglang/kernels.py:309-311)
// with inv = 1 / sqrt(mean(x^2) + eps); RoPE (modeling_flashmap.py:61-66):
//   (e, o) -> (e cos - o sin, o cos + e sin) in fp32.
template <int NP>
__device__ __forceinline__ void warp_norm_rope(const __nv_bfloat16* row, int hd, const void* w, int wdt, float eps,
                                               int mode, const RopeRef& rp, long long pos, int* err, float* re,
                                               float* ro) {
  const int lane = threadIdx.x & 31, half = hd >> 1;
  float e[NP], o[NP];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int i = lane + 32 * j;
    e[j] = o[j] = 0.0f;
    if (i < half) {
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(row + 2 * i);
      e[j] = __low2float(v);
      o[j] = __high2float(v);
      ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(e[j], e[j]), __fmul_rn(o[j], o[j])));
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), eps)));
  if (pos < 0 || pos >= rp.rows) {
    if (lane == 0) record_error(err, DEV_BAD_INDEX);
    pos = 0;
  }
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int i = lane + 32 * j;
    if (i >= half) continue;
    const float we = load_w(w, wdt, 2 * i), wo = load_w(w, wdt, 2 * i + 1);
    float xe, xo;
    if (mode == FM_NORM_DIT) {
      xe = round_bf(__fmul_rn(e[j], round_bf(__fmul_rn(we, inv))));
      xo = round_bf(__fmul_rn(o[j], round_bf(__fmul_rn(wo, inv))));
    } else {
      xe = round_bf(__fmul_rn(__fmul_rn(e[j], inv), we));
      xo = round_bf(__fmul_rn(__fmul_rn(o[j], inv), wo));
    }
    const float c = rp.cos[pos * rp.rs + (long long)i * rp.ps];
    const float s = rp.sin[pos * rp.rs + (long long)i * rp.ps];
    re[j] = __fsub_rn(__fmul_rn(xe, c), __fmul_rn(xo, s));
    ro[j] = __fadd_rn(__fmul_rn(xo, c), __fmul_rn(xe, s));
  }
}

// ------------------------------------------------------------------ q/k norm + RoPE rows
constexpr int NR_WARPS = 8;

struct NormRopeArgs {
  const __nv_bfloat16* x;
  __nv_bfloat16* out;
  long long x_ts, o_ts, tokens;
  int heads, hd;
  const void* w;
  int wdt;
  RopeRef rope;
  const void* pos;
  int pdt;
  float eps;
  int mode;
  int* err;
};

template <int NP>
__global__ void __launch_bounds__(NR_WARPS * 32) qk_norm_rope_kernel(NormRopeArgs a) {
  const long long rowi = (long long)blockIdx.x * NR_WARPS + (threadIdx.x >> 5);
  if (rowi >= a.tokens * a.heads) return;
  const long long t = rowi / a.heads;
  const int h = (int)(rowi % a.heads);
  float re[NP], ro[NP];
  warp_norm_rope<NP>(a.x + t * a.x_ts + (long long)h * a.hd, a.hd, a.w, a.wdt, a.eps, a.mode, a.rope,
                     load_pos(a.pos, a.pdt, t), a.err, re, ro);
  __nv_bfloat16* dst = a.out + t * a.o_ts + (long long)h * a.hd;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int i = lane + 32 * j;
    if (i < (a.hd >> 1)) *reinterpret_cast<__nv_bfloat162*>(dst + 2 * i) = __floats2bfloat162_rn(re[j], ro[j]);
  }
}

// ------------------------------------------------------------------ block self-attention from raw qkv
constexpr int SQ_WARPS = 4;

struct SelfQkArgs {
  const __nv_bfloat16* qkv;  // (blocks, 16, 3, heads, HD)
  __nv_bfloat16* out;        // (blocks * 16, heads * HD)
  int blocks, heads;
  const void* qn;
  const void* kn;
  int wdt;
  RopeRef rope;
  const void* pos;
  int pdt;
  float eps, scale;
  int* err;
};

template <int HD>
__global__ void __launch_bounds__(SQ_WARPS * 32) self_attn_qknorm_kernel(SelfQkArgs a) {
  extern __shared__ __align__(1024) uint8_t sq_smem[];
  constexpr int PART = 16 * HD * 2;
  constexpr int NP = HD / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // one CTA per (block, head): its warps share the 32 q/k rows, warp 0 attends
  const int it = blockIdx.x;
  const int b = it / a.heads, h = it % a.heads;
  const long long D = (long long)a.heads * HD;
  uint8_t* st = sq_smem;
  for (int r = warp; r < 16; r += SQ_WARPS) {
    const long long tok = (long long)b * 16 + r;
    const long long pos = load_pos(a.pos, a.pdt, tok);
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      float re[NP], ro[NP];
      warp_norm_rope<NP>(a.qkv + tok * 3 * D + part * D + (long long)h * HD, HD, part ? a.kn : a.qn, a.wdt, a.eps,
                         FM_NORM_DIT, a.rope, pos, a.err, re, ro);
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int i = lane + 32 * j;  // pair i: elements 2i, 2i + 1 of chunk (2i) / 8
        *reinterpret_cast<__nv_bfloat162*>(st + part * PART + blk_sw(r, i >> 2) + (i & 3) * 4) =
            __floats2bfloat162_rn(re[j], ro[j]);
      }
    }
  }
  for (int idx = threadIdx.x; idx < 16 * (HD / 8); idx += SQ_WARPS * 32) {
    const int row = idx / (HD / 8), ch = idx % (HD / 8);
    const uint4 v = *reinterpret_cast<const uint4*>(a.qkv + ((long long)b * 16 + row) * 3 * D + 2 * D +
                                                    (long long)h * HD + ch * 8);
    *reinterpret_cast<uint4*>(st + 2 * PART + blk_sw(row, ch)) = v;
  }
  __syncthreads();
  if (warp != 0) return;
  const uint32_t base = smem_u32(st);
  __nv_bfloat16* out = a.out + (long long)b * 16 * D + (long long)h * HD;
  block_attn_head<HD>(base, base + PART, base + 2 * PART, a.scale, [&](int i, int d, float lo, float hi) {
    *reinterpret_cast<__nv_bfloat162*>(out + (long long)i * D + d) = __floats2bfloat162_rn(lo, hi);
  });
}

// ------------------------------------------------------------------ paged cross-attention
// One CTA of 4 warps per (request, group of 16 query rows, head, key split).
// Each warp owns keys 16w .. 16w + 15 of every 64-key tile of its split and
// streams them through a private 3-stage cp.async pipeline (the page table
// makes every key row its own copy source; no CTA barrier inside the loop).
// e4m3 rows land raw and are widened to bf16 (exactly) in a warp-private tile.
// The 4 warps' partial softmax states, then the splits', are merged like
// cross_attn_kernel's.
constexpr int PX_STAGES = 3;
constexpr int PX_TILE = 64;

struct PagedArgs {
  const uint8_t* q;
  int q8;
  long long q_ts, q_hs;
  const int* cu;
  long long qpr;
  int groups;
  const uint8_t* k;
  const uint8_t* v;
  long long kps, khs, kts;
  int page;
  long long num_pages;
  const int* table;
  long long tstride, tcols;
  const int* seqused;
  int R, H, nsplit;
  float scale;
  const float* descales;
  int quant_q;
  __nv_bfloat16* out;
  long long o_ts, o_hs;
  int* counters;
  float* part;
  int* err;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <int HD, bool KV8>
struct PxLayout {
  static constexpr int TILE_BF = 16 * HD * 2;                  // one of K, V of a warp's 16 keys, bf16
  static constexpr int STAGE = KV8 ? 2 * 16 * HD : 2 * TILE_BF;  // raw bytes per stage
  static constexpr int CONV = KV8 ? 2 * TILE_BF : 0;           // widened K | V of the current tile
  static constexpr int WARP = PX_STAGES * STAGE + CONV;
  static constexpr int CPR = KV8 ? HD / 16 : HD / 8;           // 16-byte copies per key row
  static constexpr int PER_LANE = 2 * 16 * CPR / 32;           // copies per lane per tile
  static constexpr int MERGE = (4 * 16 * HD + 256) * 4;
  static constexpr int SMEM = (4 * WARP > MERGE ? 4 * WARP : MERGE) + 64;
};

template <int HD, bool KV8>
__global__ void __launch_bounds__(128) paged_xattn_kernel(PagedArgs a) {
  using Lay = PxLayout<HD, KV8>;
  constexpr int NT = HD / 8;
  constexpr int ESZ = KV8 ? 1 : 2;
  extern __shared__ __align__(1024) uint8_t px_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  int rest = blockIdx.x;
  const int split = rest % a.nsplit;
  rest /= a.nsplit;
  const int h = rest % a.H;
  rest /= a.H;
  const int g = rest % a.groups;
  const int r = rest / a.groups;
  const long long item = ((long long)r * a.groups + g) * a.H + h;
  int* sflag = reinterpret_cast<int*>(px_smem + Lay::SMEM - 64);
  float* sred = reinterpret_cast<float*>(px_smem + Lay::SMEM - 48);

  const long long q0 = a.cu ? (long long)a.cu[r] : (long long)r * a.qpr;
  const long long nq = a.cu ? (long long)a.cu[r + 1] - q0 : a.qpr;
  const int rows = (int)min(16LL, nq - (long long)g * 16);
  if (g == a.groups - 1 && nq > (long long)a.groups * 16 && threadIdx.x == 0 && split == 0 && h == 0)
    record_error(a.err, DEV_BAD_INDEX);  // more query rows than max_q promised
  if (rows <= 0) return;
  long long cap = a.tcols * a.page;
  int ctx = a.seqused[r];
  if (ctx < 0 || ctx > cap) {
    if (threadIdx.x == 0 && split == 0) record_error(a.err, DEV_BAD_INDEX);
    ctx = ctx < 0 ? 0 : (int)cap;
  }
  const long long qrow0 = q0 + (long long)g * 16;
  if (ctx == 0) {  // nothing to attend to: zero rows (split 0 writes them)
    if (split == 0)
      for (int idx = threadIdx.x; idx < rows * HD; idx += 128) {
        const int i = idx / HD, d = idx % HD;
        a.out[(qrow0 + i) * a.o_ts + (long long)h * a.o_hs + d] = f2bf(0.0f);
      }
    return;
  }
  const int per = ((((ctx + a.nsplit - 1) / a.nsplit) + PX_TILE - 1) / PX_TILE) * PX_TILE;
  const int k_begin = split * per;
  const int k_end = min(ctx, k_begin + per);
  if (k_begin >= ctx) return;
  const int ntiles = (k_end - k_begin + PX_TILE - 1) / PX_TILE;

  // descales of (request, head): query, key, value
  float qd = 1.0f, kd = 1.0f, vd = 1.0f;
  if (a.descales) {
    const long long rh = (long long)r * a.H + h, n = (long long)a.R * a.H;
    qd = a.descales[rh];
    kd = a.descales[n + rh];
    vd = a.descales[2 * n + rh];
  }
  if (a.quant_q) {
    // e4m3 scale of this request's bf16 query rows of head h: amax / 448
    float mx = 0.0f;
    for (long long i = warp; i < nq; i += 4) {
      const __nv_bfloat16* qr = reinterpret_cast<const __nv_bfloat16*>(a.q) + (q0 + i) * a.q_ts + (long long)h * a.q_hs;
      for (int d = lane; d < HD; d += 32) mx = fmaxf(mx, fabsf(bf2f(qr[d])));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) sred[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(sred[0], sred[1]), fmaxf(sred[2], sred[3]));
    qd = __fdiv_rn(fmaxf(mx, 1e-12f), 448.0f);
  }
  const float sscale = __fmul_rn(__fmul_rn(qd, kd), a.scale);

  // query fragments (rows gid, gid + 8 of the group; rows past `rows` are zero)
  uint32_t qa[HD / 16][4];
  {
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks)
#pragma unroll
      for (int f = 0; f < 4; ++f) {
        const int i = gid + (f & 1) * 8;
        const int c = ks * 16 + tig * 2 + (f >> 1) * 8;
        uint32_t val = 0;
        if (i < rows) {
          const long long off = (qrow0 + i) * a.q_ts + (long long)h * a.q_hs + c;
          if (a.q8) {
            const uint8_t* qb = a.q + off;
            val = pack_bf16x2(e4m3_to_f(qb[0]), e4m3_to_f(qb[1]));
          } else {
            const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(a.q) + off;
            if (a.quant_q) {
              // quantise to e4m3 (round to nearest, saturating) and widen back: exact in bf16
              const uint16_t pq = e4m3x2(__fdiv_rn(bf2f(qb[0]), qd), __fdiv_rn(bf2f(qb[1]), qd));
              val = pack_bf16x2(e4m3_to_f((uint8_t)(pq & 0xff)), e4m3_to_f((uint8_t)(pq >> 8)));
            } else {
              val = *reinterpret_cast<const uint32_t*>(qb);
            }
          }
        }
        qa[ks][f] = val;
      }
  }

  uint8_t* wbase = px_smem + warp * Lay::WARP;
  const uint32_t wbase_s = smem_u32(wbase);
  // copies of tile t of this warp's keys into stage t % PX_STAGES (one commit group per tile)
  auto issue = [&](int t) {
    if (t < ntiles) {
      const int key0 = k_begin + t * PX_TILE + 16 * warp;
      long long off = 0;
      int ok = 0;
      if (lane < 16) {
        const int p = key0 + lane;
        if (p < k_end) {
          const long long pi = p / a.page;
          const int page = a.table[(long long)r * a.tstride + pi];
          if (page >= 0 && page < a.num_pages) {
            off = (long long)page * a.kps + (long long)h * a.khs + (long long)(p % a.page) * a.kts;
            ok = 1;
          } else {
            record_error(a.err, DEV_BAD_INDEX);
          }
        }
      }
      const uint32_t sbase = wbase_s + (t % PX_STAGES) * Lay::STAGE;
#pragma unroll
      for (int u = 0; u < Lay::PER_LANE; ++u) {
        const int c = u * 32 + lane;
        const int row = c / Lay::CPR, ch = c % Lay::CPR;
        const int part = row >> 4, j = row & 15;
        const long long so = __shfl_sync(0xffffffffu, off, j);
        const int sok = __shfl_sync(0xffffffffu, ok, j);
        const uint8_t* src = (part ? a.v : a.k) + (so + (long long)ch * (16 / ESZ)) * ESZ;
        uint32_t dst;
        if constexpr (KV8)
          dst = sbase + part * (16 * HD) + j * HD + ch * 16;
        else
          dst = sbase + part * Lay::TILE_BF + blk_sw(j, ch);
        cp_async16(dst, sok ? (const void*)src : (const void*)a.k, sok ? 16u : 0u);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int t = 0; t < PX_STAGES - 1; ++t) issue(t);

  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

  for (int t = 0; t < ntiles; ++t) {
    issue(t + PX_STAGES - 1);  // into the stage consumed at t - 1 (the warp synced after it)
    cp_async_wait<PX_STAGES - 1>();
    __syncwarp();
    uint32_t kbase = wbase_s + (t % PX_STAGES) * Lay::STAGE;
    if constexpr (KV8) {
      // widen the raw e4m3 rows into the bf16 tile (8 values per step)
      const uint8_t* raw = wbase + (t % PX_STAGES) * Lay::STAGE;
      uint8_t* conv = wbase + PX_STAGES * Lay::STAGE;
      for (int c = lane; c < 2 * 16 * (HD / 8); c += 32) {
        const int row = c / (HD / 8), ch = c % (HD / 8);
        const int part = row >> 4, j = row & 15;
        const uint2 bytes = *reinterpret_cast<const uint2*>(raw + part * (16 * HD) + j * HD + ch * 8);
        uint32_t w4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t word = e < 2 ? bytes.x : bytes.y;
          const int sh = (e & 1) * 16;
          w4[e] = pack_bf16x2(e4m3_to_f((uint8_t)(word >> sh)), e4m3_to_f((uint8_t)(word >> (sh + 8))));
        }
        *reinterpret_cast<uint4*>(conv + part * Lay::TILE_BF + blk_sw(j, ch)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      __syncwarp();
      kbase = wbase_s + PX_STAGES * Lay::STAGE;
    }
    const uint32_t vbase = kbase + Lay::TILE_BF;
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
      const int kr = nt * 8 + (lane & 7);
#pragma unroll
      for (int ks = 0; ks < HD / 16; ks += 2) {
        uint32_t kb[4];
        sa_ldsm4(kbase + blk_sw(kr, 2 * ks + (lane >> 3)), kb, false);
        sa_mma(sc[nt], qa[ks], kb[0], kb[1]);
        sa_mma(sc[nt], qa[ks + 1], kb[2], kb[3]);
      }
    }
    const int kabs = k_begin + t * PX_TILE + 16 * warp;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool valid = kabs + nt * 8 + tig * 2 + e < k_end;
        sc[nt][e] = valid ? __fmul_rn(sc[nt][e], sscale) : -INFINITY;
        sc[nt][2 + e] = valid ? __fmul_rn(sc[nt][2 + e], sscale) : -INFINITY;
        mx0 = fmaxf(mx0, sc[nt][e]);
        mx1 = fmaxf(mx1, sc[nt][2 + e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float u0 = n0 == -INFINITY ? 0.0f : n0, u1 = n1 == -INFINITY ? 0.0f : n1;
    const float al0 = expf(__fsub_rn(m0, u0)), al1 = expf(__fsub_rn(m1, u1));
    m0 = n0;
    m1 = n1;
    float p[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      p[nt][0] = expf(__fsub_rn(sc[nt][0], u0));
      p[nt][1] = expf(__fsub_rn(sc[nt][1], u0));
      p[nt][2] = expf(__fsub_rn(sc[nt][2], u1));
      p[nt][3] = expf(__fsub_rn(sc[nt][3], u1));
    }
    l0 = __fadd_rn(__fmul_rn(l0, al0), __fadd_rn(__fadd_rn(p[0][0], p[0][1]), __fadd_rn(p[1][0], p[1][1])));
    l1 = __fadd_rn(__fmul_rn(l1, al1), __fadd_rn(__fadd_rn(p[0][2], p[0][3]), __fadd_rn(p[1][2], p[1][3])));
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      o[i][0] *= al0;
      o[i][1] *= al0;
      o[i][2] *= al1;
      o[i][3] *= al1;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(p[0][0], p[0][1]);
    pa[1] = pack_bf16x2(p[0][2], p[0][3]);
    pa[2] = pack_bf16x2(p[1][0], p[1][1]);
    pa[3] = pack_bf16x2(p[1][2], p[1][3]);
    const int vr = ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int dn = 0; dn < NT; dn += 2) {
      uint32_t vb[4];
      sa_ldsm4(vbase + blk_sw(vr, dn + (lane >> 4)), vb, true);
      sa_mma(o[dn], pa, vb[0], vb[1]);
      sa_mma(o[dn + 1], pa, vb[2], vb[3]);
    }
    __syncwarp();  // the stage (and the widened tile) may be refilled from here on
  }
  cp_async_wait<0>();
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 1));
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 2));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 1));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 2));
  __syncthreads();  // every warp's pipeline is drained: its shared memory is free

  float* mO = reinterpret_cast<float*>(px_smem);
  float* mM = mO + 4 * 16 * HD;
  float* mL = mM + 64;
  float* mF = mL + 64;
  float* mR = mF + 64;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int col = i * 8 + tig * 2;
    *reinterpret_cast<float2*>(&mO[(warp * 16 + gid) * HD + col]) = make_float2(o[i][0], o[i][1]);
    *reinterpret_cast<float2*>(&mO[(warp * 16 + gid + 8) * HD + col]) = make_float2(o[i][2], o[i][3]);
  }
  if (tig == 0) {
    mM[warp * 16 + gid] = m0;
    mM[warp * 16 + gid + 8] = m1;
    mL[warp * 16 + gid] = l0;
    mL[warp * 16 + gid + 8] = l1;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int i = threadIdx.x;
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
  __syncthreads();
  const int n_active = (ctx + per - 1) / per;
  constexpr int PSZ = 16 * HD + 32;
  float* mine = a.part + (item * a.nsplit + split) * PSZ;
  auto store4 = [&](int i, int d, float4 acc, float ll) {
    if (i >= rows) return;
    __nv_bfloat16* dst = a.out + (qrow0 + i) * a.o_ts + (long long)h * a.o_hs + d;
    dst[0] = f2bf(__fmul_rn(__fdiv_rn(acc.x, ll), vd));
    dst[1] = f2bf(__fmul_rn(__fdiv_rn(acc.y, ll), vd));
    dst[2] = f2bf(__fmul_rn(__fdiv_rn(acc.z, ll), vd));
    dst[3] = f2bf(__fmul_rn(__fdiv_rn(acc.w, ll), vd));
  };
  for (int v4 = threadIdx.x; v4 < 16 * HD / 4; v4 += 128) {
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
    if (n_active == 1)
      store4(i, d, acc, mR[16 + i]);
    else
      __stcg(reinterpret_cast<float4*>(mine + i * HD + d), acc);
  }
  if (n_active == 1) return;
  if (threadIdx.x < 16) {
    __stcg(mine + 16 * HD + threadIdx.x, mR[threadIdx.x]);
    __stcg(mine + 16 * HD + 16 + threadIdx.x, mR[16 + threadIdx.x]);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(a.counters + item, 1);
    sflag[0] = (old == n_active - 1);
  }
  __syncthreads();
  if (!sflag[0]) return;
  __threadfence();
  // the last split of this item merges all splits in split order
  const float* base = a.part + item * a.nsplit * PSZ;
  float* sF = mO;  // [n_active][16] weights, then [16] sums
  for (int t = threadIdx.x; t < 16; t += 128) {
    float mm = -INFINITY;
    for (int sp = 0; sp < n_active; ++sp) mm = fmaxf(mm, __ldcg(base + (long long)sp * PSZ + 16 * HD + t));
    float ll = 0.0f;
    for (int sp = 0; sp < n_active; ++sp) {
      const float* ps = base + (long long)sp * PSZ;
      const float ms = __ldcg(ps + 16 * HD + t);
      const float f = ms == -INFINITY ? 0.0f : expf(__fsub_rn(ms, mm));
      sF[sp * 16 + t] = f;
      ll = __fadd_rn(ll, __fmul_rn(__ldcg(ps + 16 * HD + 16 + t), f));
    }
    sF[n_active * 16 + t] = ll;
  }
  __syncthreads();
  for (int v4 = threadIdx.x; v4 < 16 * HD / 4; v4 += 128) {
    const int i = (v4 * 4) / HD, d = (v4 * 4) % HD;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < n_active; ++sp) {
      const float4 t4 = __ldcg(reinterpret_cast<const float4*>(base + (long long)sp * PSZ + i * HD + d));
      const float f = sF[sp * 16 + i];
      acc.x = __fadd_rn(acc.x, __fmul_rn(t4.x, f));
      acc.y = __fadd_rn(acc.y, __fmul_rn(t4.y, f));
      acc.z = __fadd_rn(acc.z, __fmul_rn(t4.z, f));
      acc.w = __fadd_rn(acc.w, __fmul_rn(t4.w, f));
    }
    store4(i, d, acc, sF[n_active * 16 + i]);
  }
  if (threadIdx.x == 0) a.counters[item] = 0;
}

// ------------------------------------------------------------------ paged-cache writers
struct WriteCtxArgs {
  const __nv_bfloat16* kv;  // (tokens, L, 2, H, D)
  int L, H, D;
  const long long* pos;
  const long long* slots;
  const void* kn;
  int kdt;
  RopeRef rope;
  const long long* cache_ptrs;
  int hpc;
  long long sb, sh, st, voff, bs;
  float eps;
  const float* scales;
  int* err;
};

template <int NP>
__global__ void __launch_bounds__(128) write_ctx_paged_kernel(WriteCtxArgs a) {
  const long long t = blockIdx.x;
  const int c = blockIdx.y;
  const long long slot = a.slots[t];
  if (slot < 0) return;
  const int lane = threadIdx.x & 31, half = a.D >> 1;
  const long long pos = a.pos[t];
  for (int s = threadIdx.x >> 5; s < a.hpc; s += 4) {
    const int gh = c * a.hpc + s;
    if (gh >= a.L * a.H) break;
    const int layer = gh / a.H, h = gh % a.H;
    const __nv_bfloat16* krow = a.kv + ((t * a.L + layer) * 2 * a.H + h) * (long long)a.D;
    const __nv_bfloat16* vrow = krow + (long long)a.H * a.D;
    float re[NP], ro[NP];
    const void* w = a.kdt == FM_DT_F32 ? (const void*)(static_cast<const float*>(a.kn) + (long long)layer * a.D)
                                       : (const void*)(static_cast<const __nv_bfloat16*>(a.kn) + (long long)layer * a.D);
    warp_norm_rope<NP>(krow, a.D, w, a.kdt, a.eps, FM_NORM_DIT, a.rope, pos, a.err, re, ro);
    const long long off = (slot / a.bs) * a.sb + (long long)s * a.sh + (slot % a.bs) * a.st;
    if (a.scales) {
      uint8_t* dst = reinterpret_cast<uint8_t*>(a.cache_ptrs[c]) + off;
      const float ks = a.scales[layer * 2], vs = a.scales[layer * 2 + 1];
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int i = lane + 32 * j;
        if (i < half) *reinterpret_cast<uint16_t*>(dst + 2 * i) = e4m3x2(__fdiv_rn(re[j], ks), __fdiv_rn(ro[j], ks));
      }
      for (int i = lane; i < half; i += 32) {
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(vrow + 2 * i);
        *reinterpret_cast<uint16_t*>(dst + a.voff + 2 * i) =
            e4m3x2(__fdiv_rn(__low2float(v), vs), __fdiv_rn(__high2float(v), vs));
      }
    } else {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.cache_ptrs[c]) + off;
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int i = lane + 32 * j;
        if (i < half) *reinterpret_cast<__nv_bfloat162*>(dst + 2 * i) = __floats2bfloat162_rn(re[j], ro[j]);
      }
      for (int i = lane; i < half; i += 32)
        *reinterpret_cast<__nv_bfloat162*>(dst + a.voff + 2 * i) =
            *reinterpret_cast<const __nv_bfloat162*>(vrow + 2 * i);
    }
  }
}

struct WritePoolArgs {
  const __nv_bfloat16* kv;  // (tokens, L, 2, KV)
  int L, KV, D;
  const long long* meta;
  const void* kn;
  int kdt;
  RopeRef rope;
  const long long* pos;
  const long long* locs;
  const int* commit;
  long long row_w;
  int fp8, mode;
  float ks, vs, eps;
  int* err;
};

template <int NP>
__global__ void __launch_bounds__(128) write_ctx_pool_kernel(WritePoolArgs a) {
  const long long t = blockIdx.x;
  const int layer = blockIdx.y;
  if (a.commit) {
    const long long rb = t / a.row_w;
    if (t - rb * a.row_w >= (long long)a.commit[rb]) return;
  }
  const long long loc = a.locs[t];
  if (loc < 0) return;
  const int lane = threadIdx.x & 31, half = a.D >> 1;
  const long long pos = a.pos[t];
  const __nv_bfloat16* row = a.kv + (t * a.L + layer) * 2 * (long long)a.KV;
  const long long kbuf = a.meta[layer * 4 + 0], vbuf = a.meta[layer * 4 + 1];
  const long long kst = a.meta[layer * 4 + 2], vst = a.meta[layer * 4 + 3];
  const void* w = a.kdt == FM_DT_F32 ? (const void*)(static_cast<const float*>(a.kn) + (long long)layer * a.D)
                                     : (const void*)(static_cast<const __nv_bfloat16*>(a.kn) + (long long)layer * a.D);
  const int nh = a.KV / a.D;
  for (int h = threadIdx.x >> 5; h < nh; h += 4) {
    float re[NP], ro[NP];
    warp_norm_rope<NP>(row + (long long)h * a.D, a.D, w, a.kdt, a.eps, a.mode, a.rope, pos, a.err, re, ro);
    const __nv_bfloat16* vrow = row + a.KV + (long long)h * a.D;
    if (a.fp8) {
      uint8_t* kd = reinterpret_cast<uint8_t*>(kbuf) + loc * kst + (long long)h * a.D;
      uint8_t* vdst = reinterpret_cast<uint8_t*>(vbuf) + loc * vst + (long long)h * a.D;
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int i = lane + 32 * j;
        if (i < half) *reinterpret_cast<uint16_t*>(kd + 2 * i) = e4m3x2(__fdiv_rn(re[j], a.ks), __fdiv_rn(ro[j], a.ks));
      }
      for (int i = lane; i < half; i += 32) {
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(vrow + 2 * i);
        *reinterpret_cast<uint16_t*>(vdst + 2 * i) =
            e4m3x2(__fdiv_rn(__low2float(v), a.vs), __fdiv_rn(__high2float(v), a.vs));
      }
    } else {
      __nv_bfloat16* kd = reinterpret_cast<__nv_bfloat16*>(kbuf) + loc * kst + (long long)h * a.D;
      __nv_bfloat16* vdst = reinterpret_cast<__nv_bfloat16*>(vbuf) + loc * vst + (long long)h * a.D;
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int i = lane + 32 * j;
        if (i < half) *reinterpret_cast<__nv_bfloat162*>(kd + 2 * i) = __floats2bfloat162_rn(re[j], ro[j]);
      }
      for (int i = lane; i < half; i += 32)
        *reinterpret_cast<__nv_bfloat162*>(vdst + 2 * i) = *reinterpret_cast<const __nv_bfloat162*>(vrow + 2 * i);
    }
  }
}

fm_status check_rope(const fm_rope_view& r) {
  if (!r.cos || !r.sin || r.rows < 1 || r.row_stride < 0 || r.pair_stride < 0)
    return set_error(FM_ERR_INVALID, "rope table: null pointer or bad strides");
  return FM_OK;
}

int pairs_per_lane(int64_t hd) { return hd <= 64 ? 1 : hd <= 128 ? 2 : hd <= 256 ? 4 : 0; }

template <template <int> class K, class A>
fm_status launch_np(int np, dim3 grid, dim3 block, cudaStream_t s, const A& a) {
  if (np == 1) return launch_kernel(K<1>::fn, grid, block, 0, s, false, a);
  if (np == 2) return launch_kernel(K<2>::fn, grid, block, 0, s, false, a);
  return launch_kernel(K<4>::fn, grid, block, 0, s, false, a);
}
template <int NP>
struct NormRopeK {
  static constexpr auto fn = qk_norm_rope_kernel<NP>;
};
template <int NP>
struct WriteCtxK {
  static constexpr auto fn = write_ctx_paged_kernel<NP>;
};
template <int NP>
struct WritePoolK {
  static constexpr auto fn = write_ctx_pool_kernel<NP>;
};

template <int HD, bool KV8>
fm_status launch_paged(const PagedArgs& a, unsigned grid, cudaStream_t s) {
  constexpr int smem = PxLayout<HD, KV8>::SMEM;
  static int configured = -1;
  int dev;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaFuncSetAttribute(paged_xattn_kernel<HD, KV8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured = dev;
  }
  return launch_kernel(paged_xattn_kernel<HD, KV8>, dim3(grid), dim3(128), smem, s, false, a);
}

}  // namespace
}  // namespace fm

using namespace fm;

extern "C" fm_status fm_qk_norm_rope(const void* x, int64_t x_token_stride, void* out, int64_t out_token_stride,
                                     int64_t tokens, int64_t heads, int64_t head_dim, const void* weight,
                                     int32_t weight_dtype, fm_rope_view rope, const void* positions,
                                     int32_t positions_dtype, float eps, int32_t norm_mode, int32_t* err,
                                     fm_stream stream) {
  if (tokens < 0 || heads < 1) return set_error(FM_ERR_SHAPE, "qk_norm_rope: bad shape");
  if (tokens == 0) return FM_OK;
  if (!x || !out || !weight) return set_error(FM_ERR_INVALID, "qk_norm_rope: null pointer");
  const int np = pairs_per_lane(head_dim);
  if (!np || head_dim % 2) return set_error(FM_ERR_UNSUPPORTED, "qk_norm_rope: head_dim must be even and <= 256");
  if (weight_dtype != FM_DT_BF16 && weight_dtype != FM_DT_F32) return set_error(FM_ERR_INVALID, "weight dtype");
  if (positions && positions_dtype != FM_DT_I32 && positions_dtype != FM_DT_I64)
    return set_error(FM_ERR_INVALID, "positions dtype");
  if (norm_mode != FM_NORM_DIT && norm_mode != FM_NORM_FUSED) return set_error(FM_ERR_INVALID, "norm mode");
  fm_status st;
  if ((st = check_rope(rope))) return st;
  if ((uintptr_t)x % 4 || (uintptr_t)out % 4 || x_token_stride % 2 || out_token_stride % 2)
    return set_error(FM_ERR_ALIGN, "qk_norm_rope: rows must be 4-byte aligned");
  NormRopeArgs a{static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), x_token_stride,
                 out_token_stride, tokens, (int)heads, (int)head_dim, weight, weight_dtype, rope_ref(rope),
                 positions, positions_dtype, eps, norm_mode, err};
  const long long rows = tokens * heads;
  return launch_np<NormRopeK>(np, dim3((unsigned)((rows + NR_WARPS - 1) / NR_WARPS)), dim3(NR_WARPS * 32),
                              static_cast<cudaStream_t>(stream), a);
}

extern "C" fm_status fm_block_self_attn_qknorm(const void* qkv, void* out, int64_t blocks, int64_t block,
                                               int64_t heads, int64_t head_dim, const void* q_norm,
                                               const void* k_norm, int32_t weight_dtype, fm_rope_view rope,
                                               const void* positions, int32_t positions_dtype, float eps,
                                               float scale, int32_t* err, fm_stream stream) {
  if (blocks < 0 || heads < 1) return set_error(FM_ERR_SHAPE, "block_self_attn_qknorm: bad shape");
  if (block != 16 || (head_dim != 64 && head_dim != 128))
    return set_error(FM_ERR_UNSUPPORTED, "block_self_attn_qknorm: block 16 and head_dim 64 or 128");
  if (blocks == 0) return FM_OK;
  if (!qkv || !out || !q_norm || !k_norm) return set_error(FM_ERR_INVALID, "block_self_attn_qknorm: null pointer");
  if ((uintptr_t)qkv % 16 || (uintptr_t)out % 4) return set_error(FM_ERR_ALIGN, "qkv must be 16-byte aligned");
  if (weight_dtype != FM_DT_BF16 && weight_dtype != FM_DT_F32) return set_error(FM_ERR_INVALID, "weight dtype");
  if (positions && positions_dtype != FM_DT_I32 && positions_dtype != FM_DT_I64)
    return set_error(FM_ERR_INVALID, "positions dtype");
  fm_status st;
  if ((st = check_rope(rope))) return st;
  SelfQkArgs a{static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out), (int)blocks, (int)heads,
               q_norm, k_norm, weight_dtype, rope_ref(rope), positions, positions_dtype, eps, scale, err};
  const unsigned grid = (unsigned)(blocks * heads);  // one CTA per (block, head)
  const size_t smem = (size_t)3 * 16 * head_dim * 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  static int configured = -1;
  int dev;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaFuncSetAttribute(self_attn_qknorm_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    cudaFuncSetAttribute(self_attn_qknorm_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    configured = dev;
  }
  if (head_dim == 128)
    return launch_kernel(self_attn_qknorm_kernel<128>, dim3(grid), dim3(SQ_WARPS * 32), smem, s, false, a);
  return launch_kernel(self_attn_qknorm_kernel<64>, dim3(grid), dim3(SQ_WARPS * 32), smem, s, false, a);
}

extern "C" int32_t fm_paged_attn_nsplit(int64_t requests, int64_t heads, int64_t max_q, int64_t max_seqlen_k,
                                        int32_t nsplit) {
  if (nsplit > 0) return nsplit;
  const int64_t groups = max_q > 0 ? (max_q + 15) / 16 : 1;
  const int64_t items = (requests > 0 ? requests : 1) * (heads > 0 ? heads : 1) * groups;
  int64_t want = (2 * (int64_t)num_sms() + items - 1) / items;
  const int64_t tiles = max_seqlen_k > 0 ? (max_seqlen_k + PX_TILE - 1) / PX_TILE : 1;
  if (want > tiles) want = tiles;
  if (want > 64) want = 64;
  return (int32_t)(want < 1 ? 1 : want);
}

extern "C" size_t fm_paged_attn_workspace_size(int64_t requests, int64_t heads, int64_t head_dim, int64_t max_q,
                                               int32_t nsplit) {
  const int64_t groups = max_q > 0 ? (max_q + 15) / 16 : 1;
  const int64_t items = requests * heads * groups;
  const size_t counters = ((size_t)items * 4 + 255) / 256 * 256;
  return counters + (size_t)items * (nsplit > 0 ? nsplit : 1) * (16 * head_dim + 32) * 4;
}

extern "C" fm_status fm_paged_cross_attn(const fm_paged_attn* p, fm_stream stream) {
  if (!p) return set_error(FM_ERR_INVALID, "paged_cross_attn: null arguments");
  if (p->requests < 0 || p->heads < 1 || p->page_size < 1 || p->page_table_cols < 0 || p->num_pages < 0)
    return set_error(FM_ERR_SHAPE, "paged_cross_attn: bad shape");
  if (p->head_dim != 64 && p->head_dim != 128) return set_error(FM_ERR_UNSUPPORTED, "paged_cross_attn: head_dim 64 or 128");
  if (p->requests == 0) return FM_OK;
  if (!p->q || !p->k || !p->v || !p->page_table || !p->seqused_k || !p->out || !p->workspace)
    return set_error(FM_ERR_INVALID, "paged_cross_attn: null pointer");
  if (!p->cu_seqlens_q && p->q_per_request < 1) return set_error(FM_ERR_SHAPE, "paged_cross_attn: no query rows");
  if (p->q_dtype != FM_DT_BF16 && p->q_dtype != FM_DT_E4M3) return set_error(FM_ERR_INVALID, "query dtype");
  if (p->kv_dtype != FM_DT_BF16 && p->kv_dtype != FM_DT_E4M3) return set_error(FM_ERR_INVALID, "cache dtype");
  if (p->quantize_q && (p->q_dtype != FM_DT_BF16 || p->kv_dtype != FM_DT_E4M3 || p->descales))
    return set_error(FM_ERR_INVALID, "quantize_q takes a bf16 query, an e4m3 cache and no descales");
  if (p->q_dtype == FM_DT_E4M3 && p->kv_dtype != FM_DT_E4M3)
    return set_error(FM_ERR_INVALID, "an e4m3 query needs an e4m3 cache");
  const int esz = p->kv_dtype == FM_DT_E4M3 ? 1 : 2;
  if ((uintptr_t)p->k % 16 || (uintptr_t)p->v % 16 || (p->kv_page_stride * esz) % 16 ||
      (p->kv_head_stride * esz) % 16 || (p->kv_token_stride * esz) % 16)
    return set_error(FM_ERR_ALIGN, "paged_cross_attn: cache rows must be 16-byte aligned");
  if (p->q_dtype == FM_DT_BF16 && ((uintptr_t)p->q % 4 || p->q_token_stride % 2 || p->q_head_stride % 2))
    return set_error(FM_ERR_ALIGN, "paged_cross_attn: query rows must be 4-byte aligned");
  const int64_t max_q = p->cu_seqlens_q ? p->max_q : p->q_per_request;
  if (max_q < 1) return set_error(FM_ERR_SHAPE, "paged_cross_attn: max_q must be positive");
  const int nsplit = fm_paged_attn_nsplit(p->requests, p->heads, max_q, p->max_seqlen_k, p->nsplit);
  const size_t need = fm_paged_attn_workspace_size(p->requests, p->heads, p->head_dim, max_q, nsplit);
  if (p->workspace_bytes < need) return set_error(FM_ERR_WORKSPACE, "paged_cross_attn: workspace %zu < %zu", p->workspace_bytes, need);
  const int groups = (int)((max_q + 15) / 16);
  const int64_t items = p->requests * p->heads * groups;
  const size_t counters = ((size_t)items * 4 + 255) / 256 * 256;
  PagedArgs a{};
  a.q = static_cast<const uint8_t*>(p->q);
  a.q8 = p->q_dtype == FM_DT_E4M3;
  a.q_ts = p->q_token_stride;
  a.q_hs = p->q_head_stride;
  a.cu = p->cu_seqlens_q;
  a.qpr = p->q_per_request;
  a.groups = groups;
  a.k = static_cast<const uint8_t*>(p->k);
  a.v = static_cast<const uint8_t*>(p->v);
  a.kps = p->kv_page_stride;
  a.khs = p->kv_head_stride;
  a.kts = p->kv_token_stride;
  a.page = (int)p->page_size;
  a.num_pages = p->num_pages;
  a.table = p->page_table;
  a.tstride = p->page_table_stride;
  a.tcols = p->page_table_cols;
  a.seqused = p->seqused_k;
  a.R = (int)p->requests;
  a.H = (int)p->heads;
  a.nsplit = nsplit;
  a.scale = p->softmax_scale;
  a.descales = p->descales;
  a.quant_q = p->quantize_q;
  a.out = static_cast<__nv_bfloat16*>(p->out);
  a.o_ts = p->out_token_stride;
  a.o_hs = p->out_head_stride;
  a.counters = static_cast<int*>(p->workspace);
  a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(p->workspace) + counters);
  a.err = p->err;
  const int64_t grid = items * nsplit;
  if (grid > 0x7fffffff) return set_error(FM_ERR_SHAPE, "paged_cross_attn: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool kv8 = p->kv_dtype == FM_DT_E4M3;
  if (p->head_dim == 128) return kv8 ? launch_paged<128, true>(a, (unsigned)grid, s) : launch_paged<128, false>(a, (unsigned)grid, s);
  return kv8 ? launch_paged<64, true>(a, (unsigned)grid, s) : launch_paged<64, false>(a, (unsigned)grid, s);
}

extern "C" fm_status fm_write_context_kv_paged(const void* kv, int64_t tokens, int64_t layers, int64_t heads,
                                               int64_t head_dim, const int64_t* positions, const int64_t* slots,
                                               const void* k_norm, int32_t k_norm_dtype, fm_rope_view rope,
                                               const int64_t* cache_ptrs, int64_t num_caches,
                                               int64_t heads_per_cache, int64_t stride_block, int64_t stride_head,
                                               int64_t stride_token, int64_t v_offset, int64_t block_size,
                                               float eps, const float* scales, int32_t* err, fm_stream stream) {
  if (tokens < 0 || layers < 1 || heads < 1 || num_caches < 1 || heads_per_cache < 1 || block_size < 1)
    return set_error(FM_ERR_SHAPE, "write_context_kv: bad shape");
  if (num_caches * heads_per_cache < layers * heads)
    return set_error(FM_ERR_SHAPE, "write_context_kv: %lld caches of %lld heads cannot hold %lld x %lld heads",
                     (long long)num_caches, (long long)heads_per_cache, (long long)layers, (long long)heads);
  if (tokens == 0) return FM_OK;
  if (!kv || !positions || !slots || !k_norm || !cache_ptrs)
    return set_error(FM_ERR_INVALID, "write_context_kv: null pointer");
  const int np = pairs_per_lane(head_dim);
  if (!np || head_dim % 2) return set_error(FM_ERR_UNSUPPORTED, "write_context_kv: head_dim must be even and <= 256");
  if (k_norm_dtype != FM_DT_BF16 && k_norm_dtype != FM_DT_F32) return set_error(FM_ERR_INVALID, "k_norm dtype");
  if (stride_block % 2 || stride_head % 2 || stride_token % 2 || v_offset % 2)
    return set_error(FM_ERR_ALIGN, "write_context_kv: strides must be even");
  fm_status st;
  if ((st = check_rope(rope))) return st;
  WriteCtxArgs a{static_cast<const __nv_bfloat16*>(kv), (int)layers, (int)heads, (int)head_dim,
                 reinterpret_cast<const long long*>(positions), reinterpret_cast<const long long*>(slots), k_norm,
                 k_norm_dtype, rope_ref(rope), reinterpret_cast<const long long*>(cache_ptrs), (int)heads_per_cache,
                 stride_block, stride_head, stride_token, v_offset, block_size, eps, scales, err};
  return launch_np<WriteCtxK>(np, dim3((unsigned)tokens, (unsigned)num_caches), dim3(128),
                              static_cast<cudaStream_t>(stream), a);
}

extern "C" fm_status fm_kv_norm_rope_write_pool(const void* kv, int64_t tokens, int64_t layers, int64_t kv_size,
                                                int64_t head_dim, const int64_t* meta, const void* k_norm,
                                                int32_t k_norm_dtype, fm_rope_view rope, const int64_t* positions,
                                                const int64_t* locs, const int32_t* commit_lens,
                                                int64_t locs_row_width, int32_t pool_dtype, int32_t norm_mode,
                                                float k_scale, float v_scale, float eps, int32_t* err,
                                                fm_stream stream) {
  if (tokens < 0 || layers < 1 || head_dim < 2 || kv_size < head_dim || kv_size % head_dim)
    return set_error(FM_ERR_SHAPE, "kv_norm_rope_write: bad shape");
  if (tokens == 0) return FM_OK;
  if (!kv || !meta || !k_norm || !positions || !locs) return set_error(FM_ERR_INVALID, "kv_norm_rope_write: null pointer");
  if (commit_lens && locs_row_width < 1) return set_error(FM_ERR_SHAPE, "kv_norm_rope_write: locs_row_width");
  const int np = pairs_per_lane(head_dim);
  if (!np || head_dim % 2) return set_error(FM_ERR_UNSUPPORTED, "kv_norm_rope_write: head_dim must be even and <= 256");
  if (k_norm_dtype != FM_DT_BF16 && k_norm_dtype != FM_DT_F32) return set_error(FM_ERR_INVALID, "k_norm dtype");
  if (pool_dtype != FM_DT_BF16 && pool_dtype != FM_DT_E4M3) return set_error(FM_ERR_INVALID, "pool dtype");
  if (norm_mode != FM_NORM_DIT && norm_mode != FM_NORM_FUSED) return set_error(FM_ERR_INVALID, "norm mode");
  fm_status st;
  if ((st = check_rope(rope))) return st;
  WritePoolArgs a{static_cast<const __nv_bfloat16*>(kv), (int)layers, (int)kv_size, (int)head_dim,
                  reinterpret_cast<const long long*>(meta), k_norm, k_norm_dtype, rope_ref(rope),
                  reinterpret_cast<const long long*>(positions), reinterpret_cast<const long long*>(locs),
                  commit_lens, locs_row_width, pool_dtype == FM_DT_E4M3, norm_mode, k_scale, v_scale, eps, err};
  return launch_np<WritePoolK>(np, dim3((unsigned)tokens, (unsigned)layers), dim3(128),
                               static_cast<cudaStream_t>(stream), a);
}
