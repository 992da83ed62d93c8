// Row-wise, noise, sampling and acceptance kernels of the FlashMap hot path,
// and their C-ABI entry points.
#include <mutex>

#include "attention.cuh"
#include "ops.cuh"
#include "philox.cuh"
#include "rows.cuh"

namespace fm {

namespace {

constexpr int RT = 256;  // threads of the row kernels

// Sum over a 256-thread block in a fixed tree: offsets 16..1 inside each
// warp, then 4, 2, 1 over the 8 warp sums.  `red` holds >= 9 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float r = lane < (RT / 32) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = RT / 64; o >= 1; o >>= 1) r = __fadd_rn(r, __shfl_down_sync(0xffffffffu, r, o));
    if (lane == 0) red[RT / 32] = r;
  }
  __syncthreads();
  const float out = red[RT / 32];
  __syncthreads();
  return out;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < RT / 32; ++w) r = fmaxf(r, red[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ int block_min_int(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_min_sync(0xffffffffu, v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int r = red[0];
  for (int w = 1; w < RT / 32; ++w) r = min(r, red[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ int block_max_int(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_max_sync(0xffffffffu, v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int r = red[0];
  for (int w = 1; w < RT / 32; ++w) r = max(r, red[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return bf2f(v); }
__device__ __forceinline__ float to_f(float v) { return v; }

// 8 consecutive elements of a row (vector `vec`), zero-padded past V
__device__ __forceinline__ void load8(const float* row, long long vec, long long V, bool aligned, float* x) {
  const long long v0 = vec * 8;
  if (aligned && v0 + 8 <= V) {
    const float4 a = *reinterpret_cast<const float4*>(row + v0);
    const float4 b = *reinterpret_cast<const float4*>(row + v0 + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = (v0 + j < V) ? row[v0 + j] : 0.0f;
  }
}

__device__ __forceinline__ void load8(const __nv_bfloat16* row, long long vec, long long V, bool aligned,
                                      float* x) {
  const long long v0 = vec * 8;
  if (aligned && v0 + 8 <= V) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row + v0);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = (v0 + j < V) ? bf2f(row[v0 + j]) : 0.0f;
  }
}

// 8 consecutive elements of a row kept as loaded (bf16: four 32-bit words,
// unpacked a pair at a time where they are used), zero-padded past V
template <typename T>
struct Raw8;

template <>
struct Raw8<__nv_bfloat16> {
  uint32_t w[4];
  __device__ __forceinline__ void load(const __nv_bfloat16* row, long long vec, long long V, bool aligned) {
    const long long v0 = vec * 8;
    if (aligned && v0 + 8 <= V) {
      const uint4 raw = *reinterpret_cast<const uint4*>(row + v0);
      w[0] = raw.x;
      w[1] = raw.y;
      w[2] = raw.z;
      w[3] = raw.w;
    } else {
      const unsigned short* h = reinterpret_cast<const unsigned short*>(row);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = (v0 + 2 * i < V) ? h[v0 + 2 * i] : 0u, hi = (v0 + 2 * i + 1 < V) ? h[v0 + 2 * i + 1] : 0u;
        w[i] = lo | (hi << 16);
      }
    }
  }
  // elements 2i, 2i + 1
  __device__ __forceinline__ float2 pair(int i) const {
    return make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
  }
};

template <>
struct Raw8<float> {
  float x[8];
  __device__ __forceinline__ void load(const float* row, long long vec, long long V, bool aligned) {
    load8(row, vec, V, aligned, x);
  }
  __device__ __forceinline__ float2 pair(int i) const { return make_float2(x[2 * i], x[2 * i + 1]); }
};

// max of x/T, and (first) argmax of the raw values, over one row
template <typename T>
__device__ void row_max_argmax(const T* row, long long V, float temperature, float* red, float* m_out,
                               long long* arg_out) {
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const long long nvec = (V + 7) / 8;
  float m = -INFINITY, bv = -INFINITY;
  long long bi = V;  // sentinel larger than any index
  // vectors i, i + RT, ... in order; four loads issued ahead of their use
  for (long long vec0 = threadIdx.x; vec0 < nvec; vec0 += 4 * RT) {
    float x[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (vec0 + u * RT < nvec) load8(row, vec0 + u * RT, V, aligned, x[u]);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long vec = vec0 + u * RT;
      if (vec >= nvec) break;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const long long v = vec * 8 + j;
        if (v >= V) break;
        if (bi == V || x[u][j] > bv) {  // strict: the first index of a tie stays
          bv = x[u][j];
          bi = v;
        }
        if (temperature > 0.0f) m = fmaxf(m, __fdiv_rn(x[u][j], temperature));
      }
    }
  }
  // block argmax: largest value, smallest index among equals
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const long long oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __shared__ float rv[RT / 32];
  __shared__ long long ri[RT / 32];
  if (lane == 0) {
    rv[warp] = bv;
    ri[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = rv[0];
    long long i = ri[0];
    for (int w = 1; w < RT / 32; ++w)
      if (rv[w] > b || (rv[w] == b && ri[w] < i)) {
        b = rv[w];
        i = ri[w];
      }
    *arg_out = i;
  }
  __syncthreads();
  *m_out = temperature > 0.0f ? block_max(m, red) : 0.0f;
}

// fixed-order sum of fm_exp(x/T - m): thread i walks vectors i, i+256, ...,
// the elements of a vector in index order.  Full vectors take fm_exp2 on
// element pairs (values identical to fm_exp), the partial last one fm_exp.
// (Vector indices are 32-bit: the callers bound V below 2^31.)
template <bool UNIT_T, typename T>
__device__ float row_sumexp_t(const T* row, long long V, float temperature, float m, float* red) {
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int nvec = (int)((V + 7) / 8), nfull = (int)(V / 8);
  const float2 neg_m = make_float2(-m, -m);  // x - m == x + (-m) exactly
  float acc = 0.0f;
  for (int vec0 = threadIdx.x; vec0 < nvec; vec0 += 4 * RT) {
    Raw8<T> x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (vec0 + u * RT < nvec) x[u].load(row, vec0 + u * RT, V, aligned);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int vec = vec0 + u * RT;
      if (vec >= nvec) break;
      // x / 1 == x exactly, so the division is skipped at T = 1
      if (vec < nfull) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 xt = x[u].pair(i);
          if (!UNIT_T) xt = make_float2(__fdiv_rn(xt.x, temperature), __fdiv_rn(xt.y, temperature));
          const float2 e = fm_exp2(__fadd2_rn(xt, neg_m));
          acc = __fadd_rn(acc, e.x);
          acc = __fadd_rn(acc, e.y);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 xp = x[u].pair(i);
          if ((long long)vec * 8 + 2 * i < V)
            acc = __fadd_rn(acc, fm_exp(__fsub_rn(UNIT_T ? xp.x : __fdiv_rn(xp.x, temperature), m)));
          if ((long long)vec * 8 + 2 * i + 1 < V)
            acc = __fadd_rn(acc, fm_exp(__fsub_rn(UNIT_T ? xp.y : __fdiv_rn(xp.y, temperature), m)));
        }
      }
    }
  }
  return block_sum(acc, red);
}

template <typename T>
__device__ float row_sumexp(const T* row, long long V, float temperature, float m, float* red) {
  return temperature == 1.0f ? row_sumexp_t<true>(row, V, temperature, m, red)
                             : row_sumexp_t<false>(row, V, temperature, m, red);
}

__device__ __forceinline__ long long range_width(long long V) {
  const long long w = (V + RT - 1) / RT;
  return (w + 7) / 8 * 8;
}

// Categorical draw over non-negative weights w(v), v < V, with uniform u:
// contiguous per-thread ranges, scan, two-level search (see the C oracle).
// A range weight functor that computes nothing in bulk (scalar weights only).
struct NoBulk {
  __device__ bool operator()(long long, float*) const { return false; }
};

// bulk(v0, w) may fill w[0..31] with the weights of v0 .. v0+31 (all < V) from
// vector loads issued together, returning false when it cannot (alignment);
// the range sum then takes the scalar weights.  Either way the sum runs in
// index order, so the result does not depend on which path ran.
template <typename F, typename B = NoBulk>
__device__ long long block_categorical(F weight, long long V, float u, float* sm, B bulk = B()) {
  const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
  const long long W = range_width(V);
  const long long lo = (long long)i * W, hi = min(lo + W, V);
  float t = 0.0f;
  long long v = lo;
  for (; v + 32 <= hi; v += 32) {
    float w[32];
    if (!bulk(v, w)) break;
#pragma unroll
    for (int j = 0; j < 32; ++j) t = __fadd_rn(t, w[j]);
  }
  for (; v < hi; ++v) t = __fadd_rn(t, weight(v));
  float h = t;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, h, off);
    if (lane >= off) h = __fadd_rn(y, h);
  }
  if (lane == 31) sm[RT + warp] = h;
  __syncthreads();
  if (i == 0) {
    float base = 0.0f;
    for (int w = 0; w < RT / 32; ++w) {
      const float tot = sm[RT + w];
      sm[RT + 8 + w] = base;
      base = (w == 0) ? tot : __fadd_rn(base, tot);
    }
  }
  __syncthreads();
  if (warp > 0) h = __fadd_rn(sm[RT + 8 + warp], h);
  sm[i] = h;
  __syncthreads();
  const float total = sm[RT - 1];
  const float target = __fmul_rn(u, total);
  int* ired = reinterpret_cast<int*>(sm + RT + 16);
  const int first = block_min_int(h > target ? i : RT, ired);
  const int lastpos = block_max_int(t > 0.0f ? i : -1, ired);
  __shared__ long long result;
  // the chosen range's weights, computed by the whole block (the running sum
  // below stays sequential, in index order)
  constexpr int WMAX = 4096;
  __shared__ float wbuf[WMAX];
  const int chosen = first < RT ? first : lastpos;
  const long long clo = chosen >= 0 ? (long long)chosen * W : 0, chi = chosen >= 0 ? min(clo + W, V) : 0;
  const bool staged = chi - clo <= WMAX;
  if (staged)
    for (long long v = clo + i; v < chi; v += RT) wbuf[v - clo] = weight(v);
  __syncthreads();
  if (i == 0) {
    long long pick = 0;
    if (chosen >= 0) {
      float run = chosen > 0 ? sm[chosen - 1] : 0.0f;
      long long last = -1;
      pick = -1;
      for (long long v = clo; v < chi; ++v) {
        const float wv = staged ? wbuf[v - clo] : weight(v);
        run = __fadd_rn(run, wv);
        if (wv > 0.0f) last = v;
        if (run > target) {
          pick = v;
          break;
        }
      }
      if (pick < 0) pick = last >= 0 ? last : clo;
    }
    result = pick;
  }
  __syncthreads();
  return result;
}

// ------------------------------------------------------------------ kernels

// One warp per row (rows.cuh gives the reduction order): 8 rows per CTA.
// Rows up to 2048 wide (one chunk round) whose width is a multiple of 8 with
// 16-byte aligned pointers keep the row and its per-column vectors in
// registers, all loaded at once; other rows take the general loop.
constexpr int ROWS_PER_CTA = RT / 32;

__device__ __forceinline__ bool vec_ok(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// the lane's chunks (lane + 32 i, i < 8) of a row: count, loaded together
__device__ __forceinline__ int lane_load8(const __nv_bfloat16* row, int nch, int lane, uint4* raw) {
  int n = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ch = lane + 32 * i;
    if (ch < nch) {
      raw[i] = *reinterpret_cast<const uint4*>(row + ch * 8);
      n = i + 1;
    }
  }
  return n;
}

// Rows wider than 2048 (up to 32 * MAXC * 8 columns): the row held in
// registers as 16-byte chunks lane + 32 i (the canonical order of rows.cuh),
// the weight / modulation chunks loaded as each output chunk is formed.
template <int MAXC>
__device__ __forceinline__ int lane_load(const __nv_bfloat16* row, int nch, int lane, uint4* raw) {
  int n = 0;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int ch = lane + 32 * i;
    if (ch < nch) {
      raw[i] = *reinterpret_cast<const uint4*>(row + ch * 8);
      n = i + 1;
    }
  }
  return n;
}
constexpr int WIDE_CHUNKS = 24;  // rows of up to 6144 columns
// Wide rows read their per-column weights (RMSNorm weight, AdaLN scale and
// shift) WIDE_GROUP chunks at a time, all of a group's 16-byte loads issued
// before its outputs are stored: read-only loads, so the compiler need not
// order them after the stores (the output may not alias a weight)
constexpr int WIDE_GROUP = 8;
__device__ __forceinline__ uint4 ldg16(const __nv_bfloat16* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void rms_row_wide(const __nv_bfloat16* xr, const __nv_bfloat16* w, __nv_bfloat16* yr,
                                             int cols, float eps, int lane) {
  const int nch = cols / 8;
  uint4 xv[WIDE_CHUNKS];
  const int n = lane_load<WIDE_CHUNKS>(xr, nch, lane, xv);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < WIDE_CHUNKS; ++i)
    if (i < n) {
      float xf[8], t[8];
      unpack_bf16x8(xv[i], xf);
#pragma unroll
      for (int e = 0; e < 8; ++e) t[e] = __fmul_rn(xf[e], xf[e]);
      s = __fadd_rn(s, chunk_tree(t, 8));
    }
  const float inv = inv_rms(warp_allsum(s), cols, eps);
#pragma unroll
  for (int g0 = 0; g0 < WIDE_CHUNKS; g0 += WIDE_GROUP) {
    uint4 wv[WIDE_GROUP];
#pragma unroll
    for (int i = 0; i < WIDE_GROUP; ++i)
      if (g0 + i < n) wv[i] = ldg16(w + (lane + 32 * (g0 + i)) * 8);
#pragma unroll
    for (int i = 0; i < WIDE_GROUP; ++i)
      if (g0 + i < n) {
        const int ch = lane + 32 * (g0 + i);
        float xf[8], wf[8], o[8];
        unpack_bf16x8(xv[g0 + i], xf);
        unpack_bf16x8(wv[i], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rms_value(xf[e], wf[e], inv);
        *reinterpret_cast<uint4*>(yr + ch * 8) = pack_bf16x8(o);
      }
  }
}

__global__ void __launch_bounds__(RT) rmsnorm_kernel(const __nv_bfloat16* x, const __nv_bfloat16* w,
                                                     __nv_bfloat16* y, long long rows, int cols, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  if (r >= rows) return;
  const __nv_bfloat16* xr = x + r * cols;
  __nv_bfloat16* yr = y + r * cols;
  if (cols % 8 == 0 && cols <= 2048 && vec_ok(xr) && vec_ok(yr) && vec_ok(w)) {
    const int nch = cols / 8;
    uint4 xv[8], wv[8];
    const int n = lane_load8(xr, nch, lane, xv);
    lane_load8(w, nch, lane, wv);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < n) {
        float xf[8], t[8];
        unpack_bf16x8(xv[i], xf);
#pragma unroll
        for (int e = 0; e < 8; ++e) t[e] = __fmul_rn(xf[e], xf[e]);
        s = __fadd_rn(s, chunk_tree(t, 8));
      }
    const float inv = inv_rms(warp_allsum(s), cols, eps);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < n) {
        float xf[8], wf[8], o[8];
        unpack_bf16x8(xv[i], xf);
        unpack_bf16x8(wv[i], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rms_value(xf[e], wf[e], inv);
        *reinterpret_cast<uint4*>(yr + (lane + 32 * i) * 8) = pack_bf16x8(o);
      }
    return;
  }
  if (cols % 8 == 0 && cols <= 32 * 8 * WIDE_CHUNKS && vec_ok(xr) && vec_ok(yr) && vec_ok(w)) {
    rms_row_wide(xr, w, yr, cols, eps, lane);
    return;
  }
  const float inv = inv_rms(warp_row_sumsq(xr, cols, lane), cols, eps);
  for (int c = lane; c < cols; c += 32) yr[c] = f2bf(rms_value(bf2f(xr[c]), bf2f(w[c]), inv));
}

// AdaLN of a row of up to NC * 256 columns with the row, scale and shift
// all loaded before the statistics (one round trip): NC = 8 for rows up to
// 2048, NC = 12 up to 3072 (the 27B map's 2560).
template <int NC>
__device__ __forceinline__ void adaln_row_upfront(const __nv_bfloat16* xr, const __nv_bfloat16* mod,
                                                  __nv_bfloat16* yr, int cols, float eps, int lane) {
  const int nch = cols / 8;
  uint4 xv[NC], sv[NC], hv[NC];
  const int n = lane_load<NC>(xr, nch, lane, xv);
  lane_load<NC>(mod, nch, lane, sv);
  lane_load<NC>(mod + cols, nch, lane, hv);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NC; ++i)
    if (i < n) {
      float xf[8];
      unpack_bf16x8(xv[i], xf);
      s = __fadd_rn(s, chunk_tree(xf, 8));
    }
  const float mean = __fdiv_rn(warp_allsum(s), (float)cols);
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < NC; ++i)
    if (i < n) {
      float xf[8], t[8];
      unpack_bf16x8(xv[i], xf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = __fsub_rn(xf[e], mean);
        t[e] = __fmul_rn(d, d);
      }
      q = __fadd_rn(q, chunk_tree(t, 8));
    }
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(warp_allsum(q), (float)cols), eps)));
#pragma unroll
  for (int i = 0; i < NC; ++i)
    if (i < n) {
      float xf[8], sc[8], sh[8], o[8];
      unpack_bf16x8(xv[i], xf);
      unpack_bf16x8(sv[i], sc);
      unpack_bf16x8(hv[i], sh);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = adaln_value(xf[e], mean, rstd, sc[e], sh[e]);
      *reinterpret_cast<uint4*>(yr + (lane + 32 * i) * 8) = pack_bf16x8(o);
    }
}

// AdaLN of one row per warp: LayerNorm statistics, then the modulated output
// (mod = [scale | shift], each `cols` wide)
__global__ void __launch_bounds__(RT) adaln_kernel(const __nv_bfloat16* x, const __nv_bfloat16* mod,
                                                   __nv_bfloat16* y, long long rows, int cols, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  if (r >= rows) return;
  const __nv_bfloat16* xr = x + r * cols;
  __nv_bfloat16* yr = y + r * cols;
  if (cols % 8 == 0 && cols <= 2048 && vec_ok(xr) && vec_ok(yr) && vec_ok(mod)) {
    adaln_row_upfront<8>(xr, mod, yr, cols, eps, lane);
    return;
  }
  if (cols % 8 == 0 && cols <= 3072 && vec_ok(xr) && vec_ok(yr) && vec_ok(mod)) {
    adaln_row_upfront<12>(xr, mod, yr, cols, eps, lane);
    return;
  }
  if (cols % 8 == 0 && cols <= 32 * 8 * WIDE_CHUNKS && vec_ok(xr) && vec_ok(yr) && vec_ok(mod)) {
    // wide rows: the same canonical order, the modulation read chunk by chunk
    const int nch = cols / 8;
    uint4 xv[WIDE_CHUNKS];
    const int n = lane_load<WIDE_CHUNKS>(xr, nch, lane, xv);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < WIDE_CHUNKS; ++i)
      if (i < n) {
        float xf[8];
        unpack_bf16x8(xv[i], xf);
        s = __fadd_rn(s, chunk_tree(xf, 8));
      }
    const float mean = __fdiv_rn(warp_allsum(s), (float)cols);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < WIDE_CHUNKS; ++i)
      if (i < n) {
        float xf[8], t[8];
        unpack_bf16x8(xv[i], xf);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = __fsub_rn(xf[e], mean);
          t[e] = __fmul_rn(d, d);
        }
        q = __fadd_rn(q, chunk_tree(t, 8));
      }
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(warp_allsum(q), (float)cols), eps)));
#pragma unroll
    for (int g0 = 0; g0 < WIDE_CHUNKS; g0 += WIDE_GROUP) {
      uint4 sv[WIDE_GROUP], hv[WIDE_GROUP];
#pragma unroll
      for (int i = 0; i < WIDE_GROUP; ++i)
        if (g0 + i < n) {
          const int ch = lane + 32 * (g0 + i);
          sv[i] = ldg16(mod + ch * 8);
          hv[i] = ldg16(mod + cols + ch * 8);
        }
#pragma unroll
      for (int i = 0; i < WIDE_GROUP; ++i)
        if (g0 + i < n) {
          const int ch = lane + 32 * (g0 + i);
          float xf[8], sc[8], sh[8], o[8];
          unpack_bf16x8(xv[g0 + i], xf);
          unpack_bf16x8(sv[i], sc);
          unpack_bf16x8(hv[i], sh);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = adaln_value(xf[e], mean, rstd, sc[e], sh[e]);
          *reinterpret_cast<uint4*>(yr + ch * 8) = pack_bf16x8(o);
        }
    }
    return;
  }
  float mean, rstd;
  warp_row_meanrstd(xr, cols, eps, lane, &mean, &rstd);
  for (int c = lane; c < cols; c += 32)
    yr[c] = f2bf(adaln_value(bf2f(xr[c]), mean, rstd, bf2f(mod[c]), bf2f(mod[cols + c])));
}

__global__ void rope_table_kernel(float* cs, float* sn, int max_pos, int hd, const float* inv_freq) {
  const int half = hd / 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)max_pos * half) return;
  const int pos = (int)(idx / half), i = (int)(idx % half);
  // modeling_flashmap.py:57-58 in fp32: angle = pos * inv_freq[i]
  const float ang = __fmul_rn((float)pos, inv_freq[i]);
  cs[idx] = cosf(ang);
  sn[idx] = sinf(ang);
}

__global__ void __launch_bounds__(RT) draft_prep_kernel(DraftPrepArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  long long id = a.anchor_ids[b];
  const int len = a.lengths[b];
  if (id < 0 || id >= a.V) {
    if (threadIdx.x == 0) record_error(a.err, DEV_BAD_INDEX);
    id = 0;
  }
  if (threadIdx.x == 0 && (len < 0 || len + a.K + 1 > a.rope_len || len >= a.cache_len))
    record_error(a.err, DEV_BAD_INDEX);
  const __nv_bfloat16* src = a.embed + id * a.Ht;
  __nv_bfloat16* dst = a.anchor_rows + (long long)b * a.Ht;
  for (int c = threadIdx.x; c < a.Ht; c += RT) dst[c] = src[c];
  if (threadIdx.x == 0) {
    a.anchor_pos[b] = len;
    a.anchor_seq[b] = b;
    if (b == 0 && a.offset_bump) *a.offset_bump += 1u;
  }
  for (int k = threadIdx.x; k < a.K; k += RT) {
    a.slot_pos[b * a.K + k] = len + 1 + k;
    a.keys[b * a.K + k] = 0ull;
  }
  // the slots' rotary factors, read once here instead of in every q/k epilogue
  const int half = a.rope_half;
  for (int i = threadIdx.x; i < a.K * half; i += RT) {
    const int k = i / half, f = i - k * half;
    int pos = len + 1 + k;
    if (pos < 0 || pos >= a.rope_len) pos = 0;  // recorded above
    a.tok_cos[(long long)b * a.K * half + i] = a.rope_cos[(long long)pos * half + f];
    a.tok_sin[(long long)b * a.K * half + i] = a.rope_sin[(long long)pos * half + f];
  }
}

__global__ void __launch_bounds__(RT) rope_gather_kernel(const int* positions, int T, const float* rope_cos,
                                                         const float* rope_sin, int rope_len, int half,
                                                         float* tok_cos, float* tok_sin, int* err) {
  const long long i = (long long)blockIdx.x * RT + threadIdx.x;
  if (i >= (long long)T * half) return;
  const int t = (int)(i / half), f = (int)(i - (long long)t * half);
  int pos = positions[t];
  if (pos < 0 || pos >= rope_len) {
    if (f == 0) record_error(err, DEV_BAD_INDEX);
    pos = 0;
  }
  tok_cos[i] = rope_cos[(long long)pos * half + f];
  tok_sin[i] = rope_sin[(long long)pos * half + f];
}

__global__ void __launch_bounds__(RT) mix_state_kernel(MixArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  if (t >= a.T) return;
  const __nv_bfloat16* pr = a.post + (long long)t * a.post_stride;
  const __nv_bfloat16* sr = a.state + (long long)t * a.Ht;
  __nv_bfloat16* orow = a.out + (long long)t * a.Ht;
  if (a.Ht % 8 == 0 && vec_ok(pr) && vec_ok(sr) && vec_ok(orow) && vec_ok(a.state_norm_w) &&
      vec_ok(a.noise_norm_w)) {
    // rounds of 8 chunks per lane (chunk lane + 32 k in round k / 8): sums in the canonical order
    const int nch = a.Ht / 8;
    float sp = 0.0f, ss = 0.0f;
    for (int rd = 0; rd * 256 < nch; ++rd) {
      uint4 pv[8], zv[8];
      const int n = lane_load8(pr + rd * 2048, nch - rd * 256, lane, pv);
      lane_load8(sr + rd * 2048, nch - rd * 256, lane, zv);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < n) {
          float f[8], t2[8];
          unpack_bf16x8(pv[i], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) t2[e] = __fmul_rn(f[e], f[e]);
          sp = __fadd_rn(sp, chunk_tree(t2, 8));
          unpack_bf16x8(zv[i], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) t2[e] = __fmul_rn(f[e], f[e]);
          ss = __fadd_rn(ss, chunk_tree(t2, 8));
        }
    }
    const float ip = inv_rms(warp_allsum(sp), a.Ht, a.eps);
    const float is = inv_rms(warp_allsum(ss), a.Ht, a.eps);
    for (int rd = 0; rd * 256 < nch; ++rd) {
      uint4 pv[8], zv[8], av[8], bv[8];
      const int n = lane_load8(pr + rd * 2048, nch - rd * 256, lane, pv);
      lane_load8(sr + rd * 2048, nch - rd * 256, lane, zv);
      lane_load8(a.state_norm_w + rd * 2048, nch - rd * 256, lane, av);
      lane_load8(a.noise_norm_w + rd * 2048, nch - rd * 256, lane, bv);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < n) {
          float pf[8], zf[8], af[8], bf_[8], o[8];
          unpack_bf16x8(pv[i], pf);
          unpack_bf16x8(zv[i], zf);
          unpack_bf16x8(av[i], af);
          unpack_bf16x8(bv[i], bf_);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = mix_value(pf[e], zf[e], af[e], bf_[e], ip, is, a.gate);
          *reinterpret_cast<uint4*>(orow + rd * 2048 + (lane + 32 * i) * 8) = pack_bf16x8(o);
        }
    }
    return;
  }
  const float ip = inv_rms(warp_row_sumsq(pr, a.Ht, lane), a.Ht, a.eps);
  const float is = inv_rms(warp_row_sumsq(sr, a.Ht, lane), a.Ht, a.eps);
  __nv_bfloat16* o = a.out + (long long)t * a.Ht;
  for (int c = lane; c < a.Ht; c += 32)
    o[c] = f2bf(mix_value(bf2f(pr[c]), bf2f(sr[c]), bf2f(a.state_norm_w[c]), bf2f(a.noise_norm_w[c]), ip, is,
                          a.gate));
}

// One CTA (NF_THREADS) per token: the variance-weighted sum of squares of its
// noise row (each thread 8 consecutive entries per step, then the warps' xor
// trees and the warps in order), then the scaled projection added to the
// uniform posterior's embedded row, 8 features per thread per step.
constexpr int NF_THREADS = 256;
__global__ void __launch_bounds__(NF_THREADS) noise_fold_kernel(NoiseFoldArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[NF_THREADS / 32];
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const __nv_bfloat16* zr = a.z + (long long)t * a.Ht;
  const __nv_bfloat16* pr = a.proj + (long long)t * a.D;
  __nv_bfloat16* orow = a.out + (long long)t * a.D;
  float acc = 0.0f;
  if (a.Ht % 8 == 0 && vec_ok(zr) && vec_ok(a.var)) {
    for (int c = threadIdx.x * 8; c < a.Ht; c += NF_THREADS * 8) {
      float zf[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(zr + c), zf);
      const float4 v0 = *reinterpret_cast<const float4*>(a.var + c);
      const float4 v1 = *reinterpret_cast<const float4*>(a.var + c + 4);
      const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(zf[e], zf[e]), vv[e]));
    }
  } else {
    for (int c = threadIdx.x; c < a.Ht; c += NF_THREADS) {
      const float zf = bf2f(zr[c]);
      acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(zf, zf), a.var[c]));
    }
  }
  acc = warp_allsum(acc);
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  float ms = 0.0f;
#pragma unroll
  for (int w = 0; w < NF_THREADS / 32; ++w) ms = __fadd_rn(ms, red[w]);
  const float scale = __fmul_rn(a.gate, __frsqrt_rn(__fadd_rn(ms, a.eps)));
  if (a.D % 8 == 0 && vec_ok(pr) && vec_ok(a.x0) && vec_ok(orow)) {
    for (int d = threadIdx.x * 8; d < a.D; d += NF_THREADS * 8) {
      float pf[8], xf[8], o[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(pr + d), pf);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(a.x0 + d), xf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __fadd_rn(xf[e], round_bf(__fmul_rn(scale, pf[e])));
      *reinterpret_cast<uint4*>(orow + d) = pack_bf16x8(o);
    }
  } else {
    for (int d = threadIdx.x; d < a.D; d += NF_THREADS)
      orow[d] = f2bf(__fadd_rn(bf2f(a.x0[d]), round_bf(__fmul_rn(scale, bf2f(pr[d])))));
  }
}

__global__ void philox_normal_bf16_kernel(__nv_bfloat16* out, long long count, uint64_t seed, uint32_t offset,
                                          const uint32_t* offset_ptr) {
  pdl_wait();
  pdl_launch_dependents();
  if (offset_ptr) offset += *offset_ptr;
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * p >= count) return;
  float z0, z1;
  normal_pair(seed, offset, p, z0, z1);
  out[2 * p] = f2bf(z0);
  if (2 * p + 1 < count) out[2 * p + 1] = f2bf(z1);
}

__global__ void philox_normal_f32_kernel(float* out, long long count, uint64_t seed, uint32_t offset,
                                         const uint32_t* offset_ptr) {
  pdl_wait();
  pdl_launch_dependents();
  if (offset_ptr) offset += *offset_ptr;
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * p >= count) return;
  float z0, z1;
  normal_pair(seed, offset, p, z0, z1);
  out[2 * p] = z0;
  if (2 * p + 1 < count) out[2 * p + 1] = z1;
}

// Row r of n_cols normals keyed by its request's seed and its position:
// seed = seeds[rows[r]] (0 when rows[r] < 0), counter offset = positions[r];
// pair p of the row uses counter (p, 0, offset, 4) like philox_normal.
__device__ __forceinline__ void put_val(__nv_bfloat16* p, float v) { *p = f2bf(v); }
__device__ __forceinline__ void put_val(float* p, float v) { *p = v; }

template <typename OutT>
__global__ void philox_normal_rows_kernel(OutT* out, long long n_rows, long long n_cols, const long long* seeds,
                                          const long long* rows, const long long* positions, float scale) {
  const long long half = (n_cols + 1) / 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_rows * half) return;
  const long long r = idx / half, p = idx - r * half;
  const long long st = rows[r];
  const uint64_t seed = st >= 0 ? (uint64_t)seeds[st] : 0ull;
  float z0, z1;
  normal_pair(seed, (uint32_t)positions[r], p, z0, z1);
  OutT* o = out + r * n_cols;
  put_val(o + 2 * p, __fmul_rn(z0, scale));
  if (2 * p + 1 < n_cols) put_val(o + 2 * p + 1, __fmul_rn(z1, scale));
}

__global__ void argmax_tokens_kernel(const unsigned long long* keys, int64_t* tokens, int n) {
  pdl_wait();
  pdl_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) tokens[i] = (int64_t)argmax_key_index(keys[i]);
}

// rows of the multi-step featurisation GEMM input
// The multi-jump state rows (modeling_flashmap.py:378-391): per token the bf16
// copy of the fp32 state and, with the posterior, softmax(c * state) in bf16.
// Rows are read as 16-byte vectors of 8 (four in flight per thread), the
// exponentials two at a time (fm_exp2); scalar loops serve unaligned rows.
__global__ void __launch_bounds__(RT) state_rows_kernel(const float* state, __nv_bfloat16* out, int T, int S,
                                                        float c, int with_posterior) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[16];
  const int t = blockIdx.x;
  const float* sr = state + (long long)t * S;
  __nv_bfloat16* st_out = out + (long long)(with_posterior ? T + t : t) * S;
  __nv_bfloat16* po = out + (long long)t * S;
  const bool vec = S % 8 == 0 && vec_ok(sr) && vec_ok(st_out) && vec_ok(po);
  const int nvec = S / 8;
  float m = -INFINITY;
  if (vec) {
    for (int v0 = threadIdx.x; v0 < nvec; v0 += 4 * RT) {
      float x[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v0 + u * RT < nvec) load8(sr, v0 + u * RT, S, true, x[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + u * RT;
        if (v >= nvec) break;
        *reinterpret_cast<uint4*>(st_out + (long long)v * 8) = pack_bf16x8(x[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) m = fmaxf(m, __fmul_rn(x[u][e], c));
      }
    }
  } else {
    for (int v = threadIdx.x; v < S; v += RT) {
      st_out[v] = f2bf(sr[v]);
      m = fmaxf(m, __fmul_rn(sr[v], c));
    }
  }
  if (!with_posterior) return;
  m = block_max(m, red);
  const float2 neg_m = make_float2(-m, -m), c2 = make_float2(c, c);
  float acc = 0.0f;
  if (vec) {
    for (int v0 = threadIdx.x; v0 < nvec; v0 += 4 * RT) {
      float x[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v0 + u * RT < nvec) load8(sr, v0 + u * RT, S, true, x[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (v0 + u * RT >= nvec) break;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 e = fm_exp2(__fadd2_rn(__fmul2_rn(make_float2(x[u][2 * i], x[u][2 * i + 1]), c2), neg_m));
          acc = __fadd_rn(__fadd_rn(acc, e.x), e.y);
        }
      }
    }
  } else {
    for (int v = threadIdx.x; v < S; v += RT) acc = __fadd_rn(acc, fm_exp(__fsub_rn(__fmul_rn(sr[v], c), m)));
  }
  const float sum = block_sum(acc, red);
  if (vec) {
    for (int v0 = threadIdx.x; v0 < nvec; v0 += 4 * RT) {
      float x[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v0 + u * RT < nvec) load8(sr, v0 + u * RT, S, true, x[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + u * RT;
        if (v >= nvec) break;
        float o[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 e = fm_exp2(__fadd2_rn(__fmul2_rn(make_float2(x[u][2 * i], x[u][2 * i + 1]), c2), neg_m));
          o[2 * i] = __fdiv_rn(e.x, sum);
          o[2 * i + 1] = __fdiv_rn(e.y, sum);
        }
        *reinterpret_cast<uint4*>(po + (long long)v * 8) = pack_bf16x8(o);
      }
    }
    return;
  }
  for (int v = threadIdx.x; v < S; v += RT)
    po[v] = f2bf(__fdiv_rn(fm_exp(__fsub_rn(__fmul_rn(sr[v], c), m)), sum));
}

// state = (a * state + b * softmax(logits row)) / d per token, the softmax's
// maximum and sum from vector passes (row_sumexp), the update from 16-byte
// vectors of logits and state
__global__ void __launch_bounds__(RT) state_update_kernel(float* state, const __nv_bfloat16* logits, long long ldl,
                                                          int S, float a, float b, float d) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[16];
  const int t = blockIdx.x;
  const __nv_bfloat16* lr = logits + (long long)t * ldl;
  float* sr = state + (long long)t * S;
  const bool vec = S % 8 == 0 && vec_ok(lr) && vec_ok(sr);
  const int nvec = S / 8;
  float m = -INFINITY;
  if (vec) {
    for (int v0 = threadIdx.x; v0 < nvec; v0 += 4 * RT) {
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        raw[u] = v0 + u * RT < nvec ? *reinterpret_cast<const uint4*>(lr + (long long)(v0 + u * RT) * 8)
                                    : make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
      __nv_bfloat162 m2 = __halves2bfloat162(__ushort_as_bfloat16(0xff80), __ushort_as_bfloat16(0xff80));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) m2 = __hmax2(m2, *reinterpret_cast<const __nv_bfloat162*>(&w[k]));
      }
      m = fmaxf(m, fmaxf(__low2float(m2), __high2float(m2)));
    }
  } else {
    for (int v = threadIdx.x; v < S; v += RT) m = fmaxf(m, bf2f(lr[v]));
  }
  m = block_max(m, red);
  const float sum = row_sumexp(lr, (long long)S, 1.0f, m, red);
  if (vec) {
    const float2 neg_m = make_float2(-m, -m);
    for (int v0 = threadIdx.x; v0 < nvec; v0 += 2 * RT) {
      uint4 raw[2];
      float4 st[2][2];
#pragma unroll
      for (int u = 0; u < 2; ++u)
        if (v0 + u * RT < nvec) {
          const long long v = v0 + u * RT;
          raw[u] = *reinterpret_cast<const uint4*>(lr + v * 8);
          st[u][0] = *reinterpret_cast<const float4*>(sr + v * 8);
          st[u][1] = *reinterpret_cast<const float4*>(sr + v * 8 + 4);
        }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const long long v = v0 + u * RT;
        if (v >= nvec) break;
        const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
        float sv[8] = {st[u][0].x, st[u][0].y, st[u][0].z, st[u][0].w, st[u][1].x, st[u][1].y, st[u][1].z, st[u][1].w};
        float o[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 x = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
          const float2 e = fm_exp2(__fadd2_rn(x, neg_m));
          const float p0 = __fdiv_rn(e.x, sum), p1 = __fdiv_rn(e.y, sum);
          o[2 * i] = __fdiv_rn(__fadd_rn(__fmul_rn(a, sv[2 * i]), __fmul_rn(b, p0)), d);
          o[2 * i + 1] = __fdiv_rn(__fadd_rn(__fmul_rn(a, sv[2 * i + 1]), __fmul_rn(b, p1)), d);
        }
        *reinterpret_cast<float4*>(sr + v * 8) = make_float4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<float4*>(sr + v * 8 + 4) = make_float4(o[4], o[5], o[6], o[7]);
      }
    }
    return;
  }
  for (int v = threadIdx.x; v < S; v += RT) {
    const float p = __fdiv_rn(fm_exp(__fsub_rn(bf2f(lr[v]), m)), sum);
    sr[v] = __fdiv_rn(__fadd_rn(__fmul_rn(a, sr[v]), __fmul_rn(b, p)), d);
  }
}

__global__ void extend_prep_kernel(ExtendPrepArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= a.rows) return;
  int lo = 0, hi = a.B;  // find b with cu[b] <= r < cu[b+1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) / 2;
    if (a.cu_rows[mid] <= r)
      lo = mid;
    else
      hi = mid;
  }
  const int pos = a.lengths[lo] + (r - a.cu_rows[lo]);
  if (pos < 0 || pos >= a.cache_len || pos >= a.rope_len) record_error(a.err, DEV_BAD_INDEX);
  a.token_seq[r] = lo;
  a.positions[r] = pos;
}

__global__ void extend_commit_kernel(const int32_t* cu, int32_t* lengths, int B) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) lengths[b] += cu[b + 1] - cu[b];
}

// ------------------------------------------------------------------ sampling / acceptance

// Row slices of the many-CTAs-per-row reductions: SLICE_VPT vectors of 8 per
// thread, loaded together.
constexpr int SLICE_VPT = 8;
constexpr long long SLICE_VECS = (long long)SLICE_VPT * RT;

template <typename T>
__global__ void __launch_bounds__(RT) row_stats_kernel(const T* logits, long long V, float temperature,
                                                       float* stats, int64_t* argmax) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[16];
  const T* row = logits + (long long)blockIdx.x * V;
  float m;
  long long am = 0;
  row_max_argmax(row, V, temperature, red, &m, &am);
  if (argmax && threadIdx.x == 0) argmax[blockIdx.x] = am;
  if (stats) {
    const float s = temperature > 0.0f ? row_sumexp(row, V, temperature, m, red) : 0.0f;
    if (threadIdx.x == 0) {
      stats[2 * blockIdx.x] = m;
      stats[2 * blockIdx.x + 1] = s;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(RT) softmax_rows_kernel(const T* logits, long long V, float temperature,
                                                          float* probs) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[16];
  const T* row = logits + (long long)blockIdx.x * V;
  float m;
  long long am;
  row_max_argmax(row, V, temperature, red, &m, &am);
  const float s = row_sumexp(row, V, temperature, m, red);
  float* pr = probs + (long long)blockIdx.x * V;
  for (long long v = threadIdx.x; v < V; v += RT)
    pr[v] = __fdiv_rn(fm_exp(__fsub_rn(__fdiv_rn(to_f(row[v]), temperature), m)), s);
}

__global__ void __launch_bounds__(RT) sample_rows_kernel(const float* probs, long long V, int K, uint64_t seed,
                                                         uint32_t offset, int64_t* tokens) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float sm[RT + 32];
  const int row = blockIdx.x, b = row / K, k = row % K;
  const float* pr = probs + (long long)row * V;
  const float u = philox_uniform(seed, (uint32_t)k, (uint32_t)b, offset, 3u);
  const bool aligned = (reinterpret_cast<uintptr_t>(pr) & 15) == 0;
  const long long pick = block_categorical([&](long long v) { return pr[v]; }, V, u, sm, [&](long long v0, float* w) {
    if (!aligned) return false;
    float x[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k) load8(pr, v0 / 8 + k, V, true, x[k]);
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) w[k * 8 + j] = x[k][j];
    return true;
  });
  if (threadIdx.x == 0) tokens[row] = pick;
}

// Argmax of target rows for greedy acceptance, with many CTAs per row: CTA
// (row, slice) reads SLICE_VECS vectors of 8 (eight 16-byte loads per thread
// issued together) and merges its best (value, first index) into the row's
// 64-bit key with atomicMax (argmax_key: larger value, then smaller index, so
// the merge is order-independent).  keys must be zero beforehand.

template <typename T>
__global__ void __launch_bounds__(RT) row_argmax_slice_kernel(const T* logits, long long V,
                                                              unsigned long long* keys) {
  pdl_wait();
  pdl_launch_dependents();
  const T* row = logits + (long long)blockIdx.x * V;
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const long long nvec = (V + 7) / 8;
  const long long v_begin = (long long)blockIdx.y * SLICE_VECS;
  if constexpr (sizeof(T) == 2) {
    if (aligned && V % 8 == 0) {
      // bf16 rows of whole vectors: the slice maximum by packed bf16x2 max, then
      // the first index holding it, searched only by the threads that hold it
      uint4 raw[SLICE_VPT];
#pragma unroll
      for (int u = 0; u < SLICE_VPT; ++u) {
        const long long vec = v_begin + u * RT + threadIdx.x;
        raw[u] = vec < nvec ? *reinterpret_cast<const uint4*>(row + vec * 8) : make_uint4(0xff80ff80u, 0xff80ff80u,
                                                                                         0xff80ff80u, 0xff80ff80u);
      }
      __nv_bfloat162 m2 = __halves2bfloat162(__ushort_as_bfloat16(0xff80), __ushort_as_bfloat16(0xff80));
#pragma unroll
      for (int u = 0; u < SLICE_VPT; ++u) {
        const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) m2 = __hmax2(m2, *reinterpret_cast<const __nv_bfloat162*>(&w[k]));
      }
      float mloc = fmaxf(__low2float(m2), __high2float(m2));
      float mb = mloc;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
      __shared__ float wm[RT / 32];
      __shared__ unsigned long long wk2[RT / 32];
      if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = mb;
      __syncthreads();
      float M = wm[0];
#pragma unroll
      for (int w = 1; w < RT / 32; ++w) M = fmaxf(M, wm[w]);
      unsigned long long key = 0ull;
      if (mloc == M) {
        for (int u = 0; u < SLICE_VPT && key == 0ull; ++u) {
          const long long vec = v_begin + u * RT + threadIdx.x;
          if (vec >= nvec) break;
          const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
          for (int j = 0; j < 8; ++j) {
            const uint32_t bits = j & 1 ? (w[j >> 1] & 0xffff0000u) : (w[j >> 1] << 16);
            if (__uint_as_float(bits) == M) {
              key = argmax_key(M, (uint32_t)(vec * 8 + j));
              break;
            }
          }
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if ((threadIdx.x & 31) == 0) wk2[threadIdx.x >> 5] = key;
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 0; w < RT / 32; ++w) key = wk2[w] > key ? wk2[w] : key;
        if (key) atomicMax(keys + blockIdx.x, key);
      }
      return;
    }
  }
  float x[SLICE_VPT][8];
#pragma unroll
  for (int u = 0; u < SLICE_VPT; ++u) {
    const long long vec = v_begin + u * RT + threadIdx.x;
    if (vec < nvec) load8(row, vec, V, aligned, x[u]);
  }
  float bv = -INFINITY;
  long long bi = -1;
#pragma unroll
  for (int u = 0; u < SLICE_VPT; ++u) {
    const long long vec = v_begin + u * RT + threadIdx.x;
    if (vec >= nvec) break;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const long long v = vec * 8 + j;
      if (v >= V) break;
      if (bi < 0 || x[u][j] > bv) {  // indices rise within the thread: the first of a tie stays
        bv = x[u][j];
        bi = v;
      }
    }
  }
  unsigned long long key = bi >= 0 ? argmax_key(bv, (uint32_t)bi) : 0ull;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
    key = other > key ? other : key;
  }
  __shared__ unsigned long long wk[RT / 32];
  if ((threadIdx.x & 31) == 0) wk[threadIdx.x >> 5] = key;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < RT / 32; ++w) key = wk[w] > key ? wk[w] : key;
    key = wk[0] > key ? wk[0] : key;
    if (key) atomicMax(keys + blockIdx.x, key);
  }
}

__global__ void accept_greedy_keys_kernel(const int64_t* draft, const unsigned long long* keys, int K,
                                          int64_t* accepted, int64_t* bonus) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;  // one thread per sequence
  const unsigned long long* kr = keys + (long long)b * (K + 1);
  int acc = 0;
  while (acc < K && draft[(long long)b * K + acc] == (int64_t)argmax_key_index(kr[acc])) ++acc;
  accepted[b] = acc;
  bonus[b] = (int64_t)argmax_key_index(kr[acc]);
}

// ---------------------------------------------------------------- rejection acceptance
// The tests and the rows' statistics (reject_*_kernel below), then the
// residual's slice totals over (request, slice) blocks (residual_slices_kernel)
// and the bonus draw (residual_pick_kernel).  The bonus is a sliced
// categorical draw: slices of CAT_SLICE = 256 ranges of CAT_RANGE weights;
// per slice the ranges' sequential sums and a block inclusive scan give its
// total; the totals are summed in slice order, the slice holding u * total is
// rescanned and its range searched in index order (the C oracle's
// fmo_categorical_sliced).
constexpr int CAT_RANGE = 32;
constexpr long long CAT_SLICE = (long long)RT * CAT_RANGE;
constexpr int CAT_MAX_SLICES = 256;

template <typename T>
struct RejectionRow {
  const T* tr;        // target row of the first rejected slot (or row K)
  const float* qr;    // the draft's probabilities of that slot (unused when all were accepted)
  float m, s, temperature;
  bool residual;      // max(0, p - q) (else the target's p)
  bool vec;           // rows 16-byte aligned
  bool unit_t;        // T == 1: x / T == x exactly, the division is skipped
  __device__ float scaled(float x) const { return unit_t ? x : __fdiv_rn(x, temperature); }
  __device__ float p(long long v) const { return __fdiv_rn(fm_exp(__fsub_rn(scaled(to_f(tr[v])), m)), s); }
  __device__ float weight(long long v) const {
    const float pv = p(v);
    if (!residual) return pv;
    const float d = __fsub_rn(pv, qr[v]);
    return d > 0.0f ? d : 0.0f;
  }
  // 32 weights of v0 .. v0 + 31 (all < V) from 16-byte loads issued together
  __device__ bool bulk(long long v0, long long V, float* w) const {
    if (!vec) return false;
    Raw8<T> x[4];
    float qv[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[k].load(tr, v0 / 8 + k, V, true);
      if (residual) load8(qr, v0 / 8 + k, V, true, qv[k]);
    }
    const float2 neg_m = make_float2(-m, -m);  // x - m == x + (-m) exactly
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float2 xp = x[k].pair(j / 2);
        const float2 e = fm_exp2(__fadd2_rn(make_float2(scaled(xp.x), scaled(xp.y)), neg_m));
        const float pv[2] = {__fdiv_rn(e.x, s), __fdiv_rn(e.y, s)};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!residual) {
            w[k * 8 + j + h] = pv[h];
          } else {
            const float d = __fsub_rn(pv[h], qv[k][j + h]);
            w[k * 8 + j + h] = d > 0.0f ? d : 0.0f;
          }
        }
      }
    return true;
  }
};

template <typename T>
__device__ RejectionRow<T> rejection_row(const T* target, const float* q, const float* stats, long long V, int K,
                                         float temperature, int b, int acc) {
  RejectionRow<T> r;
  const long long row = (long long)b * (K + 1) + acc;
  r.tr = target + row * V;
  r.qr = q + ((long long)b * K + (acc < K ? acc : 0)) * V;
  r.m = stats[2 * row];
  r.s = stats[2 * row + 1];
  r.temperature = temperature;
  r.residual = acc < K;
  r.vec = (reinterpret_cast<uintptr_t>(r.tr) & 15) == 0 && (reinterpret_cast<uintptr_t>(r.qr) & 15) == 0;
  r.unit_t = temperature == 1.0f;
  return r;
}

// this thread's range sum t and the block's inclusive scan h over slice j
// (Hillis-Steele inside each warp, then the warp totals in order); sm holds
// >= 16 floats.  bulk tells whether bw holds the range's 32 weights.
template <typename T, bool TargetOnly>
__device__ __forceinline__ void slice_scan(const RejectionRow<T>& w, long long V, long long j, float* sm, float& t,
                                           float& h, float (&bw)[CAT_RANGE], bool& bulk) {
  const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
  const long long lo = j * CAT_SLICE + (long long)i * CAT_RANGE, hi = min(lo + CAT_RANGE, V);
  RejectionRow<T> r = w;
  if (TargetOnly) r.residual = false;
  t = 0.0f;
  bulk = false;
  if (hi - lo == CAT_RANGE && r.bulk(lo, V, bw)) {
    bulk = true;
#pragma unroll
    for (int k = 0; k < 32; ++k) t = __fadd_rn(t, bw[k]);
  } else {
    for (long long v = lo; v < hi; ++v) t = __fadd_rn(t, r.weight(v));
  }
  h = t;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, h, off);
    if (lane >= off) h = __fadd_rn(y, h);
  }
  if (lane == 31) sm[warp] = h;
  __syncthreads();
  if (i == 0) {
    float base = 0.0f;
    for (int wp = 0; wp < RT / 32; ++wp) {
      const float tot = sm[wp];
      sm[8 + wp] = base;
      base = (wp == 0) ? tot : __fadd_rn(base, tot);
    }
  }
  __syncthreads();
  if (warp > 0) h = __fadd_rn(sm[8 + warp], h);
  __syncthreads();
}

// Row statistics of the rejection step.  The exact sum S = sum_v fm_exp(x_v / T - m)
// runs in a fixed slice-major order: slices of REJ_SLICE_VECS vectors of 8
// (CAT_SLICE elements); in a slice, thread i sums its REJ_VPT vectors (slice
// start + u * RT + i, u ascending) element by element, the slice total is
// block_sum's tree, and the slice totals are added in slice order (the C
// oracle's row_sumexp_sliced).  fm_exp costs ~18 instructions per element, so
// the exact sum is formed only for the rows whose outcome needs it:
//   1. reject_scan_kernel, CTA (row, chunk of 16384): the chunk's raw maximum
//      (exact) and an approximate sum of 2^((x - max) log2(e) / T) by a
//      polynomial exp2_poly2 (relative error under 5e-6), in one read;
//   2. reject_decide_kernel, one warp per request: each row's m (exact) and
//      approximate S'; a test u q < p is settled from p' = e / S' when u q lies
//      outside p' (1 -+ 2^-10), since S' and S differ by far less (fm_exp's
//      1-ulp error, exp2_poly2's 5e-6 per term and per chunk merge, a few
//      hundred rounded additions of positive terms); otherwise it stays open.  Listed
//      for the exact sum: the open tests before the first settled rejection,
//      then the bonus row (that rejection, or row K);
//   3. reject_exact_kernel, CTA (request, slice): the listed rows' exact slice totals;
//   4. reject_final_kernel, one warp per request: the open tests decided with
//      the exact sums, the accepted length, the bonus row's exact S.
constexpr int REJ_VPT = 4;
constexpr long long REJ_SLICE_VECS = (long long)REJ_VPT * RT;
static_assert(REJ_SLICE_VECS * 8 == CAT_SLICE, "one slicing for the sums and the bonus draw");
constexpr float REJ_MARGIN = 9.765625e-4f;  // 2^-10

// 2^y of two lanes, y <= 0, for the approximate sums: y clamped at -125 (a
// term below 2^-124 is invisible in a sum whose largest term is 1), n = rint(y)
// by the 1.5 * 2^23 shifter, f = y - n in [-1/2, 1/2], 2^f by the degree-5
// Taylor polynomial of e^(f ln 2) (remainder below (ln2 / 2)^6 / 720 * 2^(1/2)
// = 3.4e-6 of 2^f >= 2^(-1/2): relative error under 5e-6), 2^n from n's bits
// as in fm_exp2.  Packed fp32x2 arithmetic throughout.
__device__ __forceinline__ float2 exp2_poly2(float2 y) {
  y = make_float2(fmaxf(y.x, -125.0f), fmaxf(y.y, -125.0f));
  const float2 t = __fadd2_rn(y, make_float2(12582912.0f, 12582912.0f));
  const float2 n = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), y);
  float2 p = __ffma2_rn(make_float2(1.3333558e-3f, 1.3333558e-3f), f, make_float2(9.6181291e-3f, 9.6181291e-3f));
  p = __ffma2_rn(p, f, make_float2(5.5504109e-2f, 5.5504109e-2f));
  p = __ffma2_rn(p, f, make_float2(2.4022651e-1f, 2.4022651e-1f));
  p = __ffma2_rn(p, f, make_float2(6.9314718e-1f, 6.9314718e-1f));
  p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
  const uint32_t b0 = __float_as_uint(t.x), b1 = __float_as_uint(t.y);
  return __fmul2_rn(p, make_float2(__uint_as_float((b0 << 23) + 0x3F800000u), __uint_as_float((b1 << 23) + 0x3F800000u)));
}

// Scan chunks of REJ_SCAN_VECS vectors (16384 elements): each thread's 8
// vectors in registers, its own maximum and its sum relative to it, then one
// block merge of the (max, sum) pairs -> (chunk max, approximate chunk sum).
constexpr int REJ_SCAN_VPT = 8;
constexpr long long REJ_SCAN_VECS = (long long)REJ_SCAN_VPT * RT;

template <typename T>
__global__ void __launch_bounds__(RT) reject_scan_kernel(const T* logits, long long V, float c, int C,
                                                         float2* chunk_stats) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[16];
  const T* row = logits + (long long)blockIdx.x * V;
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const long long nvec = (V + 7) / 8, nfull = V / 8;
  const long long v0 = (long long)blockIdx.y * REJ_SCAN_VECS + threadIdx.x;
  Raw8<T> x[REJ_SCAN_VPT];
#pragma unroll
  for (int u = 0; u < REJ_SCAN_VPT; ++u)
    if (v0 + u * RT < nvec) x[u].load(row, v0 + u * RT, V, aligned);
  float mt = -INFINITY;
#pragma unroll
  for (int u = 0; u < REJ_SCAN_VPT; ++u) {
    const long long vec = v0 + u * RT;
    if (vec >= nvec) break;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 p = x[u].pair(i);
      const bool full = vec < nfull;
      if (full || vec * 8 + 2 * i < V) mt = fmaxf(mt, p.x);
      if (full || vec * 8 + 2 * i + 1 < V) mt = fmaxf(mt, p.y);
    }
  }
  float st = 0.0f;
  if (mt > -INFINITY && mt < INFINITY) {
    const float off = -mt * c;
    const float2 c2 = make_float2(c, c), off2 = make_float2(off, off);
    float2 acc2 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int u = 0; u < REJ_SCAN_VPT; ++u) {
      const long long vec = v0 + u * RT;
      if (vec >= nvec) break;
      if (vec < nfull) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc2 = __fadd2_rn(acc2, exp2_poly2(__ffma2_rn(x[u].pair(i), c2, off2)));
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 e = exp2_poly2(__ffma2_rn(x[u].pair(i), c2, off2));
          if (vec * 8 + 2 * i < V) acc2.x += e.x;
          if (vec * 8 + 2 * i + 1 < V) acc2.y += e.y;
        }
      }
    }
    st = acc2.x + acc2.y;
  }
  const float M = block_max(mt, red);
  const float scaled = (st > 0.0f && M < INFINITY) ? st * exp2_poly2(make_float2((mt - M) * c, 0.0f)).x : 0.0f;
  const float S = block_sum(scaled, red);
  if (threadIdx.x == 0) chunk_stats[(long long)blockIdx.x * C + blockIdx.y] = make_float2(M, S);
}

// list[b * (K + 1) + i], i < nlist[b]: rows of request b in ascending order;
// the last is the bonus candidate, the others open tests
template <typename T>
__global__ void __launch_bounds__(32) reject_decide_kernel(const T* target, const int64_t* draft, const float* q,
                                                           long long V, int K, float temperature, float c,
                                                           uint64_t seed, uint32_t offset, int C,
                                                           const float2* chunk_stats, float* stats, int* list,
                                                           int* nlist) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int state[];  // K entries: 0 accept, 1 reject, 2 open
  const int b = blockIdx.x, lane = threadIdx.x;
  const bool unit_t = temperature == 1.0f;
  for (int k = lane; k <= K; k += 32) {
    const long long row = (long long)b * (K + 1) + k;
    const float2* ss = chunk_stats + row * C;
    float M = -INFINITY;
    for (int j = 0; j < C; ++j) M = fmaxf(M, ss[j].x);
    // max of x / T is the rounded quotient of the raw max (division by T > 0 keeps order)
    const float m = unit_t ? M : __fdiv_rn(M, temperature);
    stats[2 * row] = m;
    if (k == K) break;
    int st = 2;
    if (M > -INFINITY && M < INFINITY) {
      float sa = 0.0f;
      for (int j = 0; j < C; ++j)
        if (ss[j].y > 0.0f) sa += ss[j].y * exp2_poly2(make_float2((ss[j].x - M) * c, 0.0f)).x;
      const long long d = draft[(long long)b * K + k];
      const float xd = to_f(target[row * V + d]);
      const float e = fm_exp(__fsub_rn(unit_t ? xd : __fdiv_rn(xd, temperature), m));
      const float pa = __fdiv_rn(e, sa);
      const float qd = q[((long long)b * K + k) * V + d];
      const float u = philox_uniform(seed, (uint32_t)k, (uint32_t)b, offset, 1u);
      const float uq = __fmul_rn(u, qd);
      if (uq < __fmul_rn(pa, 1.0f - REJ_MARGIN))
        st = 0;
      else if (uq >= __fmul_rn(pa, 1.0f + REJ_MARGIN))
        st = 1;
    }
    state[k] = st;
  }
  __syncwarp();
  if (lane == 0) {
    int* lst = list + (long long)b * (K + 1);
    int n = 0, j = 0;
    for (; j < K && state[j] != 1; ++j)
      if (state[j] == 2) lst[n++] = j;
    lst[n++] = j;
    nlist[b] = n;
  }
}

template <typename T, bool UNIT_T>
__device__ __forceinline__ float reject_exact_slice(const T* row, long long V, float temperature, float m,
                                                    long long s, float* red) {
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const long long nvec = (V + 7) / 8, nfull = V / 8;
  const long long v0 = s * REJ_SLICE_VECS + threadIdx.x;
  const float2 neg_m = make_float2(-m, -m);  // x - m == x + (-m) exactly
  Raw8<T> x[REJ_VPT];
#pragma unroll
  for (int u = 0; u < REJ_VPT; ++u)
    if (v0 + u * RT < nvec) x[u].load(row, v0 + u * RT, V, aligned);
  float acc = 0.0f;
#pragma unroll
  for (int u = 0; u < REJ_VPT; ++u) {
    const long long vec = v0 + u * RT;
    if (vec >= nvec) break;
    if (vec < nfull) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 xt = x[u].pair(i);
        if (!UNIT_T) xt = make_float2(__fdiv_rn(xt.x, temperature), __fdiv_rn(xt.y, temperature));
        const float2 e = fm_exp2(__fadd2_rn(xt, neg_m));
        acc = __fadd_rn(acc, e.x);
        acc = __fadd_rn(acc, e.y);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 xp = x[u].pair(i);
        if (vec * 8 + 2 * i < V)
          acc = __fadd_rn(acc, fm_exp(__fsub_rn(UNIT_T ? xp.x : __fdiv_rn(xp.x, temperature), m)));
        if (vec * 8 + 2 * i + 1 < V)
          acc = __fadd_rn(acc, fm_exp(__fsub_rn(UNIT_T ? xp.y : __fdiv_rn(xp.y, temperature), m)));
      }
    }
  }
  return block_sum(acc, red);
}

// CTA (b, s): slice s of each listed row of request b -> exact[b * (K + 1) + i][s]
template <typename T>
__global__ void __launch_bounds__(RT, 5) reject_exact_kernel(const T* target, long long V, int K, float temperature,
                                                             int S, const float* stats, const int* list,
                                                             const int* nlist, float* exact) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[16];
  const int b = blockIdx.x;
  const long long s = blockIdx.y;
  const int n = nlist[b];
  for (int i = 0; i < n; ++i) {
    const long long row = (long long)b * (K + 1) + list[(long long)b * (K + 1) + i];
    const float m = stats[2 * row];
    const float t = temperature == 1.0f
                        ? reject_exact_slice<T, true>(target + row * V, V, temperature, m, s, red)
                        : reject_exact_slice<T, false>(target + row * V, V, temperature, m, s, red);
    if (threadIdx.x == 0) exact[((long long)b * (K + 1) + i) * S + s] = t;
  }
}

template <typename T>
__global__ void __launch_bounds__(32) reject_final_kernel(const T* target, const int64_t* draft, const float* q,
                                                          long long V, int K, float temperature, uint64_t seed,
                                                          uint32_t offset, int S, const int* list, const int* nlist,
                                                          const float* exact, float* stats, int64_t* accepted) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x != 0) return;
  const int b = blockIdx.x;
  const int n = nlist[b];
  const int* lst = list + (long long)b * (K + 1);
  const bool unit_t = temperature == 1.0f;
  int j = lst[n - 1];
  float sj = 0.0f;
  for (int i = 0; i < n; ++i) {
    const int k = lst[i];
    const long long row = (long long)b * (K + 1) + k;
    const float* ex = exact + ((long long)b * (K + 1) + i) * S;
    float sum = 0.0f;
    for (int t = 0; t < S; ++t) sum = __fadd_rn(sum, ex[t]);
    if (i == n - 1) {
      sj = sum;
      break;
    }
    // an open test, decided with the exact sum as the C oracle decides it
    const float m = stats[2 * row];
    const long long d = draft[(long long)b * K + k];
    const float xd = to_f(target[row * V + d]);
    const float p = __fdiv_rn(fm_exp(__fsub_rn(unit_t ? xd : __fdiv_rn(xd, temperature), m)), sum);
    const float qd = q[((long long)b * K + k) * V + d];
    const float u = philox_uniform(seed, (uint32_t)k, (uint32_t)b, offset, 1u);
    if (!(__fmul_rn(u, qd) < p)) {
      j = k;
      sj = sum;
      break;
    }
  }
  stats[2 * ((long long)b * (K + 1) + j) + 1] = sj;
  accepted[b] = j;
}

// the residual's (or, all accepted, the target's) slice totals: block (b, j)
template <typename T>
__global__ void __launch_bounds__(RT) residual_slices_kernel(const T* target, const float* q, long long V, int K,
                                                             float temperature, const float* stats,
                                                             const int64_t* accepted, float* totals) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float sm[16];
  const int b = blockIdx.x;
  const long long j = blockIdx.y;
  const RejectionRow<T> w = rejection_row(target, q, stats, V, K, temperature, b, (int)accepted[b]);
  float t, h, bw[CAT_RANGE];
  bool bulk;
  slice_scan<T, false>(w, V, j, sm, t, h, bw, bulk);
  if (threadIdx.x == RT - 1) totals[(long long)b * CAT_MAX_SLICES + j] = h;
}

// the bonus: the slice totals in order, then the chosen slice and range; a
// residual with no positive weight draws from the target's distribution
template <typename T>
__global__ void __launch_bounds__(RT) residual_pick_kernel(const T* target, const float* q, long long V, int K,
                                                           float temperature, uint64_t seed, uint32_t offset,
                                                           const float* stats, const int64_t* accepted,
                                                           const float* totals, int64_t* bonus) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float sm[16];
  __shared__ float tot[CAT_MAX_SLICES], pre[CAT_MAX_SLICES];
  __shared__ float g[RT];
  __shared__ int s_choice;
  __shared__ float s_base, s_target;
  __shared__ int ired[RT / 32];
  const int b = blockIdx.x, i = threadIdx.x;
  const int S = (int)((V + CAT_SLICE - 1) / CAT_SLICE);
  RejectionRow<T> w = rejection_row(target, q, stats, V, K, temperature, b, (int)accepted[b]);
  for (int j = i; j < S; j += RT) tot[j] = totals[(long long)b * CAT_MAX_SLICES + j];
  __syncthreads();
  if (i == 0) {
    float run = 0.0f;
    for (int j = 0; j < S; ++j) {
      run = j == 0 ? tot[j] : __fadd_rn(run, tot[j]);
      pre[j] = run;
    }
  }
  __syncthreads();
  if (!(pre[S - 1] > 0.0f)) {
    // no positive residual weight: the target's distribution, its slice totals here
    w.residual = false;
    for (int j = 0; j < S; ++j) {
      float t, h, bw[CAT_RANGE];
      bool bulk;
      slice_scan<T, true>(w, V, j, sm, t, h, bw, bulk);
      if (i == RT - 1) tot[j] = h;
    }
    __syncthreads();
    if (i == 0) {
      float run = 0.0f;
      for (int j = 0; j < S; ++j) {
        run = j == 0 ? tot[j] : __fadd_rn(run, tot[j]);
        pre[j] = run;
      }
    }
    __syncthreads();
  }
  if (i == 0) {
    const float target_u = __fmul_rn(philox_uniform(seed, 0u, (uint32_t)b, offset, 2u), pre[S - 1]);
    int js = -1;
    for (int j = 0; j < S; ++j)
      if (pre[j] > target_u) {
        js = j;
        break;
      }
    if (js < 0)
      for (int j = S - 1; j >= 0; --j)
        if (tot[j] > 0.0f) {
          js = j;
          break;
        }
    s_choice = js;
    s_base = js > 0 ? pre[js - 1] : 0.0f;
    s_target = target_u;
  }
  __syncthreads();
  const int js = s_choice;
  if (js < 0) {  // every weight zero
    if (i == 0) bonus[b] = 0;
    return;
  }
  float t, h, bw[CAT_RANGE];
  bool bulk;
  if (w.residual)
    slice_scan<T, false>(w, V, js, sm, t, h, bw, bulk);
  else
    slice_scan<T, true>(w, V, js, sm, t, h, bw, bulk);
  g[i] = __fadd_rn(s_base, h);
  const float target_u = s_target;
  const int first = block_min_int(g[i] > target_u ? i : RT, ired);
  const int lastpos = block_max_int(t > 0.0f ? i : -1, ired);
  const int chosen = first < RT ? first : lastpos;
  if (chosen < 0) {
    if (i == 0) bonus[b] = js * CAT_SLICE;
    return;
  }
  // the chosen range's own thread searches it in index order (its weights
  // are still in registers when the range was loaded in bulk)
  if (i != chosen) return;
  float run = chosen > 0 ? g[chosen - 1] : s_base;
  const long long lo = js * CAT_SLICE + (long long)chosen * CAT_RANGE, hi = min(lo + CAT_RANGE, V);
  long long last = -1, pick = -1;
  if (bulk) {
#pragma unroll
    for (int k = 0; k < CAT_RANGE; ++k)
      if (pick < 0) {
        run = __fadd_rn(run, bw[k]);
        if (bw[k] > 0.0f) last = lo + k;
        if (run > target_u) pick = lo + k;
      }
  } else {
    for (long long v = lo; v < hi; ++v) {
      const float wv = w.weight(v);
      run = __fadd_rn(run, wv);
      if (wv > 0.0f) last = v;
      if (run > target_u) {
        pick = v;
        break;
      }
    }
  }
  bonus[b] = pick >= 0 ? pick : (last >= 0 ? last : lo);
}

__global__ void transpose_bf16_kernel(const __nv_bfloat16* in, __nv_bfloat16* out, long long R, long long C) {
  __shared__ __nv_bfloat16 tile[32][33];
  const long long r0 = (long long)blockIdx.y * 32, c0 = (long long)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const long long r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = in[r * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const long long c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) out[c * R + r] = tile[threadIdx.x][i];
  }
}

__global__ void time_sinusoid_kernel(__nv_bfloat16* out, int dim, float s, float t, float scale, const float* freqs) {
  const int half = dim / 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= 2 * half) return;
  const int row = idx / half, i = idx % half;
  // modeling_flashmap.py:95-96 in fp32: (t * scale) * freq
  const float arg = __fmul_rn(__fmul_rn(row == 0 ? s : t, scale), freqs[i]);
  out[row * dim + i] = f2bf(cosf(arg));
  out[row * dim + half + i] = f2bf(sinf(arg));
}

__global__ void silu_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = bf2f(x[i]);
  y[i] = f2bf(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))));
}

__global__ void add_kernel(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* y, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = f2bf(__fadd_rn(bf2f(a[i]), bf2f(b[i])));
}

inline unsigned blocks_for(long long n, int per) { return (unsigned)((n + per - 1) / per); }

}  // namespace

// ------------------------------------------------------------------ launchers
fm_status launch_rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int64_t rows,
                         int64_t cols, float eps, cudaStream_t s, bool pdl) {
  return launch_kernel(rmsnorm_kernel, dim3(blocks_for(rows, ROWS_PER_CTA)), dim3(RT), 0, s, pdl, x, w, y,
                       (long long)rows, (int)cols, eps);
}
fm_status launch_adaln(const __nv_bfloat16* x, const __nv_bfloat16* mod, __nv_bfloat16* y, int64_t rows,
                       int64_t cols, float eps, cudaStream_t s, bool pdl) {
  return launch_kernel(adaln_kernel, dim3(blocks_for(rows, ROWS_PER_CTA)), dim3(RT), 0, s, pdl, x, mod, y,
                       (long long)rows, (int)cols, eps);
}
fm_status launch_draft_prep(const DraftPrepArgs& a, cudaStream_t s, bool pdl) {
  return launch_kernel(draft_prep_kernel, dim3(a.B), dim3(RT), 0, s, pdl, a);
}

fm_status launch_rope_gather(const int* positions, int T, const float* rope_cos, const float* rope_sin, int rope_len,
                             int half, float* tok_cos, float* tok_sin, int* err, cudaStream_t s) {
  const long long n = (long long)T * half;
  if (n == 0) return FM_OK;
  return launch_kernel(rope_gather_kernel, dim3((unsigned)((n + RT - 1) / RT)), dim3(RT), 0, s, false, positions, T,
                       rope_cos, rope_sin, rope_len, half, tok_cos, tok_sin, err);
}
fm_status launch_mix_state(const MixArgs& a, cudaStream_t s, bool pdl) {
  return launch_kernel(mix_state_kernel, dim3(blocks_for(a.T, ROWS_PER_CTA)), dim3(RT), 0, s, pdl, a);
}
fm_status launch_noise_fold(const NoiseFoldArgs& a, cudaStream_t s, bool pdl) {
  return launch_kernel(noise_fold_kernel, dim3(a.T), dim3(NF_THREADS), 0, s, pdl, a);
}
fm_status launch_philox_normal_bf16(__nv_bfloat16* out, long long count, uint64_t seed, uint32_t offset,
                                    const uint32_t* offset_ptr, cudaStream_t s, bool pdl) {
  return launch_kernel(philox_normal_bf16_kernel, dim3(blocks_for((count + 1) / 2, 256)), dim3(256), 0, s, pdl,
                       out, count, seed, offset, offset_ptr);
}
fm_status launch_philox_normal_f32(float* out, long long count, uint64_t seed, uint32_t offset,
                                   const uint32_t* offset_ptr, cudaStream_t s, bool pdl) {
  return launch_kernel(philox_normal_f32_kernel, dim3(blocks_for((count + 1) / 2, 256)), dim3(256), 0, s, pdl, out,
                       count, seed, offset, offset_ptr);
}
fm_status launch_argmax_tokens(const unsigned long long* keys, int64_t* tokens, int n, cudaStream_t s, bool pdl) {
  return launch_kernel(argmax_tokens_kernel, dim3(blocks_for(n, 128)), dim3(128), 0, s, pdl, keys, tokens, n);
}
fm_status launch_state_rows(const float* state, __nv_bfloat16* out, int T, int S, float c, int with_posterior,
                            cudaStream_t s, bool pdl) {
  return launch_kernel(state_rows_kernel, dim3(T), dim3(RT), 0, s, pdl, state, out, T, S, c, with_posterior);
}
fm_status launch_state_update(float* state, const __nv_bfloat16* logits, long long ldl, int T, int S, float a,
                              float b, float d, cudaStream_t s, bool pdl) {
  return launch_kernel(state_update_kernel, dim3(T), dim3(RT), 0, s, pdl, state, logits, ldl, S, a, b, d);
}
fm_status launch_extend_prep(const ExtendPrepArgs& a, cudaStream_t s, bool pdl) {
  return launch_kernel(extend_prep_kernel, dim3(blocks_for(a.rows, 128)), dim3(128), 0, s, pdl, a);
}
fm_status launch_extend_commit(const int32_t* cu_rows, int32_t* lengths, int B, cudaStream_t s, bool pdl) {
  return launch_kernel(extend_commit_kernel, dim3(blocks_for(B, 128)), dim3(128), 0, s, pdl, cu_rows, lengths, B);
}

fm_status launch_self_attn(const SelfAttnArgs& a, int batch, cudaStream_t stream, bool pdl);
fm_status launch_cross_attn(const CrossAttnArgs& a, const CUtensorMap& tm, cudaStream_t stream, bool pdl);
size_t cross_attn_smem(int hd);

}  // namespace fm

// ====================================================================== C ABI
using namespace fm;

namespace {
cudaStream_t as_stream(fm_stream s) { return static_cast<cudaStream_t>(s); }
const __nv_bfloat16* cbf(const void* p) { return static_cast<const __nv_bfloat16*>(p); }
__nv_bfloat16* bf(void* p) { return static_cast<__nv_bfloat16*>(p); }
}  // namespace

extern "C" fm_status fm_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t cols, float eps,
                                fm_stream stream) {
  if (!x || !w || !y) return set_error(FM_ERR_INVALID, "rmsnorm: null pointer");
  if (rows <= 0 || cols <= 0) return set_error(FM_ERR_SHAPE, "rmsnorm: empty shape");
  return launch_rmsnorm(cbf(x), cbf(w), bf(y), rows, cols, eps, as_stream(stream), false);
}

extern "C" fm_status fm_adaln(const void* x, const void* mod, void* y, int64_t rows, int64_t cols, float eps,
                              fm_stream stream) {
  if (!x || !mod || !y) return set_error(FM_ERR_INVALID, "adaln: null pointer");
  if (rows <= 0 || cols <= 0) return set_error(FM_ERR_SHAPE, "adaln: empty shape");
  return launch_adaln(cbf(x), cbf(mod), bf(y), rows, cols, eps, as_stream(stream), false);
}

extern "C" fm_status fm_rope_table(float* cos_out, float* sin_out, int64_t max_pos, int64_t head_dim,
                                   const float* inv_freq, fm_stream stream) {
  if (!cos_out || !sin_out || !inv_freq) return set_error(FM_ERR_INVALID, "rope_table: null pointer");
  if (max_pos <= 0 || head_dim <= 0 || head_dim % 2) return set_error(FM_ERR_SHAPE, "rope_table: bad shape");
  const long long n = max_pos * (head_dim / 2);
  return launch_kernel(rope_table_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, as_stream(stream), false,
                       cos_out, sin_out, (int)max_pos, (int)head_dim, inv_freq);
}

extern "C" fm_status fm_philox_normal(void* out, int64_t count, uint64_t seed, uint32_t offset, fm_stream stream) {
  if (!out) return set_error(FM_ERR_INVALID, "philox_normal: null pointer");
  if (count <= 0) return FM_OK;
  return launch_philox_normal_bf16(bf(out), count, seed, offset, nullptr, as_stream(stream), false);
}

extern "C" fm_status fm_philox_normal_rows(void* out, int64_t n_rows, int64_t n_cols, const int64_t* seeds,
                                           const int64_t* rows, const int64_t* positions, float scale,
                                           fm_stream stream) {
  if (n_rows < 0 || n_cols < 0) return set_error(FM_ERR_SHAPE, "philox_normal_rows: bad shape");
  if (n_rows == 0 || n_cols == 0) return FM_OK;
  if (!out || !seeds || !rows || !positions) return set_error(FM_ERR_INVALID, "philox_normal_rows: null pointer");
  const long long pairs = n_rows * ((n_cols + 1) / 2);
  return launch_kernel(philox_normal_rows_kernel<__nv_bfloat16>, dim3(blocks_for(pairs, 256)), dim3(256), 0,
                       as_stream(stream), false, bf(out), (long long)n_rows, (long long)n_cols,
                       reinterpret_cast<const long long*>(seeds), reinterpret_cast<const long long*>(rows),
                       reinterpret_cast<const long long*>(positions), scale);
}

extern "C" fm_status fm_philox_normal_rows_f32(float* out, int64_t n_rows, int64_t n_cols, const int64_t* seeds,
                                               const int64_t* rows, const int64_t* positions, float scale,
                                               fm_stream stream) {
  if (n_rows < 0 || n_cols < 0) return set_error(FM_ERR_SHAPE, "philox_normal_rows_f32: bad shape");
  if (n_rows == 0 || n_cols == 0) return FM_OK;
  if (!out || !seeds || !rows || !positions) return set_error(FM_ERR_INVALID, "philox_normal_rows_f32: null pointer");
  const long long pairs = n_rows * ((n_cols + 1) / 2);
  return launch_kernel(philox_normal_rows_kernel<float>, dim3(blocks_for(pairs, 256)), dim3(256), 0,
                       as_stream(stream), false, out, (long long)n_rows, (long long)n_cols,
                       reinterpret_cast<const long long*>(seeds), reinterpret_cast<const long long*>(rows),
                       reinterpret_cast<const long long*>(positions), scale);
}

extern "C" fm_status fm_state_rows(const float* state, void* out, int64_t rows, int64_t cols, float evidence,
                                   int32_t with_posterior, fm_stream stream) {
  if (rows < 0 || cols < 1) return set_error(FM_ERR_SHAPE, "state_rows: bad shape");
  if (rows == 0) return FM_OK;
  if (!state || !out) return set_error(FM_ERR_INVALID, "state_rows: null pointer");
  if (rows > INT32_MAX || cols > INT32_MAX) return set_error(FM_ERR_SHAPE, "state_rows: dimension too large");
  return launch_state_rows(state, bf(out), (int)rows, (int)cols, evidence, with_posterior ? 1 : 0,
                           as_stream(stream), false);
}

extern "C" fm_status fm_state_update(float* state, const void* logits, int64_t ldl, int64_t rows, int64_t cols,
                                     float keep, float step, float denom, fm_stream stream) {
  if (rows < 0 || cols < 1 || ldl < cols) return set_error(FM_ERR_SHAPE, "state_update: bad shape");
  if (rows == 0) return FM_OK;
  if (!state || !logits) return set_error(FM_ERR_INVALID, "state_update: null pointer");
  if (rows > INT32_MAX || cols > INT32_MAX) return set_error(FM_ERR_SHAPE, "state_update: dimension too large");
  return launch_state_update(state, static_cast<const __nv_bfloat16*>(logits), ldl, (int)rows, (int)cols, keep, step,
                             denom, as_stream(stream), false);
}

extern "C" fm_status fm_mix_state(const void* post, int64_t post_stride, const void* state, const void* state_norm_w,
                                  const void* noise_norm_w, void* out, float gate, float eps, int64_t rows,
                                  int64_t cols, fm_stream stream) {
  if (rows < 0 || cols < 1) return set_error(FM_ERR_SHAPE, "mix_state: bad shape");
  if (rows == 0) return FM_OK;
  if (!post || !state || !state_norm_w || !noise_norm_w || !out) return set_error(FM_ERR_INVALID, "mix_state: null pointer");
  MixArgs a{};
  a.post = static_cast<const __nv_bfloat16*>(post);
  a.post_stride = post_stride;
  a.state = static_cast<const __nv_bfloat16*>(state);
  a.state_norm_w = static_cast<const __nv_bfloat16*>(state_norm_w);
  a.noise_norm_w = static_cast<const __nv_bfloat16*>(noise_norm_w);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.gate = gate;
  a.eps = eps;
  a.T = (int)rows;
  a.Ht = (int)cols;
  return launch_mix_state(a, as_stream(stream), false);
}

extern "C" fm_status fm_noise_fold(const void* proj, const void* z, const float* var, const void* x0, void* out,
                                   float gate, float eps, int64_t rows, int64_t cols, int64_t noise_cols,
                                   fm_stream stream) {
  if (rows < 0 || cols < 1 || noise_cols < 1) return set_error(FM_ERR_SHAPE, "noise_fold: bad shape");
  if (rows == 0) return FM_OK;
  if (!proj || !z || !var || !x0 || !out) return set_error(FM_ERR_INVALID, "noise_fold: null pointer");
  if (rows > INT32_MAX || cols > INT32_MAX || noise_cols > INT32_MAX)
    return set_error(FM_ERR_SHAPE, "noise_fold: dimension too large");
  NoiseFoldArgs a{};
  a.proj = static_cast<const __nv_bfloat16*>(proj);
  a.z = static_cast<const __nv_bfloat16*>(z);
  a.var = var;
  a.x0 = static_cast<const __nv_bfloat16*>(x0);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.gate = gate;
  a.eps = eps;
  a.T = (int)rows;
  a.D = (int)cols;
  a.Ht = (int)noise_cols;
  return launch_noise_fold(a, as_stream(stream), false);
}

extern "C" fm_status fm_block_self_attn(const void* qkv, void* out, int64_t batch, int64_t block, int64_t heads,
                                        int64_t head_dim, fm_stream stream) {
  if (!qkv || !out) return set_error(FM_ERR_INVALID, "self_attn: null pointer");
  if (batch <= 0 || block <= 0 || block > 64 || heads <= 0 || head_dim <= 0)
    return set_error(FM_ERR_SHAPE, "self_attn: bad shape");
  SelfAttnArgs a{};
  a.qkv = cbf(qkv);
  a.out = bf(out);
  a.block = (int)block;
  a.heads = (int)heads;
  a.head_dim = (int)head_dim;
  a.hidden = (int)(heads * head_dim);
  a.scale = (float)(1.0 / sqrt((double)head_dim));
  return launch_self_attn(a, (int)batch, as_stream(stream), false);
}

extern "C" size_t fm_cross_attn_workspace_size(int64_t batch, int64_t heads, int64_t head_dim, int64_t nsplit) {
  const size_t counters = ((size_t)batch * heads * sizeof(int) + 255) / 256 * 256;
  return counters + (size_t)batch * heads * nsplit * (16 * head_dim + 32) * sizeof(float);
}

extern "C" fm_status fm_cross_attn(const void* q, const void* cache, void* out, const int32_t* lengths,
                                   int64_t batch, int64_t heads, int64_t head_dim, int64_t layers, int64_t layer,
                                   int64_t cache_batch, int64_t cache_len, int64_t nsplit, void* workspace,
                                   size_t workspace_bytes, int32_t* err, fm_stream stream) {
  if (!q || !cache || !out || !lengths) return set_error(FM_ERR_INVALID, "cross_attn: null pointer");
  if (nsplit < 1 || layer < 0 || layer >= layers || batch > cache_batch)
    return set_error(FM_ERR_SHAPE, "cross_attn: bad shape");
  const size_t need = fm_cross_attn_workspace_size(batch, heads, head_dim, nsplit);
  if (!workspace || workspace_bytes < need) return set_error(FM_ERR_WORKSPACE, "cross_attn: %zu bytes needed", need);
  CUtensorMap tm;
  const uint64_t rows = (uint64_t)layers * 2 * cache_batch * heads * cache_len;
  fm_status st = make_tmap_bf16(&tm, cache, rows, (uint64_t)head_dim, (uint64_t)head_dim, 64);
  if (st) return st;
  CrossAttnArgs a{};
  a.q = cbf(q);
  a.out = bf(out);
  a.lengths = lengths;
  a.batch = (int)batch;
  a.heads = (int)heads;
  a.head_dim = (int)head_dim;
  a.hidden = (int)(heads * head_dim);
  a.layer = (int)layer;
  a.cache_batch = (int)cache_batch;
  a.cache_len = (int)cache_len;
  a.nsplit = (int)nsplit;
  a.scale = (float)(1.0 / sqrt((double)head_dim));
  const size_t counters = ((size_t)batch * heads * sizeof(int) + 255) / 256 * 256;
  a.counters = static_cast<int*>(workspace);
  a.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + counters);
  a.err = err;
  return launch_cross_attn(a, tm, as_stream(stream), false);
}

namespace {
// launch a kernel template instantiated for bf16 (dtype 0) or fp32 (dtype 1) logits
#define FM_DISPATCH_LOGITS(dtype, KERNEL, grid, ptr, ...)                                                      \
  ((dtype) == 0 ? launch_kernel(KERNEL<__nv_bfloat16>, grid, dim3(RT), 0, as_stream(stream), false,            \
                                static_cast<const __nv_bfloat16*>(ptr), __VA_ARGS__)                           \
                : launch_kernel(KERNEL<float>, grid, dim3(RT), 0, as_stream(stream), false,                   \
                                static_cast<const float*>(ptr), __VA_ARGS__))
// the same with programmatic dependent launch (kernels that call pdl_wait() before any read)
#define FM_DISPATCH_LOGITS_PDL(dtype, KERNEL, grid, ptr, ...)                                                  \
  ((dtype) == 0 ? launch_kernel(KERNEL<__nv_bfloat16>, grid, dim3(RT), 0, as_stream(stream), true,             \
                                static_cast<const __nv_bfloat16*>(ptr), __VA_ARGS__)                           \
                : launch_kernel(KERNEL<float>, grid, dim3(RT), 0, as_stream(stream), true,                    \
                                static_cast<const float*>(ptr), __VA_ARGS__))
bool bad_dtype(int32_t d) { return d != 0 && d != 1; }

// greedy acceptance through the sliced argmax: zero the keys, slice kernel, accept
fm_status greedy_sliced(const void* logits, int32_t dtype, const int64_t* draft, int64_t B, int64_t K, int64_t V,
                        int64_t* accepted, int64_t* bonus, unsigned long long* keys, fm_stream stream) {
  const long long rows = B * (K + 1);
  fm_status st = check_cuda(cudaMemsetAsync(keys, 0, (size_t)rows * 8, as_stream(stream)), "accept: key reset");
  if (st) return st;
  const long long slices = ((V + 7) / 8 + SLICE_VECS - 1) / SLICE_VECS;
  if (slices > 65535) return set_error(FM_ERR_SHAPE, "accept: vocabulary too large");
  st = FM_DISPATCH_LOGITS(dtype, row_argmax_slice_kernel, dim3((unsigned)rows, (unsigned)slices), logits,
                          (long long)V, keys);
  if (st) return st;
  return launch_kernel(accept_greedy_keys_kernel, dim3((unsigned)B), dim3(1), 0, as_stream(stream), false, draft,
                       (const unsigned long long*)keys, (int)K, accepted, bonus);
}
}  // namespace

extern "C" fm_status fm_row_stats(const void* logits, int32_t dtype, int64_t rows, int64_t V, float temperature,
                                  float* stats, int64_t* argmax, fm_stream stream) {
  if (!logits) return set_error(FM_ERR_INVALID, "row_stats: null logits");
  if (rows <= 0 || V <= 0 || V >= (1ll << 31) || bad_dtype(dtype))
    return set_error(FM_ERR_SHAPE, "row_stats: bad arguments");
  return FM_DISPATCH_LOGITS(dtype, row_stats_kernel, dim3((unsigned)rows), logits, (long long)V, temperature, stats,
                            argmax);
}

extern "C" fm_status fm_softmax_rows(const void* logits, int32_t dtype, int64_t rows, int64_t V, float temperature,
                                     float* probs, fm_stream stream) {
  if (!logits || !probs) return set_error(FM_ERR_INVALID, "softmax_rows: null pointer");
  if (rows <= 0 || V <= 0 || V >= (1ll << 31) || !(temperature > 0.0f) || bad_dtype(dtype))
    return set_error(FM_ERR_SHAPE, "softmax_rows: bad arguments");
  return FM_DISPATCH_LOGITS(dtype, softmax_rows_kernel, dim3((unsigned)rows), logits, (long long)V, temperature,
                            probs);
}

extern "C" fm_status fm_sample_rows(const void* logits, int32_t dtype, const float* probs, int64_t B, int64_t K,
                                    int64_t V, float temperature, uint64_t seed, uint32_t offset, int64_t* tokens,
                                    fm_stream stream) {
  if (!tokens) return set_error(FM_ERR_INVALID, "sample_rows: null tokens");
  if (B <= 0 || K <= 0 || V <= 0 || bad_dtype(dtype)) return set_error(FM_ERR_SHAPE, "sample_rows: bad arguments");
  if (temperature <= 0.0f) {
    if (!logits) return set_error(FM_ERR_INVALID, "sample_rows: null logits");
    // the sliced argmax of greedy acceptance: each int64 token holds its row's
    // 64-bit (value, complement index) key while the slices merge into it by
    // atomicMax, then the key is turned into its index in place
    const long long rows = B * K;
    const long long slices = ((V + 7) / 8 + SLICE_VECS - 1) / SLICE_VECS;
    if (slices > 65535 || rows >= (1ll << 31)) return set_error(FM_ERR_SHAPE, "sample_rows: too many rows or ids");
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(tokens);
    fm_status st = check_cuda(cudaMemsetAsync(keys, 0, (size_t)rows * 8, as_stream(stream)), "sample_rows: key reset");
    if (st) return st;
    st = FM_DISPATCH_LOGITS(dtype, row_argmax_slice_kernel, dim3((unsigned)rows, (unsigned)slices), logits,
                            (long long)V, keys);
    if (st) return st;
    return launch_argmax_tokens(keys, tokens, (int)rows, as_stream(stream), false);
  }
  if (!probs) return set_error(FM_ERR_INVALID, "sample_rows: T > 0 needs probs");
  return launch_kernel(sample_rows_kernel, dim3((unsigned)(B * K)), dim3(RT), 0, as_stream(stream), false, probs,
                       (long long)V, (int)K, seed, offset, tokens);
}

namespace {
// Acceptance workspace, 256-byte aligned parts.  Greedy: a 64-bit key per
// target row.  Rejection: per row (m, S), per (row, slice) the scan's (max,
// approximate sum) and the listed rows' exact slice totals, per request its
// row list and count, then the bonus draw's slice totals.
struct AcceptLayout {
  size_t stats, slices, exact, list, nlist, totals, bytes;
  AcceptLayout(int64_t B, int64_t K) {
    const size_t rows = (size_t)B * (K + 1);
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    stats = 0;
    slices = up(rows * 2 * sizeof(float));
    exact = slices + up(rows * CAT_MAX_SLICES * sizeof(float2));
    list = exact + up(rows * CAT_MAX_SLICES * sizeof(float));
    nlist = list + up(rows * sizeof(int));
    totals = nlist + up((size_t)B * sizeof(int));
    bytes = totals + up((size_t)B * CAT_MAX_SLICES * sizeof(float));
  }
};
}  // namespace

extern "C" size_t fm_accept_workspace_size(int64_t B, int64_t K) {
  if (B <= 0 || K < 0) return 0;
  return AcceptLayout(B, K).bytes;
}

extern "C" fm_status fm_accept_greedy(const void* target_logits, int32_t dtype, const int64_t* draft, int64_t B,
                                      int64_t K, int64_t V, int64_t* accepted, int64_t* bonus, void* workspace,
                                      size_t workspace_bytes, fm_stream stream) {
  if (!target_logits || !draft || !accepted || !bonus) return set_error(FM_ERR_INVALID, "accept: null pointer");
  if (B <= 0 || K <= 0 || V <= 0 || bad_dtype(dtype)) return set_error(FM_ERR_SHAPE, "accept: bad arguments");
  if (!workspace || workspace_bytes < fm_accept_workspace_size(B, K))
    return set_error(FM_ERR_WORKSPACE, "accept: workspace too small");
  return greedy_sliced(target_logits, dtype, draft, B, K, V, accepted, bonus,
                       static_cast<unsigned long long*>(workspace), stream);
}

extern "C" fm_status fm_accept_rejection(const void* target_logits, int32_t dtype, const int64_t* draft,
                                         const float* q, int64_t B, int64_t K, int64_t V, float temperature,
                                         uint64_t seed, uint32_t offset, int64_t* accepted, int64_t* bonus,
                                         void* workspace, size_t workspace_bytes, fm_stream stream) {
  if (!target_logits || !draft || !q || !accepted || !bonus) return set_error(FM_ERR_INVALID, "accept: null pointer");
  if (B <= 0 || K <= 0 || V <= 0 || !(temperature > 0.0f) || bad_dtype(dtype))
    return set_error(FM_ERR_SHAPE, "accept: bad arguments");
  if (!workspace || workspace_bytes < fm_accept_workspace_size(B, K))
    return set_error(FM_ERR_WORKSPACE, "accept: workspace too small");
  const long long cat_slices = (V + CAT_SLICE - 1) / CAT_SLICE;
  if (cat_slices > CAT_MAX_SLICES) return set_error(FM_ERR_SHAPE, "accept: vocabulary too large for the bonus draw");
  const AcceptLayout lay(B, K);
  char* ws = static_cast<char*>(workspace);
  float* stats = reinterpret_cast<float*>(ws + lay.stats);
  float2* slice_stats = reinterpret_cast<float2*>(ws + lay.slices);
  float* exact = reinterpret_cast<float*>(ws + lay.exact);
  int* list = reinterpret_cast<int*>(ws + lay.list);
  int* nlist = reinterpret_cast<int*>(ws + lay.nlist);
  float* totals = reinterpret_cast<float*>(ws + lay.totals);
  const long long rows = B * (K + 1);
  const int S = (int)cat_slices;
  const float c = (float)(1.4426950408889634 / (double)temperature);  // log2(e) / T
  cudaStream_t cs = as_stream(stream);
  const bool bf = dtype == 0;
  const void* tl = target_logits;
  fm_status st;
  // 1. chunk maxima and approximate sums
  const int C = (int)(((V + 7) / 8 + REJ_SCAN_VECS - 1) / REJ_SCAN_VECS);
  st = bf ? launch_kernel(reject_scan_kernel<__nv_bfloat16>, dim3((unsigned)rows, (unsigned)C), dim3(RT), 0, cs, true,
                          static_cast<const __nv_bfloat16*>(tl), (long long)V, c, C, slice_stats)
          : launch_kernel(reject_scan_kernel<float>, dim3((unsigned)rows, (unsigned)C), dim3(RT), 0, cs, true,
                          static_cast<const float*>(tl), (long long)V, c, C, slice_stats);
  if (st) return st;
  // 2. settled tests and the rows needing exact sums
  const size_t dsmem = (size_t)(K > 0 ? K : 1) * sizeof(int);
  if (dsmem > 48 * 1024) return set_error(FM_ERR_SHAPE, "accept: too many slots");
  st = bf ? launch_kernel(reject_decide_kernel<__nv_bfloat16>, dim3((unsigned)B), dim3(32), dsmem, cs, true,
                          static_cast<const __nv_bfloat16*>(tl), draft, q, (long long)V, (int)K, temperature, c, seed,
                          offset, C, (const float2*)slice_stats, stats, list, nlist)
          : launch_kernel(reject_decide_kernel<float>, dim3((unsigned)B), dim3(32), dsmem, cs, true,
                          static_cast<const float*>(tl), draft, q, (long long)V, (int)K, temperature, c, seed, offset,
                          C, (const float2*)slice_stats, stats, list, nlist);
  if (st) return st;
  // 3. exact slice totals of the listed rows
  st = bf ? launch_kernel(reject_exact_kernel<__nv_bfloat16>, dim3((unsigned)B, (unsigned)S), dim3(RT), 0, cs, true,
                          static_cast<const __nv_bfloat16*>(tl), (long long)V, (int)K, temperature, S,
                          (const float*)stats, (const int*)list, (const int*)nlist, exact)
          : launch_kernel(reject_exact_kernel<float>, dim3((unsigned)B, (unsigned)S), dim3(RT), 0, cs, true,
                          static_cast<const float*>(tl), (long long)V, (int)K, temperature, S, (const float*)stats,
                          (const int*)list, (const int*)nlist, exact);
  if (st) return st;
  // 4. open tests, accepted lengths, the bonus rows' exact sums
  st = bf ? launch_kernel(reject_final_kernel<__nv_bfloat16>, dim3((unsigned)B), dim3(32), 0, cs, true,
                          static_cast<const __nv_bfloat16*>(tl), draft, q, (long long)V, (int)K, temperature, seed,
                          offset, S, (const int*)list, (const int*)nlist, (const float*)exact, stats, accepted)
          : launch_kernel(reject_final_kernel<float>, dim3((unsigned)B), dim3(32), 0, cs, true,
                          static_cast<const float*>(tl), draft, q, (long long)V, (int)K, temperature, seed, offset, S,
                          (const int*)list, (const int*)nlist, (const float*)exact, stats, accepted);
  if (st) return st;
  st = FM_DISPATCH_LOGITS_PDL(dtype, residual_slices_kernel, dim3((unsigned)B, (unsigned)cat_slices), target_logits, q,
                          (long long)V, (int)K, temperature, (const float*)stats, (const int64_t*)accepted, totals);
  if (st) return st;
  return FM_DISPATCH_LOGITS_PDL(dtype, residual_pick_kernel, dim3((unsigned)B), target_logits, q, (long long)V, (int)K,
                            temperature, seed, offset, (const float*)stats, (const int64_t*)accepted,
                            (const float*)totals, bonus);
}

extern "C" fm_status fm_transpose_bf16(const void* in, void* out, int64_t rows, int64_t cols, fm_stream stream) {
  if (!in || !out) return set_error(FM_ERR_INVALID, "transpose: null pointer");
  if (rows <= 0 || cols <= 0) return set_error(FM_ERR_SHAPE, "transpose: empty shape");
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  return launch_kernel(transpose_bf16_kernel, grid, dim3(32, 8), 0, as_stream(stream), false, cbf(in), bf(out),
                       (long long)rows, (long long)cols);
}

extern "C" fm_status fm_time_sinusoid(void* out, int64_t dim, float s, float t, float scale, const float* freqs,
                                      fm_stream stream) {
  if (!out || !freqs) return set_error(FM_ERR_INVALID, "time_sinusoid: null pointer");
  if (dim <= 0 || dim % 2) return set_error(FM_ERR_SHAPE, "time_sinusoid: bad dim");
  return launch_kernel(time_sinusoid_kernel, dim3(blocks_for(dim, 256)), dim3(256), 0, as_stream(stream), false,
                       bf(out), (int)dim, s, t, scale, freqs);
}

extern "C" fm_status fm_silu(const void* x, void* y, int64_t n, fm_stream stream) {
  if (!x || !y) return set_error(FM_ERR_INVALID, "silu: null pointer");
  if (n <= 0) return FM_OK;
  return launch_kernel(silu_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, as_stream(stream), false, cbf(x), bf(y),
                       (long long)n);
}

extern "C" fm_status fm_add(const void* a, const void* b, void* y, int64_t n, fm_stream stream) {
  if (!a || !b || !y) return set_error(FM_ERR_INVALID, "add: null pointer");
  if (n <= 0) return FM_OK;
  return launch_kernel(add_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, as_stream(stream), false, cbf(a), cbf(b),
                       bf(y), (long long)n);
}

// ====================================================================== allocation-free greedy acceptance
//
// Some callers cannot allocate device memory when they accept a block: a
// serving engine that plans every device buffer before it captures its decode
// step in a CUDA graph, or host code in another language that is handed the
// logits and token buffers and has no device allocator of its own.  For them
// fm_accept_greedy_noalloc keeps its per-row argmax scratch in a fixed array
// inside this library instead of a caller workspace.
//
// The array is shared by every call on a device and keeps the last call's
// contents.  The argmax keys are merged with atomicMax and must start at
// zero: greedy_sliced clears the rows a call uses (cudaMemsetAsync on the
// call's stream) before its kernels run.  Calls that overlap on the GPU
// (different streams, no ordering) race on it.  Its device address is looked up once per device, by the first
// call made with that device current; make that first call before any stream
// capture begins.
static __device__ __align__(256) int64_t g_accept_noalloc_scratch[FM_ACCEPT_NOALLOC_MAX_ROWS];

namespace {

int64_t* accept_noalloc_scratch(fm_status* st) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static int64_t* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *st = set_error(FM_ERR_CUDA, "accept_noalloc: no usable current device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_accept_noalloc_scratch);
    if (e != cudaSuccess) {
      *st = set_error(FM_ERR_CUDA, "accept_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<int64_t*>(p);
  }
  *st = FM_OK;
  return addr[dev];
}

}  // namespace

extern "C" fm_status fm_accept_greedy_noalloc(const void* target_logits, int32_t dtype, const int64_t* draft,
                                              int64_t B, int64_t K, int64_t V, int64_t* accepted, int64_t* bonus,
                                              fm_stream stream) {
  if (!target_logits || !draft || !accepted || !bonus) return set_error(FM_ERR_INVALID, "accept_noalloc: null pointer");
  if (B <= 0 || K <= 0 || V <= 0 || bad_dtype(dtype)) return set_error(FM_ERR_SHAPE, "accept_noalloc: bad arguments");
  // B*(K+1) <= the maximum, checked without forming a product that could wrap
  if (K >= FM_ACCEPT_NOALLOC_MAX_ROWS || B > FM_ACCEPT_NOALLOC_MAX_ROWS / (K + 1))
    return set_error(FM_ERR_WORKSPACE,
                     "accept_noalloc: B=%lld, K=%lld needs more target rows (B*(K+1)) than the built-in scratch "
                     "of %d rows; use fm_accept_greedy with a workspace",
                     (long long)B, (long long)K, FM_ACCEPT_NOALLOC_MAX_ROWS);
  fm_status st;
  int64_t* am = accept_noalloc_scratch(&st);
  if (!am) return st;
  return greedy_sliced(target_logits, dtype, draft, B, K, V, accepted, bonus,
                       reinterpret_cast<unsigned long long*>(am), stream);
}
