// Row statistics of the normalisations (LayerNorm of AdaLN, RMSNorm,
// mix_state) in one canonical order, shared by every kernel that normalises
// rows so that all of them produce identical bits.
//
// One warp per row.  Lane l takes the 8-element chunks l, l+32, l+64, ... of
// the row; inside a chunk the elements are combined as a pairwise tree
// ((e0 op e1) + (e2 op e3)) + ((e4 op e5) + (e6 op e7)), and the chunk total is
// added to the lane's running sum; the 32 lane sums are then combined by an
// xor butterfly (offsets 16, 8, 4, 2, 1), so every lane ends with the total.
// A ragged last chunk treats its missing elements as absent (not as zeros
// that would shift a variance).
#pragma once

#include "common.cuh"

namespace fm {

// 8 elements of chunk `ch` (count valid ones, the rest 0)
__device__ __forceinline__ int row_chunk8(const __nv_bfloat16* row, int ch, int cols, bool aligned, float* x) {
  const int e0 = ch * 8;
  const int n = cols - e0 < 8 ? cols - e0 : 8;
  if (aligned && n == 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row + e0);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = j < n ? bf2f(row[e0 + j]) : 0.0f;
  }
  return n;
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// tree over the valid elements of a chunk (absent elements contribute nothing)
__device__ __forceinline__ float chunk_tree(const float* t, int n) {
  if (n == 8) return __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3])),
                               __fadd_rn(__fadd_rn(t[4], t[5]), __fadd_rn(t[6], t[7])));
  float s = t[0];
  for (int j = 1; j < n; ++j) s = __fadd_rn(s, t[j]);
  return s;
}

// sum of squares of a row (RMSNorm statistic)
__device__ __forceinline__ float warp_row_sumsq(const __nv_bfloat16* row, int cols, int lane) {
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  float s = 0.0f;
  for (int ch = lane; ch * 8 < cols; ch += 32) {
    float x[8], t[8];
    const int n = row_chunk8(row, ch, cols, aligned, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = __fmul_rn(x[j], x[j]);
    s = __fadd_rn(s, chunk_tree(t, n));
  }
  return warp_allsum(s);
}

// 1 / sqrt(mean of squares + eps)
__device__ __forceinline__ float inv_rms(float sumsq, int cols, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, (float)cols), eps)));
}

// mean and 1 / sqrt(var + eps) of a row (LayerNorm without affine, two passes)
__device__ __forceinline__ void warp_row_meanrstd(const __nv_bfloat16* row, int cols, float eps, int lane,
                                                  float* mean_out, float* rstd_out) {
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  float s = 0.0f;
  for (int ch = lane; ch * 8 < cols; ch += 32) {
    float x[8];
    const int n = row_chunk8(row, ch, cols, aligned, x);
    s = __fadd_rn(s, chunk_tree(x, n));
  }
  const float mean = __fdiv_rn(warp_allsum(s), (float)cols);
  float q = 0.0f;
  for (int ch = lane; ch * 8 < cols; ch += 32) {
    float x[8], t[8];
    const int n = row_chunk8(row, ch, cols, aligned, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d = __fsub_rn(x[j], mean);
      t[j] = __fmul_rn(d, d);
    }
    q = __fadd_rn(q, chunk_tree(t, n));
  }
  const float var = __fdiv_rn(warp_allsum(q), (float)cols);
  *mean_out = mean;
  *rstd_out = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// The same statistics with a lane's chunks loaded 8 at a time (one memory
// round trip per 8 chunks instead of one per chunk): rows whose width is a
// multiple of 8 and 16-byte aligned.  Loads bypass L1 (the rows may have been
// written by other SMs during the same kernel).
__device__ __forceinline__ void unpack_bf16x8(const uint4 raw, float* x) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float* v) {
  uint4 o;
  __nv_bfloat162 t;
  t = __floats2bfloat162_rn(v[0], v[1]);
  o.x = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(v[2], v[3]);
  o.y = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(v[4], v[5]);
  o.z = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(v[6], v[7]);
  o.w = *reinterpret_cast<uint32_t*>(&t);
  return o;
}

// chunks lane + 32 * (base + i), i < 8, that exist
__device__ __forceinline__ void lane_chunks8(const __nv_bfloat16* row, int nch, int lane, int base, uint4* raw) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ch = lane + 32 * (base + i);
    if (ch < nch) raw[i] = __ldcg(reinterpret_cast<const uint4*>(row) + ch);
  }
}

__device__ __forceinline__ float warp_row_sumsq_batched(const __nv_bfloat16* row, int cols, int lane) {
  const int nch = cols / 8, rounds = (nch + 255) / 256;
  float s = 0.0f;
  for (int rd = 0; rd < rounds; ++rd) {
    uint4 raw[8];
    lane_chunks8(row, nch, lane, rd * 8, raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (lane + 32 * (rd * 8 + i) < nch) {
        float x[8], t[8];
        unpack_bf16x8(raw[i], x);
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = __fmul_rn(x[j], x[j]);
        s = __fadd_rn(s, chunk_tree(t, 8));
      }
    }
  }
  return warp_allsum(s);
}

__device__ __forceinline__ void warp_row_meanrstd_batched(const __nv_bfloat16* row, int cols, float eps, int lane,
                                                          float* mean_out, float* rstd_out) {
  const int nch = cols / 8, rounds = (nch + 255) / 256;
  uint4 raw[8];
  float s = 0.0f;
  for (int rd = 0; rd < rounds; ++rd) {
    lane_chunks8(row, nch, lane, rd * 8, raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (lane + 32 * (rd * 8 + i) < nch) {
        float x[8];
        unpack_bf16x8(raw[i], x);
        s = __fadd_rn(s, chunk_tree(x, 8));
      }
    }
  }
  const float mean = __fdiv_rn(warp_allsum(s), (float)cols);
  float q = 0.0f;
  for (int rd = 0; rd < rounds; ++rd) {
    if (rounds > 1) lane_chunks8(row, nch, lane, rd * 8, raw);  // one round: still in registers
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (lane + 32 * (rd * 8 + i) < nch) {
        float x[8], t[8];
        unpack_bf16x8(raw[i], x);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = __fsub_rn(x[j], mean);
          t[j] = __fmul_rn(d, d);
        }
        q = __fadd_rn(q, chunk_tree(t, 8));
      }
    }
  }
  const float var = __fdiv_rn(warp_allsum(q), (float)cols);
  *mean_out = mean;
  *rstd_out = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// AdaLN output element: bf16(bf16(bf16(LN(x)) * bf16(1 + scale)) + shift)
__device__ __forceinline__ float adaln_value(float x, float mean, float rstd, float scale, float shift) {
  const float ln = round_bf(__fmul_rn(__fsub_rn(x, mean), rstd));
  const float one_plus = round_bf(__fadd_rn(1.0f, scale));
  const float scaled = round_bf(__fmul_rn(ln, one_plus));
  return __fadd_rn(scaled, shift);
}

// RMSNorm output element: x * bf16(w * inv)
__device__ __forceinline__ float rms_value(float x, float w, float inv) { return __fmul_rn(x, round_bf(__fmul_rn(w, inv))); }

// mix_state element: bf16(RMSNorm_s(post)) + bf16(gate * bf16(RMSNorm_n(state)))
__device__ __forceinline__ float mix_value(float post, float state, float sw, float nw, float ip, float is,
                                           float gate) {
  const float pn = round_bf(rms_value(post, sw, ip));
  const float nn = round_bf(rms_value(state, nw, is));
  return __fadd_rn(pn, round_bf(__fmul_rn(gate, nn)));
}

}  // namespace fm
