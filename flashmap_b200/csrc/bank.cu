// The banked multi-jump draft of the sglang plugin (flashmap/sglang/jump_bank.py),
// behind the C ABI:
//   * bank_rows_kernel       one chunk of bank draws: bf16 z (for z @ E) and, per
//                            later jump, softmax(a z) in bf16 and logsumexp(a z)
//   * topk_rows_kernel       a jump's prediction: the top k of a logits row with
//                            their probabilities under the row's full softmax
//   * bank_gather_kernel     rows of a bank table for the draft's slots
//   * bank_jump_rows_kernel  a later jump's two state rows per slot: the hashed
//                            normals on the support, the mass weights, and the
//                            sums over the support's embedding rows
//   * token_normals_kernel   the per-(seed, token) normals alone (parity checks)
//   * philox_randint_kernel  uniform integers (bank rows and slot seeds)
//
// A bank row holds what a jump needs over the whole vocabulary from one draw
// z: z @ E, and per later jump n, softmax(a_n z) @ E and logsumexp(a_n z); the
// E products are the library's GEMMs over these kernels' outputs.  Reductions
// use fixed 256-thread trees.
#include <climits>

#include "common.cuh"
#include "launch.cuh"
#include "philox.cuh"

namespace fm {
namespace {

constexpr int BT = 256;
constexpr int BANK_MAX_SUPPORT = 256;  // support entries per slot (jumps x top-k)

__device__ __forceinline__ float tree_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.0f;
#pragma unroll
  for (int w = 0; w < BT / 32; ++w) r = __fadd_rn(r, red[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ float tree_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < BT / 32; ++w) r = fmaxf(r, red[w]);
  __syncthreads();
  return r;
}

struct BankSlopes {
  int n;
  float v[8];
};

__global__ void __launch_bounds__(BT) bank_rows_kernel(const float* z, __nv_bfloat16* zb, __nv_bfloat16* probs,
                                                       float* log_mass, long long rows, long long cols, BankSlopes sl) {
  __shared__ float red[BT / 32];
  const long long r = blockIdx.x;
  const float* zr = z + r * cols;
  __nv_bfloat16* zo = zb + r * cols;
  for (long long c = threadIdx.x; c < cols; c += BT) zo[c] = f2bf(zr[c]);
  for (int j = 0; j < sl.n; ++j) {
    const float a = sl.v[j];
    float m = -INFINITY;
    for (long long c = threadIdx.x; c < cols; c += BT) m = fmaxf(m, __fmul_rn(a, zr[c]));
    m = tree_max(m, red);
    float acc = 0.0f;
    for (long long c = threadIdx.x; c < cols; c += BT) acc = __fadd_rn(acc, expf(__fsub_rn(__fmul_rn(a, zr[c]), m)));
    const float sum = tree_sum(acc, red);
    if (threadIdx.x == 0) log_mass[j * rows + r] = __fadd_rn(m, logf(sum));
    __nv_bfloat16* po = probs + (j * rows + r) * cols;
    for (long long c = threadIdx.x; c < cols; c += BT)
      po[c] = f2bf(__fdiv_rn(expf(__fsub_rn(__fmul_rn(a, zr[c]), m)), sum));
  }
}

// (value, index) order of a prediction: larger value first, then smaller index
__device__ __forceinline__ bool ranks_before(float a, int ia, float b, int ib) {
  return a > b || (a == b && ia < ib);
}

// orderable key of (value, index): the largest key is the first in the order
__device__ __forceinline__ unsigned long long rank_key(float v, int i) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}

template <int KM>
__global__ void __launch_bounds__(BT) topk_rows_kernel(const __nv_bfloat16* logits, long long ld, int cols, int k,
                                                       const long long* row_map, long long map_len, long long* ids,
                                                       float* probs, int* err) {
  __shared__ float red[BT / 32];
  __shared__ unsigned long long wkey[BT / 32];
  __shared__ int win_idx[KM];
  __shared__ float win_val[KM];
  const long long r = blockIdx.x;
  const __nv_bfloat16* row = logits + r * ld;
  // this thread's best k of its strided elements, sorted in rank order
  float lv[KM];
  int li[KM];
#pragma unroll
  for (int p = 0; p < KM; ++p) {
    lv[p] = -INFINITY;
    li[p] = INT_MAX;
  }
  float kv = -INFINITY;
  int ki = INT_MAX;
  for (int c = threadIdx.x; c < cols; c += BT) {
    const float x = bf2f(row[c]);
    if (!ranks_before(x, c, kv, ki)) continue;
#pragma unroll
    for (int p = KM - 1; p >= 1; --p) {
      if (p >= k) continue;
      if (ranks_before(x, c, lv[p - 1], li[p - 1])) {
        lv[p] = lv[p - 1];
        li[p] = li[p - 1];
      } else if (ranks_before(x, c, lv[p], li[p])) {
        lv[p] = x;
        li[p] = c;
      }
    }
    if (ranks_before(x, c, lv[0], li[0])) {
      lv[0] = x;
      li[0] = c;
    }
#pragma unroll
    for (int p = 0; p < KM; ++p)
      if (p == k - 1) {
        kv = lv[p];
        ki = li[p];
      }
  }
  // merge: k rounds, each taking the best head of the threads' sorted lists
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int head = 0;
  for (int round = 0; round < k; ++round) {
    float hv = -INFINITY;
    int hi = INT_MAX;
#pragma unroll
    for (int p = 0; p < KM; ++p)
      if (p == head) {
        hv = lv[p];
        hi = li[p];
      }
    const unsigned long long key = hi == INT_MAX ? 0ull : rank_key(hv, hi);
    const uint32_t kh = (uint32_t)(key >> 32);
    const uint32_t mh = __reduce_max_sync(0xffffffffu, kh);
    const uint32_t ml = __reduce_max_sync(0xffffffffu, kh == mh ? (uint32_t)key : 0u);
    if (lane == 0) wkey[warp] = ((unsigned long long)mh << 32) | ml;
    __syncthreads();
    unsigned long long best = wkey[0];
#pragma unroll
    for (int w = 1; w < BT / 32; ++w) best = wkey[w] > best ? wkey[w] : best;
    const bool mine = best != 0ull && key == best;
    if (mine) {
      win_idx[round] = hi;
      win_val[round] = hv;
      ++head;
    }
    if (best == 0ull && threadIdx.x == 0) {  // fewer than k columns
      win_idx[round] = -1;
      win_val[round] = -INFINITY;
    }
    __syncthreads();
  }
  // the full softmax's sum, for the probabilities of the winners
  const float m = win_val[0];
  float acc = 0.0f;
  for (int c = threadIdx.x; c < cols; c += BT) acc = __fadd_rn(acc, expf(__fsub_rn(bf2f(row[c]), m)));
  const float sum = tree_sum(acc, red);
  if (threadIdx.x < k) {
    const int j = threadIdx.x;
    const int c = win_idx[j];
    long long id = c;
    if (c >= 0 && row_map) {
      if (c < map_len) {
        id = row_map[c];
      } else {
        record_error(err, DEV_BAD_INDEX);
        id = -1;
      }
    }
    ids[r * k + j] = id;
    probs[r * k + j] = c >= 0 ? __fdiv_rn(expf(__fsub_rn(win_val[j], m)), sum) : 0.0f;
  }
}

__global__ void __launch_bounds__(BT) bank_gather_kernel(const __nv_bfloat16* table, long long table_rows,
                                                         long long cols, const long long* rows, __nv_bfloat16* out,
                                                         int* err) {
  const long long r = blockIdx.x;
  const long long src = rows[r];
  __nv_bfloat16* o = out + r * cols;
  if (src < 0 || src >= table_rows) {
    if (threadIdx.x == 0) record_error(err, DEV_BAD_INDEX);
    for (long long c = threadIdx.x; c < cols; c += BT) o[c] = f2bf(0.0f);
    return;
  }
  const __nv_bfloat16* s = table + src * cols;
  for (long long c = threadIdx.x; c < cols; c += BT) o[c] = s[c];
}

// two multiply-xorshift rounds (jump_bank.py:52-59, its int64 arithmetic
// taken modulo 2^32, which the masks there keep)
__device__ __forceinline__ uint32_t mix_hash(uint32_t x) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    x ^= x >> 16;
    x *= 0x45D9F3Bu;
  }
  return x ^ (x >> 16);
}

// normal of (slot seed, token id) by Box-Muller on two hashed uniforms (jump_bank.py:62-73)
__device__ __forceinline__ float token_normal(long long seed, long long id) {
  const uint32_t hid = mix_hash((uint32_t)((unsigned long long)id & 0xFFFFFFFFull) ^ 0x9E3779B9u);
  const uint32_t h1 = mix_hash(hid ^ (uint32_t)((unsigned long long)seed & 0xFFFFFFFFull));
  const uint32_t h2 = mix_hash(h1 ^ 0x68E31DA4u);
  // the divisors as fp32 (4294967297 rounds to 2^32)
  const float u1 = __fdiv_rn(__fadd_rn(__uint2float_rn(h1), 1.0f), 4294967296.0f);
  const float u2 = __fdiv_rn(__uint2float_rn(h2), 4294967296.0f);
  return __fmul_rn(sqrtf(__fmul_rn(-2.0f, logf(u1))), cosf(__fmul_rn(6.2831855f, u2)));
}

__global__ void token_normals_kernel(const long long* seeds, const long long* ids, long long R, long long L,
                                     float* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * L) return;
  out[i] = token_normal(seeds[i / L], ids[i]);
}

__global__ void __launch_bounds__(BT) bank_jump_rows_kernel(fm_bank_jump a) {
  __shared__ long long sid[BANK_MAX_SUPPORT];
  __shared__ long long srow[BANK_MAX_SUPPORT];
  __shared__ float slin[BANK_MAX_SUPPORT];
  __shared__ float swt[BANK_MAX_SUPPORT];
  __shared__ float red[BT / 32];
  const long long slot = blockIdx.x;
  const int L = a.support;
  long long row = a.rows[slot];
  if (row < 0 || row >= a.bank_rows) {
    if (threadIdx.x == 0) record_error(a.err, DEV_BAD_INDEX);
    row = 0;
  }
  const long long seed = a.seeds[slot];
  const int t = threadIdx.x;
  if (t < L) {
    long long id = a.ids[slot * L + t];
    if (id < 0 || id >= a.state_rows) {
      record_error(a.err, DEV_BAD_INDEX);
      id = 0;
    }
    sid[t] = id;
    srow[t] = a.state_map ? a.state_map[id] : id;
    slin[t] = __fmul_rn(a.betas[t / a.topk], a.probs[slot * L + t]);
  }
  __syncthreads();
  float w = 0.0f;
  if (t < L) {
    const long long id = sid[t];
    float c = 0.0f;  // every prediction's weight on this token, in support order
    bool first = true;
    for (int i = 0; i < L; ++i)
      if (sid[i] == id) {
        c = __fadd_rn(c, slin[i]);
        if (i < t) first = false;
      }
    const float shift = __fmul_rn(a.evidence, c);
    const float zv = __fmul_rn(a.temperature, token_normal(seed, id));
    w = __fmul_rn(__fmul_rn(expf(__fsub_rn(__fmul_rn(a.slope, zv), a.log_mass[row])), expm1f(shift)),
                  first ? 1.0f : 0.0f);
    swt[t] = w;
  }
  const float wsum = tree_sum(w, red);  // also orders the swt writes before the reads below
  const float denom = __fadd_rn(1.0f, wsum);
  const long long H = a.hidden;
  const __nv_bfloat16* mean = static_cast<const __nv_bfloat16*>(a.mean_embed) + row * H;
  const __nv_bfloat16* noise = static_cast<const __nv_bfloat16*>(a.noise_embed) + row * H;
  const __nv_bfloat16* embed = static_cast<const __nv_bfloat16*>(a.embed);
  __nv_bfloat16* post_out = static_cast<__nv_bfloat16*>(a.out) + slot * H;
  __nv_bfloat16* noise_out = static_cast<__nv_bfloat16*>(a.out) + (a.slots + slot) * H;
  for (long long col = t; col < H; col += BT) {
    float s0 = 0.0f, s1 = 0.0f;
    for (int j = 0; j < L; ++j) {
      const float e = bf2f(embed[srow[j] * H + col]);
      s0 = __fadd_rn(s0, __fmul_rn(round_bf(swt[j]), e));
      s1 = __fadd_rn(s1, __fmul_rn(round_bf(slin[j]), e));
    }
    post_out[col] = f2bf(__fdiv_rn(__fadd_rn(bf2f(mean[col]), s0), denom));
    noise_out[col] = f2bf(__fadd_rn(__fmul_rn(a.alpha, bf2f(noise[col])), s1));
  }
}

__global__ void philox_randint_kernel(long long* out, long long n, long long high, uint64_t seed, uint32_t offset,
                                      uint32_t purpose) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const Philox4 r = philox4x32_10((uint32_t)i, (uint32_t)(i >> 32), offset, purpose, seed);
  out[i] = (long long)(((unsigned long long)r.v[0] * (unsigned long long)high) >> 32);
}

}  // namespace
}  // namespace fm

// ====================================================================== C ABI
using namespace fm;

extern "C" fm_status fm_bank_rows(const float* z, void* z_bf16, void* probs, float* log_mass, int64_t rows,
                                  int64_t cols, const float* slopes, int32_t n_slopes, fm_stream stream) {
  if (rows < 0 || cols < 1 || n_slopes < 0 || n_slopes > 8) return set_error(FM_ERR_SHAPE, "bank_rows: bad shape");
  if (rows == 0) return FM_OK;
  if (!z || !z_bf16 || (n_slopes > 0 && (!probs || !log_mass || !slopes)))
    return set_error(FM_ERR_INVALID, "bank_rows: null pointer");
  BankSlopes sl{};
  sl.n = n_slopes;
  for (int j = 0; j < n_slopes; ++j) sl.v[j] = slopes[j];
  return launch_kernel(bank_rows_kernel, dim3((unsigned)rows), dim3(BT), 0, static_cast<cudaStream_t>(stream), false,
                       z, static_cast<__nv_bfloat16*>(z_bf16), static_cast<__nv_bfloat16*>(probs), log_mass,
                       (long long)rows, (long long)cols, sl);
}

extern "C" fm_status fm_topk_rows(const void* logits, int64_t ld, int64_t rows, int64_t cols, int32_t k,
                                  const int64_t* row_map, int64_t map_len, int64_t* ids, float* probs, int32_t* err,
                                  fm_stream stream) {
  if (rows < 0 || cols < 1 || ld < cols || k < 1 || k > 32 || cols > INT32_MAX - 1)
    return set_error(FM_ERR_SHAPE, "topk_rows: bad shape (1 <= k <= 32)");
  if (rows == 0) return FM_OK;
  if (!logits || !ids || !probs) return set_error(FM_ERR_INVALID, "topk_rows: null pointer");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* lp = static_cast<const __nv_bfloat16*>(logits);
  const auto* rm = reinterpret_cast<const long long*>(row_map);
  auto* io = reinterpret_cast<long long*>(ids);
  if (k <= 16)
    return launch_kernel(topk_rows_kernel<16>, dim3((unsigned)rows), dim3(BT), 0, s, false, lp, (long long)ld,
                         (int)cols, (int)k, rm, (long long)map_len, io, probs, err);
  return launch_kernel(topk_rows_kernel<32>, dim3((unsigned)rows), dim3(BT), 0, s, false, lp, (long long)ld,
                       (int)cols, (int)k, rm, (long long)map_len, io, probs, err);
}

extern "C" fm_status fm_bank_gather(const void* table, int64_t table_rows, int64_t cols, const int64_t* rows,
                                    int64_t n, void* out, int32_t* err, fm_stream stream) {
  if (n < 0 || cols < 1 || table_rows < 1) return set_error(FM_ERR_SHAPE, "bank_gather: bad shape");
  if (n == 0) return FM_OK;
  if (!table || !rows || !out) return set_error(FM_ERR_INVALID, "bank_gather: null pointer");
  return launch_kernel(bank_gather_kernel, dim3((unsigned)n), dim3(BT), 0, static_cast<cudaStream_t>(stream), false,
                       static_cast<const __nv_bfloat16*>(table), (long long)table_rows, (long long)cols,
                       reinterpret_cast<const long long*>(rows), static_cast<__nv_bfloat16*>(out), err);
}

extern "C" fm_status fm_bank_jump_rows(const fm_bank_jump* a, fm_stream stream) {
  if (!a) return set_error(FM_ERR_INVALID, "bank_jump_rows: null arguments");
  if (a->slots < 0 || a->hidden < 1 || a->support < 1 || a->support > BANK_MAX_SUPPORT || a->topk < 1 ||
      a->support % a->topk != 0 || a->bank_rows < 1 || a->state_rows < 1)
    return set_error(FM_ERR_SHAPE, "bank_jump_rows: bad shape (support <= %d, a multiple of topk)", BANK_MAX_SUPPORT);
  if (a->slots == 0) return FM_OK;
  if (!a->noise_embed || !a->mean_embed || !a->log_mass || !a->embed || !a->rows || !a->seeds || !a->ids ||
      !a->probs || !a->betas || !a->out)
    return set_error(FM_ERR_INVALID, "bank_jump_rows: null pointer");
  return launch_kernel(bank_jump_rows_kernel, dim3((unsigned)a->slots), dim3(BT), 0,
                       static_cast<cudaStream_t>(stream), false, *a);
}

extern "C" fm_status fm_token_normals(const int64_t* seeds, const int64_t* ids, int64_t rows, int64_t cols,
                                      float* out, fm_stream stream) {
  if (rows < 0 || cols < 0) return set_error(FM_ERR_SHAPE, "token_normals: bad shape");
  if (rows == 0 || cols == 0) return FM_OK;
  if (!seeds || !ids || !out) return set_error(FM_ERR_INVALID, "token_normals: null pointer");
  const long long n = rows * cols;
  return launch_kernel(token_normals_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), false, reinterpret_cast<const long long*>(seeds),
                       reinterpret_cast<const long long*>(ids), (long long)rows, (long long)cols, out);
}

extern "C" fm_status fm_philox_randint(int64_t* out, int64_t n, int64_t high, uint64_t seed, uint32_t offset,
                                       uint32_t purpose, fm_stream stream) {
  if (n < 0 || high < 1 || high > (int64_t)UINT32_MAX) return set_error(FM_ERR_SHAPE, "philox_randint: bad range");
  if (n == 0) return FM_OK;
  if (!out) return set_error(FM_ERR_INVALID, "philox_randint: null pointer");
  return launch_kernel(philox_randint_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), false, reinterpret_cast<long long*>(out), (long long)n,
                       (long long)high, seed, offset, purpose);
}
