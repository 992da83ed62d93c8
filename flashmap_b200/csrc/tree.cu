// Tree drafting's index work (flashmap/sglang/tree.py:9-78,
// flashmap/sglang/kernels.py:363-454), behind the C ABI:
//   * tree_build_kernel   one CTA per request: the trie of its N candidate
//                         blocks (a node per distinct prefix, its vote the
//                         number of candidates through it), the width - 1
//                         best-voted nodes (ties: shallower, then lower
//                         candidate) listed by depth then candidate, in
//                         EAGLE's encoding (id = parent * width + index)
//   * tree_commit_kernel  one CTA per request: the accepted path's KV slots
//                         to the front of its verify window in req_to_token,
//                         the path's tokens, bonus, commit and new lengths,
//                         and the context-injection slots
// Integer work only; every data-dependent index is checked.
#include "common.cuh"
#include "launch.cuh"

namespace fm {
namespace {

constexpr int TT = 256;
constexpr int TREE_MAX_CAND = 64, TREE_MAX_DEPTH = 64, TREE_MAX_SLOTS = 1024;

struct TreeSmem {
  long long cand[TREE_MAX_SLOTS];
  long long key[TREE_MAX_SLOTS];
  short common[TREE_MAX_CAND * TREE_MAX_CAND];
  short first[TREE_MAX_SLOTS];
  int node_of[TREE_MAX_SLOTS];  // 1-based node index of a kept slot, else 0
  int n_real, n_distinct, n_kept;
  long long token0;
};

__global__ void __launch_bounds__(TT) tree_build_kernel(const long long* candidates, int n, int k, int width,
                                                        long long* tokens, long long* ids, long long* stats) {
  extern __shared__ __align__(16) uint8_t tree_smem_raw[];
  TreeSmem& sm = *reinterpret_cast<TreeSmem*>(tree_smem_raw);
  const long long b = blockIdx.x;
  const int S = n * k, m = width - 1;
  if (threadIdx.x == 0) {
    sm.n_real = 0;
    sm.n_distinct = 0;
    sm.n_kept = 0;
  }
  for (int s = threadIdx.x; s < S; s += TT) {
    sm.cand[s] = candidates[b * S + s];
    sm.node_of[s] = 0;
  }
  __syncthreads();
  // common prefix length of every pair of candidates
  for (int p = threadIdx.x; p < n * n; p += TT) {
    const int i = p / n, j = p % n;
    int len = 0;
    while (len < k && sm.cand[i * k + len] == sm.cand[j * k + len]) ++len;
    sm.common[p] = (short)len;
  }
  __syncthreads();
  // per slot (i, d): votes, the lowest candidate with the prefix, the node key
  for (int s = threadIdx.x; s < S; s += TT) {
    const int i = s / k, d = s % k;
    int votes = 0, f = n;
    for (int j = 0; j < n; ++j)
      if (sm.common[i * n + j] > d) {
        ++votes;
        f = j < f ? j : f;
      }
    sm.first[s] = (short)f;
    const bool real = f == i;
    sm.key[s] = real ? (long long)votes * S + (long long)(k - 1 - d) * n + (n - 1 - i) : -1;
    if (real) {
      atomicAdd(&sm.n_real, 1);
      if (d == k - 1) atomicAdd(&sm.n_distinct, 1);
    }
  }
  __syncthreads();
  // kept: a real node among the m largest keys (real keys are distinct)
  for (int s = threadIdx.x; s < S; s += TT) {
    const long long ks = sm.key[s];
    if (ks < 0) continue;
    int rank = 0;
    for (int t = 0; t < S; ++t) rank += sm.key[t] > ks;
    if (rank < m) {
      sm.node_of[s] = 1;  // marked; numbered below
      atomicAdd(&sm.n_kept, 1);
    }
  }
  __syncthreads();
  // node index: position among the kept nodes ordered by (depth, candidate)
  int pos_of[TREE_MAX_SLOTS / TT];
#pragma unroll
  for (int r = 0; r < TREE_MAX_SLOTS / TT; ++r) {
    const int s = threadIdx.x + r * TT;
    pos_of[r] = -1;
    if (s >= S || !sm.node_of[s]) continue;
    const int os = (s % k) * n + s / k;
    int pos = 0;
    for (int t = 0; t < S; ++t)
      if (sm.node_of[t] && (t % k) * n + t / k < os) ++pos;
    pos_of[r] = pos;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < TREE_MAX_SLOTS / TT; ++r) {
    const int s = threadIdx.x + r * TT;
    if (s < S && pos_of[r] >= 0) sm.node_of[s] = pos_of[r] + 1;
  }
  __syncthreads();
  for (int s = threadIdx.x; s < S; s += TT) {
    const int idx = sm.node_of[s];
    if (!idx) continue;
    const int i = s / k, d = s % k;
    const int parent = d == 0 ? 0 : sm.node_of[sm.first[i * k + d - 1] * k + d - 1];
    tokens[b * m + idx - 1] = sm.cand[s];
    ids[b * m + idx - 1] = (long long)parent * width + idx;
    if (idx == 1) sm.token0 = sm.cand[s];
  }
  __syncthreads();
  for (int col = sm.n_kept + threadIdx.x; col < m; col += TT) {
    tokens[b * m + col] = sm.token0;
    ids[b * m + col] = col + 1;
  }
  if (threadIdx.x == 0) {
    stats[b * 2] = sm.n_real;
    stats[b * 2 + 1] = sm.n_distinct;
  }
}

__global__ void __launch_bounds__(TT) tree_commit_kernel(const int32_t* accept, const int32_t* num_correct,
                                                         const long long* window, const int32_t* predict,
                                                         const long long* req_pool, const long long* prefix,
                                                         int32_t* req_to_token, long long row_stride,
                                                         long long req_rows, int W, int D1, long long* out_tokens,
                                                         long long* bonus, int32_t* commit, long long* new_seq_lens,
                                                         long long* inject, int* err) {
  extern __shared__ __align__(16) uint8_t commit_smem_raw[];
  int* on_path = reinterpret_cast<int*>(commit_smem_raw);  // [W]
  int* path = on_path + W;                                  // [D1] node per path position, -1 past it
  const long long b = blockIdx.x;
  const int n = num_correct[b];
  for (int i = threadIdx.x; i < W; i += TT) on_path[i] = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < D1; j += TT) {
    int node = -1;
    if (j <= n) {
      node = (int)((long long)accept[b * D1 + j] - b * W);
      if (node >= W) {
        record_error(err, DEV_BAD_INDEX);
        node = -1;
      }
      if (node < 0) node = -1;
    }
    path[j] = node;
    if (node >= 0) atomicOr(&on_path[node], 1);
  }
  __syncthreads();
  const long long row = req_pool[b], base = prefix[b];
  const bool row_ok = row >= 0 && row < req_rows && base >= 0;
  if (!row_ok && threadIdx.x == 0) record_error(err, DEV_BAD_INDEX);
  int32_t* dst = req_to_token + row * row_stride + base;
  for (int j = threadIdx.x; j < D1; j += TT) {
    const int node = path[j];
    long long token = 0;
    if (node >= 0) {
      token = predict[b * W + node];
      if (row_ok && base + j < row_stride)
        dst[j] = (int32_t)window[b * W + node];
      else if (row_ok)
        record_error(err, DEV_BAD_INDEX);
    }
    out_tokens[b * D1 + j] = token;
    if (j == n) bonus[b] = token;
  }
  if (threadIdx.x == 0) {
    if (n >= D1) bonus[b] = 0;
    commit[b] = n + 1;
    new_seq_lens[b] = base + n + 1;
  }
  for (int i = threadIdx.x; i < W; i += TT) {
    const bool on = on_path[i] != 0;
    inject[b * W + i] = on ? window[b * W + i] : 0;
    if (on) continue;
    int rank = 0;  // off-path nodes before this one
    for (int t = 0; t < i; ++t) rank += on_path[t] == 0;
    const long long at = base + n + 1 + rank;
    if (row_ok && at < row_stride)
      req_to_token[row * row_stride + at] = (int32_t)window[b * W + i];
    else if (row_ok)
      record_error(err, DEV_BAD_INDEX);
  }
}

}  // namespace
}  // namespace fm

// ====================================================================== C ABI
using namespace fm;

extern "C" fm_status fm_tree_build(const int64_t* candidates, int64_t bs, int64_t n, int64_t k, int64_t width,
                                   int64_t* tokens, int64_t* ids, int64_t* stats, fm_stream stream) {
  if (bs < 0 || n < 1 || k < 1 || n > TREE_MAX_CAND || k > TREE_MAX_DEPTH || n * k > TREE_MAX_SLOTS || width < 2)
    return set_error(FM_ERR_SHAPE, "tree_build: need 1 <= N <= %d, 1 <= K <= %d, N*K <= %d, width >= 2",
                     TREE_MAX_CAND, TREE_MAX_DEPTH, TREE_MAX_SLOTS);
  if (bs == 0) return FM_OK;
  if (!candidates || !tokens || !ids || !stats) return set_error(FM_ERR_INVALID, "tree_build: null pointer");
  const size_t smem = sizeof(TreeSmem);
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(tree_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return set_error(FM_ERR_CUDA, "tree_build: cannot set shared memory size");
    attr = true;
  }
  return launch_kernel(tree_build_kernel, dim3((unsigned)bs), dim3(TT), smem, static_cast<cudaStream_t>(stream),
                       false, reinterpret_cast<const long long*>(candidates), (int)n, (int)k, (int)width,
                       reinterpret_cast<long long*>(tokens), reinterpret_cast<long long*>(ids),
                       reinterpret_cast<long long*>(stats));
}

extern "C" fm_status fm_tree_commit(const int32_t* accept, const int32_t* num_correct, const int64_t* window,
                                    const int32_t* predict, const int64_t* req_pool, const int64_t* prefix,
                                    int32_t* req_to_token, int64_t row_stride, int64_t req_rows, int64_t bs,
                                    int64_t width, int64_t depth1, int64_t* out_tokens, int64_t* bonus,
                                    int32_t* commit, int64_t* new_seq_lens, int64_t* inject_locs, int32_t* err,
                                    fm_stream stream) {
  if (bs < 0 || width < 1 || depth1 < 1 || width > 8192 || depth1 > 8192 || row_stride < 1 || req_rows < 1)
    return set_error(FM_ERR_SHAPE, "tree_commit: bad shape");
  if (bs == 0) return FM_OK;
  if (!accept || !num_correct || !window || !predict || !req_pool || !prefix || !req_to_token || !out_tokens ||
      !bonus || !commit || !new_seq_lens || !inject_locs)
    return set_error(FM_ERR_INVALID, "tree_commit: null pointer");
  const size_t smem = (size_t)(width + depth1) * sizeof(int);
  return launch_kernel(tree_commit_kernel, dim3((unsigned)bs), dim3(TT), smem, static_cast<cudaStream_t>(stream),
                       false, accept, num_correct, reinterpret_cast<const long long*>(window), predict,
                       reinterpret_cast<const long long*>(req_pool), reinterpret_cast<const long long*>(prefix),
                       req_to_token, (long long)row_stride, (long long)req_rows, (int)width, (int)depth1,
                       reinterpret_cast<long long*>(out_tokens), reinterpret_cast<long long*>(bonus), commit,
                       reinterpret_cast<long long*>(new_seq_lens), reinterpret_cast<long long*>(inject_locs), err);
}
