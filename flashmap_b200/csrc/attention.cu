// Self- and cross-attention kernels of the FlashMap DiT (see attention.cuh).
#include "attention.cuh"
#include "launch.cuh"

namespace fm {

// ------------------------------------------------------------------ self-attention
// One CTA of 256 threads per (sequence, head).  q and k rows are padded by one
// float in shared memory so the per-pair dot products read distinct banks.
constexpr int SA_THREADS = 256;

__global__ void __launch_bounds__(SA_THREADS) self_attn_kernel(SelfAttnArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x / a.heads, h = blockIdx.x % a.heads;
  const int K = a.block, hd = a.head_dim, D = a.hidden, ld = hd + 1;
  extern __shared__ float sm[];
  float* sq = sm;
  float* sk = sq + K * ld;
  float* sv = sk + K * ld;
  float* sp = sv + K * hd;  // [K][K + 1]
  float* sl = sp + K * (K + 1);
  for (int idx = threadIdx.x; idx < K * hd / 2; idx += SA_THREADS) {
    const int i = (2 * idx) / hd, d = (2 * idx) % hd;
    const __nv_bfloat16* row = a.qkv + (long long)(b * K + i) * 3 * D + h * hd + d;
    const __nv_bfloat162 q2 = *reinterpret_cast<const __nv_bfloat162*>(row);
    const __nv_bfloat162 k2 = *reinterpret_cast<const __nv_bfloat162*>(row + D);
    const __nv_bfloat162 v2 = *reinterpret_cast<const __nv_bfloat162*>(row + 2 * D);
    sq[i * ld + d] = __low2float(q2);
    sq[i * ld + d + 1] = __high2float(q2);
    sk[i * ld + d] = __low2float(k2);
    sk[i * ld + d + 1] = __high2float(k2);
    sv[i * hd + d] = __low2float(v2);
    sv[i * hd + d + 1] = __high2float(v2);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < K * K; idx += SA_THREADS) {
    const int i = idx / K, j = idx % K;
    float acc = 0.0f;
    for (int d = 0; d < hd; ++d) acc = fmaf(sq[i * ld + d], sk[j * ld + d], acc);
    sp[i * (K + 1) + j] = __fmul_rn(acc, a.scale);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < K; i += SA_THREADS) {
    float m = -INFINITY;
    for (int j = 0; j < K; ++j) m = fmaxf(m, sp[i * (K + 1) + j]);
    float l = 0.0f;
    for (int j = 0; j < K; ++j) {
      const float e = expf(__fsub_rn(sp[i * (K + 1) + j], m));
      l = __fadd_rn(l, e);
      sp[i * (K + 1) + j] = round_bf(e);  // bf16 numerators, fp32 sum
    }
    sl[i] = l;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < K * hd; idx += SA_THREADS) {
    const int i = idx / hd, d = idx % hd;
    float acc = 0.0f;
    for (int j = 0; j < K; ++j) acc = fmaf(sp[i * (K + 1) + j], sv[j * hd + d], acc);
    a.out[(long long)(b * K + i) * D + h * hd + d] = f2bf(__fdiv_rn(acc, sl[i]));
  }
}

// Blocks of 16 slots with head_dim 64 or 128: one warp per (sequence, head) on
// the tensor cores (block_attn_head, attention.cuh).
constexpr int SA_MMA_WARPS = 4;

template <int HD>
__global__ void __launch_bounds__(SA_MMA_WARPS * 32) self_attn_mma_kernel(SelfAttnArgs a, int items) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(1024) uint8_t sa_smem[];
  constexpr int PART = 16 * HD * 2;  // one of q, k, v of a head
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int it = blockIdx.x * SA_MMA_WARPS + warp;
  if (it >= items) return;
  const int b = it / a.heads, h = it % a.heads, D = a.hidden;
  uint8_t* st = sa_smem + warp * 3 * PART;
  // q | k | v rows of this head into the swizzled layout
  for (int idx = lane; idx < 3 * 16 * (HD / 8); idx += 32) {
    const int part = idx / (16 * (HD / 8)), rem = idx % (16 * (HD / 8)), row = rem / (HD / 8), ch = rem % (HD / 8);
    const uint4 v = *reinterpret_cast<const uint4*>(a.qkv + (long long)(b * 16 + row) * 3 * D + part * D + h * HD + ch * 8);
    *reinterpret_cast<uint4*>(st + part * PART + blk_sw(row, ch)) = v;
  }
  __syncwarp();
  const uint32_t base = smem_u32(st);
  __nv_bfloat16* out = a.out + (long long)(b * 16) * D + h * HD;
  block_attn_head<HD>(base, base + PART, base + 2 * PART, a.scale, [&](int i, int d, float lo, float hi) {
    *reinterpret_cast<__nv_bfloat162*>(out + (long long)i * D + d) = __floats2bfloat162_rn(lo, hi);
  });
}

fm_status launch_self_attn(const SelfAttnArgs& a, int batch, cudaStream_t stream, bool pdl) {
  const int K = a.block, hd = a.head_dim;
  if (K == 16 && (hd == 64 || hd == 128)) {
    const int items = batch * a.heads;
    const unsigned grid = (unsigned)((items + SA_MMA_WARPS - 1) / SA_MMA_WARPS);
    const size_t smem = (size_t)SA_MMA_WARPS * 3 * 16 * hd * 2;
    static int configured = -1;
    int dev;
    cudaGetDevice(&dev);
    if (configured != dev) {
      cudaFuncSetAttribute(self_attn_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
      cudaFuncSetAttribute(self_attn_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
      configured = dev;
    }
    if (hd == 128)
      return launch_kernel(self_attn_mma_kernel<128>, dim3(grid), dim3(SA_MMA_WARPS * 32), smem, stream, pdl, a, items);
    return launch_kernel(self_attn_mma_kernel<64>, dim3(grid), dim3(SA_MMA_WARPS * 32), smem, stream, pdl, a, items);
  }
  const size_t smem = (size_t)(2 * K * (hd + 1) + K * hd + K * (K + 1) + K) * sizeof(float);
  if (smem > 200 * 1024) return set_error(FM_ERR_SHAPE, "self-attention block too large");
  if (hd % 2) return set_error(FM_ERR_SHAPE, "self-attention needs an even head_dim");
  static int configured = -1;
  int dev;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaFuncSetAttribute(self_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    configured = dev;
  }
  return launch_kernel(self_attn_kernel, dim3(batch * a.heads), dim3(SA_THREADS), smem, stream, pdl, a);
}

// ------------------------------------------------------------------ cross-attention
namespace {
constexpr int XA_STAGES = 3;
}  // namespace

template <int HD>
__global__ void __launch_bounds__(128) cross_attn_kernel(const __grid_constant__ CUtensorMap tm, CrossAttnArgs a) {
  constexpr int TILE_BYTES = XA_TILE * HD * 2;  // one of K or V
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + XA_STAGES * STAGE_BYTES);
  uint64_t* empty = full + XA_STAGES;
  int* sflag = reinterpret_cast<int*>(empty + XA_STAGES);
  float* mrg = reinterpret_cast<float*>(smem);  // reused after the pipeline: [4][16*HD] O, then m, l

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / a.nsplit, split = blockIdx.x % a.nsplit;
  const int b = bh / a.heads, h = bh % a.heads;

  if (threadIdx.x == 0) {
    for (int s = 0; s < XA_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    sflag[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm);
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  volatile int* abort_flag = sflag;

  int ctx = a.lengths[b] + 1;
  if (ctx > a.cache_len || ctx < 1) {
    if (threadIdx.x == 0) record_error(a.err, DEV_BAD_INDEX);
    ctx = ctx < 1 ? 1 : a.cache_len;
  }
  const int per = xa_split_keys(ctx, a.nsplit);
  const int k_begin = split * per;
  const int k_end = min(ctx, k_begin + per);
  if (k_begin >= ctx) return;  // no keys here; the merge counts only splits that own keys
  const int ntiles = (k_end - k_begin + XA_TILE - 1) / XA_TILE;
  const long long krow = ((((long long)a.layer * 2 + 0) * a.cache_batch + b) * a.heads + h) * a.cache_len;
  const long long vrow = ((((long long)a.layer * 2 + 1) * a.cache_batch + b) * a.heads + h) * a.cache_len;

  auto issue = [&](int t) {
    const int s = t % XA_STAGES;
    uint8_t* dst = smem + s * STAGE_BYTES;
    mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
    const int row = k_begin + t * XA_TILE;
#pragma unroll
    for (int bx = 0; bx < HD / 64; ++bx) {
      tma_load_2d(dst + bx * XA_TILE * 128, &tm, &full[s], bx * 64, (int)(krow + row));
      tma_load_2d(dst + TILE_BYTES + bx * XA_TILE * 128, &tm, &full[s], bx * 64, (int)(vrow + row));
    }
  };
  if (threadIdx.x == 0)
    for (int t = 0; t < XA_STAGES - 1 && t < ntiles; ++t) issue(t);

  // queries: A fragments for HD/16 k-steps
  uint32_t qa[HD / 16][4];
  {
    const __nv_bfloat16* qb = a.q + (long long)(b * 16) * a.hidden + h * HD;
    xa_load_q<HD>(qa, [&](int row, int col) {
      return *reinterpret_cast<const uint32_t*>(qb + (long long)row * a.hidden + col);
    });
  }
  XaAcc<HD> st;
  xa_init<HD>(st);

  int consumed = 0;
  for (int t = 0; t < ntiles; ++t) {
    if (threadIdx.x == 0) {
      const int tn = t + XA_STAGES - 1;
      if (tn < ntiles) {
        bool ok = true;
        if (tn >= XA_STAGES) ok = mbar_wait(&empty[tn % XA_STAGES], (uint32_t)(tn / XA_STAGES - 1) & 1u, abort_flag);
        if (ok) {
          issue(tn);
        } else {
          record_error(a.err, DEV_TIMEOUT_EMPTY);
          *abort_flag = 1;
        }
      }
    }
    const int s = t % XA_STAGES;
    if (!mbar_wait(&full[s], (uint32_t)(t / XA_STAGES) & 1u, abort_flag)) {
      record_error(a.err, DEV_TIMEOUT_FULL);
      *abort_flag = 1;
      break;
    }
    consumed = t + 1;
    const uint32_t kbase = smem_u32(smem + s * STAGE_BYTES);
    const int key0 = 16 * warp;  // this warp's 16 keys of the tile
    xa_tile<HD>(st, qa, kbase, kbase + TILE_BYTES, key0, k_begin + t * XA_TILE + key0, k_end, a.scale);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // issued tiles that were not consumed (only after an abort) must land first
  if (threadIdx.x == 0) {
    const int issued = min(ntiles, consumed + XA_STAGES - 1);
    for (int t = consumed; t < issued; ++t) mbar_wait(&full[t % XA_STAGES], (uint32_t)(t / XA_STAGES) & 1u, nullptr);
  }
  // the pipeline's shared memory is free after xa_finish's first barrier
  const int nsp = a.nsplit;
  const int n_active = (ctx + per - 1) / per;  // splits that own keys (the rest exit above)
  float* mine = a.part + (long long)(bh * nsp + split) * (16 * HD + 32);
  const float* base = a.part + (long long)bh * nsp * (16 * HD + 32);
  __nv_bfloat16* outp = a.out + (long long)(b * 16) * a.hidden + h * HD;
  const bool merged = xa_finish<HD>(
      st, mrg, threadIdx.x, n_active, mine, base, sflag + 1, [] { __syncthreads(); },
      [&] {
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(a.counters + bh) : "memory");
        return old == n_active - 1;
      },
      [&](int i, int d, float lo, float hi) {
        *reinterpret_cast<__nv_bfloat162*>(outp + (long long)i * a.hidden + d) = __floats2bfloat162_rn(lo, hi);
      });
  if (merged && n_active > 1 && threadIdx.x == 0) a.counters[bh] = 0;
}

size_t cross_attn_smem(int hd) {
  const size_t pipe = (size_t)XA_STAGES * 2 * XA_TILE * hd * 2;
  const size_t merge = (size_t)(4 * 16 * hd + 256) * sizeof(float);
  return 1024 + (pipe > merge ? pipe : merge) + 128;
}

fm_status launch_cross_attn(const CrossAttnArgs& a, const CUtensorMap& tm, cudaStream_t stream, bool pdl) {
  const size_t smem = cross_attn_smem(a.head_dim);
  const dim3 grid(a.batch * a.heads * a.nsplit);
  static int configured64 = -1, configured128 = -1;
  int dev;
  cudaGetDevice(&dev);
  if (a.head_dim == 128) {
    if (configured128 != dev) {
      cudaFuncSetAttribute(cross_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      configured128 = dev;
    }
    return launch_kernel(cross_attn_kernel<128>, grid, dim3(128), smem, stream, pdl, tm, a);
  }
  if (a.head_dim == 64) {
    if (configured64 != dev) {
      cudaFuncSetAttribute(cross_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      configured64 = dev;
    }
    return launch_kernel(cross_attn_kernel<64>, grid, dim3(128), smem, stream, pdl, tm, a);
  }
  return set_error(FM_ERR_UNSUPPORTED, "cross-attention supports head_dim 64 or 128");
}

}  // namespace fm
