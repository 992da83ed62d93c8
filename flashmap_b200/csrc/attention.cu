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

constexpr int XA_TILE = 64;  // keys per pipeline stage
constexpr int XA_STAGES = 3;

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

}  // namespace

template <int HD>
__global__ void __launch_bounds__(128) cross_attn_kernel(const __grid_constant__ CUtensorMap tm, CrossAttnArgs a) {
  constexpr int TILE_BYTES = XA_TILE * HD * 2;  // one of K or V
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  constexpr int NT = HD / 8;  // n8 tiles over head dims
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + XA_STAGES * STAGE_BYTES);
  uint64_t* empty = full + XA_STAGES;
  int* sflag = reinterpret_cast<int*>(empty + XA_STAGES);
  float* mrg = reinterpret_cast<float*>(smem);  // reused after the pipeline: [4][16*HD] O, then m, l

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
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
  const int per = ((((ctx + a.nsplit - 1) / a.nsplit) + XA_TILE - 1) / XA_TILE) * XA_TILE;
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
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const int c = ks * 16 + tig * 2;
      qa[ks][0] = *reinterpret_cast<const uint32_t*>(qb + (long long)gid * a.hidden + c);
      qa[ks][1] = *reinterpret_cast<const uint32_t*>(qb + (long long)(gid + 8) * a.hidden + c);
      qa[ks][2] = *reinterpret_cast<const uint32_t*>(qb + (long long)gid * a.hidden + c + 8);
      qa[ks][3] = *reinterpret_cast<const uint32_t*>(qb + (long long)(gid + 8) * a.hidden + c + 8);
    }
  }
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

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
    const uint32_t vbase = kbase + TILE_BYTES;
    const int key0 = 16 * warp;  // this warp's 16 keys of the tile

    // S = Q K^T for keys key0 .. key0+15 (two n8 tiles)
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
    // scale, mask, online softmax (rows gid and gid+8)
    const int kabs = k_begin + t * XA_TILE + key0;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool valid = kabs + nt * 8 + tig * 2 + e < k_end;
        sc[nt][e] = valid ? __fmul_rn(sc[nt][e], a.scale) : -INFINITY;
        sc[nt][2 + e] = valid ? __fmul_rn(sc[nt][2 + e], a.scale) : -INFINITY;
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
    pa[0] = pack_bf16(p[0][0], p[0][1]);
    pa[1] = pack_bf16(p[0][2], p[0][3]);
    pa[2] = pack_bf16(p[1][0], p[1][1]);
    pa[3] = pack_bf16(p[1][2], p[1][3]);
    // O += P V over the 16 keys
    const int vr = key0 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int dn = 0; dn < NT; dn += 2) {
      uint32_t r0, r1, r2, r3;
      ldsm_x4_t(vbase + sw128_offset(vr, dn + (lane >> 4)), r0, r1, r2, r3);
      mma_bf16_16816(o[dn], pa, r0, r1);
      mma_bf16_16816(o[dn + 1], pa, r2, r3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // issued tiles that were not consumed (only after an abort) must land first
  if (threadIdx.x == 0) {
    const int issued = min(ntiles, consumed + XA_STAGES - 1);
    for (int t = consumed; t < issued; ++t) mbar_wait(&full[t % XA_STAGES], (uint32_t)(t / XA_STAGES) & 1u, nullptr);
  }
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 1));
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 2));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 1));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 2));
  __syncthreads();  // pipeline smem is free from here on

  // merge the 4 warps: mO[w][16][HD], mM / mL [4][16], then per-row weights
  float* mO = mrg;
  float* mM = mrg + 4 * 16 * HD;
  float* mL = mM + 64;
  float* mF = mL + 64;   // [4][16] exp(m_w - m)
  float* mR = mF + 64;   // [16] merged m, [16] merged l
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
  const int nsp = a.nsplit;
  const int n_active = (ctx + per - 1) / per;  // splits that own keys (the rest exit above)
  float* mine = a.part + (long long)(bh * nsp + split) * (16 * HD + 32);
  // each thread: 4 consecutive dims of one row per step (float4)
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
    if (n_active == 1) {
      const float ll = mR[16 + i];
      __nv_bfloat16* dst = a.out + (long long)(b * 16 + i) * a.hidden + h * HD + d;
      *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(__fdiv_rn(acc.x, ll), __fdiv_rn(acc.y, ll));
      *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __floats2bfloat162_rn(__fdiv_rn(acc.z, ll), __fdiv_rn(acc.w, ll));
    } else {
      __stcg(reinterpret_cast<float4*>(mine + i * HD + d), acc);
    }
  }
  if (n_active == 1) return;
  if (threadIdx.x < 16) {
    __stcg(mine + 16 * HD + threadIdx.x, mR[threadIdx.x]);
    __stcg(mine + 16 * HD + 16 + threadIdx.x, mR[16 + threadIdx.x]);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(a.counters + bh, 1);
    sflag[1] = (old == n_active - 1);
  }
  __syncthreads();
  if (!sflag[1]) return;
  __threadfence();
  // last split of this (sequence, head): merge all splits in split order
  const float* base = a.part + (long long)bh * nsp * (16 * HD + 32);
  float* sF = mO;  // reuse: [n_active][16] weights, then [16] l
  for (int t = threadIdx.x; t < 16; t += 128) {
    float mm = -INFINITY;
    for (int sp = 0; sp < n_active; ++sp) mm = fmaxf(mm, __ldcg(base + (long long)sp * (16 * HD + 32) + 16 * HD + t));
    float ll = 0.0f;
    for (int sp = 0; sp < n_active; ++sp) {
      const float* ps = base + (long long)sp * (16 * HD + 32);
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
      const float4 t = __ldcg(reinterpret_cast<const float4*>(base + (long long)sp * (16 * HD + 32) + i * HD + d));
      const float f = sF[sp * 16 + i];
      acc.x = __fadd_rn(acc.x, __fmul_rn(t.x, f));
      acc.y = __fadd_rn(acc.y, __fmul_rn(t.y, f));
      acc.z = __fadd_rn(acc.z, __fmul_rn(t.z, f));
      acc.w = __fadd_rn(acc.w, __fmul_rn(t.w, f));
    }
    const float ll = sF[n_active * 16 + i];
    __nv_bfloat16* dst = a.out + (long long)(b * 16 + i) * a.hidden + h * HD + d;
    *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(__fdiv_rn(acc.x, ll), __fdiv_rn(acc.y, ll));
    *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __floats2bfloat162_rn(__fdiv_rn(acc.z, ll), __fdiv_rn(acc.w, ll));
  }
  if (threadIdx.x == 0) a.counters[bh] = 0;
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
