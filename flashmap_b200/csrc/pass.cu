// Persistent single-launch draft pass (see pass.cuh).
//
// CTA roles (256 threads, one CTA per SM, cooperative launch):
//   warp 0      TMA producer: every weight tile of every GEMM stage, in stage
//               order, through an NA-slot ring; it never waits on a grid
//               barrier, so the next stage's weights stream during the barrier.
//   warp 1      tcgen05 MMA issuer and TMEM owner: pairs ring slots with the
//               stage's B operand in shared memory, accumulates in TMEM.
//   warps 2-7   workers: wait for a stage's inputs (grid barrier), build its B
//               operand, run the epilogues (warps 2-5 own the TMEM lane
//               quarters), run the cross-attention stages, arrive.
//
// Named barriers: 1 = epilogue warps 2-5 (inside epilogue16), 2 = the six
// worker warps, 3 = the cross-attention warps 2-5.  Every branch around a
// named barrier is uniform over the threads that use it: outcomes of waits
// are published through shared flags and read after a barrier.
//
// Numerics equal the multi-kernel path bit for bit: the same GEMM unit split
// (grid = SM count) and epilogues (gemm.cuh), the row statistics of rows.cuh,
// the self-attention of self_attn_kernel and the cross-attention of
// cross_attn_kernel (attention.cu), and the Philox normals of philox.cuh.
#include <algorithm>

#include "pass.cuh"
#include "philox.cuh"
#include "rows.cuh"

namespace fm {
namespace pass {

constexpr int THREADS = 256;
constexpr int NA = 5;                  // weight ring slots
constexpr int BNP = 16;                // block tokens (B rows)
constexpr int A_BYTES = 128 * 64 * 2;  // 16 KB weight tile
constexpr int B_SLOT = BNP * 64 * 2;   // 2 KB activation k-block
constexpr int B_SLOTS = 64;            // K up to 4096 per CTA range
constexpr int B_REGION = B_SLOTS * B_SLOT;
constexpr int BAR_BYTES = 256;
constexpr int FLAG_BYTES = 128;
constexpr int XCH_BYTES = 4096;  // epilogue exchange: 64 x 16 floats (SwiGLU) or 64 keys
constexpr int STAT_BYTES = 1024;
constexpr int STAGE_BYTES = 768;  // this CTA's copy of the current stage descriptor
constexpr int MAX_STAGES = 96;
constexpr int LITE_BYTES = MAX_STAGES * 32;  // the fields the producer and MMA warps read, every stage
constexpr int ROPE_BYTES = 16 * 64 * 2 * 4;   // rotary factors of the 16 slot positions, head_dim <= 128
constexpr int SMEM =
    1024 + NA * A_BYTES + B_REGION + BAR_BYTES + FLAG_BYTES + XCH_BYTES + STAT_BYTES + STAGE_BYTES + LITE_BYTES +
    ROPE_BYTES;
constexpr int TMEM_COLS = 32;
constexpr int WORKERS = 192;  // warps 2..7
constexpr int XA_TILE = 64;
constexpr int XA_STAGES = 2;
constexpr uint32_t PF_TILES = 24;
constexpr int TRACE_SLOTS = 14;  // per stage and CTA: start, inputs ready, loads issued, loads landed, operand
                                 // built, first epilogue done, last epilogue done, arrived, statistics done,
                                 // transform done; split-tile owner: contributors in, partials in, summed,
                                 // epilogue done  // weight tiles a CTA keeps requested into L2 ahead of its loads
static_assert(sizeof(Stage) <= STAGE_BYTES && sizeof(Stage) % 16 == 0, "stage slot");

struct StageLite {
  long long units;
  int type, kb, tmap, bsrc, fmap, full;
};
static_assert(sizeof(StageLite) == 32, "lite stage");
static_assert(SMEM <= 227 * 1024, "shared memory");

// flags
constexpr int F_ABORT = 0, F_SPLIT_LAST = 1, F_SEG = 2 /* 2..3 */, F_XA_LAST = 4, F_GRID = 5, F_STAGE_OK = 6,
              F_BFREE = 7, F_BLOAD = 8, F_BLOAD_OK = 9, F_FIX = 10, F_NHEADS = 11;

struct Smem {
  uint8_t* A;
  uint8_t* B;
  uint64_t *a_full, *a_empty, *acc_full, *acc_empty, *b_ready, *b_free, *xa_full, *xa_empty, *b_load, *fix;
  uint32_t* tmem_slot;
  int* flags;
  float* xch;
  unsigned long long* xch64;
  float* stats;  // [0..15] mean, [16..32] 1/std or 1/rms of up to 17 rows
  Stage* stage;
  StageLite* lite;
  float* rope;  // [2][16][head_dim / 2]: cos then sin of the slot positions
};

__device__ __forceinline__ Smem carve_smem(uint8_t* raw) {
  uint8_t* s = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  Smem m;
  m.A = s;
  m.B = s + NA * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(m.B + B_REGION);
  m.a_full = bars;
  m.a_empty = m.a_full + NA;
  m.acc_full = m.a_empty + NA;
  m.acc_empty = m.acc_full + 2;
  m.b_ready = m.acc_empty + 2;
  m.b_free = m.b_ready + 1;
  m.xa_full = m.b_free + 1;
  m.xa_empty = m.xa_full + XA_STAGES;
  m.b_load = m.xa_empty + XA_STAGES;
  m.fix = m.b_load + 1;
  uint8_t* after = m.B + B_REGION + BAR_BYTES;
  m.tmem_slot = reinterpret_cast<uint32_t*>(after);
  m.flags = reinterpret_cast<int*>(after + 16);
  m.xch = reinterpret_cast<float*>(after + FLAG_BYTES);
  m.xch64 = reinterpret_cast<unsigned long long*>(m.xch);
  m.stats = reinterpret_cast<float*>(after + FLAG_BYTES + XCH_BYTES);
  m.stage = reinterpret_cast<Stage*>(after + FLAG_BYTES + XCH_BYTES + STAT_BYTES);
  m.lite = reinterpret_cast<StageLite*>(after + FLAG_BYTES + XCH_BYTES + STAT_BYTES + STAGE_BYTES);
  m.rope = reinterpret_cast<float*>(after + FLAG_BYTES + XCH_BYTES + STAT_BYTES + STAGE_BYTES + LITE_BYTES);
  return m;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ void give_up(const PassArgs& P, volatile int* sabort, int code) {
  *sabort = 1;
  atomicExch(P.abort, 1);
  record_error(P.err, code);
}

// one thread: spin (bounded) until `target` arrivals were counted
__device__ bool grid_wait(const PassArgs& P, unsigned long long target, volatile int* sabort) {
  if (ld_acquire_u64(P.bar_count) >= target) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_u64(P.bar_count) >= target) return true;
    if ((i & 15u) == 0) {
      if (*sabort || *reinterpret_cast<volatile int*>(P.abort)) return false;
      if (global_ns() - t0 > FM_WAIT_NS) {
        give_up(P, sabort, DEV_TIMEOUT_OTHER);
        return false;
      }
    }
  }
}

// Every asynchronous copy of the pass is checked before it is issued: 16-byte
// aligned addresses and sizes, a tile's innermost coordinate on a 16-byte
// boundary, and a shared-memory destination inside [lo, hi).  A copy that
// fails is recorded (DEV_BAD_COPY) and skipped; the wait that expects its
// bytes then runs out and reports too.
__device__ __forceinline__ bool copy_checked(const PassArgs& P, const void* dst, uint32_t bytes, const void* lo,
                                             const void* hi, const void* src, int x) {
  const uintptr_t d = reinterpret_cast<uintptr_t>(dst);
  const bool ok = (d & 15) == 0 && bytes > 0 && (bytes & 15) == 0 && d >= reinterpret_cast<uintptr_t>(lo) &&
                  d + bytes <= reinterpret_cast<uintptr_t>(hi) && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                  ((x * 2) & 15) == 0;
  if (!ok) record_error(P.err, DEV_BAD_COPY);
  return ok;
}

// one thread: spin (bounded) until *counter reaches target
__device__ bool wait_count(const int* counter, int target, volatile int* sabort) {
  if (ld_acquire_s32(counter) >= target) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_s32(counter) >= target) return true;
    if ((i & 15u) == 0) {
      if (*sabort) return false;
      if (global_ns() - t0 > FM_WAIT_NS) return false;
    }
  }
}

__device__ __forceinline__ uint32_t b_offset(int r, int chunk) { return (uint32_t)(r * 128 + ((chunk ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint4 pack8(const float* v) {
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

__device__ __forceinline__ void unpack8(const __nv_bfloat16* p, float* x) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// ------------------------------------------------------------------ B operand (workers)
//
// The B region during a GEMM stage starts with the operand: nk slots of 2 KB,
// rows of 64 bf16 128-byte swizzled as TMA writes and the MMA reads them.
// Slot j holds k-block (k0 + j) mod kb ("compact"), except for a CTA of a
// copy stage that needs every k-block, which gets them in place (slot k) from
// one TMA.  Inputs arrive asynchronously, all issued at once by one thread:
//   copy        the k-blocks of the source rows (TMA)
//   AdaLN       whole input rows staged at the end of the region (one TMA)
//               and scale|shift (one bulk copy): statistics and the
//               transform read shared memory only; or, when the rows do not
//               fit, the CTA's k-blocks plus statistics from global loads
//   RMSNorm /   the single input row and the norm weight (bulk copies)
//   gather
//   mix_state   the CTA's k-blocks of z L^T (TMA), the segments of the three
//               per-column vectors (bulk copies), statistics from global loads
//   self-attn.  q|k|v of every head the k-range touches (one TMA per part)
// so an operand costs about one memory round trip.  After the build, the
// region past the operand takes the split-K partials of the fix-ups.

__device__ __host__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
// staged whole rows of an AdaLN stage and its scale|shift, at the region's end
__device__ __host__ inline size_t adaln_full_bytes(int K) { return (size_t)BNP * K * 2 + (size_t)2 * K * 2; }
// mix_state parameter segments (3 vectors of nk x 64)
__device__ __host__ inline size_t mix_param_bytes(int nk) { return (size_t)3 * nk * 128; }
// a single staged row and its norm weight
__device__ __host__ inline size_t row_stage_bytes(int K) { return align_up((size_t)K * 2, 128) * 2; }
// self-attention: staged heads (q|k|v, bf16)
__device__ __host__ inline size_t selfattn_bytes(int heads_touched, int hd) {
  return (size_t)heads_touched * 3 * BNP * hd * 2;
}

// element d of row i of a [16 x 64 * blocks] staged block group
__device__ __forceinline__ float staged_at(const uint8_t* base, int i, int d) {
  const int box = d >> 6, dd = d & 63;
  const uint32_t off = (uint32_t)(box * B_SLOT + i * 128 + ((((dd >> 3) ^ (i & 7))) << 4) + (dd & 7) * 2);
  return __uint_as_float(((uint32_t)(*reinterpret_cast<const uint16_t*>(base + off))) << 16);
}
// 8 elements (chunk ch of k-block k) of row i of a staged block group
__device__ __forceinline__ uint4 staged_chunk(const uint8_t* base, int i, int k, int ch) {
  return *reinterpret_cast<const uint4*>(base + k * B_SLOT + b_offset(i, ch));
}

// bulk copies of elements [e0, e0 + n) of a vector, in runs that do not wrap
__device__ __forceinline__ uint32_t copy_segments(const PassArgs* P, const Smem* sm, uint8_t* dst,
                                                  const __nv_bfloat16* vec, int K, int kb, int k0, int nk,
                                                  uint64_t* bar, bool issue) {
  uint32_t bytes = 0;
  int j = 0;
  while (j < nk) {
    const int k = (k0 + j) % kb;
    const int run = min(nk - j, kb - k);
    const uint32_t b = (uint32_t)((min(K, (k + run) * 64) - k * 64) * 2);
    if (issue && copy_checked(*P, dst + (size_t)j * 128, b, sm->B, sm->B + B_REGION, vec + (size_t)k * 64, 0))
      bulk_load(dst + (size_t)j * 128, vec + (size_t)k * 64, b, bar);
    bytes += b;
    j += run;
  }
  return bytes;
}

struct BMode {
  bool inplace;   // copy stage, every k-block in slot k
  bool staged;    // AdaLN with whole rows staged
};

__device__ __forceinline__ BMode b_mode(int bsrc, int fmap, int full, int kb, int nk) {
  BMode m;
  m.inplace = bsrc == BS_COPY && fmap >= 0 && nk == kb;
  m.staged = bsrc == BS_ADALN && full;
  return m;
}

// One thread: issue every asynchronous copy of this stage's operand inputs;
// returns the bytes expected on b_load (0: nothing issued).
__device__ uint32_t issue_b_loads(const Stage& S, const PassArgs& P, const Smem& sm, int K, int kb, int k0, int nk,
                                  BMode md, const int* heads, int nh) {
  const CUtensorMap* smap = S.smap >= 0 ? P.tmaps + S.smap : nullptr;
  const CUtensorMap* fmap = S.fmap >= 0 ? P.tmaps + S.fmap : nullptr;
  uint8_t* tail = sm.B + B_REGION;  // staged inputs grow down from the region's end
  uint32_t total = 0;
  // the byte count first (the barrier's transaction count), then the copies
  if (md.inplace) {
    total = (uint32_t)kb * B_SLOT;
  } else if (md.staged) {
    total = (uint32_t)(BNP * K * 2 + 2 * K * 2);
  } else if (S.bsrc == BS_COPY || S.bsrc == BS_ADALN || S.bsrc == BS_MIX) {
    total = (uint32_t)nk * B_SLOT;
    if (S.bsrc == BS_ADALN) total += 2 * copy_segments(&P, &sm, nullptr, S.mod, K, kb, k0, nk, nullptr, false);
    if (S.bsrc == BS_MIX) total += 3 * copy_segments(&P, &sm, nullptr, S.aux, K, kb, k0, nk, nullptr, false);
  } else if (S.bsrc == BS_RMSROW || S.bsrc == BS_GATHER) {
    total = (uint32_t)(K * 2) * (S.bsrc == BS_RMSROW ? 2 : 1);
  } else if (S.bsrc == BS_SELFATTN) {
    total = (uint32_t)nh * 3 * (S.head_dim / 64) * B_SLOT;
  }
  if (total == 0) return 0;
  if (smap) tmap_acquire(smap);
  if (fmap) tmap_acquire(fmap);
  fence_async_global();  // inputs written by other CTAs' generic stores, read by the async proxy
  mbar_arrive_expect_tx(sm.b_load, total);
  const uint8_t* lo = sm.B;
  const uint8_t* hi = sm.B + B_REGION;
  if (md.inplace) {
    if (copy_checked(P, sm.B, (uint32_t)kb * B_SLOT, lo, hi, nullptr, 0)) tma_load_3d(sm.B, fmap, sm.b_load, 0, 0, 0);
  } else if (md.staged) {
    uint8_t* rows = tail - (size_t)BNP * K * 2;
    if (copy_checked(P, rows, (uint32_t)(BNP * K * 2), lo, hi, nullptr, 0)) tma_load_3d(rows, fmap, sm.b_load, 0, 0, 0);
    if (copy_checked(P, rows - (size_t)2 * K * 2, (uint32_t)(2 * K * 2), lo, hi, S.mod, 0))
      bulk_load(rows - (size_t)2 * K * 2, S.mod, (uint32_t)(2 * K * 2), sm.b_load);
  } else if (S.bsrc == BS_COPY || S.bsrc == BS_ADALN || S.bsrc == BS_MIX) {
    for (int j = 0; j < nk; ++j)
      if (copy_checked(P, sm.B + j * B_SLOT, B_SLOT, lo, hi, nullptr, ((k0 + j) % kb) * 64))
        tma_load_2d(sm.B + j * B_SLOT, smap, sm.b_load, ((k0 + j) % kb) * 64, 0);
    uint8_t* parm = sm.B + (size_t)nk * B_SLOT;
    if (S.bsrc == BS_ADALN) {
      copy_segments(&P, &sm, parm, S.mod, K, kb, k0, nk, sm.b_load, true);
      copy_segments(&P, &sm, parm + (size_t)nk * 128, S.mod + K, K, kb, k0, nk, sm.b_load, true);
    } else if (S.bsrc == BS_MIX) {
      copy_segments(&P, &sm, parm, S.aux, K, kb, k0, nk, sm.b_load, true);
      copy_segments(&P, &sm, parm + (size_t)nk * 128, S.w0, K, kb, k0, nk, sm.b_load, true);
      copy_segments(&P, &sm, parm + (size_t)2 * nk * 128, S.w1, K, kb, k0, nk, sm.b_load, true);
    }
  } else if (S.bsrc == BS_RMSROW || S.bsrc == BS_GATHER) {
    const size_t rb = align_up((size_t)K * 2, 128);
    const __nv_bfloat16* row = S.src;
    if (S.bsrc == BS_GATHER) {
      long long id = P.anchor_ids[0];
      if (id < 0 || id >= P.vocab) id = 0;  // recorded as DEV_BAD_INDEX by the prep step
      row = S.aux + id * K;
    }
    if (copy_checked(P, tail - rb, (uint32_t)(K * 2), lo, hi, row, 0)) bulk_load(tail - rb, row, (uint32_t)(K * 2), sm.b_load);
    if (S.bsrc == BS_RMSROW && copy_checked(P, tail - 2 * rb, (uint32_t)(K * 2), lo, hi, S.w0, 0))
      bulk_load(tail - 2 * rb, S.w0, (uint32_t)(K * 2), sm.b_load);
  } else if (S.bsrc == BS_SELFATTN) {
    const int bx = S.head_dim / 64, D = S.heads * S.head_dim;
    uint8_t* st = sm.B + align_up((size_t)nk * B_SLOT, 1024);
    for (int i = 0; i < nh; ++i)
      for (int part = 0; part < 3; ++part)
        if (copy_checked(P, st + (size_t)(i * 3 + part) * bx * B_SLOT, (uint32_t)bx * B_SLOT, lo, hi, nullptr, 0))
          tma_load_3d(st + (size_t)(i * 3 + part) * bx * B_SLOT, fmap, sm.b_load, 0, 0,
                      (part * D + heads[i] * S.head_dim) / 64);
  }
  return total;
}

// Build the stage's B operand (all 192 workers).  Returns the bytes of the
// region that stay in use while the stage's MMAs run.
__device__ size_t build_b(const Stage& S, const PassArgs& P, const Smem& sm, int K, int kb, int k0, int nk, int wt,
                          uint32_t noise_off, uint32_t& bl_phase, volatile int* sabort, unsigned long long* ts) {
  float* stats = sm.stats;
  const int wid = wt >> 5, lane = wt & 31;
  const BMode md = b_mode(S.bsrc, S.fmap, S.full, kb, nk);
  uint8_t* tail = sm.B + B_REGION;
  // self-attention: the heads the k-range touches, in order (heads[]), and
  // each slot's index into that list (slot_head[])
  int* heads = reinterpret_cast<int*>(sm.stats + 64);
  int* slot_head = reinterpret_cast<int*>(sm.stats + 128);
  int nh = 0;
  if (S.bsrc == BS_SELFATTN) {
    if (wt == 0) {
      int n = 0, cur = -1;
      for (int j = 0; j < nk; ++j) {
        const int h = (((k0 + j) % kb) * 64) / S.head_dim;
        if (h != cur) heads[n++] = h;
        cur = h;
        slot_head[j] = n - 1;
      }
      sm.flags[F_NHEADS] = n;
    }
    named_bar_sync(2, WORKERS);
    nh = sm.flags[F_NHEADS];
  }
  // 1. the asynchronous copies
  if (wt == 0) {
    sm.flags[F_BLOAD] = (int)issue_b_loads(S, P, sm, K, kb, k0, nk, md, heads, nh);
    if (ts) ts[2] = global_ns();
  }
  // 2. meanwhile: statistics from global memory, noise, zero rows
  if (S.bsrc == BS_ADALN && !md.staged) {
    for (int r = wid; r < S.ntok; r += WORKERS / 32) {
      float mean, rstd;
      warp_row_meanrstd_batched(S.src + (long long)r * S.ld, K, S.eps, lane, &mean, &rstd);
      if (lane == 0) {
        stats[r] = mean;
        stats[16 + r] = rstd;
      }
    }
  } else if (S.bsrc == BS_MIX) {
    for (int r = wid; r <= S.ntok; r += WORKERS / 32) {  // rows of z L^T, then the shared posterior row
      const __nv_bfloat16* row = r < S.ntok ? S.src + (long long)r * S.ld : S.aux;
      const float ss = warp_row_sumsq_batched(row, K, lane);
      if (lane == 0) stats[16 + r] = inv_rms(ss, K, S.eps);
    }
  }
  if (S.bsrc == BS_NOISE || S.bsrc == BS_RMSROW || S.bsrc == BS_GATHER) {
    // noise: all rows; single-row sources: rows 1..15 stay zero
    for (int item = wt; item < nk * 128; item += WORKERS) {
      const int j = item >> 7, rem = item & 127, r = rem >> 3, ch = rem & 7;
      const int k = (k0 + j) % kb;
      const int e0 = k * 64 + ch * 8;
      uint4 out = make_uint4(0u, 0u, 0u, 0u);
      if (S.bsrc == BS_NOISE && r < S.ntok && e0 < K) {
        if (P.z) {
          out = __ldcg(reinterpret_cast<const uint4*>(P.z + (long long)r * K + e0));
        } else {
          float v[8];
          const long long f0 = (long long)r * K + e0;
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) normal_pair(P.seed, noise_off, (f0 >> 1) + pp, v[2 * pp], v[2 * pp + 1]);
          out = pack8(v);
        }
      } else if (S.bsrc != BS_NOISE && r == 0) {
        continue;  // written below from the staged row
      }
      *reinterpret_cast<uint4*>(sm.B + j * B_SLOT + b_offset(r, ch)) = out;
    }
  }
  // 3. the copies landed
  named_bar_sync(2, WORKERS);
  const uint32_t bytes = (uint32_t)sm.flags[F_BLOAD];
  if (bytes) {
    if (wt == 0) {
      const bool ok = mbar_wait(sm.b_load, bl_phase & 1u, sabort);
      if (!ok) give_up(P, sabort, DEV_TIMEOUT_FULL);
      sm.flags[F_BLOAD_OK] = ok ? 1 : 0;
      if (ts) ts[3] = global_ns();
    }
    ++bl_phase;
    named_bar_sync(2, WORKERS);
    if (!sm.flags[F_BLOAD_OK]) return (size_t)B_REGION;
  }
  // 4. statistics from shared memory, then the transforms
  if (md.staged) {
    const uint8_t* rows = tail - (size_t)BNP * K * 2;
    const __nv_bfloat16* mod = reinterpret_cast<const __nv_bfloat16*>(rows - (size_t)2 * K * 2);
    // the warp's rows (wid, wid + 6, wid + 12) side by side: independent
    // accumulations, each in the canonical order of rows.cuh
    constexpr int RW = (BNP + WORKERS / 32 - 1) / (WORKERS / 32);
    const int nch = K / 8;
    int rr[RW];
    bool live[RW];
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      rr[i] = wid + i * (WORKERS / 32);
      live[i] = rr[i] < S.ntok;
      if (!live[i]) rr[i] = 0;
    }
    float sum[RW], mean[RW];
#pragma unroll
    for (int i = 0; i < RW; ++i) sum[i] = 0.0f;
    for (int ch = lane; ch < nch; ch += 32) {
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        float x[8];
        unpack_bf16x8(staged_chunk(rows, rr[i], ch >> 3, ch & 7), x);
        sum[i] = __fadd_rn(sum[i], chunk_tree(x, 8));
      }
    }
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      mean[i] = __fdiv_rn(warp_allsum(sum[i]), (float)K);
      sum[i] = 0.0f;
    }
    for (int ch = lane; ch < nch; ch += 32) {
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        float x[8], t[8];
        unpack_bf16x8(staged_chunk(rows, rr[i], ch >> 3, ch & 7), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = __fsub_rn(x[e], mean[i]);
          t[e] = __fmul_rn(d, d);
        }
        sum[i] = __fadd_rn(sum[i], chunk_tree(t, 8));
      }
    }
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      const float var = __fdiv_rn(warp_allsum(sum[i]), (float)K);
      if (lane == 0 && live[i]) {
        stats[rr[i]] = mean[i];
        stats[16 + rr[i]] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, S.eps)));
      }
    }
    named_bar_sync(2, WORKERS);
    if (ts && wt == 0) ts[8] = global_ns();
    for (int item = wt; item < nk * 128; item += WORKERS) {
      const int j = item >> 7, rem = item & 127, r = rem >> 3, ch = rem & 7;
      const int k = (k0 + j) % kb;
      float x[8], sc[8], sh[8], v[8];
      unpack_bf16x8(staged_chunk(rows, r, k, ch), x);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(mod + k * 64 + ch * 8), sc);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(mod + K + k * 64 + ch * 8), sh);
      const float mean = stats[r], rstd = stats[16 + r];
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = adaln_value(x[t], mean, rstd, sc[t], sh[t]);
      *reinterpret_cast<uint4*>(sm.B + j * B_SLOT + b_offset(r, ch)) = pack8(v);
    }
    if (ts && wt == 0) ts[9] = global_ns();
    return (size_t)nk * B_SLOT;
  }
  if (S.bsrc == BS_RMSROW || S.bsrc == BS_GATHER) {
    const size_t rb = align_up((size_t)K * 2, 128);
    const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(tail - rb);
    const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(tail - 2 * rb);
    if (S.bsrc == BS_RMSROW) {
      if (wid == 0) {
        const float inv = inv_rms(warp_row_sumsq(row, K, lane), K, S.eps);
        if (lane == 0) stats[16] = inv;
      }
      named_bar_sync(2, WORKERS);
    }
    for (int item = wt; item < nk * 8; item += WORKERS) {
      const int j = item >> 3, ch = item & 7;
      const int e0 = ((k0 + j) % kb) * 64 + ch * 8;
      uint4 out = make_uint4(0u, 0u, 0u, 0u);
      if (e0 < K) {
        out = *reinterpret_cast<const uint4*>(row + e0);
        if (S.bsrc == BS_RMSROW) {
          float x[8], wv[8], v[8];
          unpack_bf16x8(out, x);
          unpack_bf16x8(*reinterpret_cast<const uint4*>(w + e0), wv);
#pragma unroll
          for (int t = 0; t < 8; ++t) v[t] = rms_value(x[t], wv[t], stats[16]);
          out = pack8(v);
        }
      }
      *reinterpret_cast<uint4*>(sm.B + j * B_SLOT + b_offset(0, ch)) = out;
    }
    return (size_t)nk * B_SLOT;
  }
  if (S.bsrc == BS_ADALN || S.bsrc == BS_MIX) {
    const uint8_t* parm = sm.B + (size_t)nk * B_SLOT;
    for (int item = wt; item < nk * 128; item += WORKERS) {
      const int j = item >> 7, rem = item & 127, r = rem >> 3, ch = rem & 7;
      const int k = (k0 + j) % kb;
      if (k * 64 + ch * 8 >= K) continue;  // zero fill from the copy
      uint4* slot = reinterpret_cast<uint4*>(sm.B + j * B_SLOT + b_offset(r, ch));
      float x[8], v[8], p0[8], p1[8];
      unpack_bf16x8(*slot, x);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(parm + j * 128 + ch * 16), p0);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(parm + (size_t)nk * 128 + j * 128 + ch * 16), p1);
      if (S.bsrc == BS_ADALN) {
        const float mean = stats[r], rstd = stats[16 + r];
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = adaln_value(x[t], mean, rstd, p0[t], p1[t]);
      } else {
        float p2[8];
        unpack_bf16x8(*reinterpret_cast<const uint4*>(parm + (size_t)2 * nk * 128 + j * 128 + ch * 16), p2);
        const float ip = stats[16 + S.ntok], is = stats[16 + r];
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = mix_value(p0[t], x[t], p1[t], p2[t], ip, is, S.gate);
      }
      *slot = pack8(v);
    }
    return (size_t)nk * B_SLOT + (S.bsrc == BS_MIX ? mix_param_bytes(nk) : (size_t)2 * nk * 128);
  }
  if (S.bsrc == BS_SELFATTN) {
    // one warp per touched head, on the tensor cores (block_attn_head,
    // attention.cuh, as the kernel sequence computes it); each writes the
    // columns of its head that fall in this CTA's k-range into their slots
    const int hd = S.head_dim, bx = hd / 64;
    const uint8_t* st = sm.B + align_up((size_t)nk * B_SLOT, 1024);
    for (int hi = wid; hi < nh; hi += WORKERS / 32) {
      const uint32_t q = smem_u32(st + (size_t)(hi * 3 + 0) * bx * B_SLOT);
      const int h = heads[hi];
      auto store = [&](int i, int d, float lo, float hi2) {
        const int k = (h * hd + d) >> 6;
        const int j = (k - k0 + kb) % kb;
        if (j >= nk) return;
        const int dd = d & 63;
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi2);
        *reinterpret_cast<__nv_bfloat162*>(sm.B + j * B_SLOT + b_offset(i, dd >> 3) + (dd & 7) * 2) = v;
      };
      if (hd == 128)
        block_attn_head<128>(q, q + bx * B_SLOT, q + 2 * bx * B_SLOT, S.scale, store);
      else
        block_attn_head<64>(q, q + bx * B_SLOT, q + 2 * bx * B_SLOT, S.scale, store);
    }
    if (ts && wt == 0) ts[9] = global_ns();
    return (size_t)nk * B_SLOT;
  }
  return md.inplace ? (size_t)kb * B_SLOT : (size_t)nk * B_SLOT;
}

// ------------------------------------------------------------------ cross-attention (warps 2-5)

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t packbf(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t xa_sw128(int row, int chunk) {
  const int box = chunk >> 3, cin = chunk & 7;
  return (uint32_t)(box * (XA_TILE * 128) + row * 128 + ((cin ^ (row & 7)) << 4));
}
// one lane waits, the warp shares the outcome (keeps the warp converged)
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* sabort) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, sabort) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// One (sequence-head, split) item of the cross-attention of layer `layer`:
// cross_attn_kernel (attention.cu) run by warps 2-5 of a persistent CTA.  The
// K/V tiles go through a 2-stage TMA ring counted across items by `xt`.
template <int HD>
__device__ void xattn_item(const PassArgs& P, const Smem& sm, int layer, int bh, int split, int t, uint32_t& xt,
                           volatile int* sabort) {
  constexpr int TILE_BYTES = XA_TILE * HD * 2;
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  constexpr int NT = HD / 8;
  const CrossAttnArgs& a = P.xa;
  const int warp = t >> 5, lane = t & 31, gid = lane >> 2, tig = lane & 3;
  const int b = bh / a.heads, h = bh % a.heads;
  uint8_t* stage_base = sm.B;
  float* mrg = reinterpret_cast<float*>(sm.B + XA_STAGES * STAGE_BYTES);
  int ctx = a.lengths[b] + 1;
  if (ctx > a.cache_len || ctx < 1) ctx = ctx < 1 ? 1 : a.cache_len;  // recorded by the prep step
  const int per = ((((ctx + a.nsplit - 1) / a.nsplit) + XA_TILE - 1) / XA_TILE) * XA_TILE;
  const int k_begin = split * per;
  if (k_begin >= ctx) return;
  const int k_end = min(ctx, k_begin + per);
  const int ntiles = (k_end - k_begin + XA_TILE - 1) / XA_TILE;
  const long long krow = ((((long long)layer * 2 + 0) * a.cache_batch + b) * a.heads + h) * a.cache_len;
  const long long vrow = ((((long long)layer * 2 + 1) * a.cache_batch + b) * a.heads + h) * a.cache_len;
  const uint32_t xt0 = xt;
  xt = xt0 + ntiles;

  // tile tl of this item into ring stage (xt0 + tl) % XA_STAGES, once the four
  // warps released the tile that stage held before (only thread 0 issues)
  int issued = 0;
  auto issue_next = [&]() -> bool {
    const uint32_t g = xt0 + issued;
    const int s = g % XA_STAGES;
    if (g >= XA_STAGES && !mbar_wait(&sm.xa_empty[s], ((g / XA_STAGES) - 1) & 1u, sabort)) {
      give_up(P, sabort, DEV_TIMEOUT_EMPTY);
      return false;
    }
    uint8_t* dst = stage_base + s * STAGE_BYTES;
    mbar_arrive_expect_tx(&sm.xa_full[s], STAGE_BYTES);
    const int row = k_begin + issued * XA_TILE;
#pragma unroll
    for (int bx = 0; bx < HD / 64; ++bx) {
      if (copy_checked(P, dst + bx * XA_TILE * 128, XA_TILE * 128, sm.B, sm.B + B_REGION, nullptr, bx * 64))
        tma_load_2d(dst + bx * XA_TILE * 128, P.cache_map, &sm.xa_full[s], bx * 64, (int)(krow + row));
      if (copy_checked(P, dst + TILE_BYTES + bx * XA_TILE * 128, XA_TILE * 128, sm.B, sm.B + B_REGION, nullptr, bx * 64))
        tma_load_2d(dst + TILE_BYTES + bx * XA_TILE * 128, P.cache_map, &sm.xa_full[s], bx * 64, (int)(vrow + row));
    }
    ++issued;
    return true;
  };
  if (t == 0) {
    for (int tl = 0; tl < XA_STAGES && tl < ntiles; ++tl)
      if (!issue_next()) break;
  }
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
  for (int tl = 0; tl < ntiles; ++tl) {
    // keep XA_STAGES tiles in flight: tile tl+1 goes into the stage tile tl-1 used
    if (t == 0 && tl >= 1 && issued == tl + XA_STAGES - 1 && issued < ntiles) issue_next();
    const uint32_t g = xt0 + tl;
    const int s = g % XA_STAGES;
    if (!warp_wait(&sm.xa_full[s], (g / XA_STAGES) & 1u, sabort)) {
      if (lane == 0) give_up(P, sabort, DEV_TIMEOUT_FULL);
      break;
    }
    const uint32_t kbase = smem_u32(stage_base + s * STAGE_BYTES);
    const uint32_t vbase = kbase + TILE_BYTES;
    const int key0 = 16 * warp;
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
      const int kr = key0 + nt * 8 + (lane & 7);
#pragma unroll
      for (int ks = 0; ks < HD / 16; ks += 2) {
        uint32_t r0, r1, r2, r3;
        ldsm4(kbase + xa_sw128(kr, 2 * ks + (lane >> 3)), r0, r1, r2, r3);
        mma16816(sc[nt], qa[ks], r0, r1);
        mma16816(sc[nt], qa[ks + 1], r2, r3);
      }
    }
    const int kabs = k_begin + tl * XA_TILE + key0;
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
    pa[0] = packbf(p[0][0], p[0][1]);
    pa[1] = packbf(p[0][2], p[0][3]);
    pa[2] = packbf(p[1][0], p[1][1]);
    pa[3] = packbf(p[1][2], p[1][3]);
    const int vr = key0 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int dn = 0; dn < NT; dn += 2) {
      uint32_t r0, r1, r2, r3;
      ldsm4t(vbase + xa_sw128(vr, dn + (lane >> 4)), r0, r1, r2, r3);
      mma16816(o[dn], pa, r0, r1);
      mma16816(o[dn + 1], pa, r2, r3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.xa_empty[s]);
  }
  named_bar_sync(3, 128);
  // tiles issued but never consumed (only after a wait gave up) land before the smem is reused
  if (t == 0 && *sabort) {
    for (int tl = issued > XA_STAGES ? issued - XA_STAGES : 0; tl < issued; ++tl) {
      const uint32_t g = xt0 + tl;
      mbar_wait(&sm.xa_full[g % XA_STAGES], (g / XA_STAGES) & 1u, nullptr);
    }
  }
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 1));
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 2));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 1));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 2));
  float* mO = mrg;
  float* mM = mrg + 4 * 16 * HD;
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
  named_bar_sync(3, 128);
  if (t < 16) {
    float mm = -INFINITY;
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, mM[w * 16 + t]);
    float ll = 0.0f;
    for (int w = 0; w < 4; ++w) {
      const float f = mM[w * 16 + t] == -INFINITY ? 0.0f : expf(__fsub_rn(mM[w * 16 + t], mm));
      mF[w * 16 + t] = f;
      ll = __fadd_rn(ll, __fmul_rn(mL[w * 16 + t], f));
    }
    mR[t] = mm;
    mR[16 + t] = ll;
  }
  named_bar_sync(3, 128);
  const int nsp = a.nsplit;
  const int n_active = (ctx + per - 1) / per;
  float* mine = a.part + (long long)(bh * nsp + split) * (16 * HD + 32);
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
      __nv_bfloat16* dst = a.out + (long long)(b * 16 + i) * a.hidden + h * HD + d;
      *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(__fdiv_rn(acc.x, ll), __fdiv_rn(acc.y, ll));
      *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __floats2bfloat162_rn(__fdiv_rn(acc.z, ll), __fdiv_rn(acc.w, ll));
    } else {
      __stcg(reinterpret_cast<float4*>(mine + i * HD + d), acc);
    }
  }
  if (n_active == 1) {
    named_bar_sync(3, 128);
    return;
  }
  if (t < 16) {
    __stcg(mine + 16 * HD + t, mR[t]);
    __stcg(mine + 16 * HD + 16 + t, mR[16 + t]);
  }
  __threadfence();
  named_bar_sync(3, 128);
  if (t == 0) {
    const int old = atomicAdd(a.counters + bh, 1);
    sm.flags[F_XA_LAST] = (old == n_active - 1);
  }
  named_bar_sync(3, 128);
  const bool last = sm.flags[F_XA_LAST] != 0;
  named_bar_sync(3, 128);  // the flag is rewritten by the next item
  if (!last) return;
  __threadfence();
  const float* base = a.part + (long long)bh * nsp * (16 * HD + 32);
  float* sF = mO;
  if (t < 16) {
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
  named_bar_sync(3, 128);
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
      const float4 tv = __ldcg(reinterpret_cast<const float4*>(base + (long long)sp * (16 * HD + 32) + i * HD + d));
      const float f = sF[sp * 16 + i];
      acc.x = __fadd_rn(acc.x, __fmul_rn(tv.x, f));
      acc.y = __fadd_rn(acc.y, __fmul_rn(tv.y, f));
      acc.z = __fadd_rn(acc.z, __fmul_rn(tv.z, f));
      acc.w = __fadd_rn(acc.w, __fmul_rn(tv.w, f));
    }
    const float ll = sF[n_active * 16 + i];
    __nv_bfloat16* dst = a.out + (long long)(b * 16 + i) * a.hidden + h * HD + d;
    *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(__fdiv_rn(acc.x, ll), __fdiv_rn(acc.y, ll));
    *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __floats2bfloat162_rn(__fdiv_rn(acc.z, ll), __fdiv_rn(acc.w, ll));
  }
  if (t == 0) a.counters[bh] = 0;
  named_bar_sync(3, 128);
}

// ------------------------------------------------------------------ one accumulator segment (warps 2-5)

// The epilogue side of gemm_bf16_tc<16, EPI> (gemm.cuh) for one segment: the
// units [seg_begin, seg_end) of one tile.  Returns false when the wait for
// the accumulator gave up (uniformly over the 128 threads).
template <int EPI>
__device__ bool run_segment(const GemmArgs& a, const Smem& sm, uint32_t tmem, int seg, long long u0, long long seg_begin,
                            long long seg_end, long long U, int G, int c, uint8_t* fx, uint32_t fx_cap,
                            uint32_t& fx_phase, volatile int* sabort, unsigned long long* ts) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, r = q * 32 + lane;
  const int kb = a.kb;
  const int tile = (int)(seg_begin / kb);
  const int acc = seg & 1;
  if (threadIdx.x == 64) {
    const bool ok = mbar_wait(&sm.acc_full[acc], (uint32_t)(seg >> 1) & 1u, sabort);
    if (!ok) {
      *sabort = 1;
      record_error(a.err, DEV_TIMEOUT_ACC);
    }
    sm.flags[F_SEG + (seg & 1)] = ok ? 1 : 0;
  }
  named_bar_sync(1, 128);
  if (!sm.flags[F_SEG + (seg & 1)]) return false;
  tc_fence_after();
  const int m = tile * 128 + r;
  const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BNP);
  const bool whole = (seg_begin == (long long)tile * kb) && (seg_end == (long long)(tile + 1) * kb);
  if (whole) {
    float v[16];
    tmem_ld_x16(taddr, v);
    tmem_wait_ld();
    epilogue16<EPI>(a, v, r, m, tile, 0, sm.xch, sm.xch64);
  } else {
    // split tile: its owner is the CTA holding the tile's first k-block (for
    // which this is the last segment); the others hand it their partials
    const long long c_first = cta_of_unit((long long)tile * kb, U, G);
    const long long c_last = cta_of_unit((long long)(tile + 1) * kb - 1, U, G);
    const int ncon = (int)(c_last - c_first + 1);
    constexpr uint32_t PART = BNP * 128 * 4;  // one contributor's partial tile
    if (c != c_first) {
      // a contributor's segment is its first one: slot 0
      float* mine = a.ws + ((long long)(c * 2) * BNP) * 128;
      float v[16];
      tmem_ld_x16(taddr, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) __stcg(mine + (long long)j * 128 + r, v[j]);
      named_bar_sync(1, 128);
      if (threadIdx.x == 64) red_release_add(a.counters + tile, 1);
    } else {
      float own[16], v[16];
      tmem_ld_x16(taddr, own);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = 0.0f;
      const bool staged = fx != nullptr && (uint32_t)ncon * PART <= fx_cap;
      if (threadIdx.x == 64) {
        // every other contributor arrived (bounded wait), then their partials
        // in one round trip when shared memory has room
        bool ok = wait_count(a.counters + tile, ncon - 1, sabort);
        if (ts) ts[10] = global_ns();
        if (ok) {
          a.counters[tile] = 0;  // every contributor of this use has arrived
          if (staged) {
            fence_async_global();
            mbar_arrive_expect_tx(sm.fix, (uint32_t)(ncon - 1) * PART);
            for (long long cc = c_first + 1; cc <= c_last; ++cc) {
              uint8_t* d = fx + (cc - c_first) * PART;
              const float* src = a.ws + ((cc * 2) * BNP) * 128;
              if ((reinterpret_cast<uintptr_t>(d) & 15) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                  d >= sm.B && d + PART <= sm.B + B_REGION)
                bulk_load(d, src, PART, sm.fix);
              else
                record_error(a.err, DEV_BAD_COPY);
            }
            ok = mbar_wait(sm.fix, fx_phase & 1u, sabort);
          }
        }
        if (ts) ts[11] = global_ns();
        if (!ok) {
          *sabort = 1;
          record_error(a.err, DEV_TIMEOUT_OTHER);
        }
        sm.flags[F_FIX] = ok ? 1 : 0;
      }
      if (staged) ++fx_phase;
      named_bar_sync(1, 128);
      const bool ok = sm.flags[F_FIX] != 0;
      named_bar_sync(1, 128);  // the flag is rewritten by the next fix-up
      if (!ok) return false;
      // partials summed in contributor order (the owner is the first)
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], own[j]);
      if (staged) {
        for (long long cc = c_first + 1; cc <= c_last; ++cc) {
          const float* p = reinterpret_cast<const float*>(fx + (cc - c_first) * PART) + r;
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], p[j * 128]);
        }
      } else {
        for (long long cc0 = c_first + 1; cc0 <= c_last; cc0 += 4) {
          float tv[4][16];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const long long cc = cc0 + q4 <= c_last ? cc0 + q4 : c_last;
            const float* p = a.ws + ((cc * 2) * BNP) * 128 + r;
#pragma unroll
            for (int j = 0; j < 16; ++j) tv[q4][j] = __ldcg(p + (long long)j * 128);
          }
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            if (cc0 + q4 <= c_last) {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], tv[q4][j]);
            }
        }
      }
      if (ts && threadIdx.x == 64) ts[12] = global_ns();
      epilogue16<EPI>(a, v, r, m, tile, 0, sm.xch, sm.xch64);
      if (ts && threadIdx.x == 64) ts[13] = global_ns();
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
  return true;
}

__device__ bool run_segment_any(int epi, const GemmArgs& a, const Smem& sm, uint32_t tmem, int seg, long long u0,
                                long long sb, long long se, long long U, int G, int c, uint8_t* fx, uint32_t fx_cap,
                                uint32_t& fxp, volatile int* sabort, unsigned long long* ts) {
  switch (epi) {
    case EPI_STORE: return run_segment<EPI_STORE>(a, sm, tmem, seg, u0, sb, se, U, G, c, fx, fx_cap, fxp, sabort, ts);
    case EPI_GELU: return run_segment<EPI_GELU>(a, sm, tmem, seg, u0, sb, se, U, G, c, fx, fx_cap, fxp, sabort, ts);
    case EPI_SWIGLU: return run_segment<EPI_SWIGLU>(a, sm, tmem, seg, u0, sb, se, U, G, c, fx, fx_cap, fxp, sabort, ts);
    case EPI_RESID: return run_segment<EPI_RESID>(a, sm, tmem, seg, u0, sb, se, U, G, c, fx, fx_cap, fxp, sabort, ts);
    case EPI_QKNORM: return run_segment<EPI_QKNORM>(a, sm, tmem, seg, u0, sb, se, U, G, c, fx, fx_cap, fxp, sabort, ts);
    case EPI_KVCACHE: return run_segment<EPI_KVCACHE>(a, sm, tmem, seg, u0, sb, se, U, G, c, fx, fx_cap, fxp, sabort, ts);
    case EPI_LOGITS: return run_segment<EPI_LOGITS>(a, sm, tmem, seg, u0, sb, se, U, G, c, fx, fx_cap, fxp, sabort, ts);
    default: return false;
  }
}

// Units [u0, u1) of a GEMM stage owned by CTA c: the stage runs on
// min(U, grid) CTAs (as the kernel sequence launches it), so that every
// participating CTA owns at least one unit; Gs is that CTA count.
__device__ __forceinline__ int stage_units(long long U, int G, int c, long long* u0, long long* u1) {
  const int Gs = U < (long long)G ? (int)U : G;
  if (c < Gs) {
    *u0 = (long long)c * U / Gs;
    *u1 = (long long)(c + 1) * U / Gs;
  } else {
    *u0 = *u1 = 0;
  }
  return Gs;
}

__device__ __forceinline__ long long seg_end_of(long long u, long long u1, int kb) {
  const long long e = (u / kb + 1) * kb;
  return e < u1 ? e : u1;
}

// ------------------------------------------------------------------ the kernel

__global__ void __launch_bounds__(THREADS, 1) pass_kernel(const __grid_constant__ PassArgs P) {
  extern __shared__ uint8_t smem_raw[];
  const Smem sm = carve_smem(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;
  volatile int* sabort = sm.flags + F_ABORT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NA; ++s) {
      mbar_init(&sm.a_full[s], 1);
      mbar_init(&sm.a_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], 4);
    }
    mbar_init(sm.b_ready, 1);
    mbar_init(sm.b_free, 1);
    for (int s = 0; s < XA_STAGES; ++s) {
      mbar_init(&sm.xa_full[s], 1);
      mbar_init(&sm.xa_empty[s], 4);
    }
    mbar_init(sm.b_load, 1);
    mbar_init(sm.fix, 1);
    for (int i = 0; i < 16; ++i) sm.flags[i] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  for (int s = threadIdx.x; s < P.n_stages; s += THREADS) {
    const Stage& S = P.stages[s];
    StageLite l;
    l.units = S.ep.units;
    l.type = S.type;
    l.kb = S.ep.kb;
    l.tmap = S.tmap;
    l.bsrc = S.bsrc;
    l.fmap = S.fmap;
    l.full = S.full;
    sm.lite[s] = l;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;
  const uint32_t bump = P.offset_ptr ? *reinterpret_cast<volatile uint32_t*>(P.offset_ptr) + 1u : 0u;
  const uint32_t noise_off = P.offset + bump;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t i = 0;
      bool ok = true;
      // L2 prefetch cursor over the same (stage, unit) sequence, PF tiles
      // ahead of the loads: the weights of the next stages stream from HBM
      // while the current stage waits on its inputs
      struct Cursor {
        int s = -1, kb = 1;
        long long u = 0, u1 = 0;
        const CUtensorMap* map = nullptr;
      } pf;
      uint32_t pf_n = 0;
      auto prefetch_to = [&](uint32_t upto) {
        while (pf_n < upto) {
          if (pf.u >= pf.u1) {
            do {
              ++pf.s;
            } while (pf.s < P.n_stages && sm.lite[pf.s].type != ST_GEMM);
            if (pf.s >= P.n_stages) return;
            const StageLite T = sm.lite[pf.s];
            stage_units(T.units, G, c, &pf.u, &pf.u1);
            pf.kb = T.kb;
            pf.map = P.tmaps + T.tmap;
            tmap_acquire(pf.map);
            continue;
          }
          tma_prefetch_l2_2d(pf.map, (int)(pf.u % pf.kb) * 64, (int)(pf.u / pf.kb) * 128);
          ++pf.u;
          ++pf_n;
        }
      };
      for (int s = 0; s < P.n_stages && ok; ++s) {
        const StageLite S = sm.lite[s];
        if (S.type != ST_GEMM) continue;
        const long long U = S.units;
        long long u0, u1;
        stage_units(U, G, c, &u0, &u1);
        const int kb = S.kb;
        const CUtensorMap* map = P.tmaps + S.tmap;
        if (u1 > u0) tmap_acquire(map);
        for (long long u = u0; u < u1; ++u, ++i) {
          if (P.pf_tiles) prefetch_to(i + (uint32_t)P.pf_tiles);
          const int slot = i % NA;
          const uint32_t round = i / NA;
          if (round > 0 && !mbar_wait(&sm.a_empty[slot], (round - 1) & 1u, sabort)) {
            record_error(P.err, DEV_TIMEOUT_EMPTY);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.a_full[slot], A_BYTES);
          if (copy_checked(P, sm.A + slot * A_BYTES, A_BYTES, sm.A, sm.A + NA * A_BYTES, nullptr, (int)(u % kb) * 64))
            tma_load_2d_hint(sm.A + slot * A_BYTES, map, &sm.a_full[slot], (int)(u % kb) * 64, (int)(u / kb) * 128,
                             pol);
        }
      }
      if (!ok) *sabort = 1;
      // every issued tile lands before the CTA's shared memory goes away
      for (uint32_t j = i > (uint32_t)NA ? i - NA : 0u; j < i; ++j)
        mbar_wait(&sm.a_full[j % NA], (j / NA) & 1u, nullptr);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128, BNP);
      uint32_t i = 0, gs = 0;
      int seg = 0;
      bool ok = true;
      for (int s = 0; s < P.n_stages && ok; ++s) {
        const StageLite S = sm.lite[s];
        if (S.type != ST_GEMM) continue;
        if (!mbar_wait(sm.b_ready, gs & 1u, sabort)) {
          record_error(P.err, DEV_TIMEOUT_OTHER);
          ok = false;
          break;
        }
        tc_fence_after();
        const long long U = S.units;
        long long u0, u1;
        stage_units(U, G, c, &u0, &u1);
        const int kb = S.kb;
        const int k0 = (int)(u0 % kb);
        const bool any = u1 > u0;
        const int nk = (int)((u1 - u0) < kb ? (u1 - u0) : kb);
        const int kbase = b_mode(S.bsrc, S.fmap, S.full, kb, nk).inplace ? 0 : k0;  // slot of k-block k: (k - kbase) mod kb
        for (long long u = u0; u < u1 && ok; ++seg) {
          const long long seg_begin = u, seg_end = seg_end_of(u, u1, kb);
          const int acc = seg & 1;
          if (seg >= 2 && !mbar_wait(&sm.acc_empty[acc], ((uint32_t)(seg >> 1) - 1) & 1u, sabort)) {
            record_error(P.err, DEV_TIMEOUT_ACC);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + (uint32_t)(acc * BNP);
          for (; u < seg_end; ++u, ++i) {
            const int slot = i % NA;
            if (!mbar_wait(&sm.a_full[slot], (i / NA) & 1u, sabort)) {
              record_error(P.err, DEV_TIMEOUT_FULL);
              ok = false;
              break;
            }
            tc_fence_after();
            const int bs = ((int)(u % kb) - kbase + kb) % kb;
            const uint64_t ad = sdesc_k_sw128(smem_u32(sm.A + slot * A_BYTES));
            const uint64_t bd = sdesc_k_sw128(smem_u32(sm.B + bs * B_SLOT));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16(d_tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), IDESC,
                        (u > seg_begin || kk > 0) ? 1u : 0u);
            umma_commit(&sm.a_empty[slot]);
          }
          if (!ok) break;
          umma_commit(&sm.acc_full[acc]);
        }
        if (!ok) break;
        // the B operand may be rebuilt once this stage's MMAs completed
        if (any)
          umma_commit(sm.b_free);
        else
          mbar_arrive(sm.b_free);
        ++gs;
      }
      if (!ok) *sabort = 1;
    }
  } else {
    // ---------------------------------------------------------------- workers (warps 2..7)
    const int wt = threadIdx.x - 64;
    uint32_t gs = 0, xt = 0, bl_phase = 0, fx_phase = 0;
    int seg = 0;
    uint8_t* fx = nullptr;
    uint32_t fx_cap = 0;
    if (c == 0) {
      // prep: the anchor row's position and sequence, the slots' positions, argmax keys
      const int len = P.lengths[0];
      if (wt == 0) {
        const long long id = P.anchor_ids[0];
        if (id < 0 || id >= P.vocab || len < 0 || len + P.block + 1 > P.rope_len || len >= P.cache_len)
          record_error(P.err, DEV_BAD_INDEX);
        P.anchor_pos[0] = len;
        P.anchor_seq[0] = 0;
      }
      for (int k = wt; k < P.block; k += WORKERS) {
        P.slot_pos[k] = len + 1 + k;
        P.keys[k] = 0ull;
      }
    }
    unsigned long long* trace = P.trace ? P.trace + (size_t)c * P.n_stages * TRACE_SLOTS : nullptr;
    {
      // rotary factors of the block slots (positions len + 1 + k) for the q/k norms
      const int len = P.lengths[0];
      for (int i = wt; i < P.block * P.rope_half; i += WORKERS) {
        const int k = i / P.rope_half, f = i % P.rope_half;
        int pos = len + 1 + k;
        if (pos < 0 || pos >= P.rope_len) pos = 0;  // recorded as DEV_BAD_INDEX by the prep step
        sm.rope[k * P.rope_half + f] = P.rope_cos[(long long)pos * P.rope_half + f];
        sm.rope[(BNP + k) * P.rope_half + f] = P.rope_sin[(long long)pos * P.rope_half + f];
      }
    }
    for (int s = 0; s < P.n_stages; ++s) {
      unsigned long long* ts = trace ? trace + s * TRACE_SLOTS : nullptr;
      if (ts && wt == 0) ts[0] = global_ns();
      {
        // this stage's descriptor into shared memory (loops below read it often)
        const uint4* src = reinterpret_cast<const uint4*>(P.stages + s);
        uint4* dst = reinterpret_cast<uint4*>(sm.stage);
        for (int i = wt; i < (int)(sizeof(Stage) / 16); i += WORKERS) dst[i] = __ldg(src + i);
      }
      named_bar_sync(2, WORKERS);
      const Stage& S = *sm.stage;
      if (S.wait >= 0) {
        if (wt == 0) sm.flags[F_GRID] = grid_wait(P, (unsigned long long)(S.wait + 1) * G, sabort) ? 1 : 0;
        named_bar_sync(2, WORKERS);
        if (!sm.flags[F_GRID]) break;
      }
      if ((S.type == ST_GEMM || S.type == ST_XATTN) && gs > 0) {
        // the B region is shared: the last GEMM stage's MMAs must have released it
        if (wt == 0) {
          const bool ok = mbar_wait(sm.b_free, (gs - 1) & 1u, sabort);
          if (!ok) give_up(P, sabort, DEV_TIMEOUT_OTHER);
          sm.flags[F_BFREE] = ok ? 1 : 0;
        }
        named_bar_sync(2, WORKERS);
        if (!sm.flags[F_BFREE]) break;
      }
      if (ts && wt == 0) ts[1] = global_ns();
      if (S.type == ST_GEMM) {
        const long long U = S.ep.units;
        long long u0, u1;
        const int Gs = stage_units(U, G, c, &u0, &u1);
        const int kb = S.ep.kb;
        if (wt == 0) {
          // the pass's split-K buffers (two parities: a stage that starts without
          // a barrier may overlap the fix-up of the stage before it) and the
          // draft call's LM-head output
          GemmArgs& a = sm.stage->ep;
          const int par = s & 1;
          a.ws = P.ws + (long long)par * G * 2 * BNP * 128;
          a.counters = P.counters + (long long)par * P.max_tiles;
          a.err = P.err;
          if (S.epi == EPI_QKNORM) {
            a.tok_cos = sm.rope;
            a.tok_sin = sm.rope + BNP * P.rope_half;
          }
          if (S.is_lm) {
            a.out = P.logits;
            a.ldo = P.ldl;
            a.scatter = P.scatter;
            a.argmax_keys = P.keys;
          }
        }
        if (u1 > u0) {
          const int k0 = (int)(u0 % kb);
          const int nk = (int)((u1 - u0) < kb ? (u1 - u0) : kb);
          const size_t used = build_b(S, P, sm, S.ep.K, kb, k0, nk, wt, noise_off, bl_phase, sabort, ts);
          fence_async_smem();
          // the epilogue's fix-up may stage partials past the operand
          fx = sm.B + align_up(used, 1024);
          fx_cap = (uint32_t)(B_REGION - align_up(used, 1024));
        }
        named_bar_sync(2, WORKERS);
        if (wt == 0) {
          mbar_arrive(sm.b_ready);
          if (ts) ts[4] = global_ns();
        }
        if (warp < 6) {
          bool first = true;
          for (long long u = u0; u < u1; ++seg) {
            const long long seg_begin = u;
            u = seg_end_of(u, u1, kb);
            if (!run_segment_any(S.epi, sm.stage->ep, sm, tmem, seg, u0, seg_begin, u, U, Gs, c, fx, fx_cap, fx_phase,
                                 sabort, ts))
              break;
            if (ts && wt == 0 && first) ts[5] = global_ns();
            first = false;
          }
          if (ts && wt == 0) ts[6] = global_ns();
        } else {
          for (long long u = u0; u < u1; ++seg) u = seg_end_of(u, u1, kb);  // keep the segment count in step
        }
        ++gs;
      } else if (S.type == ST_XATTN) {
        if (warp < 6) {
          fence_async_global();  // cache rows written by other CTAs' epilogues are read by TMA
          if (wt == 0) tmap_acquire(P.cache_map);
          const int items = P.xa.batch * P.xa.heads * P.xa.nsplit;
          for (int it = c; it < items; it += G) {
            const int bh = it / P.xa.nsplit, split = it % P.xa.nsplit;
            if (P.xa.head_dim == 128)
              xattn_item<128>(P, sm, S.xa_layer, bh, split, wt, xt, sabort);
            else
              xattn_item<64>(P, sm, S.xa_layer, bh, split, wt, xt, sabort);
            if (ts && wt == 0 && it == c) ts[5] = global_ns();
          }
          if (ts && wt == 0) ts[6] = global_ns();
        }
      } else if (S.type == ST_FINAL) {
        if (c == 0 && P.tokens)
          for (int k = wt; k < P.block; k += WORKERS) P.tokens[k] = (int64_t)argmax_key_index(P.keys[k]);
      }
      // stage done: check for an abort uniformly, then arrive
      named_bar_sync(2, WORKERS);
      if (wt == 0) sm.flags[F_STAGE_OK] = *sabort ? 0 : 1;
      named_bar_sync(2, WORKERS);
      if (!sm.flags[F_STAGE_OK]) break;
      if (wt == 0) {
        if (ts) ts[7] = global_ns();
        __threadfence();
        atomicAdd(P.bar_count, 1ull);
      }
    }
    if (wt == 0 && *sabort) atomicExch(P.abort, 1);
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0) {
    // the last CTA out resets the pass's words; every CTA has read them by now
    __threadfence();
    const unsigned long long done = atomicAdd(P.bar_exit, 1ull);
    if (done == (unsigned long long)G - 1) {
      *P.bar_count = 0ull;
      *P.bar_exit = 0ull;
      *P.abort = 0;
      if (P.offset_ptr) *P.offset_ptr = bump;
      __threadfence();
    }
  }
}

}  // namespace pass

// ------------------------------------------------------------------ host side

size_t pass_smem_bytes() { return (size_t)pass::SMEM; }
int pass_b_slots() { return pass::B_SLOTS; }
int pass_max_stages() { return pass::MAX_STAGES; }
size_t pass_b_region() { return (size_t)pass::B_REGION; }
size_t pass_stage_b_bytes(int bsrc, int nk, int K, int head_dim, bool staged_rows) {
  using namespace pass;
  const size_t slots = (size_t)nk * B_SLOT;
  switch (bsrc) {
    case BS_SELFATTN: {
      const int nh = std::min(nk, (nk * 64 + head_dim - 1) / head_dim + 1);
      return align_up(slots, 1024) + selfattn_bytes(nh, head_dim);
    }
    case BS_ADALN:
      return staged_rows ? align_up(slots, 1024) + adaln_full_bytes(K) : slots + (size_t)2 * nk * 128;
    case BS_MIX:
      return slots + mix_param_bytes(nk);
    case BS_RMSROW:
    case BS_GATHER:
      return slots + row_stage_bytes(K);
    default:
      return slots;
  }
}

static bool pass_configure() {
  static int configured = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (configured == dev) return true;
  if (cudaFuncSetAttribute(pass::pass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pass::SMEM) != cudaSuccess)
    return false;
  configured = dev;
  return true;
}

int pass_grid() {
  if (!pass_configure()) return 0;
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, pass::pass_kernel, pass::THREADS, pass::SMEM) !=
      cudaSuccess)
    return 0;
  return blocks >= 1 ? num_sms() : 0;
}

fm_status pass_launch(const pass::PassArgs& P, int grid, cudaStream_t stream) {
  if (!pass_configure()) return set_error(FM_ERR_CUDA, "pass: cannot set the shared memory size");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(pass::THREADS);
  cfg.dynamicSmemBytes = pass::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, pass::pass_kernel, P);
  if (e != cudaSuccess) return set_error(FM_ERR_LAUNCH, "pass: launch failed: %s", cudaGetErrorString(e));
  ++launch_counter();
  return FM_OK;
}

}  // namespace fm
