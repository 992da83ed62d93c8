// Persistent single-launch draft pass (batch 1, one jump): the whole of
// modeling_flashmap.py:422-479 in one cooperative kernel.
//
// The pass is a static list of stages.  GEMM stages stream one weight matrix
// (tcgen05, as in gemm.cuh) with a fused epilogue; the B operand (the 16
// block tokens) is built by worker warps straight into shared memory with the
// stage's input transform (copy, AdaLN, RMSNorm, mix-state, Philox noise,
// anchor-row gather, self-attention).  The cross-attention is a stage of its
// own.  Stages that read another CTA's output first wait on a grid barrier:
// one arrival counter per pass, stage w complete when it reaches (w + 1) x grid.
// That count is exact only when every wait names the stage right before it
// and no two stages in a row skip their wait; the host builder checks both.  The producer warp streams the
// weights of every stage through one TMA ring without ever waiting on a
// barrier, so the weight stream of the next stage overlaps the barrier of
// the current one.
#pragma once

#include "attention.cuh"
#include "gemm.cuh"
#include "launch.cuh"

namespace fm {
namespace pass {

enum StageType : int { ST_GEMM = 0, ST_XATTN = 1, ST_FINAL = 2 };
enum BSource : int {
  BS_COPY = 0,      // rows of an activation buffer
  BS_ADALN = 1,     // LayerNorm(x) * bf16(1 + scale) + shift (modeling_flashmap.py:112-115)
  BS_RMSROW = 2,    // RMSNorm of row 0 (the anchor row, :69-80)
  BS_GATHER = 3,    // embedding row of the anchor token (:453)
  BS_NOISE = 4,     // one-step noise z: Philox normals, or a caller-given z
  BS_MIX = 5,       // mix_state of the uniform posterior and z L^T (:393-399)
  BS_SELFATTN = 6,  // self-attention of the block (:188, :144-147)
};

struct Stage {
  int type;
  int wait;  // stage whose grid barrier must complete before this stage reads its inputs (-1: none)
  int tmap;  // weight tensor map (GEMM)
  int smap;  // source activation of the B rows, one 64-column block per box, -1: none
  int fmap;  // the same source as whole rows in one box (or, self-attention, one head part), -1: none
  int full;  // AdaLN: the whole input rows are staged (statistics from shared memory)
  int ntok;  // valid B rows
  int bsrc;
  int heads, head_dim;
  float scale, eps, gate;
  long long ld;
  const __nv_bfloat16* src;
  const __nv_bfloat16* mod;
  const __nv_bfloat16* w0;
  const __nv_bfloat16* w1;
  const __nv_bfloat16* aux;
  int epi;
  int is_lm;      // the LM head: output pointer comes from the draft call
  int xa_layer;   // cross-attention layer
  GemmArgs ep;    // geometry (M, N, K, kb, m_tiles, units) and epilogue arguments
};

struct PassArgs {
  const Stage* stages;
  int n_stages;
  const CUtensorMap* tmaps;      // weight maps, 64-byte aligned, device memory
  const CUtensorMap* cache_map;  // the context cache as [rows, head_dim]
  unsigned long long* bar_count;  // grid-barrier arrivals of this pass (zero between passes)
  unsigned long long* bar_exit;   // CTAs that finished; the last one zeroes the words of the pass
  int* abort;                     // set by a CTA that gave up; zeroed by the last CTA out
  int* err;
  float* ws;        // split-K partials: [2 parities][grid][2 slots][16][128]
  int* counters;    // [2 parities][max_tiles]
  int max_tiles;
  const int64_t* anchor_ids;
  const int32_t* lengths;
  const __nv_bfloat16* z;
  uint64_t seed;
  uint32_t offset;
  uint32_t* offset_ptr;
  int* anchor_pos;
  int* anchor_seq;
  int* slot_pos;
  unsigned long long* keys;
  int64_t* tokens;
  unsigned long long* trace;  // optional [grid][n_stages][10] timestamps (ns)
  int pf_tiles;               // weight tiles a CTA keeps requested into L2 ahead of its loads (0: none)
  __nv_bfloat16* logits;
  long long ldl;
  int scatter;
  int rope_len, cache_len, block;
  const float* rope_cos;  // [rope_len][rope_half]
  const float* rope_sin;
  int rope_half;
  long long vocab;
  CrossAttnArgs xa;
};

}  // namespace pass

// host side (pass.cu)
size_t pass_smem_bytes();
// B-operand k-blocks a CTA can hold; bytes of the B region, and the bytes a
// stage of that B source with nk k-blocks uses of it
int pass_b_slots();
int pass_max_stages();
size_t pass_b_region();
size_t pass_stage_b_bytes(int bsrc, int nk, int K, int head_dim, bool staged_rows);
// CTAs of the persistent launch (one per SM), or 0 when it cannot be resident
int pass_grid();
fm_status pass_launch(const pass::PassArgs& P, int grid, cudaStream_t stream);

}  // namespace fm
