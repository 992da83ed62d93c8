// The streamed single-launch draft pass (batch 1, one jump): the whole of
// modeling_flashmap.py:422-479 as one cooperative kernel with one CTA per SM.
//
// Why one launch: a batch-1 draft is ~70 dependent steps, and its weight
// matrices (2.4 GB at Qwen3-8B sizing) do not depend on the activations.  In
// this pass every CTA streams the weight tiles of all its work, stage after
// stage, through a shared-memory ring (and, further ahead, into L2) without
// ever waiting on an activation; only the small token-side operand of a
// stage waits for the stage before it.  So the HBM stream runs on while the
// short dependent steps (operand build, tensor-core MMA, split-K reduction,
// epilogue) follow one another across the grid.
//
// Stages (the host builds the list, the kernel interprets it):
//   GEMM  Y[16, M] = B[16, K] W[M, K]^T on tcgen05 (weights as the 128-row A
//         operand, the 16 block tokens as N = 16), the (tile, k-block) units
//         split evenly over the grid (stream-K, the split of gemm_bf16_tc).
//         The B operand is built in shared memory from its source rows with
//         the stage's input transform (Philox noise, embedding row, RMSNorm,
//         mix_state, AdaLN, copy); partial tiles are finished by the last
//         contributor to arrive, summing the partials in contributor order;
//         the fused epilogues are those of gemm_bf16_tc.  The q|k|v GEMM's
//         last tile of each head group also runs that group's block
//         self-attention, so the o projection reads finished attention rows.
//   XATTN the block's cross-attention over the context cache, (head, key
//         split) items whose K/V tiles stream through the same ring.
//   FINAL the argmax tokens.
// A stage's inputs are ready when the completion counter of the stage it
// depends on reaches its piece count (tiles, head groups or heads).  The
// row statistics an AdaLN / RMSNorm / mix_state operand needs are produced
// per 128-feature tile by the producing stage's epilogue and combined in
// tile order by the consumer.
//
// Every wait is bounded (FM_WAIT_NS); a wait that runs out records an error
// code and raises an abort word that makes every CTA leave its loop, drain
// its copies and exit.  Counters return to zero by the end of every launch.
#pragma once

#include "attention.cuh"
#include "gemm.cuh"
#include "launch.cuh"

namespace fm {
namespace stream {

using bf16 = __nv_bfloat16;

constexpr int THREADS = 256;              // warps: 0 weights, 1 MMA, 2-5 epilogue / attention, 6-7 operand
constexpr int NA = 8;                     // weight ring slots
constexpr int A_BYTES = 128 * 64 * 2;     // one 128 x 64 weight tile
constexpr int NB = 16;                    // operand ring slots
constexpr int B_BYTES = 16 * 64 * 2;      // one 16 x 64 operand block
constexpr int BATCH = 8;                  // operand blocks whose source rows are staged per round
constexpr int STAGE_SLOT = B_BYTES;       // the 16 source rows of one block
constexpr int MAX_TRANSFORM_UNITS = 16;   // units per CTA of a transform stage (their constant rows staged at once)
constexpr int CONST_SLOT = 3 * 128;       // up to three constant rows of one block
constexpr int MAX_MAPS = 112;

enum Kind : int { K_PREP = 0, K_GEMM = 1, K_XATTN = 2, K_FINAL = 3, K_NOISE = 4, K_ANORM = 5 };
// operand sources: rows copied by TMA, or computed from staged rows (mix_state, AdaLN)
enum BKind : int { B_COPY = 0, B_MIX = 1, B_ADALN = 2 };
enum EKind : int { E_STORE = 0, E_GELU = 1, E_SWIGLU = 2, E_RESID = 3, E_QKV = 4, E_QNORM = 5, E_KVCACHE = 6,
                   E_LOGITS = 7 };
enum Stats : int { S_NONE = 0, S_LN = 1, S_SQ = 2 };

struct alignas(16) Stage {
  int kind;
  int dep, dep2;     // stages whose completion this stage's inputs need (-1: none)
  int pieces;        // completion count of this stage per draft
  // GEMM: the units are split over `vg` of the CTAs, virtual CTA v being CTA
  // (v + rot) % grid, so that the small stages of a chain spread over the grid
  int vg, rot;
  int map;           // weight tensor map (index into Params::maps)
  int bmap;          // B_COPY: the operand source's tensor map ([rows, K], boxes of 16 x 64)
  int bkind, ekind, stats;
  int ntok;          // operand rows that hold data (16, or 1 for the anchor row)
  const bf16* src;   // operand source rows [ntok, K] (stride ld)
  long long ld;
  const bf16* mod;   // B_ADALN: scale | shift rows (K each)
  const bf16* w0;    // B_RMSROW: norm weight; B_MIX: state_norm weight
  const bf16* w1;    // B_MIX: noise_norm weight
  const bf16* aux;   // B_MIX: uniform-posterior row; K_PREP: the embedding [V, count]
  bf16* dst;         // K_PREP: anchor row; K_NOISE: noise rows; K_ANORM: normalised anchor row
  long long count;   // elements of dst
  const float* stats_in;  // statistics of the source rows: [tiles][16][2]
  int stats_tiles;
  float* stats_out;  // this stage's statistics: [m_tiles][16][2]
  float eps, gate;
  float* ws;         // split-K partials [virtual CTA][2 slots][128 rows][16 tokens]
  unsigned long long* tickets;  // [m_tiles] contributors arrived
  unsigned long long* groups;   // E_QKV: [D / 128] finished tiles of each (q, k, v) group
  bf16* attn;        // E_QKV: block self-attention output [16, D]
  GemmArgs ep;       // geometry and epilogue arguments (gemm.cuh)
  // XATTN
  int layer, nsplit;
  const bf16* q;     // [16, D] normed + roped queries
  bf16* out;         // [16, D]
  float* part;       // [heads * nsplit][16 * hd + 32]
  unsigned long long* xtickets;  // [heads] splits arrived
};

struct Params {
  CUtensorMap maps[MAX_MAPS];  // the weights' maps, then the context cache's
  const Stage* stages;
  int n_stages;
  int cache_map;
  unsigned long long* done;    // [n_stages] completion counters
  unsigned long long* words;   // [0] CTAs out, [1] abort
  unsigned long long* all_tickets;  // every ticket of the pass (zeroed after an abort)
  long long n_tickets;
  int* err;
  // per call
  const int64_t* anchor_ids;
  const int32_t* lengths;
  const bf16* z;               // caller's one-step noise [16, Ht] or null (Philox)
  uint64_t seed;
  uint32_t offset;
  uint32_t* offset_ptr;
  bf16* logits;
  long long ldl;
  int scatter;
  int64_t* tokens;
  unsigned long long* keys;    // [16] argmax keys
  int lm_stage;
  // model
  const float* rope_cos;
  const float* rope_sin;
  int rope_len, half;
  int cache_len, cache_batch, heads, head_dim, hidden, target_hidden, vocab, block;
  float scale;
};

// host side (stream.cu)
size_t smem_bytes();
// CTAs of the pass on this device (one per SM), or 0 when they cannot all be resident
int grid_size();
fm_status launch(const Params* P, int grid, cudaStream_t stream);

}  // namespace stream
}  // namespace fm
