// Host-side plan of one GEMM launch (tensor maps + arguments).
#pragma once

#include "gemm.cuh"
#include "launch.cuh"

namespace fm {

struct GemmPlan {
  CUtensorMap tmA;
  CUtensorMap tmB;
  GemmArgs args;
  int bn;
  int cg;  // CTAs per tile: 1, or 2 (a CTA pair launched as a cluster of two)
  int epi;
  int grid;
  size_t smem;
  unsigned long long* trace;  // optional per-CTA timestamps (diagnostics), else null
};

// Block width (tokens per tile) used for N tokens.
int gemm_bn_for(int64_t N);
// CTAs per tile for that block width (2: 256 x 256 pair tiles).
int gemm_cg_for(int bn);
// Split-K counters of a GEMM launch of this shape (one per 128-row tile and block).
int64_t gemm_counter_slots(int64_t M, int64_t N);
// Workspace bytes for the split-K partials of a GEMM launch of this shape.
size_t gemm_partials_bytes(int64_t M, int64_t N, int64_t K);
// Fill `p` for Y = X W^T.  Epilogue-specific fields of p->args are left zero
// for the caller to set.  ws/counters: split-K partials and per-tile counters.
fm_status gemm_prepare(GemmPlan* p, const void* W, int64_t M, int64_t K, int64_t ldw, const void* X, int64_t N,
                       int64_t ldx, int epi, float* ws, int* counters, int* err);
fm_status gemm_launch(const GemmPlan& p, cudaStream_t stream, bool pdl);

}  // namespace fm
