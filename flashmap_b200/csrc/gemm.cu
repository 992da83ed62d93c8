// Host side of the tcgen05 GEMM: template dispatch, plans and the C ABI.
#include <cstdlib>

#include "gemm_plan.cuh"

namespace fm {

namespace {

using GemmKernel = void (*)(const CUtensorMap, const CUtensorMap, const GemmArgs, unsigned long long*);

template <int BN, int CG = 1>
struct BnTable {
  static GemmKernel get(int epi) {
    switch (epi) {
      case EPI_STORE: return gemm_bf16_tc<BN, EPI_STORE, CG>;
      case EPI_GELU: return gemm_bf16_tc<BN, EPI_GELU, CG>;
      case EPI_SWIGLU: return gemm_bf16_tc<BN, EPI_SWIGLU, CG>;
      case EPI_RESID: return gemm_bf16_tc<BN, EPI_RESID, CG>;
      case EPI_QKNORM: return gemm_bf16_tc<BN, EPI_QKNORM, CG>;
      case EPI_KVCACHE: return gemm_bf16_tc<BN, EPI_KVCACHE, CG>;
      case EPI_LOGITS: return gemm_bf16_tc<BN, EPI_LOGITS, CG>;
      case EPI_F32: return gemm_bf16_tc<BN, EPI_F32, CG>;
      default: return nullptr;
    }
  }
  static size_t smem() { return GemmShape<BN, CG>::SMEM; }
};

GemmKernel kernel_for(int bn, int epi, int cg, size_t* smem) {
  if (cg == 2) {
    if (bn != 256) return nullptr;
    *smem = BnTable<256, 2>::smem();
    return BnTable<256, 2>::get(epi);
  }
  switch (bn) {
    case 16: *smem = BnTable<16>::smem(); return BnTable<16>::get(epi);
    case 32: *smem = BnTable<32>::smem(); return BnTable<32>::get(epi);
    case 64: *smem = BnTable<64>::smem(); return BnTable<64>::get(epi);
    case 128: *smem = BnTable<128>::smem(); return BnTable<128>::get(epi);
    case 256: *smem = BnTable<256>::smem(); return BnTable<256>::get(epi);
    default: return nullptr;
  }
}

// cudaFuncSetAttribute once per (device, kernel)
bool ensure_smem_attr(GemmKernel k, size_t smem) {
  static thread_local int cached_dev = -1;
  static thread_local GemmKernel done[64];
  static thread_local int ndone = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    ndone = 0;
    cached_dev = dev;
  }
  for (int i = 0; i < ndone; ++i)
    if (done[i] == k) return true;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return false;
  if (ndone < 64) done[ndone++] = k;
  return true;
}

}  // namespace

// FM_GEMM_BN_MAX (tuning experiments) caps the block width.
int gemm_bn_for(int64_t N) {
  static const int cap = [] {
    const char* e = getenv("FM_GEMM_BN_MAX");
    const int v = e ? atoi(e) : 256;
    return (v == 64 || v == 128 || v == 256) ? v : 256;
  }();
  int bn = N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256;
  return bn > cap && cap >= 64 && N > 64 ? cap : bn;
}

// CTAs per tile: 256-token blocks run as CTA pairs (256 x 256 tiles, one
// M = 256 MMA per k-block); FM_GEMM_PAIR=0 (tuning experiments) keeps them on
// single CTAs.
int gemm_cg_for(int bn) {
  static const bool pair = [] {
    const char* e = getenv("FM_GEMM_PAIR");
    return !(e && atoi(e) == 0);
  }();
  return bn == 256 && pair ? 2 : 1;
}

namespace {

// Pairs that can be resident at once (clusters of two, one CTA per SM): the
// split-K fix-up waits for contributors, so every pair of a launch must be
// resident together.  Queried once per (device, kernel); num_sms() / 2 when
// the query is unavailable (sizing without a device).
int64_t resident_pairs(GemmKernel k, size_t smem) {
  static thread_local int cached_dev = -1;
  static thread_local GemmKernel keys[64];
  static thread_local int vals[64];
  static thread_local int n = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return num_sms() / 2;
  if (dev != cached_dev) {
    n = 0;
    cached_dev = dev;
  }
  for (int i = 0; i < n; ++i)
    if (keys[i] == k) return vals[i];
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    cudaGetLastError();
    return num_sms() / 2;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(num_sms() & ~1));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();
    return num_sms() / 2;
  }
  const int v = clusters < num_sms() / 2 ? clusters : num_sms() / 2;
  if (n < 64) {
    keys[n] = k;
    vals[n] = v;
    ++n;
  }
  return v;
}

}  // namespace

// Units are split over `groups` (CTAs, or pairs for cg = 2): one group per SM
// (pair of SMs) by default, `cap_groups` at most.  FM_GEMM_CTAS_PER_SM
// (tuning experiments) scales single-CTA grids; the result never exceeds the
// unit count.  Wide blocks (BN >= 64, finished by their head from staged
// partials) are split over at most 2 groups per tile when that still occupies
// half the groups (each head then stages one partial), else over at most 8
// (FM_GEMM_MAX_SPLIT overrides the cap for tuning experiments).
//
// Long reductions (K >= 512 k-blocks, the state vocabulary's E_S^T GEMMs)
// with about as many tiles as groups take whole tiles instead: the grid is
// the largest divisor of the tile count that fits, every group starts its
// tiles at k = 0, and the groups advance through K together, so each k-block
// of A and B is read from DRAM once and served to the other tiles from L2
// (stream-K would start every group at its own k offset, and the
// vocabulary-sized B panel, larger than L2, would be re-read per m-tile).
// Returns CTAs.
// `sizing` (workspace bounds) skips the two whole-tile schedules: the
// stream-K grid bounds theirs for the same shape, and a plan sizes its
// partials at its largest token counts, which must then bound every smaller
// call's stream-K grid as well.
static int64_t gemm_grid_for(int64_t units, int64_t tiles, int bn, int cg, int64_t cap_groups, bool sizing = false,
                             bool whole_short = false) {
  static const int per_sm = [] {
    const char* e = getenv("FM_GEMM_CTAS_PER_SM");
    const int v = e ? atoi(e) : 1;
    return v >= 1 && v <= 4 ? v : 1;
  }();
  static const int split_env = [] {
    const char* e = getenv("FM_GEMM_MAX_SPLIT");
    const int v = e ? atoi(e) : 0;
    return v >= 1 && v <= 8 ? v : 0;
  }();
  const int64_t avail = cg == 2 ? cap_groups : (int64_t)num_sms() * per_sm;
  const int64_t kb = tiles > 0 ? units / tiles : 0;
  // Short reductions of wide blocks (at most 40 k-blocks) with no more tiles
  // than groups: one whole tile per group.  A split tile's fix-up (partials
  // published, waited for, staged and summed by its head) costs more than the
  // half of such a mainloop it saves.  Only for the DiT layers' residual,
  // q/k-norm, GELU and SwiGLU GEMMs (`whole_short`): the context-extension GEMMs keep the split
  // schedule, under which a context extended in chunks equals one extended at
  // once bit for bit (their k segmentation then does not change with the rows).
  if (!sizing && whole_short && bn >= 64 && kb <= 40 && !split_env) {
    if (tiles <= avail) return tiles * cg;
    // w whole tiles per group when they divide evenly and still occupy five
    // eighths of the groups (each group's first epilogue overlaps its next
    // mainloop; the <= 40 k-blocks a group adds cost less than a split's fix-up)
    const int64_t w = (tiles + avail - 1) / avail;
    if (tiles % w == 0 && (tiles / w) * 8 >= avail * 5) return (tiles / w) * cg;
  }
  if (!sizing && kb >= 512 && tiles * 4 >= avail * 3 && !split_env) {
    for (int64_t g = avail < tiles ? avail : tiles; g * 4 >= avail * 3; --g)
      if (tiles % g == 0) return g * cg;
  }
  int64_t g = avail;
  if (bn >= 64) {
    const int64_t max_split = split_env ? split_env : (tiles * 2 >= avail / 2 ? 2 : 8);
    if (g > tiles * max_split) g = tiles * max_split;
  }
  return (units < g ? units : g) * cg;
}

namespace {
struct GemmGeom {
  int bn, cg;
  int64_t m_tiles, n_tiles, kb, units, grid_bound;
};
// m_tiles counts tiles of 128 * cg rows; grid_bound is the largest grid (CTAs)
// a launch of this shape uses (workspace sizing).
GemmGeom gemm_geom(int64_t M, int64_t N, int64_t K) {
  GemmGeom g;
  g.bn = gemm_bn_for(N);
  g.cg = gemm_cg_for(g.bn);
  g.m_tiles = (M + 128 * g.cg - 1) / (128 * g.cg);
  g.n_tiles = (N + g.bn - 1) / g.bn;
  g.kb = (K + 63) / 64;
  g.units = g.m_tiles * g.n_tiles * g.kb;
  g.grid_bound = gemm_grid_for(g.units, g.m_tiles * g.n_tiles, g.bn, g.cg, num_sms() / 2, true);
  return g;
}
}  // namespace

size_t gemm_partials_bytes(int64_t M, int64_t N, int64_t K) {
  const GemmGeom g = gemm_geom(M, N, K);
  return (size_t)g.grid_bound * 2 * g.bn * 128 * sizeof(float);
}

int64_t gemm_counter_slots(int64_t M, int64_t N) {
  const GemmGeom g = gemm_geom(M, N, 64);
  return g.m_tiles * g.cg * g.n_tiles;
}

fm_status gemm_prepare(GemmPlan* p, const void* W, int64_t M, int64_t K, int64_t ldw, const void* X, int64_t N,
                       int64_t ldx, int epi, float* ws, int* counters, int* err) {
  if (!W || !X) return set_error(FM_ERR_INVALID, "gemm: null operand");
  if (M <= 0 || N <= 0 || K <= 0) return set_error(FM_ERR_SHAPE, "gemm: empty shape M=%lld N=%lld K=%lld",
                                                   (long long)M, (long long)N, (long long)K);
  if (K % 8 != 0 || ldw % 8 != 0 || ldx % 8 != 0)
    return set_error(FM_ERR_ALIGN, "gemm: K and leading dimensions must be multiples of 8 (16 bytes)");
  if (M >= (1ll << 31) || N >= (1ll << 31)) return set_error(FM_ERR_SHAPE, "gemm: dimension too large");
  *p = GemmPlan{};
  const GemmGeom g = gemm_geom(M, N, K);
  const int bn = g.bn, cg = g.cg;
  fm_status st = make_tmap_bf16(&p->tmA, W, (uint64_t)M, (uint64_t)K, (uint64_t)ldw, 128);
  if (st) return st;
  // a pair's CTAs each stage half of the block's token rows
  st = make_tmap_bf16(&p->tmB, X, (uint64_t)N, (uint64_t)K, (uint64_t)ldx, (uint32_t)(bn / cg));
  if (st) return st;
  GemmArgs& a = p->args;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.kb = (int)g.kb;
  a.m_tiles = (int)g.m_tiles;
  a.n_tiles = (int)g.n_tiles;
  a.units = (long long)g.units;
  a.ws = ws;
  a.counters = counters;
  a.err = err;
  p->bn = bn;
  p->cg = cg;
  p->epi = epi;
  size_t smem = 0;
  GemmKernel k = kernel_for(bn, epi, cg, &smem);
  if (!k) return set_error(FM_ERR_UNSUPPORTED, "gemm: no kernel for epilogue %d", epi);
  p->smem = smem;
  const int64_t cap = cg == 2 ? resident_pairs(k, smem) : 0;
  p->grid = (int)gemm_grid_for(a.units, (int64_t)a.m_tiles * a.n_tiles, bn, cg, cap, false,
                               epi == EPI_RESID || epi == EPI_QKNORM || epi == EPI_GELU || epi == EPI_SWIGLU);
  return FM_OK;
}

fm_status gemm_launch(const GemmPlan& p, cudaStream_t stream, bool pdl) {
  size_t smem = 0;
  GemmKernel k = kernel_for(p.bn, p.epi, p.cg, &smem);
  if (!k) return set_error(FM_ERR_UNSUPPORTED, "gemm: no kernel for bn %d epilogue %d", p.bn, p.epi);
  const bool split_possible = p.grid > p.cg || p.args.units > p.args.kb;
  if (split_possible && (!p.args.ws || !p.args.counters))
    return set_error(FM_ERR_WORKSPACE, "gemm: split-K workspace missing");
  if (!ensure_smem_attr(k, smem)) return set_error(FM_ERR_CUDA, "gemm: cannot set shared memory size");
  if (p.cg == 1) return launch_kernel(k, dim3(p.grid), dim3(192), smem, stream, pdl, p.tmA, p.tmB, p.args, p.trace);
  if (p.grid % 2 != 0) return set_error(FM_ERR_LAUNCH, "gemm: a pair grid must be even");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k, p.tmA, p.tmB, p.args, p.trace);
  if (e != cudaSuccess) return set_error(FM_ERR_LAUNCH, "gemm pair launch failed: %s", cudaGetErrorString(e));
  ++launch_counter();
  return FM_OK;
}

}  // namespace fm

using namespace fm;

extern "C" size_t fm_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  const size_t tiles = (size_t)gemm_counter_slots(M, N);
  return 256 + ((tiles * sizeof(int) + 255) / 256) * 256 + gemm_partials_bytes(M, N, K);
}

static fm_status gemm_bf16_call(const void* W, const void* X, void* out, int64_t M, int64_t N, int64_t K,
                                int64_t ldo, const void* bias, const void* gate, int epilogue, void* workspace,
                                size_t workspace_bytes, int32_t* err, uint64_t* trace, fm_stream stream) {
  if (!out) return set_error(FM_ERR_INVALID, "gemm: null output");
  if (epilogue != EPI_STORE && epilogue != EPI_GELU && epilogue != EPI_SWIGLU && epilogue != EPI_RESID &&
      epilogue != EPI_F32)
    return set_error(FM_ERR_UNSUPPORTED, "gemm: epilogue %d is not exposed here", epilogue);
  if (epilogue == EPI_RESID && !gate) return set_error(FM_ERR_INVALID, "gemm: residual epilogue needs a gate");
  if (epilogue == EPI_SWIGLU && M % 128 != 0)
    return set_error(FM_ERR_SHAPE, "gemm: swiglu needs M a multiple of 128 (64 features per tile)");
  const size_t need = fm_gemm_workspace_size(M, N, K);
  if (!workspace || workspace_bytes < need)
    return set_error(FM_ERR_WORKSPACE, "gemm: workspace of %zu bytes needed", need);
  const size_t tiles = (size_t)gemm_counter_slots(M, N);
  char* wsb = static_cast<char*>(workspace);
  int* counters = reinterpret_cast<int*>(wsb + 256);
  float* partials = reinterpret_cast<float*>(wsb + 256 + ((tiles * sizeof(int) + 255) / 256) * 256);
  GemmPlan p;
  fm_status st = gemm_prepare(&p, W, M, K, K, X, N, K, epilogue, partials, counters, err);
  if (st) return st;
  p.args.out = static_cast<__nv_bfloat16*>(out);
  p.args.out32 = static_cast<float*>(out);
  p.args.ldo = ldo;
  p.args.bias = static_cast<const __nv_bfloat16*>(bias);
  p.args.gate = static_cast<const __nv_bfloat16*>(gate);
  p.trace = reinterpret_cast<unsigned long long*>(trace);
  return gemm_launch(p, static_cast<cudaStream_t>(stream), false);
}

extern "C" fm_status fm_gemm_bf16(const void* W, const void* X, void* out, int64_t M, int64_t N, int64_t K,
                                  int64_t ldo, const void* bias, const void* gate, int epilogue, void* workspace,
                                  size_t workspace_bytes, int32_t* err, fm_stream stream) {
  return gemm_bf16_call(W, X, out, M, N, K, ldo, bias, gate, epilogue, workspace, workspace_bytes, err, nullptr,
                        stream);
}

extern "C" int32_t fm_gemm_grid(int64_t M, int64_t N, int64_t K) {
  return (int32_t)gemm_geom(M, N, K).grid_bound;
}

#ifdef FM_DEBUG_TRACE
// Debug builds only (not exported by the product library): the same call
// recording per-CTA global-timer stamps (ns) into trace [grid][16].
extern "C" fm_status fm_gemm_bf16_trace(const void* W, const void* X, void* out, int64_t M, int64_t N, int64_t K,
                                        int64_t ldo, const void* bias, const void* gate, int epilogue,
                                        void* workspace, size_t workspace_bytes, int32_t* err, uint64_t* trace,
                                        fm_stream stream) {
  if (!trace) return set_error(FM_ERR_INVALID, "gemm trace: null trace buffer");
  return gemm_bf16_call(W, X, out, M, N, K, ldo, bias, gate, epilogue, workspace, workspace_bytes, err, trace,
                        stream);
}
#endif  // FM_DEBUG_TRACE
