// Host-side helpers shared by the C-ABI implementation files: error state,
// kernel launch with programmatic dependent launch, TMA descriptor encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <utility>

#include "../../include/flashmap_b200.h"

namespace fm {

fm_status set_error(fm_status code, const char* fmt, ...);

// kernels launched by this thread through launch_kernel (for launch accounting)
long long& launch_counter();

inline fm_status check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FM_OK;
  return set_error(FM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Launch `kernel` with the programmatic-stream-serialization attribute when
// `pdl` is set: the kernel may then start while the previous kernel of the
// stream finishes, and must call griddepcontrol.wait before it touches data
// that kernel produces (every kernel of this library does).
template <typename... KArgs, typename... Args>
fm_status launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                        Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return set_error(FM_ERR_LAUNCH, "kernel launch failed: %s", cudaGetErrorString(e));
  ++launch_counter();
  return FM_OK;
}

// 2D bf16 tensor map over a row-major [rows, cols] matrix with leading
// dimension ld (elements): boxes of [box_rows x 64] with 128-byte swizzling.
fm_status make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows);

// The same matrix viewed as [cols / 64][rows][64] (cols % 64 == 0): boxes of
// box_blocks consecutive 64-column blocks of box_rows rows, each block landing
// as its own 128-byte-swizzled [box_rows x 64] tile.
fm_status make_tmap_bf16_blocks(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                                uint32_t box_rows, uint32_t box_blocks);

int num_sms();

}  // namespace fm
