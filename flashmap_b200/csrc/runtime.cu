// Library runtime: error state, device checks, TMA descriptor encoding.
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "launch.cuh"

namespace fm {

namespace {
thread_local char g_last_error[512] = "";

// cuTensorMapEncodeTiled, resolved through the runtime so the library does
// not link libcuda directly.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

fm_status set_error(fm_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

long long& launch_counter() {
  static thread_local long long n = 0;
  return n;
}

int num_sms() {
  static thread_local int dev_cached = -1, sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != dev_cached) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    dev_cached = dev;
  }
  return sms;
}

fm_status make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return set_error(FM_ERR_ALIGN, "TMA base not 16-byte aligned");
  if ((ld * 2) % 16 != 0) return set_error(FM_ERR_ALIGN, "TMA row stride not a multiple of 16 bytes");
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(FM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu ld=%llu box=%u", (int)r,
                     (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)ld, box_rows);
  return FM_OK;
}

fm_status make_tmap_bf16_blocks(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                                uint32_t box_rows, uint32_t box_blocks) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return set_error(FM_ERR_ALIGN, "TMA base not 16-byte aligned");
  if ((ld * 2) % 16 != 0) return set_error(FM_ERR_ALIGN, "TMA row stride not a multiple of 16 bytes");
  if (cols % 64 != 0 || box_blocks == 0 || box_blocks > 256 || box_blocks > cols / 64)
    return set_error(FM_ERR_SHAPE, "block view needs cols %% 64 == 0 and 1..256 blocks per box");
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(FM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {ld * 2, 128};
  cuuint32_t box[3] = {64, box_rows, box_blocks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FM_ERR_CUDA, "cuTensorMapEncodeTiled (blocks) failed (%d) rows=%llu cols=%llu box=%u", (int)r,
                     (unsigned long long)rows, (unsigned long long)cols, box_blocks);
  return FM_OK;
}

}  // namespace fm

extern "C" const char* fm_last_error(void) { return fm::g_last_error; }

extern "C" int fm_version(void) { return 1; }

extern "C" fm_status fm_check_device(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fm::set_error(FM_ERR_CUDA, "no CUDA device: %s", cudaGetErrorString(e));
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fm::set_error(FM_ERR_ARCH, "device %d is sm_%d%d; this library is built for sm_100a", dev, major, minor);
  return FM_OK;
}
