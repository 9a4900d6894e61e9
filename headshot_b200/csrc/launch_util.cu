// launch_util.cu — host helpers shared by the kernel launchers: TMA tensor
// maps, the dynamic shared-memory limit of large-smem kernels, and the SM
// count that sizes persistent grids.
//
// cuTensorMapEncodeTiled is a driver API function; it is reached through the
// runtime's driver entry point so the library links only the CUDA runtime.
#include <cuda.h>

#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "hs_internal.h"

namespace hs {

EncodeTiledFn encode_tiled_fn() {
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

bool make_row_map(CUtensorMap* map, const void* base, const RowLayout& l, bool bf16, uint32_t t, uint32_t heads,
                  uint32_t seqs, uint32_t box_rows, std::string* err) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) {
    if (err) *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(t), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(seqs)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(l.t) * 2, static_cast<cuuint64_t>(l.h) * 2,
                           static_cast<cuuint64_t>(l.s) * 2};
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

cudaError_t ensure_dynamic_smem(const void* func, int bytes) {
  // A kernel's attributes belong to its instance in the current device's
  // context, so the limit is raised once per (kernel, device) pair.
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& d : done)
    if (d.first == func && d.second == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.emplace_back(func, dev);
  return e;
}

int current_sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace hs
