// Per-device launch configuration shared by the kernel launchers.
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace so3lr_b200 {

void allow_dynamic_smem(const void *func, std::size_t bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void *, int>> done;
  int dev = 0;
  SO3_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({func, dev})) return;
  SO3_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)));
  done.insert({func, dev});
}

}  // namespace so3lr_b200
