// Periodic-image codes shared by the edge builder, the pair geometry and the
// long-range kernel.
#pragma once
#include "kernels.cuh"

namespace so3lr_b200 {

__host__ __device__ inline int pack_image(int a, int b, int c) {
  return ((a + 512) << 20) | ((b + 512) << 10) | (c + 512);
}
__device__ inline void unpack_image(int code, int &a, int &b, int &c) {
  a = ((code >> 20) & 1023) - 512;
  b = ((code >> 10) & 1023) - 512;
  c = (code & 1023) - 512;
}
__device__ inline int negate_image(int code) {
  int a, b, c;
  unpack_image(code, a, b, c);
  return pack_image(-a, -b, -c);
}
constexpr int kZeroImage = (512 << 20) | (512 << 10) | 512;

}  // namespace so3lr_b200
