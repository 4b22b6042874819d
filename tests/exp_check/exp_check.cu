// Accuracy of the kernels' own exp (Tang's table-driven method, common.cuh
// exp_tang) and of SiLU / SiLU' built on it with a Newton reciprocal, against
// CUDA's exp and IEEE division, on a dense grid of each range.
//   exp_check          prints the largest errors per range; exit status 0
//                      when exp <= 2 ulp, SiLU <= 8 ulp and the SiLU' error
//                      is at most 4e-15 (1 + |x|) everywhere
#include <cmath>
#include <cstdio>
#include <vector>

#include "../../so3lr_b200/csrc/common.cuh"

using so3lr_b200::exp_tang;
using so3lr_b200::sigmoid;

__device__ double ulps(double a, double b) {
  if (a == b) return 0.0;
  int e;
  frexp(fmax(fabs(a), fabs(b)), &e);
  return fabs(a - b) / ldexp(1.0, e - 53);
}

__global__ void k_errors(int n, double lo, double hi, double *out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double x = lo + (hi - lo) * (i + 0.37) / n;
  const double s_ref = 1.0 / (1.0 + exp(-x)), s = sigmoid(x);
  out[3 * i + 0] = ulps(exp_tang(x), exp(x));
  out[3 * i + 1] = ulps(x * s, x / (1.0 + exp(-x)));
  // SiLU' = s (1 + x (1 - s)): an error in s reaches it multiplied by up to 1 + |x|
  out[3 * i + 2] = fabs(s * (1.0 + x * (1.0 - s)) - s_ref * (1.0 + x * (1.0 - s_ref))) / (1.0 + fabs(x));
}

int main() {
  const int n = 1 << 20;
  double *d = nullptr;
  if (cudaMalloc(&d, sizeof(double) * 3 * n) != cudaSuccess) {
    std::printf("no device memory\n");
    return 2;
  }
  std::vector<double> h(3 * static_cast<std::size_t>(n));
  const double ranges[3][2] = {{-40.0, 40.0}, {-700.0, 700.0}, {-1e-3, 1e-3}};
  bool ok = true;
  for (const auto &rg : ranges) {
    k_errors<<<(n + 255) / 256, 256>>>(n, rg[0], rg[1], d);
    if (cudaMemcpy(h.data(), d, sizeof(double) * 3 * n, cudaMemcpyDeviceToHost) != cudaSuccess) {
      std::printf("CUDA error: %s\n", cudaGetErrorString(cudaGetLastError()));
      return 2;
    }
    double mx[3] = {0.0, 0.0, 0.0};
    for (int i = 0; i < n; ++i)
      for (int k = 0; k < 3; ++k) mx[k] = std::fmax(mx[k], h[3 * static_cast<std::size_t>(i) + k]);
    std::printf("range [%g, %g]: exp %.2f ulp, silu %.2f ulp, silu' %.3e (1 + |x|)\n", rg[0], rg[1], mx[0], mx[1],
                mx[2]);
    ok = ok && mx[0] <= 2.0 && mx[1] <= 8.0 && mx[2] <= 4e-15;
  }
  cudaFree(d);
  std::printf("%s\n", ok ? "EXP CHECK OK" : "EXP CHECK FAIL");
  return ok ? 0 : 1;
}
