// Whether FP64 tensor (DMMA) and FP64 scalar (DFMA) work share one pipe: half
// the warps of every CTA issue m8n8k4 DMMA chains, the other half DFMA chains;
// mode 1 runs the DMMA half only, mode 2 the DFMA half only, mode 3 both.
// If the two were independent, mode 3 would take max(mode 1, mode 2).
// In-bounds microbenchmark: registers only, one 8-byte output buffer.
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 fp64_pipe_share.cu -o fp64_pipe_share && ./fp64_pipe_share
#include <cstdio>
#include <cuda_runtime.h>
__device__ __forceinline__ void mma884(double &c0, double &c1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n" : "+d"(c0), "+d"(c1) : "d"(a), "d"(b));
}
// warps 0-3 and 8-11 of a 512-thread CTA run DMMA if mode & 1; warps 4-7 and 12-15 run DFMA if mode & 2
__global__ void k(int iters, int mode, double seed, double *out) {
  const int warp = threadIdx.x >> 5;
  double s = 0;
  if (((warp >> 2) & 1) == 0 && (mode & 1)) {
    double c[16][2];
    for (int i = 0; i < 16; ++i) c[i][0] = c[i][1] = 0;
    const double a = seed * threadIdx.x, b = seed + threadIdx.x;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int i = 0; i < 16; ++i) mma884(c[i][0], c[i][1], a, b);
    }
    for (int i = 0; i < 16; ++i) s += c[i][0] + c[i][1];
  } else if (((warp >> 2) & 1) == 1 && (mode & 2)) {
    double x[16];
    for (int i = 0; i < 16; ++i) x[i] = seed * (threadIdx.x + i);
    const double m = 1.0 + seed;
    for (int it = 0; it < iters * 4; ++it) {
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = fma(x[i], m, seed);
    }
    for (int i = 0; i < 16; ++i) s += x[i];
  }
  if (s == 1234.5) out[0] = s;
}
int main() {
  double *out; cudaMalloc(&out, 8);
  const int iters = 20000, threads = 512, grid = 148;
  k<<<grid, threads>>>(10, 3, 1e-9, out);
  cudaDeviceSynchronize();
  for (int mode : {1, 2, 3}) {
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    cudaEventRecord(a);
    k<<<grid, threads>>>(iters, mode, 1e-9, out);
    cudaEventRecord(b); cudaEventSynchronize(b);
    float ms; cudaEventElapsedTime(&ms, a, b);
    const double dmma_flop = (mode & 1) ? double(grid) * (threads / 64) * 32 * 0 + double(grid) * (threads / 64) * iters * 16 * 512.0 : 0;
    const double dfma_flop = (mode & 2) ? double(grid) * (threads / 64) * 32 * iters * 4 * 16 * 2.0 : 0;
    printf("mode %d (%s): %.3f ms  DMMA %.2f TF/s  DFMA %.2f TF/s\n", mode, mode == 1 ? "DMMA only" : mode == 2 ? "DFMA only" : "both",
           ms, dmma_flop / (ms * 1e-3) / 1e12, dfma_flop / (ms * 1e-3) / 1e12);
  }
  printf("%s\n", cudaGetErrorString(cudaGetLastError()));
  return 0;
}
