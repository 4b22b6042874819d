// FP64 tensor-core (DMMA) throughput of every mma.sync f64 shape, and a check of
// the fragment layouts the kernels rely on (D = A B against a host product).
// In-bounds microbenchmark: registers only, one 8-byte output buffer.
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 fp64_mma_peak.cu -o fp64_mma_peak && ./fp64_mma_peak
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <vector>
#include <cuda_runtime.h>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("CUDA %s: %s\n", #x, cudaGetErrorString(e)); exit(1);} } while (0)

__device__ __forceinline__ void mma884(double (&c)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
               : "+d"(c[0]), "+d"(c[1]) : "d"(a), "d"(b));
}
__device__ __forceinline__ void mma1684(double (&c)[4], const double (&a)[2], double b) {
  asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
               : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3]) : "d"(a[0]), "d"(a[1]), "d"(b));
}
__device__ __forceinline__ void mma1688(double (&c)[4], const double (&a)[4], const double (&b)[2]) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
               : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3]) : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}
__device__ __forceinline__ void mma16816(double (&c)[4], const double (&a)[8], const double (&b)[4]) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7,%8,%9,%10,%11}, {%12,%13,%14,%15}, {%0,%1,%2,%3};\n"
               : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
               : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]),
                 "d"(b[0]), "d"(b[1]), "d"(b[2]), "d"(b[3]));
}

template <int SHAPE, int CH>
__global__ void k_tput(int iters, double seed, double *out) {
  double acc[CH][4];
  for (int c = 0; c < CH; ++c) for (int j = 0; j < 4; ++j) acc[c][j] = 0.0;
  double a[8], b[4];
  for (int j = 0; j < 8; ++j) a[j] = seed * (threadIdx.x + j + 1);
  for (int j = 0; j < 4; ++j) b[j] = seed * (threadIdx.x - j);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      if (SHAPE == 0) { double (&cc)[2] = *reinterpret_cast<double (*)[2]>(acc[c]); mma884(cc, a[c & 7], b[c & 3]); }
      if (SHAPE == 1) { double aa[2] = {a[0], a[1]}; mma1684(acc[c], aa, b[0]); }
      if (SHAPE == 2) { double aa[4] = {a[0], a[1], a[2], a[3]}; double bb[2] = {b[0], b[1]}; mma1688(acc[c], aa, bb); }
      if (SHAPE == 3) { mma16816(acc[c], *reinterpret_cast<double (*)[8]>(a), *reinterpret_cast<double (*)[4]>(b)); }
    }
  }
  double s = 0;
  for (int c = 0; c < CH; ++c) for (int j = 0; j < 4; ++j) s += acc[c][j];
  if (s == 12345.678) out[0] = s;
}

// layout check: D = A(16xK) * B(Kx8), A row-major, B stored as B[k][n]
template <int SHAPE>
__global__ void k_layout(const double *A, const double *B, double *D) {
  const int lane = threadIdx.x, g = lane >> 2, t = lane & 3;
  double c[4] = {0, 0, 0, 0};
  if (SHAPE == 1) {  // m16n8k4
    double a[2] = {A[g * 4 + t], A[(g + 8) * 4 + t]};
    mma1684(c, a, B[t * 8 + g]);
  } else if (SHAPE == 2) {  // m16n8k8
    double a[4] = {A[g * 8 + t], A[(g + 8) * 8 + t], A[g * 8 + t + 4], A[(g + 8) * 8 + t + 4]};
    double b[2] = {B[t * 8 + g], B[(t + 4) * 8 + g]};
    mma1688(c, a, b);
  } else {  // m16n8k16
    double a[8], b[4];
    for (int j = 0; j < 4; ++j) {
      a[2 * j] = A[g * 16 + t + 4 * j];
      a[2 * j + 1] = A[(g + 8) * 16 + t + 4 * j];
      b[j] = B[(t + 4 * j) * 8 + g];
    }
    mma16816(c, a, b);
  }
  D[g * 8 + 2 * t] = c[0];
  D[g * 8 + 2 * t + 1] = c[1];
  D[(g + 8) * 8 + 2 * t] = c[2];
  D[(g + 8) * 8 + 2 * t + 1] = c[3];
}

template <int SHAPE>
void check_layout(const char *name, int K) {
  std::vector<double> A(16 * K), B(K * 8), D(128), R(128, 0.0);
  for (int i = 0; i < 16 * K; ++i) A[i] = (i * 37 % 101) * 0.01 - 0.5;
  for (int i = 0; i < K * 8; ++i) B[i] = (i * 53 % 97) * 0.013 - 0.6;
  for (int m = 0; m < 16; ++m) for (int n = 0; n < 8; ++n) for (int k = 0; k < K; ++k) R[m * 8 + n] += A[m * K + k] * B[k * 8 + n];
  double *dA, *dB, *dD;
  CK(cudaMalloc(&dA, 8 * 16 * K)); CK(cudaMalloc(&dB, 8 * K * 8)); CK(cudaMalloc(&dD, 8 * 128));
  CK(cudaMemcpy(dA, A.data(), 8 * 16 * K, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dB, B.data(), 8 * K * 8, cudaMemcpyHostToDevice));
  k_layout<SHAPE><<<1, 32>>>(dA, dB, dD);
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpy(D.data(), dD, 8 * 128, cudaMemcpyDeviceToHost));
  double err = 0;
  for (int i = 0; i < 128; ++i) err = fmax(err, fabs(D[i] - R[i]));
  printf("layout %-10s max|D-R| = %.3e %s\n", name, err, err < 1e-12 ? "OK" : "MISMATCH");
  cudaFree(dA); cudaFree(dB); cudaFree(dD);
}

template <int SHAPE, int CH>
void tput(const char *name, int warps_per_cta, int ctas_per_sm, double flop_per_mma) {
  double *out; CK(cudaMalloc(&out, 8));
  const int iters = 4000;
  const int grid = 148 * ctas_per_sm;
  k_tput<SHAPE, CH><<<grid, 32 * warps_per_cta>>>(10, 1e-3, out);
  CK(cudaDeviceSynchronize());
  cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
  cudaEventRecord(e0);
  k_tput<SHAPE, CH><<<grid, 32 * warps_per_cta>>>(iters, 1e-3, out);
  cudaEventRecord(e1);
  CK(cudaEventSynchronize(e1));
  float ms; cudaEventElapsedTime(&ms, e0, e1);
  const double flops = double(grid) * warps_per_cta * iters * CH * flop_per_mma;
  printf("%-10s chains=%2d warps/SM=%3d : %6.2f TFLOP/s\n", name, CH, warps_per_cta * ctas_per_sm, flops / (ms * 1e-3) / 1e12);
  cudaFree(out);
}

int main() {
  check_layout<1>("m16n8k4", 4);
  check_layout<2>("m16n8k8", 8);
  check_layout<3>("m16n8k16", 16);
  for (int w : {4, 8, 16, 32}) {
    tput<0, 8>("m8n8k4", 4, w / 4, 512);
    tput<0, 16>("m8n8k4", 4, w / 4, 512);
    tput<1, 8>("m16n8k4", 4, w / 4, 1024);
    tput<2, 4>("m16n8k8", 4, w / 4, 2048);
    tput<2, 8>("m16n8k8", 4, w / 4, 2048);
    tput<3, 4>("m16n8k16", 4, w / 4, 4096);
    tput<3, 8>("m16n8k16", 4, w / 4, 4096);
  }
  return 0;
}
