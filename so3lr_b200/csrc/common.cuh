// Shared device definitions for the SO3LR B200 kernels.
//
// Fixed model shape (the capability table in model_host.cpp refuses anything
// else): F = 128 invariant features, 4 heads of 32 channels, equivariant
// degrees l = 1..4 (24 channels), 32 Bernstein radial functions, 32-wide
// hidden layer in the equivariant filter branch.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace so3lr_b200 {

constexpr int kF = 128;       // invariant features
constexpr int kHeads = 4;     // attention heads == equivariant degrees
constexpr int kHW = 32;       // head width
constexpr int kEV = 24;       // equivariant channels (l = 1..4)
constexpr int kR = 32;        // radial basis functions
constexpr int kEH = 32;       // hidden width of the ev filter branch (F / 4)
constexpr int kQKV = 5 * kF;  // q, k, v, q_ev, k_ev per node, head-major [4][5][32]
constexpr int kIntW = 136;    // 132-wide interaction layer padded to a multiple of 8
constexpr int kHeadHidden = 128;
constexpr int kHirsh = 64;
constexpr int kHeadCat = 2 * kHeadHidden + kHirsh;  // fused first layers of the 3 heads
constexpr int kMaxLayers = 8;
constexpr int kPairScalars = 32;  // per pair, per block: alpha / s for both directions
// Algorithmic FLOPs of the two filter MLPs of one pair, one direction of the
// pass (forward, or the reverse input gradients): 2 filters x (R F + F F + 4 H + H F)
// multiply-adds x 2. The reverse's first-layer recompute is not counted.
constexpr double kFilterFlopsPerPair = 2.0 * (kR * kF + kF * kF + 4 * kEH + kEH * kF) * 2.0;

inline void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
}
// number of kernels this library has launched in the process (every launcher
// calls SO3_LAUNCH exactly once per kernel launch)
long long &launch_counter();
#define SO3_CUDA(x) ::so3lr_b200::cuda_check((x), #x)
#define SO3_LAUNCH(what) (++::so3lr_b200::launch_counter(), ::so3lr_b200::cuda_check(cudaGetLastError(), what))

// degree slot of equivariant channel m (0..23): 3 + 5 + 7 + 9
__host__ __device__ inline int degree_of_channel(int m) { return m < 3 ? 0 : (m < 8 ? 1 : (m < 15 ? 2 : 3)); }
// (-1)^l for the degree slot (l = slot + 1): odd l flips sign under v -> -v
__host__ __device__ inline double parity_sign(int slot) { return (slot & 1) ? 1.0 : -1.0; }

// FP64 tensor-core MMA: D(8x8) = A(8x4, row) * B(4x8, col) + C.
// Fragment ownership (lane = threadIdx.x % 32, g = lane >> 2, t = lane & 3):
//   a = A[g][t], b = B[t][g], c0/c1 = C[g][2t], C[g][2t+1].
__device__ __forceinline__ void dmma(double &c0, double &c1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
               : "+d"(c0), "+d"(c1)
               : "d"(a), "d"(b));
}

__device__ __forceinline__ double silu(double x) { return x / (1.0 + exp(-x)); }
__device__ __forceinline__ double silu_prime(double x) {
  const double s = 1.0 / (1.0 + exp(-x));
  return s * (1.0 + x * (1.0 - s));
}

// Device view of the model weights (all float64, row-major as stored in the
// `.so3lr` file unless noted).
struct FilterW {
  const double *w0, *b0;  // [128][32], [128]   rbf -> hidden
  const double *w1, *b1;  // [128][128], [128]  hidden -> filter
  const double *v0, *c0;  // [32][4], [32]      L0 -> ev hidden
  const double *v1, *c1;  // [128][32], [128]   ev hidden -> filter
  // The same matrices as DMMA B operands in fragment-major order (see
  // fragment_major in evaluator.cu): B(k, n) of a K x N operand sits at
  // [k/4][n/32][lane = 4 (n%8) + k%4][(n%32)/8].
  const double *w0t_f;    // K=32,  N=128: B(r, j) = w0[j][r]   forward layer 0 / reverse recompute
  const double *w1t_f;    // K=128, N=128: B(j, o) = w1[o][j]   forward layer 1
  const double *v1t_f;    // K=32,  N=128: B(h, o) = v1[o][h]   forward ev layer 1
  const double *w1_f;     // K=128, N=128: B(o, j) = w1[o][j]   reverse through layer 1
  const double *v1_f;     // K=128, N=32:  B(o, h) = v1[o][h]   reverse through ev layer 1
  const double *w0_f;     // K=128, N=32:  B(j, r) = w0[j][r]   reverse through layer 0
};
struct BlockW {
  FilterW finv, fev;
  const double *cg_att, *cg_int;   // [24]
  const double *qkv_fwd;           // [4 heads][160 out (proj,o)][32 in]   (B col layout)
  const double *qkv_rev;           // [4 heads][32 out i][160 in (proj,o)] (B col layout)
  const double *ln1w, *ln1b, *ln2w, *ln2b;  // [128]
  const double *mlp1w, *mlp1b, *mlp2w, *mlp2b;  // [128][128], [128]
  const double *intw, *intb;       // padded [136][136], [136]
};
struct HeadsW {
  const double *w1cat, *b1cat;     // [320][128], [320]: energy, charge, Hirshfeld first layers
  const double *e_w2;              // [128]
  double e_b2;
  const double *e_scale, *e_shift; // [118]
  const double *c_w2;              // [128]
  double c_b2;
  const double *c_emb;             // [100]
  const double *h_w2, *h_b2;       // [64][64], [64]
  const double *h_qemb, *h_vshift; // [100][64], [100]
};
struct RadialW {
  const double *b;                 // [32]
  const double *k, *kr;            // [32] as doubles
  double gamma;
};

}  // namespace so3lr_b200
