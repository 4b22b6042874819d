// Shared device definitions for the SO3LR B200 kernels.
//
// Model shapes. The kernels are compiled once per supported model width: the
// translation units whose code depends on the width (attention, filters, node
// layers, evaluator) are built with SO3LR_FEATURES = 128 and again with 256,
// and each build's code lives in its own namespace (so3lr_b200::f128 /
// so3lr_b200::f256, opened with SO3LR_SHAPE_BEGIN). Everything else is
// width-independent and built once.
//   F = 128: 4 heads of 32, degrees {1,2,3,4} (24 equivariant channels),
//            32 Bernstein radial functions, 32-wide ev-filter hidden layer
//            (the released SO3LR v1/s/m shape);
//   F = 256: 8 heads of 32, degrees {1,1,2,2,3,3,4,4} (48 channels), 64 radial
//            functions, 64-wide ev-filter hidden layer (the "l" shape).
// The capability table in model_host.cpp refuses every other shape.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <stdexcept>
#include <string>

#ifndef SO3LR_FEATURES
#define SO3LR_FEATURES 128
#endif
#if SO3LR_FEATURES == 128
#define SO3LR_SHAPE_NS f128
#elif SO3LR_FEATURES == 256
#define SO3LR_SHAPE_NS f256
#else
#error "SO3LR_FEATURES must be 128 or 256"
#endif
#define SO3LR_SHAPE_BEGIN \
  namespace so3lr_b200 {  \
  inline namespace SO3LR_SHAPE_NS {
#define SO3LR_SHAPE_END \
  }                     \
  }

namespace so3lr_b200 {

constexpr int kSH = 24;       // distinct real harmonics l = 1..4 (per pair)
constexpr int kHW = 32;       // head width
constexpr int kHeadHidden = 128;
constexpr int kHirsh = 64;
constexpr int kHeadCat = 2 * kHeadHidden + kHirsh;  // fused first layers of the 3 heads
constexpr int kHeadCatC6 = kHeadCat + kHirsh;        // ... and of the optional C6 ratio head
constexpr int kMaxLayers = 8;

}  // namespace so3lr_b200

SO3LR_SHAPE_BEGIN
constexpr int kF = SO3LR_FEATURES;   // invariant features
constexpr int kHeads = kF / kHW;     // attention heads == equivariant degree slots
constexpr int kR = kF / 4;           // radial basis functions
constexpr int kEH = kF / 4;          // hidden width of the ev filter branch
constexpr int kQKV = 5 * kF;         // q, k, v, q_ev, k_ev per node, head-major [heads][5][32]
constexpr int kIntW = (kF + kHeads + 7) / 8 * 8;  // interaction layer (F + heads) padded to a multiple of 8
// equivariant channels: degree slot s has 2 l_s + 1 channels, l_s = s + 1
// (F = 128) or s / 2 + 1 (F = 256, every degree twice)
constexpr int kDupDegrees = kHeads / 4;
__host__ __device__ constexpr int slot_degree(int s) { return s / kDupDegrees + 1; }
__host__ __device__ constexpr int slot_width(int s) { return 2 * slot_degree(s) + 1; }
// first channel of slot s: every degree below l_s fills kDupDegrees slots
// of 2 l + 1 channels (sum = l_s^2 - 1 per copy), then the earlier copies of l_s
__host__ __device__ constexpr int slot_offset(int s) {
  return kDupDegrees * (slot_degree(s) * slot_degree(s) - 1) + (s % kDupDegrees) * slot_width(s);
}
constexpr int kEV = slot_offset(kHeads);  // 24 or 48
// per pair, per block: the cutoff-gradient weight and the ev attention
// coefficients of both directions per head (+1 pad: rows of 16-byte chunks)
constexpr int kPairScalars = 2 * kHeads + 2;
// Algorithmic FLOPs of the two filter MLPs of one pair, one direction of the
// pass (forward, or the reverse input gradients): 2 filters x (R F + F F + H EH + EH F)
// multiply-adds x 2. The reverse's first-layer recompute is not counted.
constexpr double kFilterFlopsPerPair = 2.0 * (kR * kF + kF * kF + kHeads * kEH + kEH * kF) * 2.0;

// degree slot of equivariant channel m
__host__ __device__ inline int degree_of_channel(int m) {
  int s = 0;
#pragma unroll
  for (int k = 1; k < kHeads; ++k) s += m >= slot_offset(k) ? 1 : 0;
  return s;
}
// the distinct harmonic (0..23, l = 1..4 ascending) that channel m carries
__host__ __device__ inline int sh_of_channel(int m) {
  const int s = degree_of_channel(m), l = slot_degree(s);
  return l * l - 1 + (m - slot_offset(s));
}
// (-1)^l of a degree slot: odd l flips sign under v -> -v
__host__ __device__ inline double parity_sign(int slot) { return (slot_degree(slot) & 1) ? -1.0 : 1.0; }
SO3LR_SHAPE_END

namespace so3lr_b200 {

inline void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
}
// number of kernels this library has launched in the process (every launcher
// calls SO3_LAUNCH exactly once per kernel launch)
std::atomic<long long> &launch_counter();
#define SO3_CUDA(x) ::so3lr_b200::cuda_check((x), #x)

// Allow `bytes` of dynamic shared memory for kernel `func` on the current
// device. The attribute is per device, so it is set once per (kernel, device),
// thread-safely (launch.cpp).
void allow_dynamic_smem(const void *func, std::size_t bytes);
#define SO3_LAUNCH(what) (++::so3lr_b200::launch_counter(), ::so3lr_b200::cuda_check(cudaGetLastError(), what))


// FP64 tensor-core MMA: D(8x8) = A(8x4, row) * B(4x8, col) + C.
// Fragment ownership (lane = threadIdx.x % 32, g = lane >> 2, t = lane & 3):
//   a = A[g][t], b = B[t][g], c0/c1 = C[g][2t], C[g][2t+1].
__device__ __forceinline__ void dmma(double &c0, double &c1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
               : "+d"(c0), "+d"(c1)
               : "d"(a), "d"(b));
}

// exp(x) by Tang's table-driven method (P. T. P. Tang, "Table-driven
// implementation of the exponential function in IEEE floating-point
// arithmetic", ACM TOMS 15(2), 1989): x = (32 m + j) ln2/32 + r with
// |r| <= ln2/64, exp(x) = 2^m 2^(j/32) (1 + p(r)), p the degree-6 Taylor
// polynomial of exp(r) - 1 (truncation below 4e-18). 2^(j/32) is a table of
// correctly rounded doubles; ln2/32 is split into L1 (42 significant bits, so
// N L1 is exact) and L2. Arguments are clamped to [-700, 700], which keeps every
// result normal. Measured against CUDA's exp over [-700, 700]: at most 1 ulp.
static __device__ const double kExp2Frac[32] = {
    0x1.0000000000000p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0, 0x1.11301d0125b51p+0,
    0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0, 0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0,
    0x1.306fe0a31b715p+0, 0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,
    0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0, 0x1.6247eb03a5585p+0,
    0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0, 0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0,
    0x1.8ace5422aa0dbp+0, 0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f090p+0, 0x1.a5503b23e255dp+0,
    0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0, 0x1.cb720dcef9069p+0,
    0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0, 0x1.ea4afa2a490dap+0, 0x1.f50765b6e4540p+0,
};
__device__ __forceinline__ double exp_tang(double x) {
  x = fmin(fmax(x, -700.0), 700.0);
  const double shifter = 0x1.8p52;            // 1.5 * 2^52: rounds to an integer in the low bits
  const double inv_l = 0x1.71547652b82fep+5;  // 32 / ln2
  const double l1 = 0x1.62e42fefa3800p-6, l2 = 0x1.ef35793c76730p-50;  // ln2 / 32 = l1 + l2
  const double t = fma(x, inv_l, shifter);
  const double nd = t - shifter;
  const int n = static_cast<int>(__double_as_longlong(t) - __double_as_longlong(shifter));
  const int j = n & 31, m = n >> 5;
  double r = fma(-nd, l1, x);
  r = fma(-nd, l2, r);
  const double q = fma(fma(fma(fma(r, 1.0 / 720.0, 1.0 / 120.0), r, 1.0 / 24.0), r, 1.0 / 6.0), r, 0.5);
  const double p = fma(r * r, q, r);
  const double s = __ldg(&kExp2Frac[j]);
  const double v = fma(s, p, s);  // in [1, 2): adding m to the exponent field keeps it normal
  return __longlong_as_double(__double_as_longlong(v) + (static_cast<long long>(m) << 52));
}
// 1/d for d >= 1: hardware reciprocal estimate refined by two Newton steps
__device__ __forceinline__ double rcp_newton(double d) {
  double y;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(d));
  double e = fma(-d, y, 1.0);
  y = fma(y, e, y);
  e = fma(-d, y, 1.0);
  return fma(y, e, y);
}
__device__ __forceinline__ double sigmoid(double x) { return rcp_newton(1.0 + exp_tang(-x)); }
// FP64 tensor-core MMA: D(16x8) = A(16x8, row) * B(8x8, col) + C. Fragment
// ownership (g = lane >> 2, t = lane & 3; k slots s0 = t, s1 = t + 4):
//   a = {A[g][s0], A[g+8][s0], A[g][s1], A[g+8][s1]}, b = {B[s0][g], B[s1][g]},
//   c = {C[g][2t], C[g][2t+1], C[g+8][2t], C[g+8][2t+1]}.
__device__ __forceinline__ void dmma16(double (&c)[4], const double (&a)[4], const double (&b)[2]) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};\n"
               : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
               : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}

// A fragment of an m16n8k8 DMMA from a row-major shared-memory tile whose MMA k
// slots t and t + 4 of k-step ks are the physical columns 8 ks + 2t and
// 8 ks + 2t + 1 (a permutation of the contraction index; the B operand uses the
// same one), so a lane's two values of a row are one 16-byte load:
// a = {A[r+g][c], A[r+g+8][c], A[r+g][c+1], A[r+g+8][c+1]}, c = 8 ks + 2t
__device__ __forceinline__ void load_afrag(const double *A, int lda, int r, int ks, int g, int t, double (&a)[4]) {
  const double2 x = *reinterpret_cast<const double2 *>(A + (r + g) * lda + 8 * ks + 2 * t);
  const double2 y = *reinterpret_cast<const double2 *>(A + (r + g + 8) * lda + 8 * ks + 2 * t);
  a[0] = x.x;
  a[1] = y.x;
  a[2] = x.y;
  a[3] = y.y;
}

// 16-byte global -> shared copies that bypass registers
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ double silu(double x) { return x * sigmoid(x); }
__device__ __forceinline__ double silu_prime(double x) {
  const double s = sigmoid(x);
  return s * (1.0 + x * (1.0 - s));
}

// Device view of the model weights (all float64, row-major as stored in the
// `.so3lr` file unless noted).
struct FilterW {
  const double *w0, *b0;  // [128][32], [128]   rbf -> hidden
  const double *w1, *b1;  // [128][128], [128]  hidden -> filter
  const double *v0, *c0;  // [32][4], [32]      L0 -> ev hidden
  const double *v1, *c1;  // [128][32], [128]   ev hidden -> filter
  const double *bc1;      // [128]: b1 + c1, the filter's total output bias
  // The same matrices as m16n8k8 DMMA B operands in fragment-major order (see
  // fragment_major in evaluator.cu): B(k, n) of a K x N operand sits at
  // [k/8][n/32][lane = 4 (n%8) + (k%8)/2][(n%32)/8][k%2].
  const double *w0t_f;    // K=32,  N=128: B(r, j) = w0[j][r]   forward layer 0 / reverse recompute
  const double *w1t_f;    // K=128, N=128: B(j, o) = w1[o][j]   forward layer 1
  const double *v1t_f;    // K=32,  N=128: B(h, o) = v1[o][h]   forward ev layer 1
  const double *w1_f;     // K=128, N=128: B(o, j) = w1[o][j]   reverse through layer 1
  const double *v1_f;     // K=128, N=32:  B(o, h) = v1[o][h]   reverse through ev layer 1
  const double *w0_f;     // K=128, N=32:  B(j, r) = w0[j][r]   reverse through layer 0
};
// The filter matrices for the mixed-precision kernels (filter_mixed.cu): every
// fragment-major operand of FilterW split into two TF32 parts, x = hi + lo up to
// 2^-22 |x| (hi = x rounded to TF32, lo = the rest rounded to TF32), in float;
// biases and the ev branch's first layer in float. Same fragment-major order as
// FilterW, with floats in place of doubles.
struct FilterW32 {
  const float *b0, *bc1;           // [128]
  const float *v0, *c0;            // [32][4], [32]
  const float *w0t_h, *w0t_l, *w1t_h, *w1t_l, *v1t_h, *v1t_l;  // forward operands
  const float *w1_h, *w1_l, *v1_h, *v1_l, *w0_h, *w0_l;        // reverse operands
  // forward operands for the tcgen05 kernel (filter_tc.cu): six [128 x 32]
  // K-chunks -- W0, W1 columns 0-31, 32-63, 64-95, 96-127, V1 -- each as a TF32
  // hi tile then a lo tile of 16 KB in the 128-byte-swizzled K-major layout of
  // the tensor core's shared-memory operands (32 KB per chunk, 192 KB in all)
  const float *tc_fwd;
  // reverse operands for the tcgen05 kernel: for K-chunk c = 0..3 a 40 KB group
  // [W1^T chunk (128 rows) hi | lo][V1^T chunk (32 rows) hi | lo], then for
  // c = 0..3 an 8 KB group [W0^T chunk (32 rows) hi | lo], same layout
  const float *tc_rev;
};
// Per-block constants of the tcgen05 filter kernels, passed by value as kernel
// parameters (the constant bank: one broadcast read per warp instead of a
// global load on the epilogue's critical path). Index 0: invariant filter, 1: ev.
struct TcFwdConsts {
  float b0[2][128], bc1[2][128], v0[2][128], c0[2][32];
  double rb[32], rk[32], rkr[32], gamma;  // radial basis
  double cg[24];                          // L0 weights of the block's attention
};
struct TcRevConsts {
  double v0[2][128], c0[2][32];
  double cg[24];
};
struct BlockW {
  FilterW finv, fev;
  FilterW32 finv32, fev32;
  const double *cg_att, *cg_int;   // [24]
  const double *qkv_fwd;           // [4 heads][160 out (proj,o)][32 in]   (B col layout)
  const double *qkv_rev;           // [4 heads][32 out i][160 in (proj,o)] (B col layout)
  const double *ln1w, *ln1b, *ln2w, *ln2b;  // [128]
  const double *mlp1w, *mlp1b, *mlp2w, *mlp2b;  // [128][128], [128]
  const double *intw, *intb;       // padded [136][136], [136]
};
struct HeadsW {
  const double *w1cat, *b1cat;     // [ldh][128], [ldh]: energy, charge, Hirshfeld (, C6) first layers
  const double *e_w2;              // [128]
  double e_b2;
  const double *e_scale, *e_shift; // [118]
  const double *c_w2;              // [128]
  double c_b2;
  const double *c_emb;             // [100]
  const double *h_w2, *h_b2;       // [64][64], [64]
  const double *h_w2t;             // [64][64]: h_w2 transposed ([in][out])
  const double *h_qemb, *h_vshift; // [100][64], [100]
  double h_sqrt_k;                 // sqrt(number of keys); keys beyond it are zero-padded to 64
  // optional C6 ratio head (c6_w2 == nullptr when absent), same layout
  const double *c6_w2, *c6_b2, *c6_w2t, *c6_qemb, *c6_vshift;
  double c6_sqrt_k;
  int ldh;                         // row width of the fused first layers: kHeadCat or kHeadCatC6
};
struct RadialW {
  const double *b;                 // [32]
  const double *k, *kr;            // [32] as doubles
  double gamma;
};

}  // namespace so3lr_b200
