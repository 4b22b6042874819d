// Mixed-precision pair-filter MLPs (the opt-in SO3LR_PRECISION_MIXED mode):
// the same pair tiles, data flow and outputs as the float64 kernels of
// filter.cu, with every GEMM on the TF32 tensor cores in three passes and
// float32 accumulation, and the hidden-layer SiLU in float32.
//
// Three-pass TF32 ("3xTF32"): an operand x is held as two TF32 numbers,
// x = hi + lo with hi = x rounded to TF32 and lo = (x - hi) rounded to TF32, and
// A B = A_lo B_hi + A_hi B_lo + A_hi B_hi (the A_lo B_lo term is below float32
// resolution). The products are float32-accurate; plain TF32 (one pass) is not
// accurate enough here (force MAE 2e-4 eV/A against float64 on a 1,029-atom
// water box, against 1.6e-7 with three passes). Weights are split once at load
// time (FilterW32); activations are split when they are written to shared
// memory, once per element, not per warp that reads them.
//
// Everything around the GEMMs stays float64: the radial basis and its
// derivative, the L0 invariants, the filters written for the attention
// kernels, the reverse's radial, harmonic and L0 gradients, and the pair tail.
// The float32 silu' values take the float64 path's buffer (half of it).
//
// m16n8k8 TF32 fragments have the ownership of the float64 ones
// (common.cuh: a = {A[g][s0], A[g+8][s0], A[g][s1], A[g+8][s1]}, b = {B[s0][g],
// B[s1][g]}), so the permuted-k shared-memory tiles and the fragment-major
// weight order carry over with floats in place of doubles.
#include <cooperative_groups.h>

#include "filter_common.cuh"
#include "kernels.cuh"

SO3LR_SHAPE_BEGIN
namespace {

__device__ __forceinline__ float tf32_hi(float x) {
  unsigned r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// x = hi + lo, both TF32
__device__ __forceinline__ void split_tf32(float x, float &hi, float &lo) {
  hi = tf32_hi(x);
  lo = tf32_hi(x - hi);
}
__device__ __forceinline__ void store_split2(float *h, float *l, float x0, float x1) {
  float h0, l0, h1, l1;
  split_tf32(x0, h0, l0);
  split_tf32(x1, h1, l1);
  *reinterpret_cast<float2 *>(h) = make_float2(h0, h1);
  *reinterpret_cast<float2 *>(l) = make_float2(l0, l1);
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], const float (&a)[4], const float (&b)[2]) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};\n"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(__float_as_uint(a[0])), "r"(__float_as_uint(a[1])), "r"(__float_as_uint(a[2])),
                 "r"(__float_as_uint(a[3])), "r"(__float_as_uint(b[0])), "r"(__float_as_uint(b[1])));
}
// c += a b in three passes, the small terms first
__device__ __forceinline__ void mma_3x(float (&c)[4], const float (&ah)[4], const float (&al)[4],
                                       const float (&bh)[2], const float (&bl)[2]) {
  mma_tf32(c, al, bh);
  mma_tf32(c, ah, bl);
  mma_tf32(c, ah, bh);
}

// A fragment from a float tile with the permuted k slots of load_afrag
__device__ __forceinline__ void load_afrag32(const float *A, int lda, int r, int ks, int g, int t, float (&a)[4]) {
  const float2 x = *reinterpret_cast<const float2 *>(A + (r + g) * lda + 8 * ks + 2 * t);
  const float2 y = *reinterpret_cast<const float2 *>(A + (r + g + 8) * lda + 8 * ks + 2 * t);
  a[0] = x.x;
  a[1] = y.x;
  a[2] = x.y;
  a[3] = y.y;
}
// B fragments of a fragment-major float operand (8 floats per lane and k-step)
template <int NB>
__device__ __forceinline__ void load_bfrag32(const float *__restrict__ Bf, int ks, int nslab, int slab, int ni0,
                                             int lane, float (&b)[NB][2]) {
  const float2 *q = reinterpret_cast<const float2 *>(Bf + ((size_t)(ks * nslab + slab) * 32 + lane) * 8) + ni0;
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    const float2 v = __ldg(q + j);
    b[j][0] = v.x;
    b[j][1] = v.y;
  }
}

// acc += A(64 x K, split tile) * B(K x 128, split operand): warp slab 64 x 16
template <int K>
__device__ inline void mma3_64x16(float (&acc)[4][2][4], const float *Ah, const float *Al, int lda,
                                  const float *__restrict__ Bh, const float *__restrict__ Bl, int wc, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll 2
  for (int ks = 0; ks < K / 8; ++ks) {
    float bh[2][2], bl[2][2];
    load_bfrag32<2>(Bh, ks, 4, wc >> 1, (wc & 1) * 2, lane, bh);
    load_bfrag32<2>(Bl, ks, 4, wc >> 1, (wc & 1) * 2, lane, bl);
#pragma unroll
    for (int mi = 0; mi < 4; ++mi) {
      float ah[4], al[4];
      load_afrag32(Ah, lda, mi * 16, ks, g, t, ah);
      load_afrag32(Al, lda, mi * 16, ks, g, t, al);
#pragma unroll
      for (int ni = 0; ni < 2; ++ni) mma_3x(acc[mi][ni], ah, al, bh[ni], bl[ni]);
    }
  }
}

// acc += A(rows r0.., K, split tile) * B(K x 32, split operand): warp tile 16 x 16
template <int K>
__device__ inline void mma3_16x16(float (&acc)[2][4], const float *Ah, const float *Al, int lda, int r0,
                                  const float *__restrict__ Bh, const float *__restrict__ Bl, int wc, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll 4
  for (int ks = 0; ks < K / 8; ++ks) {
    float ah[4], al[4], bh[2][2], bl[2][2];
    load_afrag32(Ah, lda, r0, ks, g, t, ah);
    load_afrag32(Al, lda, r0, ks, g, t, al);
    load_bfrag32<2>(Bh, ks, 1, 0, 2 * wc, lane, bh);
    load_bfrag32<2>(Bl, ks, 1, 0, 2 * wc, lane, bl);
#pragma unroll
    for (int j = 0; j < 2; ++j) mma_3x(acc[j], ah, al, bh[j], bl[j]);
  }
}

__device__ __forceinline__ float sigmoid_f(float x) { return __frcp_rn(1.0f + __expf(-x)); }

}  // namespace

// ---------------------------------------------------------------------------
// forward: f_inv[p][128], f_ev[p][128] (float64), silu' (float), d rbf/dr
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 2) k_filter_forward_mixed(
    int P, const double *__restrict__ geo, const int *__restrict__ pa, const int *__restrict__ pb,
    const double *__restrict__ ev, const double *__restrict__ cg, FilterW32 finv, FilterW32 fev, RadialW rad,
    double *__restrict__ f_inv, double *__restrict__ f_ev, float *__restrict__ sp, double *__restrict__ drbf) {
  extern __shared__ float smf[];
  float *rbf_h = smf;               // TP x LDR
  float *rbf_l = rbf_h + TP * LDR;
  float *u_h = rbf_l + TP * LDR;    // TP x LDU
  float *u_l = u_h + TP * LDU;
  float *w_h = u_l + TP * LDU;      // TP x LDR
  float *w_l = w_h + TP * LDR;
  double *l0 = reinterpret_cast<double *>(w_l + TP * LDR);  // TP x 4
  double *rr = l0 + TP * 4;                                 // TP
  const int p0 = blockIdx.x * TP;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  if (tid < TP) {
    const int p = p0 + tid;
    rr[tid] = p < P ? geo[(size_t)p * kGeo] : 1.0;
  }
  compute_l0(P, p0, pa, pb, ev, cg, l0);
  __syncthreads();
  {  // radial basis in float64 (as the float64 path), kept split; d rbf/dr from the same values
    const int pl = tid >> 2, k0 = (tid & 3) * 8;
    const double r = rr[pl];
    const double raw_x = exp(-rad.gamma * r);
    double x = raw_x;
    if (x < 1.0e-6) x = 1.0e-6;
    if (x > 1.0 - 1.0e-6) x = 1.0 - 1.0e-6;
    const double lx = log(x), l1x = log(1.0 - x);
    const bool live = raw_x > 1.0e-6 && raw_x < 1.0 - 1.0e-6;
    const double ratio = live ? raw_x / (1.0 - raw_x) : 0.0;
    double d[8];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const int k = k0 + j;
      const double v0 = exp_tang(rad.b[k] + rad.k[k] * lx + rad.kr[k] * l1x);
      const double v1 = exp_tang(rad.b[k + 1] + rad.k[k + 1] * lx + rad.kr[k + 1] * l1x);
      store_split2(rbf_h + pl * LDR + k, rbf_l + pl * LDR + k, float(v0), float(v1));
      d[j] = live ? v0 * (-rad.gamma * rad.k[k] + rad.gamma * rad.kr[k] * ratio) : 0.0;
      d[j + 1] = live ? v1 * (-rad.gamma * rad.k[k + 1] + rad.gamma * rad.kr[k + 1] * ratio) : 0.0;
    }
    const int p = p0 + pl;
    if (drbf != nullptr && p < P) {
      double2 *dst = reinterpret_cast<double2 *>(drbf + (size_t)p * kR + k0);
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_double2(d[2 * j], d[2 * j + 1]);
    }
  }
  for (int filt = 0; filt < 2; ++filt) {
    const FilterW32 &W = filt ? fev : finv;
    double *out = filt ? f_ev : f_inv;
    {  // ev branch hidden layer: w = silu(L0 V0^T + c0), 64 x 32, float32
      const int pl = tid >> 2, j0 = (tid & 3) * 8;
      const float l00 = float(l0[pl * 4]), l01 = float(l0[pl * 4 + 1]), l02 = float(l0[pl * 4 + 2]),
                  l03 = float(l0[pl * 4 + 3]);
#pragma unroll
      for (int j = j0; j < j0 + 8; j += 2) {
        float s2[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int jj = j + q;
          const float s = l00 * W.v0[jj * 4] + l01 * W.v0[jj * 4 + 1] + l02 * W.v0[jj * 4 + 2] +
                          l03 * W.v0[jj * 4 + 3] + W.c0[jj];
          s2[q] = s * sigmoid_f(s);
        }
        store_split2(w_h + pl * LDR + j, w_l + pl * LDR + j, s2[0], s2[1]);
      }
    }
    __syncthreads();  // rbf (first filter) and w are in shared memory
    float acc[4][2][4];
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
      for (int ni = 0; ni < 2; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = acc[mi][ni][2] = acc[mi][ni][3] = 0.0f;
    mma3_64x16<kR>(acc, rbf_h, rbf_l, LDR, W.w0t_h, W.w0t_l, warp, lane);
    // hidden layer u = silu(pre) to shared memory (split), silu'(pre) for the
    // reverse in the float64 path's order (sp_offset, in floats)
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
      for (int ni = 0; ni < 2; ++ni) {
        const int col = warp * 16 + ni * 8 + 2 * t;
        const float bb0 = W.b0[col], bb1 = W.b0[col + 1];
        float *sp_blk = sp + sp_offset(blockIdx.x, filt, (mi >> 1) * 4 + (warp >> 1)) +
                        (((mi & 1) * 4 + (warp & 1) * 2 + ni) * 2) * 64;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int row = mi * 16 + hf * 8 + g;
          const float x0 = acc[mi][ni][2 * hf] + bb0, x1 = acc[mi][ni][2 * hf + 1] + bb1;
          const float s0 = sigmoid_f(x0), s1 = sigmoid_f(x1);
          store_split2(u_h + row * LDU + col, u_l + row * LDU + col, x0 * s0, x1 * s1);
          *reinterpret_cast<float2 *>(sp_blk + hf * 64 + lane * 2) =
              make_float2(s0 * (1.0f + x0 * (1.0f - s0)), s1 * (1.0f + x1 * (1.0f - s1)));
        }
        acc[mi][ni][0] = acc[mi][ni][1] = acc[mi][ni][2] = acc[mi][ni][3] = 0.0f;
      }
    __syncthreads();
    mma3_64x16<kF>(acc, u_h, u_l, LDU, W.w1t_h, W.w1t_l, warp, lane);
    mma3_64x16<kEH>(acc, w_h, w_l, LDR, W.v1t_h, W.v1t_l, warp, lane);
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = mi * 16 + hf * 8 + g;
        const int p = p0 + row;
        if (p >= P) continue;
#pragma unroll
        for (int ni = 0; ni < 2; ++ni) {
          const int col = warp * 16 + ni * 8 + 2 * t;
          double2 v;
          v.x = double(acc[mi][ni][2 * hf] + W.bc1[col]);
          v.y = double(acc[mi][ni][2 * hf + 1] + W.bc1[col + 1]);
          *reinterpret_cast<double2 *>(out + (size_t)p * kF + col) = v;
        }
      }
    __syncthreads();
  }
}

void launch_filter_forward_mixed(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                                 const double *cg_att, const FilterW32 &finv, const FilterW32 &fev,
                                 const RadialW &rad, double *f_inv, double *f_ev, float *sp, double *drbf,
                                 cudaStream_t s) {
  if (P == 0) return;
  const size_t smem = sizeof(float) * (TP * LDR * 4 + TP * LDU * 2) + sizeof(double) * (TP * 4 + TP);
  allow_dynamic_smem(reinterpret_cast<const void *>(k_filter_forward_mixed), smem);
  k_filter_forward_mixed<<<(P + TP - 1) / TP, 256, smem, s>>>(P, geo, pair_a, pair_b, ev, cg_att, finv, fev, rad,
                                                               f_inv, f_ev, sp, drbf);
  SO3_LAUNCH("filter_forward_mixed");
}

// ---------------------------------------------------------------------------
// reverse: the float64 path's k_filter_reverse with its three GEMMs in three
// TF32 passes (one 2-CTA cluster per tile, one filter per CTA; the radial-basis
// and L0 gradients of CTA 1 reach CTA 0 through distributed shared memory in
// float64, and CTA 0 finishes the pair exactly as the float64 kernel does)
// ---------------------------------------------------------------------------
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 2) k_filter_reverse_mixed(
    int P, const double *__restrict__ geo, const int *__restrict__ pa, const int *__restrict__ pb,
    const double *__restrict__ ev, const double *__restrict__ cg, FilterW finv, FilterW fev, FilterW32 finv32,
    FilterW32 fev32, const double *__restrict__ g_filt_inv, const double *__restrict__ g_filt_ev,
    const float *__restrict__ sp, const double *__restrict__ drbf, const double *__restrict__ gA,
    const double *__restrict__ pair_sc, int need_l0, int accumulate, double *__restrict__ g_r,
    double *__restrict__ g_y, double *__restrict__ gl0) {
  namespace cgrp = cooperative_groups;
  cgrp::cluster_group cluster = cgrp::this_cluster();
  const int f = static_cast<int>(cluster.block_rank());  // 0: invariant filter, 1: ev filter
  extern __shared__ float smf[];
  float *gF_h = smf;                // TP x LDU: filter gradient, then the hidden pre-activation gradient
  float *gF_l = gF_h + TP * LDU;
  double *gw = reinterpret_cast<double *>(gF_l + TP * LDU);  // TP x LDR: ev-hidden, then radial-basis gradient
  double *l0 = gw + TP * LDR;       // TP x 4
  double *gl = l0 + TP * 4;         // TP x 4
  const int tile = blockIdx.x >> 1;
  const int p0 = tile * TP;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const FilterW32 &W32 = f ? fev32 : finv32;
  const double *v0 = f ? fev.v0 : finv.v0;
  const double *c0 = f ? fev.c0 : finv.c0;
  const float *sp_tile = sp + sp_offset(tile, f, warp);

  {  // the filter gradient (float64) into the split tile
    const double *src = f ? g_filt_ev : g_filt_inv;
    for (int idx = tid; idx < TP * (kF / 2); idx += blockDim.x) {
      const int row = idx / (kF / 2), c = 2 * (idx % (kF / 2));
      double2 v = make_double2(0.0, 0.0);
      if (p0 + row < P) v = __ldg(reinterpret_cast<const double2 *>(src + (size_t)(p0 + row) * kF + c));
      store_split2(gF_h + row * LDU + c, gF_l + row * LDU + c, float(v.x), float(v.y));
    }
  }
  // the forward's silu' values of this warp's part of the tile (4 KB) into L2
  for (int c = lane; c < 16 * 64 * 4 / 128; c += 32)
    asm volatile("prefetch.global.L2 [%0];\n" ::"l"(reinterpret_cast<const char *>(sp_tile) + 128 * c));
  gl[tid] = 0.0;
  compute_l0(P, p0, pa, pb, need_l0 ? ev : nullptr, cg, l0);
  __syncthreads();

  // gradient of the hidden layer: (gF W1) * silu'(pre), warp slab 64 x 16
  float acc[4][2][4];
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 2; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = acc[mi][ni][2] = acc[mi][ni][3] = 0.0f;
  mma3_64x16<kF>(acc, gF_h, gF_l, LDU, W32.w1_h, W32.w1_l, warp, lane);
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 2; ++ni) {
      const float *sp_blk = sp + sp_offset(tile, f, (mi >> 1) * 4 + (warp >> 1)) +
                            (((mi & 1) * 4 + (warp & 1) * 2 + ni) * 2) * 64;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const float2 s = __ldg(reinterpret_cast<const float2 *>(sp_blk + hf * 64 + lane * 2));
        acc[mi][ni][2 * hf] *= s.x;
        acc[mi][ni][2 * hf + 1] *= s.y;
      }
    }
  // ev branch: g_w = gF V1 (64 x 32), warp tile 16 x 16
  const int wr = warp >> 1, wc = warp & 1;
  float gwa[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) gwa[j][0] = gwa[j][1] = gwa[j][2] = gwa[j][3] = 0.0f;
  mma3_16x16<kF>(gwa, gF_h, gF_l, LDU, wr * 16, W32.v1_h, W32.v1_l, wc, lane);
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int row = wr * 16 + hf * 8 + g, col = wc * 16 + j * 8 + 2 * t;
      *reinterpret_cast<double2 *>(gw + row * LDR + col) =
          make_double2(double(gwa[j][2 * hf]), double(gwa[j][2 * hf + 1]));
    }
  __syncthreads();  // every warp is done reading gF
  // the hidden pre-activation gradient replaces gF (split)
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 2; ++ni)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = mi * 16 + hf * 8 + g, col = warp * 16 + ni * 8 + 2 * t;
        store_split2(gF_h + row * LDU + col, gF_l + row * LDU + col, acc[mi][ni][2 * hf], acc[mi][ni][2 * hf + 1]);
      }
  __syncthreads();
  // radial-basis gradient g_rbf = g_pre W0 (64 x 32), warp tile 16 x 16
  float grb[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) grb[j][0] = grb[j][1] = grb[j][2] = grb[j][3] = 0.0f;
  mma3_16x16<kF>(grb, gF_h, gF_l, LDU, wr * 16, W32.w0_h, W32.w0_l, wc, lane);
  // L0 gradient (float64, as the float64 path): g_pe = g_w * silu'(L0 V0^T + c0),
  // gl[d] = sum_j g_pe[j] V0[j][d]
  if (need_l0) {
    {
      const int pl = tid >> 2, j0 = (tid & 3) * 8;
      const double l00 = l0[pl * 4], l01 = l0[pl * 4 + 1], l02 = l0[pl * 4 + 2], l03 = l0[pl * 4 + 3];
#pragma unroll
      for (int j = j0; j < j0 + 8; ++j) {
        const double pe = l00 * v0[j * 4] + l01 * v0[j * 4 + 1] + l02 * v0[j * 4 + 2] + l03 * v0[j * 4 + 3] + c0[j];
        gw[pl * LDR + j] *= silu_prime(pe);
      }
    }
    __syncthreads();
    const int pl = tid >> 2, d = tid & 3;
    double s = 0.0;
#pragma unroll 8
    for (int j = 0; j < kEH; ++j) s += gw[pl * LDR + j] * v0[j * 4 + d];
    gl[pl * 4 + d] = s;
  }
  __syncthreads();  // gw is read
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int row = wr * 16 + hf * 8 + g, col = wc * 16 + j * 8 + 2 * t;
      *reinterpret_cast<double2 *>(gw + row * LDR + col) =
          make_double2(double(grb[j][2 * hf]), double(grb[j][2 * hf + 1]));
    }
  // rank 0 prefetches the per-pair inputs of the radial and harmonic gradients
  // into the free gF region (float64 rows)
  double *sc = reinterpret_cast<double *>(gF_h);  // TP x 10 pair scalars
  double *geos = sc + TP * kPairScalars;          // TP x 8 geometry
  double *drs = geos + TP * kGeo;                 // TP x 32 radial-basis derivatives
  if (f == 0) {
    stage_rows<kPairScalars>(sc, kPairScalars, pair_sc, p0, P);
    stage_rows<kGeo>(geos, kGeo, geo, p0, P);
    stage_rows<kR>(drs, kR, drbf, p0, P);
    cp_async_commit();
  }
  cluster.sync();  // both CTAs' radial-basis and L0 gradients are in shared memory
  if (f == 0) {
    const double *rgw = cluster.map_shared_rank(gw, 1);
    const double *rgl = cluster.map_shared_rank(gl, 1);
    for (int idx = tid; idx < TP * kR; idx += blockDim.x) {
      const int row = idx / kR, c = idx % kR;
      gw[row * LDR + c] += rgw[row * LDR + c];
    }
    gl[tid] += rgl[tid];
  }
  cluster.sync();  // rank 1 stays resident until rank 0 has read its shared memory
  if (f != 0) return;
  cp_async_wait<0>();
  __syncthreads();

  // per pair: radial gradient (basis and cutoff terms) and harmonic gradient,
  // summed over the blocks (the float64 kernel's finish, unchanged)
  const int pl = tid >> 2, q = tid & 3;
  const int p = p0 + pl;
  double gr = 0.0;
#pragma unroll
  for (int j = 0; j < 8; ++j) gr += gw[pl * LDR + 8 * q + j] * drs[pl * kR + 8 * q + j];
  const double *s = sc + pl * kPairScalars;
  const double dphi = geos[pl * kGeo + 5], phi = geos[pl * kGeo + 4];
  if (q == 0) gr += __dmul_rn(s[0], dphi);
  gr += __shfl_xor_sync(0xffffffffu, gr, 1);
  gr += __shfl_xor_sync(0xffffffffu, gr, 2);
  if (p < P) {
    if (q == 0) g_r[p] = accumulate ? g_r[p] + gr : gr;
    const int a = pa[p], b = pb[p];
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      const int m = 6 * q + j;
      const int d = degree_of_channel(m);
      const double y = __dmul_rn(phi, __dadd_rn(__dmul_rn(s[1 + d], gA[(size_t)a * kEV + m]),
                                                parity_sign(d) * __dmul_rn(s[5 + d], gA[(size_t)b * kEV + m])));
      double *dst = g_y + (size_t)p * kEV + m;
      *dst = accumulate ? *dst + y : y;
    }
    if (need_l0) gl0[(size_t)p * 4 + q] = gl[pl * 4 + q];
  }
}

void launch_filter_reverse_mixed(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                                 const double *cg_att, const FilterW &finv, const FilterW &fev,
                                 const FilterW32 &finv32, const FilterW32 &fev32, const double *g_filt_inv,
                                 const double *g_filt_ev, const float *sp, const double *drbf, const double *gA,
                                 const double *pair_sc, bool need_l0, bool accumulate, double *g_r, double *g_y,
                                 double *gl0, cudaStream_t s) {
  if (P == 0) return;
  const size_t smem = sizeof(float) * (TP * LDU * 2) + sizeof(double) * (TP * LDR + TP * 8);
  allow_dynamic_smem(reinterpret_cast<const void *>(k_filter_reverse_mixed), smem);
  const int tiles = (P + TP - 1) / TP;
  k_filter_reverse_mixed<<<2 * tiles, 256, smem, s>>>(P, geo, pair_a, pair_b, ev, cg_att, finv, fev, finv32, fev32,
                                                       g_filt_inv, g_filt_ev, sp, drbf, gA, pair_sc, need_l0 ? 1 : 0,
                                                       accumulate ? 1 : 0, g_r, g_y, gl0);
  SO3_LAUNCH("filter_reverse_mixed");
}

SO3LR_SHAPE_END
