// Radial/equivariant filter MLPs of the attention block, forward and reverse,
// evaluated once per undirected short-range pair on FP64 tensor cores (DMMA).
//
// Reference: src/kokkos_integrated_block0.cpp:138-163 (cutoff + Bernstein basis),
// :166-192 (edge L0 invariants), :194-255 (the two filter MLPs); reverse:
// src/kokkos_block2_attention_input_reverse.cpp:186-336 (filter input gradients,
// L0 reverse, radial/cutoff reverse) and src/kokkos_learned_energy_forces.cpp:241-306
// (geometry VJP).
//
// Why pairs: the filter of directed edge s->r depends on |x_r - x_s| and on
// sum (ev_s - ev_r)^2, both symmetric in (s, r), so both directions share one
// value. The reference evaluates it for every directed edge; here each pair
// evaluates it once and both directions read it. In reverse, the filter VJP is
// linear in the incoming gradient, so the two directions' gradients are summed
// first and pushed through the MLP once.
//
// Tile: 64 pairs per CTA, 8 warps, each warp owns a 32x32 block of the 64x128
// output and issues m8n8k4 DMMA on fragments read from shared memory (pair
// activations) and L2-resident weights.
#include <cooperative_groups.h>

#include "kernels.cuh"
#include "sh.cuh"

namespace so3lr_b200 {
namespace {

constexpr int TP = 64;     // pairs per tile
constexpr int LDU = 132;   // padded stride of 128-wide smem tiles (conflict-free fragment reads)
constexpr int LDR = 36;    // padded stride of 32-wide smem tiles

// silu'(hidden pre-activation) of the rbf branch, written by the forward and
// read by the reverse in the accumulator order of their common warp tiling:
// [tile][filter][warp][mi][ni][lane][2] (64 x 128 values per tile and filter,
// 512 contiguous bytes per warp and (mi, ni))
__device__ __forceinline__ size_t sp_offset(int tile, int filt, int warp) {
  return (((size_t)tile * 2 + filt) * 8 + warp) * (16 * 64);
}

__device__ inline void compute_rbf(const double *rr, double *rbf, const RadialW &rad) {
  const int pl = threadIdx.x >> 2;
  const int k0 = (threadIdx.x & 3) * 8;
  const double r = rr[pl];
  double x = exp(-rad.gamma * r);
  if (x < 1.0e-6) x = 1.0e-6;
  if (x > 1.0 - 1.0e-6) x = 1.0 - 1.0e-6;
  const double lx = log(x), l1x = log(1.0 - x);
#pragma unroll
  for (int k = k0; k < k0 + 8; ++k) rbf[pl * LDR + k] = exp_tang(rad.b[k] + rad.k[k] * lx + rad.kr[k] * l1x);
}

__device__ inline void compute_l0(int P, int p0, const int *pa, const int *pb, const double *ev, const double *cg,
                                  double *l0) {
  const int pl = threadIdx.x >> 2, d = threadIdx.x & 3;
  const int p = p0 + pl;
  double v = 0.0;
  if (ev != nullptr && p < P) {
    const int a = pa[p], b = pb[p];
    const int m0 = d == 0 ? 0 : (d == 1 ? 3 : (d == 2 ? 8 : 15));
    const int m1 = d == 0 ? 3 : (d == 1 ? 8 : (d == 2 ? 15 : 24));
    for (int m = m0; m < m1; ++m) {
      const double diff = ev[(size_t)b * kEV + m] - ev[(size_t)a * kEV + m];
      v += diff * diff * cg[m];
    }
  }
  l0[pl * 4 + d] = v;
}

// b[ni] = B(4 ks + t, 32 slab + 8 ni + g) of a fragment-major operand with
// `nslab` column slabs: 32 contiguous bytes per lane, 1 KB per warp
__device__ __forceinline__ void load_bfrag(const double *__restrict__ Bf, int ks, int nslab, int slab, int lane,
                                           double (&b)[4]) {
  const double2 *q = reinterpret_cast<const double2 *>(Bf + ((size_t)(ks * nslab + slab) * 32 + lane) * 4);
  const double2 x = __ldg(q), y = __ldg(q + 1);
  b[0] = x.x;
  b[1] = x.y;
  b[2] = y.x;
  b[3] = y.y;
}

// warp tile 32 x 32 (rows 32 wm.., cols 32 wn..):
// acc += A(64 x K, smem, row stride lda) * B(K x 128, fragment-major)
template <int K>
__device__ inline void mma_32x32(double (&acc)[4][4][2], const double *A, int lda, const double *__restrict__ Bf,
                                 int wm, int wn, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll 4
  for (int ks = 0; ks < K / 4; ++ks) {
    double a[4], b[4];
#pragma unroll
    for (int mi = 0; mi < 4; ++mi) a[mi] = A[(wm * 32 + mi * 8 + g) * lda + 4 * ks + t];
    load_bfrag(Bf, ks, 4, wn, lane, b);
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) dmma(acc[mi][ni][0], acc[mi][ni][1], a[mi], b[ni]);
  }
}

// warp tile 8 x 32 (rows row0..row0+7, all 32 columns), two K halves as
// independent accumulation chains: acc += A(rows, K, smem lda) * B(K x 32, fragment-major)
template <int K>
__device__ inline void mma_8x32(double (&acc)[4][2], const double *A, int lda, int row0,
                                const double *__restrict__ Bf, int lane) {
  const int g = lane >> 2, t = lane & 3;
  double acc2[4][2];
#pragma unroll
  for (int ni = 0; ni < 4; ++ni) acc2[ni][0] = acc2[ni][1] = 0.0;
#pragma unroll 4
  for (int ks = 0; ks < K / 8; ++ks) {
    const double a0 = A[(row0 + g) * lda + 4 * ks + t];
    const double a1 = A[(row0 + g) * lda + K / 2 + 4 * ks + t];
    double b0[4], b1[4];
    load_bfrag(Bf, ks, 1, 0, lane, b0);
    load_bfrag(Bf, ks + K / 8, 1, 0, lane, b1);
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) {
      dmma(acc[ni][0], acc[ni][1], a0, b0[ni]);
      dmma(acc2[ni][0], acc2[ni][1], a1, b1[ni]);
    }
  }
#pragma unroll
  for (int ni = 0; ni < 4; ++ni) {
    acc[ni][0] += acc2[ni][0];
    acc[ni][1] += acc2[ni][1];
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// forward: f_inv[p][128], f_ev[p][128]
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_filter_forward(int P, const double *__restrict__ geo,
                                                        const int *__restrict__ pa, const int *__restrict__ pb,
                                                        const double *__restrict__ ev, const double *__restrict__ cg,
                                                        FilterW finv, FilterW fev, RadialW rad,
                                                        double *__restrict__ f_inv, double *__restrict__ f_ev,
                                                        double *__restrict__ sp) {
  extern __shared__ double sm[];
  double *rbf = sm;               // TP x LDR
  double *u = rbf + TP * LDR;     // TP x LDU
  double *w = u + TP * LDU;       // TP x LDR
  double *l0 = w + TP * LDR;      // TP x 4
  double *rr = l0 + TP * 4;       // TP
  const int p0 = blockIdx.x * TP;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wm = warp >> 2, wn = warp & 3;
  if (tid < TP) {
    const int p = p0 + tid;
    rr[tid] = p < P ? geo[(size_t)p * kGeo] : 1.0;
  }
  compute_l0(P, p0, pa, pb, ev, cg, l0);
  __syncthreads();
  compute_rbf(rr, rbf, rad);
  __syncthreads();
  for (int filt = 0; filt < 2; ++filt) {
    const FilterW &W = filt ? fev : finv;
    double *out = filt ? f_ev : f_inv;
    {  // ev branch hidden layer: w = silu(L0 V0^T + c0), 64 x 32
      const int pl = tid >> 2, j0 = (tid & 3) * 8;
      const double l00 = l0[pl * 4], l01 = l0[pl * 4 + 1], l02 = l0[pl * 4 + 2], l03 = l0[pl * 4 + 3];
#pragma unroll
      for (int j = j0; j < j0 + 8; ++j) {
        const double s = l00 * W.v0[j * 4] + l01 * W.v0[j * 4 + 1] + l02 * W.v0[j * 4 + 2] + l03 * W.v0[j * 4 + 3];
        w[pl * LDR + j] = silu(s + W.c0[j]);
      }
    }
    double acc[4][4][2];
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = 0.0;
    mma_32x32<kR>(acc, rbf, LDR, W.w0t_f, wm, wn, lane);
    // hidden layer u = silu(pre) to shared memory, and silu'(pre) for the
    // reverse pass straight from the accumulators in fragment order
    double *sp_tile = sp + sp_offset(blockIdx.x, filt, warp);
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) {
        const int row = wm * 32 + mi * 8 + g, col = wn * 32 + ni * 8 + 2 * t;
        const double x0 = acc[mi][ni][0] + W.b0[col], x1 = acc[mi][ni][1] + W.b0[col + 1];
        const double s0 = sigmoid(x0), s1 = sigmoid(x1);
        u[row * LDU + col] = x0 * s0;
        u[row * LDU + col + 1] = x1 * s1;
        *reinterpret_cast<double2 *>(sp_tile + (mi * 4 + ni) * 64 + lane * 2) =
            make_double2(s0 * (1.0 + x0 * (1.0 - s0)), s1 * (1.0 + x1 * (1.0 - s1)));
        acc[mi][ni][0] = acc[mi][ni][1] = 0.0;
      }
    __syncthreads();
    mma_32x32<kF>(acc, u, LDU, W.w1t_f, wm, wn, lane);
    mma_32x32<kEH>(acc, w, LDR, W.v1t_f, wm, wn, lane);
#pragma unroll
    for (int mi = 0; mi < 4; ++mi) {
      const int row = wm * 32 + mi * 8 + g;
      const int p = p0 + row;
      if (p >= P) continue;
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) {
        const int col = wn * 32 + ni * 8 + 2 * t;
        double2 v;
        v.x = (acc[mi][ni][0] + W.b1[col]) + W.c1[col];
        v.y = (acc[mi][ni][1] + W.b1[col + 1]) + W.c1[col + 1];
        *reinterpret_cast<double2 *>(out + (size_t)p * kF + col) = v;
      }
    }
    __syncthreads();
  }
}

void launch_filter_forward(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                           const double *cg_att, const FilterW &finv, const FilterW &fev, const RadialW &rad,
                           double *f_inv, double *f_ev, double *sp, cudaStream_t s) {
  if (P == 0) return;
  const size_t smem = sizeof(double) * (TP * LDR * 2 + TP * LDU + TP * 4 + TP);
  static bool configured = false;
  if (!configured) {
    SO3_CUDA(cudaFuncSetAttribute(k_filter_forward, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    configured = true;
  }
  k_filter_forward<<<(P + TP - 1) / TP, 256, smem, s>>>(P, geo, pair_a, pair_b, ev, cg_att, finv, fev, rad, f_inv,
                                                         f_ev, sp);
  SO3_LAUNCH("filter_forward");
}

// ---------------------------------------------------------------------------
// reverse: filter input gradients for both directions of every pair, then the
// radial, cutoff and spherical-harmonic gradients accumulated into gv[p] (3)
// and, when ev is live, the L0 gradient gl0[p][4].
// g_filt_inv/g_filt_ev[p][128]: dL/d(filter) with both directions summed,
// written by the attention reverse. pair_sc[p][32] = alpha_inv, alpha_ev, s_inv,
// s_ev for the direction into the pair's primary receiver ([0:16]) and out of it.
// All per-tile inputs are streamed into shared memory with cp.async at kernel
// start so the tensor-core work never waits on a gather.
// ---------------------------------------------------------------------------
namespace {
__device__ inline void cp_async16(void *smem, const void *gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ inline void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ inline void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// copy a TP x width block of a row-major global array (row stride = width) to
// shared memory with row stride lds; rows beyond P are zero-filled
template <int WIDTH>
__device__ inline void stage_rows(double *dst, int lds, const double *src, int p0, int P) {
  constexpr int chunks = WIDTH / 2;  // 16-byte chunks per row
  for (int idx = threadIdx.x; idx < TP * chunks; idx += blockDim.x) {
    const int row = idx / chunks, c = idx % chunks;
    double *d = dst + row * lds + 2 * c;
    if (p0 + row < P) {
      cp_async16(d, src + (size_t)(p0 + row) * WIDTH + 2 * c);
    } else {
      d[0] = 0.0;
      d[1] = 0.0;
    }
  }
}

}  // namespace

// One cluster of two CTAs per tile of TP pairs: CTA rank 0 pushes the gradient
// of the invariant filter through its MLP, rank 1 that of the ev filter. Each
// CTA holds one 64 x 128 gradient tile (109 KB of shared memory, <= 128
// registers per thread), so two CTAs fit on an SM. The radial-basis and L0
// gradients of rank 1 are read by rank 0 through distributed shared memory and
// added to its own (rank 0 + rank 1, a fixed order), and rank 0 finishes the
// pair: radial/cutoff derivative, spherical-harmonic VJP, Cartesian gradient.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 2) k_filter_reverse(
    int P, const double *__restrict__ geo, const int *__restrict__ pa, const int *__restrict__ pb,
    const double *__restrict__ ev, const double *__restrict__ cg, FilterW finv, FilterW fev, RadialW rad,
    const double *__restrict__ g_filt_inv, const double *__restrict__ g_filt_ev, const double *__restrict__ sp,
    const double *__restrict__ gA, const double *__restrict__ pair_sc, int need_l0, double *__restrict__ gv,
    double *__restrict__ gl0) {
  namespace cgrp = cooperative_groups;
  cgrp::cluster_group cluster = cgrp::this_cluster();
  const int f = static_cast<int>(cluster.block_rank());  // 0: invariant filter, 1: ev filter
  extern __shared__ double sm[];
  double *gF = sm;                // TP x LDU: filter gradient, then the hidden pre-activation gradient
  double *gw = gF + TP * LDU;     // TP x LDR: ev-hidden gradient, then the radial-basis gradient
  double *l0 = gw + TP * LDR;     // TP x 4
  double *gl = l0 + TP * 4;       // TP x 4
  const int tile = blockIdx.x >> 1;
  const int p0 = tile * TP;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wm = warp >> 2, wn = warp & 3;
  // this CTA's filter (selected field by field so the parameters stay in registers)
  const double *w1_f = f ? fev.w1_f : finv.w1_f;
  const double *v1_f = f ? fev.v1_f : finv.v1_f;
  const double *w0_f = f ? fev.w0_f : finv.w0_f;
  const double *v0 = f ? fev.v0 : finv.v0;
  const double *c0 = f ? fev.c0 : finv.c0;
  const double *sp_tile = sp + sp_offset(tile, f, warp);

  stage_rows<kF>(gF, LDU, f ? g_filt_ev : g_filt_inv, p0, P);
  cp_async_commit();
  // the forward's silu' values of this warp's part of the tile (8 KB) into L2
  for (int c = lane; c < 16 * 64 * 8 / 128; c += 32)
    asm volatile("prefetch.global.L2 [%0];\n" ::"l"(reinterpret_cast<const char *>(sp_tile) + 128 * c));
  gl[tid] = 0.0;
  compute_l0(P, p0, pa, pb, need_l0 ? ev : nullptr, cg, l0);
  cp_async_wait<0>();
  __syncthreads();

  // gradient of the hidden layer: (gF W1) * silu'(pre), warp tile 32 x 32
  double acc[4][4][2];
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = 0.0;
  mma_32x32<kF>(acc, gF, LDU, w1_f, wm, wn, lane);
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) {
      const double2 s = __ldg(reinterpret_cast<const double2 *>(sp_tile + (mi * 4 + ni) * 64 + lane * 2));
      acc[mi][ni][0] *= s.x;
      acc[mi][ni][1] *= s.y;
    }
  // ev branch: g_w = gF V1 (64 x 32), warp w owns rows 8w..8w+7
  double gwa[4][2];
#pragma unroll
  for (int ni = 0; ni < 4; ++ni) gwa[ni][0] = gwa[ni][1] = 0.0;
  mma_8x32<kF>(gwa, gF, LDU, warp * 8, v1_f, lane);
  __syncthreads();  // every warp is done reading gF
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) {
      const int row = wm * 32 + mi * 8 + g, col = wn * 32 + ni * 8 + 2 * t;
      gF[row * LDU + col] = acc[mi][ni][0];
      gF[row * LDU + col + 1] = acc[mi][ni][1];
    }
#pragma unroll
  for (int ni = 0; ni < 4; ++ni) {
    const int row = warp * 8 + g, col = ni * 8 + 2 * t;
    gw[row * LDR + col] = gwa[ni][0];
    gw[row * LDR + col + 1] = gwa[ni][1];
  }
  __syncthreads();
  // radial-basis gradient g_rbf = g_pre W0 (64 x 32)
  double grb[4][2];
#pragma unroll
  for (int ni = 0; ni < 4; ++ni) grb[ni][0] = grb[ni][1] = 0.0;
  mma_8x32<kF>(grb, gF, LDU, warp * 8, w0_f, lane);
  // L0 gradient: g_pe = g_w * silu'(L0 V0^T + c0), gl[d] = sum_j g_pe[j] V0[j][d]
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
  __syncthreads();  // gw and gF reads are done
#pragma unroll
  for (int ni = 0; ni < 4; ++ni) {
    const int row = warp * 8 + g, col = ni * 8 + 2 * t;
    gw[row * LDR + col] = grb[ni][0];
    gw[row * LDR + col + 1] = grb[ni][1];
  }
  // rank 0 prefetches the tail's per-pair inputs into the free gF region
  double *sc = gF;                        // TP x 32
  double *geos = sc + TP * kPairScalars;  // TP x 8
  double *ybuf = geos + TP * kGeo;        // TP x kEV
  if (f == 0) {
    stage_rows<kPairScalars>(sc, kPairScalars, pair_sc, p0, P);
    stage_rows<kGeo>(geos, kGeo, geo, p0, P);
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

  // per pair, phase 1 (warp per pair): radial + cutoff gradient and the
  // harmonic gradient gY (pair orientation) -> shared memory
  double *grs = l0;  // TP radial gradients (the L0 inputs are no longer needed)
  for (int pl = warp; pl < TP; pl += 8) {
    const int p = p0 + pl;
    if (p >= P) continue;
    const double *gp = geos + pl * kGeo;
    const double r = gp[0], phi = gp[4], dphi = gp[5];
    // Bernstein derivative (block2_attention_input_reverse.cpp:322-333); lane k
    // evaluates basis function k (the same arithmetic as compute_rbf)
    const double raw_x = exp(-rad.gamma * r);
    double gr = 0.0;
    if (raw_x > 1.0e-6 && raw_x < 1.0 - 1.0e-6) {
      const double rbf_k = exp_tang(rad.b[lane] + rad.k[lane] * log(raw_x) + rad.kr[lane] * log(1.0 - raw_x));
      const double dl = -rad.gamma * rad.k[lane] + rad.gamma * rad.kr[lane] * raw_x / (1.0 - raw_x);
      gr = gw[pl * LDR + lane] * rbf_k * dl;
    }
    // cutoff gradient: sum over heads of alpha*s for both directions; the two
    // directions are added first (a commutative add), so the result does not
    // depend on which endpoint the pair is stored from
    const double *s = sc + pl * kPairScalars;
    const int h = lane & 3, which = lane >> 2;
    if (which < 2) {
      const int ai = which == 0 ? 0 : 4;  // (alpha_inv, s_inv) or (alpha_ev, s_ev)
      gr += __dmul_rn(__dadd_rn(__dmul_rn(s[ai + h], s[ai + 8 + h]), __dmul_rn(s[16 + ai + h], s[16 + ai + 8 + h])),
                      dphi);
    }
    if (lane < kEV) {
      const int d = degree_of_channel(lane);
      const double gAa = gA[(size_t)pa[p] * kEV + lane], gAb = gA[(size_t)pb[p] * kEV + lane];
      ybuf[pl * kEV + lane] =
          __dmul_rn(phi, __dadd_rn(__dmul_rn(s[4 + d], gAa), parity_sign(d) * __dmul_rn(s[20 + d], gAb)));
    }
    for (int off = 16; off > 0; off >>= 1) gr += __shfl_xor_sync(0xffffffffu, gr, off);
    if (lane == 0) grs[pl] = gr;
    if (need_l0 && lane < 4) gl0[(size_t)p * 4 + lane] = gl[pl * 4 + lane];
  }
  __syncthreads();
  // phase 2 (thread per pair): spherical-harmonic VJP and the Cartesian pair gradient
  if (tid < TP && p0 + tid < P) {
    const int p = p0 + tid;
    const double *gp = geos + tid * kGeo;
    const double r = gp[0], ux = gp[1], uy = gp[2], uz = gp[3];
    double gux, guy, guz;
    real_sh_vjp(ux, uy, uz, ybuf + tid * kEV, gux, guy, guz);
    const double rad_c = ux * gux + uy * guy + uz * guz;
    const double ir = r > 1.0e-14 ? 1.0 / r : 0.0;
    const double gr = grs[tid];
    gv[3 * p] += gr * ux + (gux - ux * rad_c) * ir;
    gv[3 * p + 1] += gr * uy + (guy - uy * rad_c) * ir;
    gv[3 * p + 2] += gr * uz + (guz - uz * rad_c) * ir;
  }
}

void launch_filter_reverse(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                           const double *cg_att, const FilterW &finv, const FilterW &fev, const RadialW &rad,
                           const double *g_filt_inv, const double *g_filt_ev, const double *sp, const double *gA,
                           const double *pair_sc, bool need_l0, double *gv, double *gl0, cudaStream_t s) {
  if (P == 0) return;
  const size_t smem = sizeof(double) * (TP * LDU + TP * LDR + 8 * TP);
  static_assert(TP * (kPairScalars + kGeo + kEV) <= TP * LDU, "tail inputs must fit in the gradient tile");
  static bool configured = false;
  if (!configured) {
    SO3_CUDA(cudaFuncSetAttribute(k_filter_reverse, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    configured = true;
  }
  const int tiles = (P + TP - 1) / TP;
  k_filter_reverse<<<2 * tiles, 256, smem, s>>>(P, geo, pair_a, pair_b, ev, cg_att, finv, fev, rad, g_filt_inv,
                                                g_filt_ev, sp, gA, pair_sc, need_l0 ? 1 : 0, gv, gl0);
  SO3_LAUNCH("filter_reverse");
}

}  // namespace so3lr_b200
