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
// Tile: TP pairs per CTA (64 for F = 128, 32 for F = 256), 8 warps, m16n8k8
// DMMA on fragments read from shared memory (pair activations, one 16-byte load
// per row) and L2-resident weights prepared in fragment order (16-byte loads per
// lane and k-step). The F-wide GEMMs give each warp a TP x (F / 8) column slab
// of the TP x F output, so every weight column is fetched from L2 by one warp of
// the CTA only; the R- and EH-wide ones use 16x16 warp blocks.
#include <cooperative_groups.h>

#include "filter_common.cuh"
#include "kernels.cuh"
#include "sh.cuh"

SO3LR_SHAPE_BEGIN
namespace {

// b[j] = {B(8 ks + 2t, n), B(8 ks + 2t + 1, n)}, n = 32 slab + 8 (ni0 + j) + g, for
// j < NB, from a fragment-major operand with `nslab` column slabs (8
// contiguous doubles per lane and k-step)
template <int NB>
__device__ __forceinline__ void load_bfrag(const double *__restrict__ Bf, int ks, int nslab, int slab, int ni0,
                                           int lane, double (&b)[NB][2]) {
  const double2 *q = reinterpret_cast<const double2 *>(Bf + ((size_t)(ks * nslab + slab) * 32 + lane) * 8) + ni0;
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    const double2 v = __ldg(q + j);
    b[j][0] = v.x;
    b[j][1] = v.y;
  }
}

// warp slab TP x (F / 8) (all rows, cols wc F / 8 ..) as kMT x kNB m16n8
// blocks: each weight column is read by one warp of the CTA only
// acc += A(TP x K, smem, row stride lda) * B(K x F, fragment-major)
template <int K>
__device__ inline void mma_64x16(double (&acc)[kMT][kNB][4], const double *A, int lda,
                                 const double *__restrict__ Bf, int wc, int lane) {
  const int g = lane >> 2, t = lane & 3;
  constexpr int kCW = kF / 8;  // columns per warp
#pragma unroll 2
  for (int ks = 0; ks < K / 8; ++ks) {
    double b[kNB][2];
    load_bfrag<kNB>(Bf, ks, kF / 32, (wc * kCW) / 32, ((wc * kCW) % 32) / 8, lane, b);
#pragma unroll
    for (int mi = 0; mi < kMT; ++mi) {
      double a[4];
      load_afrag(A, lda, mi * 16, ks, g, t, a);
#pragma unroll
      for (int ni = 0; ni < kNB; ++ni) dmma16(acc[mi][ni], a, b[ni]);
    }
  }
}

// warp tile 16 x 16 (rows r0.., cols 16 wc..) of a TP x kR output (kR == kEH),
// the two K halves as independent accumulation chains:
// acc += A(rows, K, smem lda) * B(K x kR, fragment-major)
template <int K>
__device__ inline void mma_16x16(double (&acc)[2][4], const double *A, int lda, int r0,
                                 const double *__restrict__ Bf, int wc, int lane) {
  const int g = lane >> 2, t = lane & 3;
  double acc2[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) acc2[j][0] = acc2[j][1] = acc2[j][2] = acc2[j][3] = 0.0;
#pragma unroll 2
  for (int ks = 0; ks < K / 16; ++ks) {
    double a0[4], a1[4], b0[2][2], b1[2][2];
    load_afrag(A, lda, r0, ks, g, t, a0);
    load_afrag(A, lda, r0, ks + K / 16, g, t, a1);
    if constexpr (kR == 32) {  // one 32-column slab
      load_bfrag<2>(Bf, ks, 1, 0, 2 * wc, lane, b0);
      load_bfrag<2>(Bf, ks + K / 16, 1, 0, 2 * wc, lane, b1);
    } else {
      load_bfrag<2>(Bf, ks, kR / 32, wc >> 1, (wc & 1) * 2, lane, b0);
      load_bfrag<2>(Bf, ks + K / 16, kR / 32, wc >> 1, (wc & 1) * 2, lane, b1);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      dmma16(acc[j], a0, b0[j]);
      dmma16(acc2[j], a1, b1[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int v = 0; v < 4; ++v) acc[j][v] += acc2[j][v];
}

}  // namespace

// ---------------------------------------------------------------------------
// forward: f_inv[p][F], f_ev[p][F]
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 2) k_filter_forward(int P, const double *__restrict__ geo,
                                                        const int *__restrict__ pa, const int *__restrict__ pb,
                                                        const double *__restrict__ ev, const double *__restrict__ cg,
                                                        FilterW finv, FilterW fev, RadialW rad,
                                                        double *__restrict__ f_inv, double *__restrict__ f_ev,
                                                        double *__restrict__ sp, double *__restrict__ drbf) {
  extern __shared__ double sm[];
  double *rbf = sm;               // TP x LDR
  double *u = rbf + TP * LDR;     // TP x LDU
  double *w = u + TP * LDU;       // TP x LDR
  double *l0 = w + TP * LDR;      // TP x kHeads
  double *rr = l0 + TP * kHeads;  // TP
  const int p0 = blockIdx.x * TP;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  if (tid < TP) {
    const int p = p0 + tid;
    rr[tid] = p < P ? geo[(size_t)p * kGeo] : 1.0;
  }
  compute_l0(P, p0, pa, pb, ev, cg, l0);
  {  // the radial basis reads its pair's distance itself: no barrier between
     // the L0 loads and the basis functions
    const int p = p0 + tid / kTPP;
    compute_rbf(p < P ? geo[(size_t)p * kGeo] : 1.0, rbf, rad);
  }
  __syncthreads();
  if (drbf != nullptr) {
    // d rbf_k / dr for the reverse pass (Bernstein derivative,
    // block2_attention_input_reverse.cpp:322-333): zero where the basis is clamped
    const int pl = (tid >> kTPPLog), k0 = ((tid & (kTPP - 1))) * 8;
    const int p = p0 + pl;
    if (p < P) {
      const double raw_x = exp(-rad.gamma * rr[pl]);
      const bool live = raw_x > 1.0e-6 && raw_x < 1.0 - 1.0e-6;
      const double ratio = live ? raw_x / (1.0 - raw_x) : 0.0;
      double d[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = k0 + j;
        d[j] = live ? rbf[pl * LDR + k] * (-rad.gamma * rad.k[k] + rad.gamma * rad.kr[k] * ratio) : 0.0;
      }
      double2 *dst = reinterpret_cast<double2 *>(drbf + (size_t)p * kR + k0);
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_double2(d[2 * j], d[2 * j + 1]);
    }
  }
  for (int filt = 0; filt < 2; ++filt) {
    const FilterW &W = filt ? fev : finv;
    double *out = filt ? f_ev : f_inv;
    {  // ev branch hidden layer: w = silu(L0 V0^T + c0), TP x EH
      const int pl = (tid >> kTPPLog), j0 = ((tid & (kTPP - 1))) * (kEH / kTPP);
      if constexpr (kHeads == 4) {
        const double l00 = l0[pl * 4], l01 = l0[pl * 4 + 1], l02 = l0[pl * 4 + 2], l03 = l0[pl * 4 + 3];
#pragma unroll
        for (int j = j0; j < j0 + 8; ++j) {
          const double s = l00 * W.v0[j * 4] + l01 * W.v0[j * 4 + 1] + l02 * W.v0[j * 4 + 2] + l03 * W.v0[j * 4 + 3];
          w[pl * LDR + j] = silu(s + W.c0[j]);
        }
      } else {
        double lv[kHeads];
#pragma unroll
        for (int d = 0; d < kHeads; ++d) lv[d] = l0[pl * kHeads + d];
#pragma unroll
        for (int j = j0; j < j0 + kEH / kTPP; ++j) {
          double s = lv[0] * W.v0[j * kHeads];
#pragma unroll
          for (int d = 1; d < kHeads; ++d) s += lv[d] * W.v0[j * kHeads + d];
          w[pl * LDR + j] = silu(s + W.c0[j]);
        }
      }
    }
    double acc[kMT][kNB][4];
#pragma unroll
    for (int mi = 0; mi < kMT; ++mi)
#pragma unroll
      for (int ni = 0; ni < kNB; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = acc[mi][ni][2] = acc[mi][ni][3] = 0.0;
    mma_64x16<kR>(acc, rbf, LDR, W.w0t_f, warp, lane);
    // hidden layer u = silu(pre) to shared memory, and silu'(pre) for the
    // reverse pass in the accumulator order of the reverse's 32 x 32 warp tiling
#pragma unroll
    for (int mi = 0; mi < kMT; ++mi)
#pragma unroll
      for (int ni = 0; ni < kNB; ++ni) {
        const int col = warp * (kF / 8) + ni * 8 + 2 * t;
        const double bb0 = W.b0[col], bb1 = W.b0[col + 1];
        double *sp_blk = sp + sp_block(blockIdx.x, filt, warp, mi, ni);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {  // rows g and g + 8 of the m16 block
          const int row = mi * 16 + hf * 8 + g;
          const double x0 = acc[mi][ni][2 * hf] + bb0, x1 = acc[mi][ni][2 * hf + 1] + bb1;
          const double s0 = sigmoid(x0), s1 = sigmoid(x1);
          *reinterpret_cast<double2 *>(u + row * LDU + col) = make_double2(x0 * s0, x1 * s1);
          *reinterpret_cast<double2 *>(sp_blk + hf * 64 + lane * 2) =
              make_double2(s0 * (1.0 + x0 * (1.0 - s0)), s1 * (1.0 + x1 * (1.0 - s1)));
        }
        acc[mi][ni][0] = acc[mi][ni][1] = acc[mi][ni][2] = acc[mi][ni][3] = 0.0;
      }
    __syncthreads();
    mma_64x16<kF>(acc, u, LDU, W.w1t_f, warp, lane);
    mma_64x16<kEH>(acc, w, LDR, W.v1t_f, warp, lane);
#pragma unroll
    for (int mi = 0; mi < kMT; ++mi)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = mi * 16 + hf * 8 + g;
        const int p = p0 + row;
        if (p >= P) continue;
#pragma unroll
        for (int ni = 0; ni < kNB; ++ni) {
          const int col = warp * (kF / 8) + ni * 8 + 2 * t;
          double2 v;
          v.x = acc[mi][ni][2 * hf] + W.bc1[col];
          v.y = acc[mi][ni][2 * hf + 1] + W.bc1[col + 1];
          *reinterpret_cast<double2 *>(out + (size_t)p * kF + col) = v;
        }
      }
    __syncthreads();
  }
}

void launch_filter_forward(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                           const double *cg_att, const FilterW &finv, const FilterW &fev, const RadialW &rad,
                           double *f_inv, double *f_ev, double *sp, double *drbf, cudaStream_t s) {
  if (P == 0) return;
  const size_t smem = sizeof(double) * (TP * LDR * 2 + TP * LDU + TP * kHeads + TP);
  allow_dynamic_smem(reinterpret_cast<const void *>(k_filter_forward), smem);
  k_filter_forward<<<(P + TP - 1) / TP, 256, smem, s>>>(P, geo, pair_a, pair_b, ev, cg_att, finv, fev, rad, f_inv,
                                                         f_ev, sp, drbf);
  SO3_LAUNCH("filter_forward");
}

// ---------------------------------------------------------------------------
// reverse: filter input gradients for both directions of every pair, then the
// radial, cutoff and spherical-harmonic gradients accumulated into gv[p] (3)
// and, when ev is live, the L0 gradient gl0[p][kHeads].
// g_filt_inv/g_filt_ev[p][128]: dL/d(filter) with both directions summed,
// written by the attention reverse. pair_sc[p][10] = the cutoff-gradient weight
// sum_h (alpha s) over both directions and both attentions, then the ev
// attention coefficient per head into ([1:5]) and out of ([5:9]) the pair's
// primary receiver.
// All per-tile inputs are streamed into shared memory with cp.async at kernel
// start so the tensor-core work never waits on a gather.
// ---------------------------------------------------------------------------

// One cluster of two CTAs per tile of TP pairs: CTA rank 0 pushes the gradient
// of the invariant filter through its MLP, rank 1 that of the ev filter. Each
// CTA holds one TP x F gradient tile (64 x 128 or 32 x 256: 109 KB of shared
// memory with the rest, <= 128 registers per thread), so two CTAs fit on an SM. The radial-basis and L0
// gradients of rank 1 are read by rank 0 through distributed shared memory and
// added to its own (rank 0 + rank 1, a fixed order), and rank 0 finishes the
// pair: radial/cutoff derivative, spherical-harmonic VJP, Cartesian gradient.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 2) k_filter_reverse(
    int P, const double *__restrict__ geo, const int *__restrict__ pa, const int *__restrict__ pb,
    const double *__restrict__ ev, const double *__restrict__ cg, FilterW finv, FilterW fev, RadialW rad,
    const double *__restrict__ g_filt_inv, const double *__restrict__ g_filt_ev, const double *__restrict__ sp,
    const double *__restrict__ drbf, const double *__restrict__ gA, const double *__restrict__ pair_sc, int need_l0,
    int accumulate, double *__restrict__ g_r, double *__restrict__ g_y, double *__restrict__ gl0) {
  namespace cgrp = cooperative_groups;
  cgrp::cluster_group cluster = cgrp::this_cluster();
  const int f = static_cast<int>(cluster.block_rank());  // 0: invariant filter, 1: ev filter
  extern __shared__ double sm[];
  double *gF = sm;                // TP x LDU: filter gradient, then the hidden pre-activation gradient
  double *gw = gF + TP * LDU;     // TP x LDR: ev-hidden gradient, then the radial-basis gradient
  double *l0 = gw + TP * LDR;     // TP x kHeads
  double *gl = l0 + TP * kHeads;  // TP x kHeads
  const int tile = blockIdx.x >> 1;
  const int p0 = tile * TP;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  // this CTA's filter (selected field by field so the parameters stay in registers)
  const double *w1_f = f ? fev.w1_f : finv.w1_f;
  const double *v1_f = f ? fev.v1_f : finv.v1_f;
  const double *w0_f = f ? fev.w0_f : finv.w0_f;
  const double *v0 = f ? fev.v0 : finv.v0;
  const double *c0 = f ? fev.c0 : finv.c0;
  const double *sp_tile = sp + sp_offset(tile, f, warp);  // this warp's eighth of the tile's silu', prefetched below

  stage_rows<kF>(gF, LDU, f ? g_filt_ev : g_filt_inv, p0, P);
  cp_async_commit();
  // the forward's silu' values of this warp's part of the tile (8 KB) into L2
  for (int c = lane; c < 16 * 64 * 8 / 128; c += 32)
    asm volatile("prefetch.global.L2 [%0];\n" ::"l"(reinterpret_cast<const char *>(sp_tile) + 128 * c));
  gl[tid] = 0.0;
  compute_l0(P, p0, pa, pb, need_l0 ? ev : nullptr, cg, l0);
  cp_async_wait<0>();
  __syncthreads();

  // gradient of the hidden layer: (gF W1) * silu'(pre), warp slab TP x F/8
  // (hidden units F/8 warp ..); silu' is read in the order the forward wrote
  // it (sp_block)
  double acc[kMT][kNB][4];
#pragma unroll
  for (int mi = 0; mi < kMT; ++mi)
#pragma unroll
    for (int ni = 0; ni < kNB; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = acc[mi][ni][2] = acc[mi][ni][3] = 0.0;
  mma_64x16<kF>(acc, gF, LDU, w1_f, warp, lane);
#pragma unroll
  for (int mi = 0; mi < kMT; ++mi)
#pragma unroll
    for (int ni = 0; ni < kNB; ++ni) {
      const double *sp_blk = sp + sp_block(tile, f, warp, mi, ni);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const double2 s = __ldg(reinterpret_cast<const double2 *>(sp_blk + hf * 64 + lane * 2));
        acc[mi][ni][2 * hf] *= s.x;
        acc[mi][ni][2 * hf + 1] *= s.y;
      }
    }
  // ev branch: g_w = gF V1 (TP x EH), warp tile 16 x 16
  const int wr = (warp >> (kEH / 32)), wc = (warp & (kEH / 16 - 1));
  double gwa[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) gwa[j][0] = gwa[j][1] = gwa[j][2] = gwa[j][3] = 0.0;
  mma_16x16<kF>(gwa, gF, LDU, wr * 16, v1_f, wc, lane);
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int row = wr * 16 + hf * 8 + g, col = wc * 16 + j * 8 + 2 * t;
      *reinterpret_cast<double2 *>(gw + row * LDR + col) = make_double2(gwa[j][2 * hf], gwa[j][2 * hf + 1]);
    }
  __syncthreads();  // every warp is done reading gF
  // the hidden pre-activation gradient replaces gF in shared memory
#pragma unroll
  for (int mi = 0; mi < kMT; ++mi)
#pragma unroll
    for (int ni = 0; ni < kNB; ++ni)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = mi * 16 + hf * 8 + g, col = warp * (kF / 8) + ni * 8 + 2 * t;
        *reinterpret_cast<double2 *>(gF + row * LDU + col) = make_double2(acc[mi][ni][2 * hf], acc[mi][ni][2 * hf + 1]);
      }
  __syncthreads();
  // radial-basis gradient g_rbf = g_pre W0 (TP x R), warp tile 16 x 16
  double grb[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) grb[j][0] = grb[j][1] = grb[j][2] = grb[j][3] = 0.0;
  mma_16x16<kF>(grb, gF, LDU, wr * 16, w0_f, wc, lane);
  // L0 gradient: g_pe = g_w * silu'(L0 V0^T + c0), gl[d] = sum_j g_pe[j] V0[j][d]
  if (need_l0) {
    {
      const int pl = (tid >> kTPPLog), j0 = ((tid & (kTPP - 1))) * (kEH / kTPP);
      if constexpr (kHeads == 4) {
        const double l00 = l0[pl * 4], l01 = l0[pl * 4 + 1], l02 = l0[pl * 4 + 2], l03 = l0[pl * 4 + 3];
#pragma unroll
        for (int j = j0; j < j0 + 8; ++j) {
          const double pe = l00 * v0[j * 4] + l01 * v0[j * 4 + 1] + l02 * v0[j * 4 + 2] + l03 * v0[j * 4 + 3] + c0[j];
          gw[pl * LDR + j] *= silu_prime(pe);
        }
      } else {
        double lv[kHeads];
#pragma unroll
        for (int d = 0; d < kHeads; ++d) lv[d] = l0[pl * kHeads + d];
#pragma unroll
        for (int j = j0; j < j0 + kEH / kTPP; ++j) {
          double pe = lv[0] * v0[j * kHeads];
#pragma unroll
          for (int d = 1; d < kHeads; ++d) pe += lv[d] * v0[j * kHeads + d];
          gw[pl * LDR + j] *= silu_prime(pe + c0[j]);
        }
      }
    }
    __syncthreads();
    const int pl = (tid >> kTPPLog), d = (tid & (kTPP - 1));
    double s = 0.0;
#pragma unroll 8
    for (int j = 0; j < kEH; ++j) s += gw[pl * LDR + j] * v0[j * kHeads + d];
    gl[pl * kHeads + d] = s;
  }
  __syncthreads();  // gw is read
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int row = wr * 16 + hf * 8 + g, col = wc * 16 + j * 8 + 2 * t;
      *reinterpret_cast<double2 *>(gw + row * LDR + col) = make_double2(grb[j][2 * hf], grb[j][2 * hf + 1]);
    }
  // Each rank finishes half of the tile's pairs: rank f takes rows
  // [f TP/2, (f+1) TP/2). It prefetches those pairs' inputs of the radial and
  // harmonic gradients into its free gF region, then adds the two ranks'
  // radial-basis and L0 gradients of its rows (rank 0's + rank 1's, the same
  // order on either rank), reading the other rank's through distributed
  // shared memory.
  constexpr int kHalf = TP / 2;
  const int r0 = f * kHalf;
  double *sc = gF;                           // kHalf x kPairScalars pair scalars
  double *geos = sc + kHalf * kPairScalars;  // kHalf x 8 geometry
  double *drs = geos + kHalf * kGeo;         // kHalf x kR radial-basis derivatives
  stage_rows<kPairScalars>(sc, kPairScalars, pair_sc, p0 + r0, P, kHalf);
  stage_rows<kGeo>(geos, kGeo, geo, p0 + r0, P, kHalf);
  stage_rows<kR>(drs, kR, drbf, p0 + r0, P, kHalf);
  cp_async_commit();
  cluster.sync();  // both CTAs' radial-basis and L0 gradients are in shared memory
  {
    const double *rgw = cluster.map_shared_rank(gw, f ^ 1);
    const double *rgl = cluster.map_shared_rank(gl, f ^ 1);
    for (int idx = tid; idx < kHalf * kR; idx += blockDim.x) {
      const int row = r0 + idx / kR, c = idx % kR;
      const double mine = gw[row * LDR + c], other = rgw[row * LDR + c];
      gw[row * LDR + c] = f == 0 ? mine + other : other + mine;
    }
    if (tid < kHalf * kHeads) {
      const int i = r0 * kHeads + tid;
      const double mine = gl[i], other = rgl[i];
      gl[i] = f == 0 ? mine + other : other + mine;
    }
  }
  cluster.sync();  // neither CTA leaves while the other reads its shared memory
  cp_async_wait<0>();
  __syncthreads();

  // Per pair: the radial gradient g_r = sum_k g_rbf[k] d rbf_k/dr + the cutoff
  // term, and the harmonic gradient g_Y[m]; both are summed over the blocks
  // (written by the first block reversed, added by the others) and turned into
  // the Cartesian pair gradient once per evaluation (launch_pair_tail).
  // 8 threads per pair: thread q sums basis functions kR/8 q .. and handles the
  // distinct harmonics 3q, 3q + 1, 3q + 2; a harmonic of degree l collects the
  // channels of every slot of degree l (one slot for F = 128, two for F = 256),
  // slot by slot.
  constexpr int kRq = kR / 8;
  const int pl = tid >> 3, q = tid & 7;
  if (pl >= kHalf) return;
  const int p = p0 + r0 + pl;
  double gr = 0.0;
#pragma unroll
  for (int j = 0; j < kRq; ++j) gr += gw[(r0 + pl) * LDR + kRq * q + j] * drs[pl * kR + kRq * q + j];
  const double *s = sc + pl * kPairScalars;
  const double dphi = geos[pl * kGeo + 5], phi = geos[pl * kGeo + 4];
  if (q == 0) gr += __dmul_rn(s[0], dphi);  // cutoff gradient (its weight is orientation-independent)
  gr += __shfl_xor_sync(0xffffffffu, gr, 1);
  gr += __shfl_xor_sync(0xffffffffu, gr, 2);
  gr += __shfl_xor_sync(0xffffffffu, gr, 4);
  if (p < P) {
    if (q == 0) g_r[p] = accumulate ? g_r[p] + gr : gr;
    const int a = pa[p], b = pb[p];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int m = 3 * q + j;  // distinct harmonic
      const int l = m < 3 ? 1 : (m < 8 ? 2 : (m < 15 ? 3 : 4));
      double v = 0.0;
#pragma unroll
      for (int k = 0; k < kDupDegrees; ++k) {
        const int d = (l - 1) * kDupDegrees + k;  // slot
        const int c = slot_offset(d) + (m - (l * l - 1));
        const double t = __dadd_rn(__dmul_rn(s[1 + d], gA[(size_t)a * kEV + c]),
                                   parity_sign(d) * __dmul_rn(s[1 + kHeads + d], gA[(size_t)b * kEV + c]));
        v = k == 0 ? t : __dadd_rn(v, t);
      }
      const double y = __dmul_rn(phi, v);
      double *dst = g_y + (size_t)p * kSH + m;
      *dst = accumulate ? *dst + y : y;
    }
    if (need_l0 && q < kHeads) gl0[(size_t)p * kHeads + q] = gl[(r0 + pl) * kHeads + q];
  }
}

void launch_filter_reverse(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                           const double *cg_att, const FilterW &finv, const FilterW &fev, const RadialW &rad,
                           const double *g_filt_inv, const double *g_filt_ev, const double *sp, const double *drbf,
                           const double *gA, const double *pair_sc, bool need_l0, bool accumulate, double *g_r,
                           double *g_y, double *gl0, cudaStream_t s) {
  if (P == 0) return;
  const size_t smem = sizeof(double) * (TP * LDU + TP * LDR + 2 * kHeads * TP);
  static_assert(TP * (kPairScalars + kGeo + kR) <= TP * LDU, "per-pair inputs must fit in the gradient tile");
  allow_dynamic_smem(reinterpret_cast<const void *>(k_filter_reverse), smem);
  const int tiles = (P + TP - 1) / TP;
  k_filter_reverse<<<2 * tiles, 256, smem, s>>>(P, geo, pair_a, pair_b, ev, cg_att, finv, fev, rad, g_filt_inv,
                                                g_filt_ev, sp, drbf, gA, pair_sc, need_l0 ? 1 : 0,
                                                accumulate ? 1 : 0, g_r, g_y, gl0);
  SO3_LAUNCH("filter_reverse");
}

// ---------------------------------------------------------------------------
// Cartesian pair gradient from the block-summed radial and harmonic gradients:
// gv[p] += g_r u + (J_Y^T g_Y - u (u . J_Y^T g_Y)) / r, with J_Y the Jacobian of
// the harmonic polynomials (learned_energy_forces.cpp:241-306)
// ---------------------------------------------------------------------------
__global__ void k_pair_tail(int P, const double *__restrict__ geo, const double *__restrict__ g_r,
                            const double *__restrict__ g_y, double *__restrict__ gv) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= P) return;
  const double *gp = geo + (size_t)p * kGeo;
  const double r = gp[0], ux = gp[1], uy = gp[2], uz = gp[3];
  double y[kSH];
#pragma unroll
  for (int m = 0; m < kSH; m += 2) {
    const double2 v = *reinterpret_cast<const double2 *>(g_y + (size_t)p * kSH + m);
    y[m] = v.x;
    y[m + 1] = v.y;
  }
  double gux, guy, guz;
  real_sh_vjp(ux, uy, uz, y, gux, guy, guz);
  const double rad_c = ux * gux + uy * guy + uz * guz;
  const double ir = r > 1.0e-14 ? 1.0 / r : 0.0;
  const double gr = g_r[p];
  gv[3 * (size_t)p] += gr * ux + (gux - ux * rad_c) * ir;
  gv[3 * (size_t)p + 1] += gr * uy + (guy - uy * rad_c) * ir;
  gv[3 * (size_t)p + 2] += gr * uz + (guz - uz * rad_c) * ir;
}

void launch_pair_tail(int P, const double *geo, const double *g_r, const double *g_y, double *gv, cudaStream_t s) {
  if (P == 0) return;
  k_pair_tail<<<(P + 127) / 128, 128, 0, s>>>(P, geo, g_r, g_y, gv);
  SO3_LAUNCH("pair_tail");
}

SO3LR_SHAPE_END
