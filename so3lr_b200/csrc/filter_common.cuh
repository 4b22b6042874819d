// Pair tiles shared by the float64 (filter.cu) and the mixed-precision
// (filter_mixed.cu) pair-filter kernels: tile shape, shared-memory row
// strides, the order in which the forward stores silu' for the reverse, and the
// per-pair radial basis and L0 invariants.
#pragma once

#include "kernels.cuh"

SO3LR_SHAPE_BEGIN
namespace {

constexpr int TP = kFilterTile;  // pairs per tile: 64 (F = 128), 32 (F = 256)
// threads of a 256-thread CTA per pair of the tile; equal to the number of
// degree slots, so thread d of a pair owns slot d of its L0 invariants
constexpr int kTPP = 256 / TP;
constexpr int kTPPLog = kTPP == 4 ? 2 : 3;
static_assert(kTPP == kHeads, "a pair's threads must match its degree slots");
static_assert(kEH == kR, "the ev-hidden and radial-basis tiles share one row stride");
// Row strides of the shared-memory tiles. A quarter-warp's 16-byte fragment
// access covers 64 bytes of two rows; a stride of 8 (mod 16) doubles puts the
// second row in the other half of the 32 banks.
constexpr int LDU = kF + 8;   // F-wide tiles
constexpr int LDR = kR + 8;   // R-wide (and EH-wide) tiles
// the float64 kernels' warp slabs: each of the 8 warps owns kF / 8 output
// columns of an F-wide GEMM, as kMT x kNB m16n8 blocks
constexpr int kMT = TP / 16, kNB = kF / 64;

// silu'(hidden pre-activation) of the rbf branch, written by the forward and
// read by the reverse in accumulator order:
// [tile][filter][block][mi][ni][half][lane][2] with 32 x 32 blocks (block =
// 4 (row / 32) + col / 32; 512 contiguous bytes per block and (mi, ni, half)).
// A 64x16 warp slab's m16n8 block (mi, ni) is one such 512-byte run.
__device__ __forceinline__ size_t sp_offset(int tile, int filt, int warp) {
  return (((size_t)tile * 2 + filt) * 8 + warp) * (16 * 64);
}
// start of the 2 x 64 doubles (rows g and g + 8, lane-major pairs) of block
// (mi, ni) of warp `warp`'s slab: the F = 128 order above; for F = 256 simply
// [tile][filter][warp][mi][ni]
__device__ __forceinline__ size_t sp_block(int tile, int filt, int warp, int mi, int ni) {
  if constexpr (kF == 128)
    return sp_offset(tile, filt, (mi >> 1) * 4 + (warp >> 1)) + (((mi & 1) * 4 + (warp & 1) * 2 + ni) * 2) * 64;
  else
    return (((size_t)tile * 2 + filt) * 8 + warp) * (kMT * kNB * 128) + (size_t)(mi * kNB + ni) * 128;
}

// r: the distance of this thread's pair (pair threadIdx.x / kTPP of the tile)
__device__ inline void compute_rbf(double r, double *rbf, const RadialW &rad) {
  const int pl = threadIdx.x / kTPP;
  const int k0 = (threadIdx.x % kTPP) * 8;
  double x = exp(-rad.gamma * r);
  if (x < 1.0e-6) x = 1.0e-6;
  if (x > 1.0 - 1.0e-6) x = 1.0 - 1.0e-6;
  const double lx = log(x), l1x = log(1.0 - x);
#pragma unroll
  for (int k = k0; k < k0 + 8; ++k) rbf[pl * LDR + k] = exp_tang(rad.b[k] + rad.k[k] * lx + rad.kr[k] * l1x);
}

__device__ inline void compute_l0(int P, int p0, const int *pa, const int *pb, const double *ev, const double *cg,
                                  double *l0) {
  const int pl = threadIdx.x / kTPP, d = threadIdx.x % kTPP;
  const int p = p0 + pl;
  double v = 0.0;
  if (ev != nullptr && p < P) {
    const int a = pa[p], b = pb[p];
    int m0, m1;
    if constexpr (kHeads == 4) {
      m0 = d == 0 ? 0 : (d == 1 ? 3 : (d == 2 ? 8 : 15));
      m1 = d == 0 ? 3 : (d == 1 ? 8 : (d == 2 ? 15 : 24));
    } else {
      m0 = slot_offset(d);
      m1 = m0 + slot_width(d);
    }
    // a degree slot has at most 9 channels: all loads first, then the sum in
    // channel order
    constexpr int kMaxW = 9;
    double eb[kMaxW], ea[kMaxW];
#pragma unroll
    for (int q = 0; q < kMaxW; ++q) {
      const int m = m0 + q;
      eb[q] = m < m1 ? ev[(size_t)b * kEV + m] : 0.0;
      ea[q] = m < m1 ? ev[(size_t)a * kEV + m] : 0.0;
    }
#pragma unroll
    for (int q = 0; q < kMaxW; ++q) {
      const int m = m0 + q;
      if (m < m1) {
        const double diff = eb[q] - ea[q];
        v += diff * diff * cg[m];
      }
    }
  }
  l0[pl * kHeads + d] = v;
}

// copy an nrows x width block of a row-major global array (row stride = width)
// to shared memory with row stride lds; rows beyond P are zero-filled
template <int WIDTH>
__device__ inline void stage_rows(double *dst, int lds, const double *src, int p0, int P, int nrows = TP) {
  constexpr int chunks = WIDTH / 2;  // 16-byte chunks per row
  for (int idx = threadIdx.x; idx < nrows * chunks; idx += blockDim.x) {
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
SO3LR_SHAPE_END
