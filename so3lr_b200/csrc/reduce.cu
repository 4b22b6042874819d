// Exact, order-independent global sums.
//
// Every double is rounded once to a 128-bit fixed-point integer with 64
// fractional bits, the integers are summed (integer addition is associative),
// and the total is converted back once. The result does not depend on how the
// atoms are split across thread blocks or across GPUs, which is what makes the
// energies and the charge conservation bit-identical for 1, 2, 4 and 8 GPUs.
// The reference reduces these quantities with float atomics and MPI_Allreduce
// (pair_so3lr_native_mpi.cpp:1624-1633, 1690-1697; output_heads.cpp:441-442).
#include "kernels.cuh"

namespace so3lr_b200 {
namespace {

// round(v * 2^64) as a signed 128-bit integer (|v| < 2^62)
__device__ inline __int128 to_fixed(double v) {
  if (v == 0.0 || !isfinite(v)) return 0;
  int e = 0;
  const double m = frexp(v, &e);  // v = m 2^e, 0.5 <= |m| < 1
  const long long mi = static_cast<long long>(ldexp(m, 53));  // exact
  const int shift = e - 53 + 64;
  __int128 r = mi;
  if (shift >= 0) {
    r <<= shift;
  } else if (shift > -120) {
    const int s = -shift;
    const __int128 half = static_cast<__int128>(1) << (s - 1);
    r = (r >= 0) ? ((r + half) >> s) : -((-r + half) >> s);
  } else {
    r = 0;
  }
  return r;
}

__device__ inline double from_fixed(__int128 s) {
  const bool neg = s < 0;
  unsigned __int128 u = neg ? static_cast<unsigned __int128>(-s) : static_cast<unsigned __int128>(s);
  const double hi = static_cast<double>(static_cast<unsigned long long>(u >> 64));
  const double lo = static_cast<double>(static_cast<unsigned long long>(u));
  const double v = hi + ldexp(lo, -64);
  return neg ? -v : v;
}

// Block (seg, blk) of a grid of nseg x nblk blocks sums the rows of segment seg
// with index = blk * blockDim + tid (mod nblk * blockDim) and writes
// out[(blk * nseg * ncol + seg * ncol + col) * 2 + {0,1}] = (hi, lo). Integer
// addition is exact, so how the rows are split over blocks does not matter.
__global__ void k_fixed_segment_sum(const int *__restrict__ start, const double *__restrict__ v, int stride, int ncol,
                                    long long *__restrict__ out) {
  __shared__ long long buf_hi[256];
  __shared__ unsigned long long buf_lo[256];
  const int seg = blockIdx.x, blk = blockIdx.y, nblk = gridDim.y;
  const int count = gridDim.x * ncol;
  const int b = start[seg], e = start[seg + 1];
  for (int col = 0; col < ncol; ++col) {
    __int128 acc = 0;
    for (int i = b + blk * blockDim.x + threadIdx.x; i < e; i += nblk * blockDim.x)
      acc += to_fixed(v[(size_t)i * stride + col]);
    buf_hi[threadIdx.x] = static_cast<long long>(acc >> 64);
    buf_lo[threadIdx.x] = static_cast<unsigned long long>(acc);
    __syncthreads();
    if (threadIdx.x == 0) {
      __int128 total = 0;
      for (int t = 0; t < blockDim.x; ++t)
        total += (static_cast<__int128>(buf_hi[t]) << 64) | static_cast<__int128>(buf_lo[t]);
      const size_t k = (size_t)blk * count + (size_t)seg * ncol + col;
      out[k * 2] = static_cast<long long>(total >> 64);
      out[k * 2 + 1] = static_cast<long long>(static_cast<unsigned long long>(total));
    }
    __syncthreads();
  }
}

// out[k] = double(sum over parts p of parts[p][k])
__global__ void k_fixed_finish(const long long *__restrict__ parts, int nparts, int count, double *__restrict__ out) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= count) return;
  __int128 total = 0;
  for (int p = 0; p < nparts; ++p) {
    const long long hi = parts[((size_t)p * count + k) * 2];
    const unsigned long long lo = static_cast<unsigned long long>(parts[((size_t)p * count + k) * 2 + 1]);
    total += (static_cast<__int128>(hi) << 64) | static_cast<__int128>(lo);
  }
  out[k] = from_fixed(total);
}

}  // namespace

void launch_fixed_segment_sum(int nseg, int nblk, const int *start, const double *v, int stride, int ncol,
                              long long *parts, cudaStream_t s) {
  if (nseg == 0) return;
  k_fixed_segment_sum<<<dim3(nseg, nblk), 256, 0, s>>>(start, v, stride, ncol, parts);
  SO3_LAUNCH("fixed_segment_sum");
}

void launch_fixed_finish(const long long *parts, int nparts, int count, double *out, cudaStream_t s) {
  if (count == 0) return;
  k_fixed_finish<<<(count + 127) / 128, 128, 0, s>>>(parts, nparts, count, out);
  SO3_LAUNCH("fixed_finish");
}

}  // namespace so3lr_b200
