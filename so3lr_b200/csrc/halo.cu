// Halo rows of the spatial decomposition.
//
// A GPU needs another GPU's rows only for the atoms that are short-range
// neighbours of its own atoms (the attention gathers, the filter inputs, the
// sender role of the reverse). The neighbour lists are symmetric bit for bit
// (cells.cuh evaluates every separation in a canonical orientation), so the
// rows GPU s must send to GPU r -- its own atoms with a neighbour owned by r --
// are exactly the rows r finds it needs in its own lists. Block features and
// adjoints are refreshed by exchanging only these rows with NCCL send/receive;
// positions and the long-range charges (which reach 12 A) stay all-gathered.
#include "kernels.cuh"

namespace so3lr_b200 {
namespace {

// send_flag[peer * stride + r] = 1 if owned row r has a neighbour owned by peer;
// recv_flag[b] = 1 for every foreign row b in an owned row's neighbour list
__global__ void k_halo_mark(int n, int row0, int stride, int rank, const int *__restrict__ row_start,
                            const int *__restrict__ nbr, int *__restrict__ send_flag, int *__restrict__ recv_flag) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  for (int e = row_start[r]; e < row_start[r + 1]; ++e) {
    const int b = nbr[e];
    const int peer = b / stride;
    if (peer == rank) continue;
    send_flag[peer * stride + r] = 1;
    recv_flag[b] = 1;
  }
}

// list[pos[i]] = base(i) + i % stride for flagged i; base = row0 for sends
// (owned rows), 0 for receives (global rows)
__global__ void k_halo_compact(int count, int stride, int base, const int *__restrict__ flag,
                               const int *__restrict__ pos, int *__restrict__ list) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count || !flag[i]) return;
  list[pos[i]] = base >= 0 ? base + i % stride : i;
}

// offsets[p] = pos[p * stride] (p < nranks), offsets[nranks] = total
__global__ void k_halo_offsets(int nranks, int stride, const int *__restrict__ pos, const int *__restrict__ total,
                               long long *__restrict__ offsets) {
  const int p = threadIdx.x;
  if (p < nranks) offsets[p] = pos[p * stride];
  if (p == nranks) offsets[p] = *total;
}

__global__ void k_halo_pack(int count, const int *__restrict__ rows, const double *__restrict__ a, int wa,
                            const double *__restrict__ b, int wb, double *__restrict__ buf) {
  const int w = wa + wb;
  const long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= (long long)count * w) return;
  const int i = int(k / w), c = int(k % w);
  const size_t row = rows[i];
  buf[k] = c < wa ? a[row * wa + c] : b[row * wb + (c - wa)];
}

__global__ void k_halo_unpack(int count, const int *__restrict__ rows, const double *__restrict__ buf, double *a,
                              int wa, double *b, int wb) {
  const int w = wa + wb;
  const long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= (long long)count * w) return;
  const int i = int(k / w), c = int(k % w);
  const size_t row = rows[i];
  if (c < wa) a[row * wa + c] = buf[k];
  else b[row * wb + (c - wa)] = buf[k];
}

}  // namespace

void launch_halo_lists(int n_own, int row0, int stride, int nranks, int rank, const int *row_start, const int *nbr,
                       int *send_flag, int *recv_flag, int *send_pos, int *recv_pos, int *send_rows, int *recv_rows,
                       long long *offsets, int *totals, int *scan_scratch, cudaStream_t s) {
  const int count = nranks * stride;
  SO3_CUDA(cudaMemsetAsync(send_flag, 0, sizeof(int) * count, s));
  SO3_CUDA(cudaMemsetAsync(recv_flag, 0, sizeof(int) * count, s));
  if (n_own > 0) {
    k_halo_mark<<<(n_own + 127) / 128, 128, 0, s>>>(n_own, row0, stride, rank, row_start, nbr, send_flag, recv_flag);
    SO3_LAUNCH("halo_mark");
  }
  exclusive_scan(send_flag, send_pos, count, totals, scan_scratch, s);
  exclusive_scan(recv_flag, recv_pos, count, totals + 1, scan_scratch, s);
  k_halo_compact<<<(count + 255) / 256, 256, 0, s>>>(count, stride, row0, send_flag, send_pos, send_rows);
  SO3_LAUNCH("halo_compact");
  k_halo_compact<<<(count + 255) / 256, 256, 0, s>>>(count, stride, -1, recv_flag, recv_pos, recv_rows);
  SO3_LAUNCH("halo_compact");
  k_halo_offsets<<<1, 64, 0, s>>>(nranks, stride, send_pos, totals, offsets);
  SO3_LAUNCH("halo_offsets");
  k_halo_offsets<<<1, 64, 0, s>>>(nranks, stride, recv_pos, totals + 1, offsets + nranks + 1);
  SO3_LAUNCH("halo_offsets");
}

void launch_halo_pack(int count, const int *rows, const double *a, int wa, const double *b, int wb, double *buf,
                      cudaStream_t s) {
  if (count == 0) return;
  const long long total = (long long)count * (wa + wb);
  k_halo_pack<<<unsigned((total + 255) / 256), 256, 0, s>>>(count, rows, a, wa, b, wb, buf);
  SO3_LAUNCH("halo_pack");
}

void launch_halo_unpack(int count, const int *rows, const double *buf, double *a, int wa, double *b, int wb,
                        cudaStream_t s) {
  if (count == 0) return;
  const long long total = (long long)count * (wa + wb);
  k_halo_unpack<<<unsigned((total + 255) / 256), 256, 0, s>>>(count, rows, buf, a, wa, b, wb);
  SO3_LAUNCH("halo_unpack");
}

}  // namespace so3lr_b200
