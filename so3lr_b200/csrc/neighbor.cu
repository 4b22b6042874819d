// Edge builder: cell lists -> deterministic short-range CSR -> undirected pairs.
//
// Replaces the reference's LAMMPS-list snapshot + candidate compaction
// (plugins/lammps/pair_so3lr_native_mpi.cpp:76-105, 258-373;
// src/lammps_neighbor_adapter.cpp:122-212). The reference keeps every directed
// candidate with 0 < r^2 < rc^2 (pair_so3lr_native_mpi.cpp:283-286); so does this
// builder, from positions alone, every step.
//
// Output layout (all device, int32 indices):
//   row_start[N+1]            CSR over receivers
//   nbr[E], img[E]            sender atom and packed periodic image of the sender
//   edge_pair[E]              pair id (>= 0: edge is the pair's primary direction,
//                             ~pid: reverse direction)
//   pair_a[P], pair_b[P], pair_img[P], pair_edge[P]   primary receiver, sender,
//                             sender image, primary edge
// The edge vector is v = xw[r] - (xw[s] + img * L) with xw the wrapped positions.
// Each receiver's entries are sorted by (sender, image), so the CSR does not depend
// on the cell layout or on thread scheduling.
#include "cells.cuh"

namespace so3lr_b200 {

// ---- exclusive scan (deterministic, three-phase) --------------------------
namespace {
constexpr int kScanBlock = 1024;

__global__ void k_scan_blocks(const int *in, int *out, int *block_sums, int n) {
  __shared__ int buf[kScanBlock];
  const int i = blockIdx.x * kScanBlock + threadIdx.x;
  const int v = i < n ? in[i] : 0;
  buf[threadIdx.x] = v;
  __syncthreads();
  for (int off = 1; off < kScanBlock; off <<= 1) {
    const int t = threadIdx.x >= off ? buf[threadIdx.x - off] : 0;
    __syncthreads();
    buf[threadIdx.x] += t;
    __syncthreads();
  }
  if (i < n) out[i] = buf[threadIdx.x] - v;
  if (threadIdx.x == kScanBlock - 1) block_sums[blockIdx.x] = buf[threadIdx.x];
}

__global__ void k_scan_add(int *out, const int *block_offsets, int n, int *total, const int *block_sums,
                           int nblocks) {
  const int i = blockIdx.x * kScanBlock + threadIdx.x;
  if (i < n) out[i] += block_offsets[blockIdx.x];
  if (i == 0) *total = block_offsets[nblocks - 1] + block_sums[nblocks - 1];
}
}  // namespace

// out[i] = sum_{j<i} in[i]; *total = sum. scratch must hold 2*ceil(n/1024)+2 ints.
void exclusive_scan(const int *in, int *out, int n, int *total, int *scratch, cudaStream_t s) {
  const int nb = (n + kScanBlock - 1) / kScanBlock;
  if (nb == 0) {
    SO3_CUDA(cudaMemsetAsync(total, 0, sizeof(int), s));
    return;
  }
  int *bsum = scratch;
  int *boff = scratch + nb + 1;
  k_scan_blocks<<<nb, kScanBlock, 0, s>>>(in, out, bsum, n);
  SO3_LAUNCH("scan_blocks");
  if (nb > 1) {
    if (nb > kScanBlock) {
      // recursive for very large inputs
      exclusive_scan(bsum, boff, nb, boff + nb, scratch + 2 * nb + 2, s);
    } else {
      int *dummy = boff + nb;
      k_scan_blocks<<<1, kScanBlock, 0, s>>>(bsum, boff, dummy, nb);
      SO3_LAUNCH("scan_top");
    }
  } else {
    SO3_CUDA(cudaMemsetAsync(boff, 0, sizeof(int), s));
  }
  k_scan_add<<<nb, kScanBlock, 0, s>>>(out, boff, n, total, bsum, nb);
  SO3_LAUNCH("scan_add");
}
std::size_t scan_scratch_ints(std::size_t n) {
  std::size_t nb = (n + kScanBlock - 1) / kScanBlock;
  std::size_t need = 2 * nb + 2;
  if (nb > kScanBlock) need += scan_scratch_ints(nb);
  return need + 8;
}

// ---- cell list ---------------------------------------------------------------
__global__ void k_wrap_assign(int n, const double *__restrict__ x, CellGrid g, const int *__restrict__ tag,
                              double *__restrict__ xw, int *__restrict__ cell, int *__restrict__ cell_count) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (tag != nullptr && tag[i] < 0) {  // padding row of a rank-major layout: not an atom
    cell[i] = -1;
    xw[3 * i] = xw[3 * i + 1] = xw[3 * i + 2] = 0.0;
    return;
  }
  int cc[3];
  for (int d = 0; d < 3; ++d) {
    double p = x[3 * i + d] - g.lo[d];
    if (g.open_cells) {  // no wrap: the position stays, the cell is clamped
      xw[3 * i + d] = x[3 * i + d];
    } else {
      p -= floor(p / g.len[d]) * g.len[d];
      if (p >= g.len[d]) p -= g.len[d];
      if (p < 0.0) p = 0.0;
      xw[3 * i + d] = p + g.lo[d];
    }
    const double fc = p * g.ncell[d] / g.len[d];
    const int c = fc < 0.0 ? 0 : (fc >= double(g.ncell[d]) ? g.ncell[d] - 1 : int(fc));
    cc[d] = c < 0 ? 0 : (c >= g.ncell[d] ? g.ncell[d] - 1 : c);
  }
  const int c = (cc[2] * g.ncell[1] + cc[1]) * g.ncell[0] + cc[0];
  cell[i] = c;
  atomicAdd(&cell_count[c], 1);
}

__global__ void k_cell_fill(int n, const int *__restrict__ cell, const int *__restrict__ cell_start,
                            int *__restrict__ cell_fill, int *__restrict__ cell_atoms) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int c = cell[i];
  if (c < 0) return;
  const int slot = atomicAdd(&cell_fill[c], 1);
  cell_atoms[cell_start[c] + slot] = i;
}

// Sort the atoms of every cell by global tag: the fill above is
// scheduling-dependent, and the tag order does not depend on how rows are laid
// out across GPUs.
// One warp per cell: the cell's atoms in ascending tag order (tags, or atom
// indices without tags, are unique), each placed at the count of smaller keys;
// a cell of more than kCsCap atoms is sorted by one lane in place.
constexpr int kCsWarps = 4, kCsCap = 64;
__global__ void __launch_bounds__(kCsWarps * 32) k_cell_sort(int ncells, const int *__restrict__ cell_start,
                                                             const int *__restrict__ cell_count,
                                                             const int *__restrict__ tag, int *__restrict__ cell_atoms) {
  __shared__ int sk[kCsWarps][kCsCap], sv[kCsWarps][kCsCap];
  const int wl = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * kCsWarps + wl;
  if (c >= ncells) return;
  int *a = cell_atoms + cell_start[c];
  const int m = cell_count[c];
  if (m <= kCsCap) {
    for (int e = lane; e < m; e += 32) {
      const int v = a[e];
      sv[wl][e] = v;
      sk[wl][e] = tag ? tag[v] : v;
    }
    __syncwarp();
    for (int e = lane; e < m; e += 32) {
      const int key = sk[wl][e];
      int rank = 0;
      for (int q = 0; q < m; ++q) rank += sk[wl][q] < key ? 1 : 0;
      a[rank] = sv[wl][e];
    }
    return;
  }
  if (lane != 0) return;
  for (int i = 1; i < m; ++i) {
    const int v = a[i];
    const int vt = tag ? tag[v] : v;
    int j = i - 1;
    while (j >= 0 && (tag ? tag[a[j]] : a[j]) > vt) {
      a[j + 1] = a[j];
      --j;
    }
    a[j + 1] = v;
  }
}

// Short-range neighbour rows: the degree of every owned atom (kFill = false),
// then its CSR row (kFill = true). One warp per owned atom, the lanes testing 32 consecutive candidates of a contiguous
// run of cells at a time (a stencil row of cells with one periodic shift, or an
// image's atom range). The separation d = x_i - (x_j + shift) is evaluated in
// a canonical orientation: from the endpoint with the smaller global tag (for
// an atom and its own periodic image, from the positive image), the other
// endpoint negating the same rounded result. Both atoms of a pair therefore see
// bit-identical |d|, so every inclusion test is symmetric and the neighbour
// lists of different GPUs agree exactly. The fill compacts the
// accepted candidates into shared memory (ballot + prefix) and writes each at
// its rank in the canonical order (sender's global tag, image), which the
// lanes compute by counting smaller keys; a row longer than kSrCap is written
// unsorted and sorted by one lane (insertion sort in global memory).
constexpr int kSrWarps = 8;
constexpr int kSrCap = 256;
template <bool kFill>
__global__ void __launch_bounds__(kSrWarps * 32) k_sr_warp(
    int n, int row0, const double *__restrict__ xw, CellGrid g, const int *__restrict__ cell,
    const int *__restrict__ cell_start, const int *__restrict__ cell_count, const int *__restrict__ cell_atoms,
    const int *__restrict__ image_of, const int *__restrict__ image_start, double rc2, int reach,
    const int *__restrict__ tag, int *__restrict__ deg, const int *__restrict__ row_start, int *__restrict__ nbr,
    int *__restrict__ img) {
  __shared__ long long skey[kFill ? kSrWarps : 1][kFill ? kSrCap : 1];
  __shared__ int sj[kFill ? kSrWarps : 1][kFill ? kSrCap : 1];
  const int wl = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kSrWarps + wl;
  if (r >= n) return;
  const int i = row0 + r;
  const double xi = xw[3 * i], yi = xw[3 * i + 1], zi = xw[3 * i + 2];
  const int ti = tag ? tag[i] : i;
  const int rb = kFill ? row_start[r] : 0;
  int count = 0;
  // candidates cell_atoms[s..e) (or atoms s..e when not cell ordered) with the
  // periodic shift (sx, sy, sz)
  auto run = [&](int s, int e, bool cell_ordered, bool periodic, int sx, int sy, int sz) {
    const int code = periodic ? pack_image(sx, sy, sz) : kZeroImage;
    const double shx = sx * g.len[0], shy = sy * g.len[1], shz = sz * g.len[2];
    const bool positive = sz > 0 || (sz == 0 && (sy > 0 || (sy == 0 && sx > 0)));
    for (int base = s; base < e; base += 32) {
      const int k = base + lane;
      bool valid = false;
      int j = 0, tj = 0;
      if (k < e) {
        j = cell_ordered ? cell_atoms[k] : k;
        tj = tag ? tag[j] : j;
        double dx, dy, dz;
        if (!periodic) {
          dx = xi - xw[3 * j];
          dy = yi - xw[3 * j + 1];
          dz = zi - xw[3 * j + 2];
        } else if (ti < tj || (ti == tj && positive)) {
          dx = xi - (xw[3 * j] + shx);
          dy = yi - (xw[3 * j + 1] + shy);
          dz = zi - (xw[3 * j + 2] + shz);
        } else {  // the other endpoint's expression, negated
          dx = -(xw[3 * j] - (xi - shx));
          dy = -(xw[3 * j + 1] - (yi - shy));
          dz = -(xw[3 * j + 2] - (zi - shz));
        }
        const double r2 = dx * dx + dy * dy + dz * dz;
        valid = r2 > 0.0 && r2 < rc2;
      }
      const unsigned mask = __ballot_sync(0xffffffffu, valid);
      if (kFill && valid) {
        const int slot = count + __popc(mask & ((1u << lane) - 1u));
        if (slot < kSrCap) {
          skey[wl][slot] = (long long)tj * 4294967296LL + code;
          sj[wl][slot] = j;
        } else {
          nbr[rb + slot] = j;
          img[rb + slot] = code;
        }
      }
      count += __popc(mask);
    }
  };
  if (!g.periodic && !g.open_cells) {
    const int im = image_of[i];
    run(image_start[im], image_start[im + 1], false, false, 0, 0, 0);
  } else if (g.open_cells) {  // one open system on a clamped, non-wrapping grid
    const int nx = g.ncell[0], ny = g.ncell[1], nz = g.ncell[2];
    const int c = cell[i];
    const int cx = c % nx, cy = (c / nx) % ny, cz = c / (nx * ny);
    for (int wz = max(0, cz - reach); wz <= min(nz - 1, cz + reach); ++wz)
      for (int wy = max(0, cy - reach); wy <= min(ny - 1, cy + reach); ++wy) {
        const int row = (wz * ny + wy) * nx;
        const int lo = max(0, cx - reach), hi = min(nx - 1, cx + reach);
        run(cell_start[row + lo], cell_start[row + hi] + cell_count[row + hi], true, false, 0, 0, 0);
      }
  } else {
    const int nx = g.ncell[0], ny = g.ncell[1], nz = g.ncell[2];
    const int c = cell[i];
    const int cx = c % nx, cy = (c / nx) % ny, cz = c / (nx * ny);
    for (int oz = -reach; oz <= reach; ++oz) {
      int wz = cz + oz, sz = 0;
      while (wz < 0) { wz += nz; --sz; }
      while (wz >= nz) { wz -= nz; ++sz; }
      for (int oy = -reach; oy <= reach; ++oy) {
        int wy = cy + oy, sy = 0;
        while (wy < 0) { wy += ny; --sy; }
        while (wy >= ny) { wy -= ny; ++sy; }
        const int row = (wz * ny + wy) * nx;
        // x runs of constant periodic shift: cells [lo, hi] of one row are contiguous
        const int sx_lo = (cx - reach >= 0) ? 0 : -((reach - cx + nx - 1) / nx);
        const int sx_hi = (cx + reach) / nx;
        for (int sx = sx_lo; sx <= sx_hi; ++sx) {
          const int lo = max(0, cx - reach - sx * nx), hi = min(nx - 1, cx + reach - sx * nx);
          if (lo > hi) continue;
          run(cell_start[row + lo], cell_start[row + hi] + cell_count[row + hi], true, true, sx, sy, sz);
        }
      }
    }
  }
  if (!kFill) {
    if (lane == 0) deg[r] = count;
    return;
  }
  __syncwarp();
  if (count <= kSrCap) {
    for (int e = lane; e < count; e += 32) {
      const long long key = skey[wl][e];
      int rank = 0;
      for (int t = 0; t < count; ++t) rank += skey[wl][t] < key ? 1 : 0;
      nbr[rb + rank] = sj[wl][e];
      img[rb + rank] = int(key & 0xffffffffLL);
    }
    return;
  }
  // long row: the first kSrCap entries join the others in global memory, then
  // one lane sorts the row in the canonical order
  for (int e = lane; e < kSrCap; e += 32) {
    nbr[rb + e] = sj[wl][e];
    img[rb + e] = int(skey[wl][e] & 0xffffffffLL);
  }
  __syncwarp();
  if (lane != 0) return;
  for (int a = 1; a < count; ++a) {
    const int vj = nbr[rb + a], vc = img[rb + a];
    const int vt = tag ? tag[vj] : vj;
    int b = a - 1;
    while (b >= 0) {
      const int bt = tag ? tag[nbr[rb + b]] : nbr[rb + b];
      if (!(bt > vt || (bt == vt && img[rb + b] > vc))) break;
      nbr[rb + b + 1] = nbr[rb + b];
      img[rb + b + 1] = img[rb + b];
      --b;
    }
    nbr[rb + b + 1] = vj;
    img[rb + b + 1] = vc;
  }
}

// Designated ("primary") edge of every pair and reverse-edge lookup. A pair is
// owned by the designated edge's receiver. When both endpoints are owned here,
// the designated edge is the canonical one (smaller global tag receives; for a
// self-image pair, the positive image); when the sender is not owned here the
// owned receiver's edge is designated and there is no local reverse edge.
__global__ void k_edge_primary(int n, int row0, const int *__restrict__ row_start, const int *__restrict__ nbr,
                               const int *__restrict__ img, const int *__restrict__ tag, int *__restrict__ primary,
                               int *__restrict__ rev, int *__restrict__ error_flag) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;  // one warp per owned atom, a lane per edge
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const int i = row0 + r;
  const int ti = tag ? tag[i] : i;
  for (int e = row_start[r] + lane; e < row_start[r + 1]; e += 32) {
    const int j = nbr[e], code = img[e];
    const int tj = tag ? tag[j] : j;
    const bool canonical = ti < tj || (ti == tj && code > kZeroImage);
    const bool owned_j = j >= row0 && j < row0 + n;
    if (!owned_j) {
      primary[e] = 1;
      rev[e] = -1;
      continue;
    }
    primary[e] = canonical ? 1 : 0;
    const int want = negate_image(code);
    const int rj = j - row0;
    int lo = row_start[rj], hi = row_start[rj + 1] - 1, found = -1;
    while (lo <= hi) {
      const int mid = (lo + hi) >> 1;
      const int mj = nbr[mid], mc = img[mid];
      const int mt = tag ? tag[mj] : mj;
      if (mj == i && mc == want) { found = mid; break; }
      if (mt < ti || (mt == ti && mc < want)) lo = mid + 1; else hi = mid - 1;
    }
    rev[e] = found;
    if (found < 0) atomicExch(error_flag, 1);
  }
}

__global__ void k_pair_fill(int n, int row0, const int *__restrict__ row_start, const int *__restrict__ nbr,
                            const int *__restrict__ img, const int *__restrict__ tag, const int *__restrict__ primary,
                            const int *__restrict__ pair_scan, int *__restrict__ edge_pair, int *__restrict__ pair_a,
                            int *__restrict__ pair_b, int *__restrict__ pair_img, int *__restrict__ pair_edge,
                            int *__restrict__ pair_canon) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;  // one warp per owned atom, a lane per edge
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const int i = row0 + r;
  const int ti = tag ? tag[i] : i;
  for (int e = row_start[r] + lane; e < row_start[r + 1]; e += 32) {
    if (!primary[e]) continue;
    const int p = pair_scan[e];
    const int j = nbr[e];
    const int tj = tag ? tag[j] : j;
    edge_pair[e] = p;
    pair_a[p] = i;
    pair_b[p] = j;
    pair_img[p] = img[e];
    pair_edge[p] = e;
    pair_canon[p] = (ti < tj || (ti == tj && img[e] > kZeroImage)) ? 1 : 0;
  }
}

__global__ void k_pair_reverse(int E, const int *__restrict__ primary, const int *__restrict__ rev,
                               int *__restrict__ edge_pair) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  if (!primary[e] && rev[e] >= 0) edge_pair[e] = ~edge_pair[rev[e]];
}

// ---- host driver ---------------------------------------------------------------
void build_cells(NeighborState &nb, int n, const double *x, cudaStream_t s) {
  const bool cells = nb.grid.periodic || nb.grid.open_cells;
  const int nc = cells ? nb.grid.ncell[0] * nb.grid.ncell[1] * nb.grid.ncell[2] : 1;
  nb.ncells = nc;
  if (!cells) {
    SO3_CUDA(cudaMemcpyAsync(nb.xw, x, sizeof(double) * 3 * n, cudaMemcpyDeviceToDevice, s));
    return;
  }
  SO3_CUDA(cudaMemsetAsync(nb.cell_count, 0, sizeof(int) * nc, s));
  SO3_CUDA(cudaMemsetAsync(nb.cell_fill, 0, sizeof(int) * nc, s));
  k_wrap_assign<<<(n + 255) / 256, 256, 0, s>>>(n, x, nb.grid, nb.tag, nb.xw, nb.cell, nb.cell_count);
  SO3_LAUNCH("wrap_assign");
  exclusive_scan(nb.cell_count, nb.cell_start, nc, nb.scan_total, nb.scan_scratch, s);
  k_cell_fill<<<(n + 255) / 256, 256, 0, s>>>(n, nb.cell, nb.cell_start, nb.cell_fill, nb.cell_atoms);
  SO3_LAUNCH("cell_fill");
  k_cell_sort<<<(nc + kCsWarps - 1) / kCsWarps, kCsWarps * 32, 0, s>>>(nc, nb.cell_start, nb.cell_count, nb.tag,
                                                                      nb.cell_atoms);
  SO3_LAUNCH("cell_sort");
}

int sr_reach(const CellGrid &g, double rc) {
  if (!g.periodic && !g.open_cells) return 0;
  int reach = 1;
  for (int d = 0; d < 3; ++d) {
    const double cl = g.len[d] / g.ncell[d];
    reach = std::max(reach, int(std::ceil(rc / cl - 1e-12)));
  }
  return reach;
}

void count_sr(NeighborState &nb, double rc, cudaStream_t s) {
  const int reach = sr_reach(nb.grid, rc);
  const int n = nb.n_own;
  if (n > 0) {
    k_sr_warp<false><<<(n + kSrWarps - 1) / kSrWarps, kSrWarps * 32, 0, s>>>(
        n, nb.row0, nb.xw, nb.grid, nb.cell, nb.cell_start, nb.cell_count, nb.cell_atoms, nb.image_of,
        nb.image_start, rc * rc, reach, nb.tag, nb.deg, nullptr, nullptr, nullptr);
    SO3_LAUNCH("sr_count");
  }
  exclusive_scan(nb.deg, nb.row_start, n, nb.row_start + n, nb.scan_scratch, s);
}

void fill_sr(NeighborState &nb, double rc, int E, cudaStream_t s) {
  const int reach = sr_reach(nb.grid, rc);
  const int n = nb.n_own;
  if (n > 0) {
    k_sr_warp<true><<<(n + kSrWarps - 1) / kSrWarps, kSrWarps * 32, 0, s>>>(
        n, nb.row0, nb.xw, nb.grid, nb.cell, nb.cell_start, nb.cell_count, nb.cell_atoms, nb.image_of,
        nb.image_start, rc * rc, reach, nb.tag, nullptr, nb.row_start, nb.nbr, nb.img);
    SO3_LAUNCH("sr_fill");
  }
  k_edge_primary<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.img, nb.tag,
                                                       nb.primary, nb.rev, nb.error_flag);
  SO3_LAUNCH("edge_primary");
  exclusive_scan(nb.primary, nb.pair_scan, E, nb.scan_total, nb.scan_scratch, s);
}

void fill_pairs(NeighborState &nb, int E, cudaStream_t s) {
  const int n = nb.n_own;
  k_pair_fill<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.img, nb.tag, nb.primary,
                                               nb.pair_scan, nb.edge_pair, nb.pair_a, nb.pair_b, nb.pair_img,
                                               nb.pair_edge, nb.pair_canon);
  SO3_LAUNCH("pair_fill");
  if (E > 0) {
    k_pair_reverse<<<(E + 255) / 256, 256, 0, s>>>(E, nb.primary, nb.rev, nb.edge_pair);
    SO3_LAUNCH("pair_reverse");
  }
}

}  // namespace so3lr_b200
