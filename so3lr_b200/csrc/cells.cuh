// Cell-list helpers shared by the edge builder and the long-range kernel.
#pragma once
#include "kernels.cuh"

namespace so3lr_b200 {

__host__ __device__ inline int pack_image(int a, int b, int c) {
  return ((a + 512) << 20) | ((b + 512) << 10) | (c + 512);
}
__device__ inline void unpack_image(int code, int &a, int &b, int &c) {
  a = ((code >> 20) & 1023) - 512;
  b = ((code >> 10) & 1023) - 512;
  c = (code & 1023) - 512;
}
__device__ inline int negate_image(int code) {
  int a, b, c;
  unpack_image(code, a, b, c);
  return pack_image(-a, -b, -c);
}
constexpr int kZeroImage = (512 << 20) | (512 << 10) | 512;

// Visit every candidate (j, image) of atom i: periodic cell stencil or the
// atom's own image range (open boundaries / turbo packs). The separation
// d = x_i - (x_j + shift) is evaluated in a canonical orientation: from the
// endpoint with the smaller global tag (for an atom and its own periodic image,
// from the positive image), the other endpoint negating the same rounded
// result. Both atoms of a pair therefore see bit-identical |d|, so every
// inclusion test is symmetric and the neighbour lists of different GPUs agree
// exactly. tag: global tag per row (nullptr: the row index).
template <class Visit>
__device__ inline void for_each_candidate(int i, const double *__restrict__ xw, const CellGrid &g,
                                          const int *__restrict__ cell, const int *__restrict__ cell_start,
                                          const int *__restrict__ cell_count, const int *__restrict__ cell_atoms,
                                          const int *__restrict__ image_of, const int *__restrict__ image_start,
                                          int reach, const int *__restrict__ tag, Visit &&visit) {
  const double xi = xw[3 * i], yi = xw[3 * i + 1], zi = xw[3 * i + 2];
  if (!g.periodic && !g.open_cells) {
    const int im = image_of[i];
    const int s = image_start[im], e = image_start[im + 1];
    for (int j = s; j < e; ++j) {
      const double dx = xi - xw[3 * j], dy = yi - xw[3 * j + 1], dz = zi - xw[3 * j + 2];
      visit(j, kZeroImage, dx, dy, dz);
    }
    return;
  }
  if (g.open_cells) {  // one open system on a clamped, non-wrapping grid
    const int c = cell[i];
    const int cx = c % g.ncell[0], cy = (c / g.ncell[0]) % g.ncell[1], cz = c / (g.ncell[0] * g.ncell[1]);
    for (int wz = max(0, cz - reach); wz <= min(g.ncell[2] - 1, cz + reach); ++wz)
      for (int wy = max(0, cy - reach); wy <= min(g.ncell[1] - 1, cy + reach); ++wy)
        for (int wx = max(0, cx - reach); wx <= min(g.ncell[0] - 1, cx + reach); ++wx) {
          const int cc = (wz * g.ncell[1] + wy) * g.ncell[0] + wx;
          const int *a = cell_atoms + cell_start[cc];
          const int m = cell_count[cc];
          for (int t = 0; t < m; ++t) {
            const int j = a[t];
            visit(j, kZeroImage, xi - xw[3 * j], yi - xw[3 * j + 1], zi - xw[3 * j + 2]);
          }
        }
    return;
  }
  const int c = cell[i];
  const int cx = c % g.ncell[0], cy = (c / g.ncell[0]) % g.ncell[1], cz = c / (g.ncell[0] * g.ncell[1]);
  for (int oz = -reach; oz <= reach; ++oz) {
    int wz = cz + oz, sz = 0;
    while (wz < 0) { wz += g.ncell[2]; --sz; }
    while (wz >= g.ncell[2]) { wz -= g.ncell[2]; ++sz; }
    for (int oy = -reach; oy <= reach; ++oy) {
      int wy = cy + oy, sy = 0;
      while (wy < 0) { wy += g.ncell[1]; --sy; }
      while (wy >= g.ncell[1]) { wy -= g.ncell[1]; ++sy; }
      for (int ox = -reach; ox <= reach; ++ox) {
        int wx = cx + ox, sx = 0;
        while (wx < 0) { wx += g.ncell[0]; --sx; }
        while (wx >= g.ncell[0]) { wx -= g.ncell[0]; ++sx; }
        const int cc = (wz * g.ncell[1] + wy) * g.ncell[0] + wx;
        const int code = pack_image(sx, sy, sz);
        const double shx = sx * g.len[0], shy = sy * g.len[1], shz = sz * g.len[2];
        const int *a = cell_atoms + cell_start[cc];
        const int m = cell_count[cc];
        for (int t = 0; t < m; ++t) {
          const int j = a[t];
          const int ti = tag ? tag[i] : i, tj = tag ? tag[j] : j;
          const bool positive = sz > 0 || (sz == 0 && (sy > 0 || (sy == 0 && sx > 0)));
          double dx, dy, dz;
          if (ti < tj || (ti == tj && positive)) {
            dx = xi - (xw[3 * j] + shx);
            dy = yi - (xw[3 * j + 1] + shy);
            dz = zi - (xw[3 * j + 2] + shz);
          } else {  // the other endpoint's expression, negated
            dx = -(xw[3 * j] - (xi - shx));
            dy = -(xw[3 * j + 1] - (yi - shy));
            dz = -(xw[3 * j + 2] - (zi - shz));
          }
          visit(j, code, dx, dy, dz);
        }
      }
    }
  }
}

}  // namespace so3lr_b200
