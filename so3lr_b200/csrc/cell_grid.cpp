#include "cell_grid.hpp"

#include <algorithm>
#include <cmath>
#include <string>

#include "model_host.hpp"

namespace so3lr_b200 {

CellGrid plan_cell_grid(bool periodic, const double lo[3], const double len[3], double sr_cut, bool open_cells,
                        int n, const double *host_x) {
  CellGrid g;
  g.periodic = periodic ? 1 : 0;
  for (int d = 0; d < 3; ++d) {
    g.lo[d] = lo[d];
    g.len[d] = periodic ? len[d] : 1.0;
    // clamped before the integer conversion; an oversized grid is refused below
    g.ncell[d] = periodic ? int(std::min(std::max(std::floor(len[d] / sr_cut), 1.0), double(1 << 20))) : 1;
  }
  if (open_cells) {
    // one open system: a non-wrapping grid over the bounding box of the
    // positions given now (atoms that later leave it go to the nearest
    // boundary cell, which keeps the neighbour search exact)
    double mn[3] = {1e300, 1e300, 1e300}, mx[3] = {-1e300, -1e300, -1e300};
    for (int i = 0; i < n; ++i)
      for (int d = 0; d < 3; ++d) {
        const double v = host_x[3 * static_cast<long long>(i) + d];
        if (!std::isfinite(v)) throw Error("SO3LR: position of atom " + std::to_string(i) + " is not finite");
        mn[d] = std::min(mn[d], v);
        mx[d] = std::max(mx[d], v);
      }
    g.open_cells = 1;
    for (int d = 0; d < 3; ++d) {
      const double margin = 0.5;
      g.lo[d] = mn[d] - margin;
      g.len[d] = std::max(mx[d] - mn[d] + 2.0 * margin, sr_cut);
      g.ncell[d] = int(std::min(std::floor(g.len[d] / sr_cut), 4096.0));
      if (g.ncell[d] < 1) g.ncell[d] = 1;
    }
    // a sparse system (atoms far apart) would need more cells than atoms:
    // coarser cells (still no smaller than the cutoff) keep the grid small
    while ((long long)g.ncell[0] * g.ncell[1] * g.ncell[2] > (1LL << 22))
      for (int d = 0; d < 3; ++d) g.ncell[d] = std::max(1, g.ncell[d] / 2);
  }
  const long long ncells = (long long)g.ncell[0] * g.ncell[1] * g.ncell[2];
  if (ncells > (1 << 26)) throw Error("SO3LR: periodic box is too large for the cell grid");
  return g;
}

}  // namespace so3lr_b200
