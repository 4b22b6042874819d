// Cell grid of the neighbour search: the plain description shared by the
// kernels (kernels.cuh) and its host-side planning (cell_grid.cpp), which has
// no CUDA dependency.
#pragma once

namespace so3lr_b200 {

// periodic: cells tile the box and wrap. open_cells: a single open-boundary
// system of many atoms on a non-wrapping grid over its bounding box; atoms
// outside the grid go to the nearest boundary cell, which keeps every pair
// within one cell size in neighbouring cells. Neither: every atom scans its
// own image's index range (small open systems and turbo packs).
struct CellGrid {
  int periodic = 0;
  int open_cells = 0;
  double lo[3] = {0, 0, 0};
  double len[3] = {1, 1, 1};
  int ncell[3] = {1, 1, 1};
};

// The grid for a system: a periodic box gets cells no smaller than sr_cut
// (at most 2^20 per dimension); with open_cells, the bounding box of the n
// host positions plus a 0.5 A margin gets cells no smaller than sr_cut, at
// most 4096 per dimension and 2^22 in total (coarser cells for sparse
// systems). Throws so3lr_b200::Error for a non-finite position or a grid of
// more than 2^26 cells.
CellGrid plan_cell_grid(bool periodic, const double lo[3], const double len[3], double sr_cut, bool open_cells,
                        int n, const double *host_x);

}  // namespace so3lr_b200
