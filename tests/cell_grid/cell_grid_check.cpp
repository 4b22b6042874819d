// Host-side planning of the neighbour-search cell grid (so3lr_b200/csrc/cell_grid.cpp):
// periodic boxes, open systems (dense, sparse, one far atom) and refusals.
// Prints "CELL GRID OK" when every check passes.
#include <cmath>
#include <cstdio>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "cell_grid.hpp"

using so3lr_b200::CellGrid;
using so3lr_b200::plan_cell_grid;

static int fails = 0;
static void check(bool ok, const std::string &what) {
  if (!ok) {
    std::printf("FAIL %s\n", what.c_str());
    ++fails;
  }
}

// cells no smaller than the cutoff (or a single cell), bounded counts, and (open grids) every atom inside
static void invariants(const CellGrid &g, double rc, const std::vector<double> &x, const std::string &what) {
  long long total = 1;
  for (int d = 0; d < 3; ++d) {
    check(g.ncell[d] >= 1, what + ": at least one cell per dimension");
    // (a periodic box shorter than the cutoff is one cell; the stencil then reaches several images)
    check(g.ncell[d] == 1 || g.len[d] / g.ncell[d] >= rc * (1 - 1e-12), what + ": cells no smaller than the cutoff");
    total *= g.ncell[d];
  }
  check(total <= (1LL << 26), what + ": at most 2^26 cells");
  if (g.open_cells) {
    check(total <= (1LL << 22), what + ": open grids at most 2^22 cells");
    for (int d = 0; d < 3; ++d) check(g.ncell[d] <= 4096, what + ": open grids at most 4096 cells per dimension");
    for (std::size_t i = 0; i < x.size(); ++i) {
      const int d = int(i % 3);
      check(x[i] >= g.lo[d] && x[i] <= g.lo[d] + g.len[d], what + ": atoms inside the grid");
    }
  }
}

static std::vector<double> cloud(int n, double half, std::mt19937_64 &rng) {
  std::uniform_real_distribution<double> u(-half, half);
  std::vector<double> x(3 * static_cast<std::size_t>(n));
  for (double &v : x) v = u(rng);
  return x;
}

int main() {
  const double rc = 4.5, lo[3] = {0, 0, 0};
  std::mt19937_64 rng(7);
  {  // the 24,000-atom box of the benchmark
    const double len[3] = {62.14784361731874, 62.14784361731874, 62.14784361731874};
    const CellGrid g = plan_cell_grid(true, lo, len, rc, false, 0, nullptr);
    check(g.periodic == 1 && g.open_cells == 0, "periodic flags");
    check(g.ncell[0] == 13 && g.ncell[1] == 13 && g.ncell[2] == 13, "13 cells per dimension");
    invariants(g, rc, {}, "periodic 62 A");
  }
  {  // a box smaller than the cutoff: one cell
    const double len[3] = {3.0, 12.0, 9.0};
    const CellGrid g = plan_cell_grid(true, lo, len, rc, false, 0, nullptr);
    check(g.ncell[0] == 1 && g.ncell[1] == 2 && g.ncell[2] == 2, "small periodic box");
    invariants(g, rc, {}, "periodic small");
  }
  {  // a box too large for any grid is refused, not converted past the int range
    const double len[3] = {1e9, 1e9, 1e9};
    bool threw = false;
    try {
      plan_cell_grid(true, lo, len, rc, false, 0, nullptr);
    } catch (const std::runtime_error &e) {
      threw = std::string(e.what()).find("too large") != std::string::npos;
    }
    check(threw, "huge periodic box refused");
  }
  {  // an open droplet
    const std::vector<double> x = cloud(912, 15.0, rng);
    const CellGrid g = plan_cell_grid(false, lo, lo, rc, true, 912, x.data());
    check(g.open_cells == 1 && g.periodic == 0, "open flags");
    invariants(g, rc, x, "open droplet");
  }
  {  // a sparse open system: coarser cells keep the grid small
    const std::vector<double> x = cloud(600, 5e5, rng);
    const CellGrid g = plan_cell_grid(false, lo, lo, rc, true, 600, x.data());
    invariants(g, rc, x, "open sparse");
  }
  {  // one atom far away along x
    std::vector<double> x = cloud(1000, 20.0, rng);
    x[0] = 1e6;
    const CellGrid g = plan_cell_grid(false, lo, lo, rc, true, 1000, x.data());
    check(g.ncell[0] <= 4096, "far atom: x cells bounded");
    invariants(g, rc, x, "open far atom");
  }
  {  // a non-finite position is refused
    std::vector<double> x = cloud(600, 10.0, rng);
    x[5] = std::nan("");
    bool threw = false;
    try {
      plan_cell_grid(false, lo, lo, rc, true, 600, x.data());
    } catch (const std::runtime_error &e) {
      threw = std::string(e.what()).find("not finite") != std::string::npos;
    }
    check(threw, "NaN position refused");
  }
  {  // without open_cells an open system has the trivial grid
    const std::vector<double> x = cloud(100, 10.0, rng);
    const CellGrid g = plan_cell_grid(false, lo, lo, rc, false, 100, x.data());
    check(g.open_cells == 0 && g.ncell[0] == 1 && g.ncell[1] == 1 && g.ncell[2] == 1, "index-range scan grid");
  }
  std::printf("%s\n", fails ? "CELL GRID FAIL" : "CELL GRID OK");
  return fails ? 1 : 0;
}
