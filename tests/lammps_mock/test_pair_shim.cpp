// Drives the so3lr/b200 pair style through the mock LAMMPS API.
//   test_pair_shim parse MODEL          pair_style/pair_coeff parsing and refusals
//   test_pair_shim run MODEL INPUT      one compute; INPUT holds "L n" then n lines "type x y z"
//                                       (types 1 = O, 2 = H); prints JSON with energy, virial, forces
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <string>
#include <vector>

#include "pair_so3lr_b200.h"

using namespace LAMMPS_NS;

static int expect_error(const char *what, const std::function<void()> &fn, const char *needle) {
  try {
    fn();
  } catch (const std::runtime_error &e) {
    if (std::strstr(e.what(), needle)) return 0;
    std::printf("FAIL %s: wrong message: %s\n", what, e.what());
    return 1;
  }
  std::printf("FAIL %s: no error\n", what);
  return 1;
}

static int parse_checks(const char *model) {
  int fails = 0;
  LAMMPS lmp;
  lmp.atom.ntypes = 2;
  lmp.atom.resize(3);
  PairSO3LRB200 pair(&lmp);
  {
    char *args[] = {(char *)"a", (char *)"b", (char *)"c", (char *)"d"};
    fails += expect_error("too many pair_style args", [&] { pair.settings(4, args); }, "Illegal pair_style");
  }
  {
    char *args[] = {(char *)"/nonexistent/model.so3lr"};
    fails += expect_error("missing model", [&] { pair.settings(1, args); }, "cannot open");
  }
  {
    char *args[] = {(char *)"*", (char *)"*", (char *)"O"};
    fails += expect_error("wrong coeff count", [&] { pair.coeff(3, args); }, "must be '* * E1");
  }
  {
    char *args[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"Xx"};
    fails += expect_error("unknown element", [&] { pair.coeff(4, args); }, "Unknown SO3LR element");
  }
  {
    char *args[] = {(char *)"*", (char *)"*", (char *)"o", (char *)"1"};
    pair.coeff(4, args);
    if (pair.type_atomic_number(1) != 8 || pair.type_atomic_number(2) != 1) {
      std::printf("FAIL element map\n");
      ++fails;
    }
  }
  {
    char *args[] = {(char *)model};
    bool gpu_ok = true;
    try {
      pair.settings(1, args);
    } catch (const std::runtime_error &e) {
      gpu_ok = false;
      if (!std::strstr(e.what(), "on the GPU")) {
        std::printf("FAIL settings with a valid model: %s\n", e.what());
        ++fails;
      }
    }
    if (pair.short_range_cutoff() != 4.5 || pair.long_range_cutoff() != 12.0) {
      std::printf("FAIL cutoffs %g %g\n", pair.short_range_cutoff(), pair.long_range_cutoff());
      ++fails;
    }
    if (pair.init_one(1, 2) != 4.5) {
      std::printf("FAIL init_one\n");
      ++fails;
    }
    if (gpu_ok) {
      lmp.force.newton_pair = 0;
      fails += expect_error("newton off", [&] { pair.init_style(); }, "requires newton pair on");
      lmp.force.newton_pair = 1;
      lmp.domain.zperiodic = 0;
      fails += expect_error("mixed boundaries", [&] { pair.init_style(); }, "'p p p'");
      lmp.domain.zperiodic = 1;
      // 3 atoms O, H, H with charge 1, multiplicity 1: 9 electrons cannot be a singlet
      lmp.atom.type[0] = 1;
      lmp.atom.type[1] = 2;
      lmp.atom.type[2] = 2;
      char *args3[] = {(char *)model, (char *)"1", (char *)"1"};
      pair.settings(3, args3);
      char *cargs[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"H"};
      pair.coeff(4, cargs);
      fails += expect_error("charge parity", [&] { pair.init_style(); }, "cannot have multiplicity");
    }
  }
  std::printf("%s\n", fails ? "PARSE FAIL" : "PARSE OK");
  return fails ? 1 : 0;
}

static int run(const char *model, const char *input) {
  std::ifstream in(input);
  double L;
  int n;
  in >> L >> n;
  LAMMPS lmp;
  lmp.atom.ntypes = 2;
  lmp.atom.resize(n);
  for (int i = 0; i < n; ++i) in >> lmp.atom.type[i] >> lmp.atom.x[i][0] >> lmp.atom.x[i][1] >> lmp.atom.x[i][2];
  for (int d = 0; d < 3; ++d) lmp.domain.prd[d] = L;
  PairSO3LRB200 pair(&lmp);
  char *sargs[] = {(char *)model};
  pair.settings(1, sargs);
  char *cargs[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"H"};
  pair.coeff(4, cargs);
  pair.init_style();
  pair.compute(1 | 2, 1 | 4);
  std::printf("{\"energy\": %.17g, \"virial\": [", pair.eng_vdwl);
  for (int k = 0; k < 6; ++k) std::printf(k ? ", %.17g" : "%.17g", pair.virial[k]);
  std::printf("], \"eatom_sum\": %.17g, \"forces\": [", [&] {
    double s = 0;
    for (int i = 0; i < n; ++i) s += pair.eatom[i];
    return s;
  }());
  for (int i = 0; i < n; ++i)
    std::printf(i ? ", [%.17g, %.17g, %.17g]" : "[%.17g, %.17g, %.17g]", lmp.atom.f[i][0], lmp.atom.f[i][1],
                lmp.atom.f[i][2]);
  std::printf("], \"vatom\": [");
  for (int i = 0; i < n; ++i) {
    std::printf(i ? ", [" : "[");
    for (int k = 0; k < 6; ++k) std::printf(k ? ", %.17g" : "%.17g", pair.vatom[i][k]);
    std::printf("]");
  }
  std::printf("], \"log\": \"%s\"}\n", lmp.log.substr(0, lmp.log.size() - 1).c_str());
  return 0;
}

int main(int argc, char **argv) {
  if (argc >= 3 && std::string(argv[1]) == "parse") return parse_checks(argv[2]);
  if (argc >= 4 && std::string(argv[1]) == "run") return run(argv[2], argv[3]);
  std::printf("usage: test_pair_shim parse MODEL | run MODEL INPUT\n");
  return 2;
}
