// Drives the so3lr/b200 and so3lr/b200/turbo pair styles through the mock LAMMPS API.
//   test_pair_shim parse MODEL          pair_style/pair_coeff parsing and refusals
//   test_pair_shim run MODEL INPUT      one compute; INPUT holds "L n" then n lines "type x y z"
//                                       (types 1 = O, 2 = H); prints JSON with energy, virial, forces
//   test_pair_shim run-reversed-tags MODEL INPUT
//                                       the same with atom i tagged n - i
//   test_pair_shim run-duplicate-tag MODEL INPUT
//                                       the same with atoms 0 and 1 sharing a tag (refused)
//   test_pair_shim repeat MODEL INPUT [CHARGE MULT]
//                                       four computes; prints the style's log and warnings
//   test_pair_shim turbo-parse MODEL    so3lr/b200/turbo parsing and refusals on one rank, and a
//                                       coordinator failure reaching every partition of a universe
//   test_pair_shim turbo-run MODEL INPUT
//                                       one image per partition, partitions run as threads of a
//                                       universe; INPUT holds "K" then per image "n charge mult" and
//                                       n lines "type x y z"; prints one JSON line per image
//   test_pair_shim multirank MODEL INPUT NRANKS
//                                       so3lr/b200 on NRANKS MPI ranks (threads, one GPU each);
//                                       INPUT as for run; atom i lives on rank (7 i) % NRANKS with
//                                       tag i + 1; prints one JSON line per rank
//   test_pair_shim rank-failure MODEL   two ranks, only rank 1 cannot load the model
//   test_pair_shim plugin               lammpsplugin_init registers both styles; their
//                                       creators build the pair objects
//   test_pair_shim turbo-refuse MODEL INPUT
//                                       the same universe with image 1 periodic and image 2 given
//                                       an impossible multiplicity: every partition must stop
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <sstream>
#include <string>
#include <vector>

#include "lammpsplugin.h"
#include "pair_so3lr_b200.h"
#include "pair_so3lr_b200_turbo.h"

extern "C" void lammpsplugin_init(void *lmp, void *handle, void *regfunc);

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

// four computes of the atoms in INPUT; prints the pair style's log and warnings
static int repeat(const char *model, const char *input, const char *charge = nullptr, const char *mult = nullptr) {
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
  char *sargs[] = {(char *)model, (char *)charge, (char *)mult};
  pair.settings(charge && mult ? 3 : 1, sargs);
  char *cargs[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"H"};
  pair.coeff(4, cargs);
  pair.init_style();
  for (int k = 0; k < 4; ++k) pair.compute(1, 0);
  std::printf("%s%s", lmp.log.c_str(), lmp.error.warnings.c_str());
  return 0;
}

static int run(const char *model, const char *input, bool reverse_tags = false, bool duplicate_tag = false) {
  std::ifstream in(input);
  double L;
  int n;
  in >> L >> n;
  LAMMPS lmp;
  lmp.atom.ntypes = 2;
  lmp.atom.resize(n);
  if (reverse_tags)
    for (int i = 0; i < n; ++i) lmp.atom.tag[i] = n - i;
  if (duplicate_tag && n > 1) lmp.atom.tag[1] = lmp.atom.tag[0];
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
  std::string log = lmp.log;  // one JSON string: the log's lines joined by " | "
  while (!log.empty() && log.back() == '\n') log.pop_back();
  for (std::size_t p = log.find('\n'); p != std::string::npos; p = log.find('\n', p)) log.replace(p, 1, " | ");
  std::printf("], \"log\": \"%s\"}\n", log.c_str());
  return 0;
}

static int multirank(const char *model, const char *input, int nranks) {
  std::ifstream in(input);
  double L;
  int n;
  in >> L >> n;
  std::vector<int> type(n);
  std::vector<double> x(3 * static_cast<std::size_t>(n));
  for (int i = 0; i < n; ++i) in >> type[i] >> x[3 * i] >> x[3 * i + 1] >> x[3 * i + 2];
  std::vector<std::string> out(nranks);
  auto errs = mpi_stub_run(nranks, [&](int r) {
    std::vector<int> mine;
    for (int i = 0; i < n; ++i)
      if ((7 * i) % nranks == r) mine.push_back(i);
    LAMMPS lmp;
    lmp.comm.me = r;
    lmp.comm.nprocs = nranks;
    lmp.atom.ntypes = 2;
    lmp.atom.resize(static_cast<int>(mine.size()));
    lmp.atom.natoms = n;
    for (std::size_t j = 0; j < mine.size(); ++j) {
      const int i = mine[j];
      lmp.atom.tag[j] = i + 1;
      lmp.atom.type[j] = type[i];
      for (int d = 0; d < 3; ++d) lmp.atom.x[j][d] = x[3 * static_cast<std::size_t>(i) + d];
    }
    for (int d = 0; d < 3; ++d) lmp.domain.prd[d] = L;
    PairSO3LRB200 pair(&lmp);
    char *sargs[] = {(char *)model};
    pair.settings(1, sargs);
    char *cargs[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"H"};
    pair.coeff(4, cargs);
    pair.init_style();
    pair.compute(1 | 2, 1 | 4);
    std::ostringstream s;
    s.precision(17);
    s << "{\"rank\": " << r << ", \"energy\": " << pair.eng_vdwl << ", \"virial\": [";
    for (int k = 0; k < 6; ++k) s << (k ? ", " : "") << pair.virial[k];
    s << "], \"tags\": [";
    for (std::size_t j = 0; j < mine.size(); ++j) s << (j ? ", " : "") << lmp.atom.tag[j];
    s << "], \"eatom\": [";
    for (std::size_t j = 0; j < mine.size(); ++j) s << (j ? ", " : "") << pair.eatom[j];
    s << "], \"forces\": [";
    for (std::size_t j = 0; j < mine.size(); ++j)
      s << (j ? ", [" : "[") << lmp.atom.f[j][0] << ", " << lmp.atom.f[j][1] << ", " << lmp.atom.f[j][2] << "]";
    s << "], \"vatom\": [";
    for (std::size_t j = 0; j < mine.size(); ++j) {
      s << (j ? ", [" : "[");
      for (int k = 0; k < 6; ++k) s << (k ? ", " : "") << pair.vatom[j][k];
      s << "]";
    }
    s << "]}";
    out[r] = s.str();
  });
  int rc = 0;
  for (int r = 0; r < nranks; ++r) {
    if (errs[r]) {
      try {
        std::rethrow_exception(errs[r]);
      } catch (const std::exception &e) {
        std::printf("ERROR rank %d: %s\n", r, e.what());
      }
      rc = 1;
    } else {
      std::printf("%s\n", out[r].c_str());
    }
  }
  return rc;
}

// two MPI ranks (threads) where only rank 1 cannot load the model: rank 1
// reports its own error, rank 0 learns of it instead of waiting
static int rank_failure(const char *model) {
  std::vector<std::string> msgs(2, "no error");
  auto errs = mpi_stub_run(2, [&](int r) {
    LAMMPS lmp;
    lmp.comm.me = r;
    lmp.comm.nprocs = 2;
    lmp.atom.ntypes = 2;
    lmp.atom.resize(3);
    PairSO3LRB200 pair(&lmp);
    char *good[] = {(char *)model};
    char *bad[] = {(char *)"/nonexistent/model.so3lr"};
    pair.settings(1, r == 1 ? bad : good);
  });
  for (int r = 0; r < 2; ++r)
    if (errs[r]) {
      try {
        std::rethrow_exception(errs[r]);
      } catch (const std::exception &e) {
        msgs[r] = e.what();
      }
    }
  const bool ok = msgs[1].find("cannot open") != std::string::npos &&
                  msgs[0].find("failed on another MPI rank") != std::string::npos;
  std::printf("rank 0: %s\nrank 1: %s\n%s\n", msgs[0].c_str(), msgs[1].c_str(),
              ok ? "RANK FAILURE OK" : "RANK FAILURE FAIL");
  return ok ? 0 : 1;
}

static int turbo_parse_checks(const char *model) {
  int fails = 0;
  {
    LAMMPS lmp;
    lmp.atom.ntypes = 2;
    lmp.atom.resize(3);
    lmp.domain.xperiodic = lmp.domain.yperiodic = lmp.domain.zperiodic = 0;
    PairSO3LRB200Turbo pair(&lmp);
    char *many[] = {(char *)"a", (char *)"b", (char *)"c", (char *)"d"};
    fails += expect_error("turbo: too many pair_style args", [&] { pair.settings(4, many); },
                          "Illegal pair_style so3lr/b200/turbo");
    char *missing[] = {(char *)"/nonexistent/model.so3lr"};
    fails += expect_error("turbo: missing model", [&] { pair.settings(1, missing); }, "cannot open");
    char *bad[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"Qq"};
    fails += expect_error("turbo: unknown element", [&] { pair.coeff(4, bad); }, "Unknown SO3LR element");
    char *good[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"H"};
    pair.coeff(4, good);
    if (pair.type_atomic_number(1) != 8 || pair.type_atomic_number(2) != 1) {
      std::printf("FAIL turbo element map\n");
      ++fails;
    }
    // a universe of one partition is refused (the reference needs at least two images)
    char *args[] = {(char *)model};
    bool gpu_ok = true;
    try {
      pair.settings(1, args);
    } catch (const std::runtime_error &e) {
      gpu_ok = false;
      if (!std::strstr(e.what(), "coordinator SO3LR model on the GPU")) {
        std::printf("FAIL turbo settings with a valid model: %s\n", e.what());
        ++fails;
      }
    }
    if (gpu_ok) {
      if (pair.long_range_cutoff() != 12.0 || pair.init_one(1, 2) != 12.0) {
        std::printf("FAIL turbo cutoffs\n");
        ++fails;
      }
      fails += expect_error("turbo: one partition", [&] { pair.init_style(); }, "multiple one-rank partitions");
    }
  }
  // two partitions: the coordinator's failure to load a model reaches both
  std::vector<std::string> msgs(2);
  auto errs = mpi_stub_run(2, [&](int r) {
    LAMMPS lmp;
    lmp.universe.me = r;
    lmp.universe.nprocs = lmp.universe.nworlds = 2;
    lmp.universe.iworld = r;
    lmp.atom.ntypes = 2;
    lmp.atom.resize(3);
    PairSO3LRB200Turbo pair(&lmp);
    pair.world = MPI_COMM_SELF;
    char *missing[] = {(char *)"/nonexistent/model.so3lr"};
    pair.settings(1, missing);
  });
  for (int r = 0; r < 2; ++r) {
    std::string what = "no error";
    if (errs[r]) {
      try {
        std::rethrow_exception(errs[r]);
      } catch (const std::runtime_error &e) {
        what = e.what();
      }
    }
    if (what.find("Cannot initialize the coordinator SO3LR model: ") == std::string::npos) {
      std::printf("FAIL turbo coordinator failure on partition %d: %s\n", r, what.c_str());
      ++fails;
    }
  }
  std::printf("%s\n", fails ? "TURBO PARSE FAIL" : "TURBO PARSE OK");
  return fails ? 1 : 0;
}

struct TurboImage {
  int n = 0;
  double charge = 0.0, mult = 1.0;
  std::vector<int> type;
  std::vector<double> x;
};

static std::vector<TurboImage> read_images(const char *input) {
  std::ifstream in(input);
  int k = 0;
  in >> k;
  std::vector<TurboImage> images(k);
  for (TurboImage &im : images) {
    in >> im.n >> im.charge >> im.mult;
    im.type.resize(im.n);
    im.x.resize(3 * static_cast<std::size_t>(im.n));
    for (int i = 0; i < im.n; ++i) in >> im.type[i] >> im.x[3 * i] >> im.x[3 * i + 1] >> im.x[3 * i + 2];
  }
  return images;
}

// one partition of the turbo universe: rank r holds image r
static void setup_partition(LAMMPS &lmp, const TurboImage &im, int r, int nimg) {
  lmp.universe.me = r;
  lmp.universe.nprocs = lmp.universe.nworlds = nimg;
  lmp.universe.iworld = r;
  lmp.atom.ntypes = 2;
  lmp.atom.resize(im.n);
  for (int i = 0; i < im.n; ++i) {
    lmp.atom.type[i] = im.type[i];
    for (int d = 0; d < 3; ++d) lmp.atom.x[i][d] = im.x[3 * static_cast<std::size_t>(i) + d];
  }
  lmp.domain.xperiodic = lmp.domain.yperiodic = lmp.domain.zperiodic = 0;
}

static int turbo_run(const char *model, const char *input) {
  const std::vector<TurboImage> images = read_images(input);
  const int nimg = static_cast<int>(images.size());
  std::vector<std::string> out(nimg);
  auto errs = mpi_stub_run(nimg, [&](int r) {
    const TurboImage &im = images[r];
    LAMMPS lmp;
    setup_partition(lmp, im, r, nimg);
    PairSO3LRB200Turbo pair(&lmp);
    pair.world = MPI_COMM_SELF;
    std::string q = std::to_string(im.charge), m = std::to_string(im.mult);
    char *sargs[] = {(char *)model, (char *)q.c_str(), (char *)m.c_str()};
    pair.settings(3, sargs);
    char *cargs[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"H"};
    pair.coeff(4, cargs);
    pair.init_style();
    // first step: every image wants F dot r and per-atom virials
    pair.compute(1 | 2, 2 | 4);
    std::ostringstream s;
    s.precision(17);
    double esum = 0.0;
    for (int i = 0; i < im.n; ++i) esum += pair.eatom[i];
    s << "{\"image\": " << r << ", \"energy\": " << pair.eng_vdwl << ", \"eatom_sum\": " << esum
      << ", \"virial\": [";
    for (int k = 0; k < 6; ++k) s << (k ? ", " : "") << pair.virial[k];
    s << "], \"forces\": [";
    for (int i = 0; i < im.n; ++i)
      s << (i ? ", [" : "[") << lmp.atom.f[i][0] << ", " << lmp.atom.f[i][1] << ", " << lmp.atom.f[i][2] << "]";
    s << "], \"vatom\": [";
    for (int i = 0; i < im.n; ++i) {
      s << (i ? ", [" : "[");
      for (int k = 0; k < 6; ++k) s << (k ? ", " : "") << pair.vatom[i][k];
      s << "]";
    }
    // second step: only image 0 wants per-atom virials; results must repeat
    const std::vector<double> f1 = lmp.atom.f_data;
    const double e1 = pair.eng_vdwl;
    std::fill(lmp.atom.f_data.begin(), lmp.atom.f_data.end(), 0.0);
    pair.compute(1, r == 0 ? (2 | 4) : 2);
    const bool repeat = lmp.atom.f_data == f1 && pair.eng_vdwl == e1;
    std::string log = lmp.log;
    for (char &c : log)
      if (c == '\n') c = '|';
    s << "], \"repeat_equal\": " << (repeat ? "true" : "false") << ", \"evaluations\": " << pair.evaluations()
      << ", \"log\": \"" << log << "\"}";
    out[r] = s.str();
  });
  int rc = 0;
  for (int r = 0; r < nimg; ++r) {
    if (errs[r]) {
      try {
        std::rethrow_exception(errs[r]);
      } catch (const std::exception &e) {
        std::printf("ERROR image %d: %s\n", r, e.what());
      }
      rc = 1;
    } else {
      std::printf("%s\n", out[r].c_str());
    }
  }
  return rc;
}

static int turbo_refuse(const char *model, const char *input) {
  const std::vector<TurboImage> images = read_images(input);
  const int nimg = static_cast<int>(images.size());
  auto errs = mpi_stub_run(nimg, [&](int r) {
    const TurboImage &im = images[r];
    LAMMPS lmp;
    setup_partition(lmp, im, r, nimg);
    if (r == 1) lmp.domain.xperiodic = lmp.domain.yperiodic = lmp.domain.zperiodic = 1;
    PairSO3LRB200Turbo pair(&lmp);
    pair.world = MPI_COMM_SELF;
    // image 2: an even electron count cannot be a doublet
    std::string q = std::to_string(im.charge), m = r == 2 ? "2" : std::to_string(im.mult);
    char *sargs[] = {(char *)model, (char *)q.c_str(), (char *)m.c_str()};
    pair.settings(3, sargs);
    char *cargs[] = {(char *)"*", (char *)"*", (char *)"O", (char *)"H"};
    pair.coeff(4, cargs);
    pair.init_style();
    pair.compute(1, 0);
  });
  const char *expect[3] = {"another partition refused", "requires non-periodic boundaries",
                           "so3lr/b200/turbo image 2: charge"};
  int fails = 0;
  for (int r = 0; r < nimg; ++r) {
    std::string what = "no error";
    if (errs[r]) {
      try {
        std::rethrow_exception(errs[r]);
      } catch (const std::exception &e) {
        what = e.what();
      }
    }
    const char *want = expect[r < 3 ? r : 0];
    if (what.find(want) == std::string::npos) {
      std::printf("FAIL partition %d: expected '%s', got '%s'\n", r, want, what.c_str());
      ++fails;
    }
  }
  std::printf("%s\n", fails ? "TURBO REFUSE FAIL" : "TURBO REFUSE OK");
  return fails ? 1 : 0;
}

static std::vector<std::string> g_registered;
static void register_style(lammpsplugin_t *p, void *lmp) {
  g_registered.push_back(std::string(p->style) + " " + p->name);
  Pair *pair = reinterpret_cast<Pair *>(p->creator.v1(lmp));
  const bool ok = pair != nullptr && pair->manybody_flag == 1 && pair->one_coeff == 1;
  std::printf("%s %s %s %s\n", p->style, p->name, ok ? "constructed" : "BAD", p->version);
  delete pair;
}

static int plugin_check() {
  LAMMPS lmp;
  int handle = 0;
  lammpsplugin_init(&lmp, &handle, reinterpret_cast<void *>(&register_style));
  const bool ok = g_registered.size() == 2 && g_registered[0] == "pair so3lr/b200" &&
                  g_registered[1] == "pair so3lr/b200/turbo";
  std::printf("%s\n", ok ? "PLUGIN OK" : "PLUGIN FAIL");
  return ok ? 0 : 1;
}

int main(int argc, char **argv) {
  if (argc >= 2 && std::string(argv[1]) == "plugin") return plugin_check();
  if (argc >= 3 && std::string(argv[1]) == "rank-failure") return rank_failure(argv[2]);
  if (argc >= 3 && std::string(argv[1]) == "parse") return parse_checks(argv[2]);
  if (argc >= 4 && std::string(argv[1]) == "run") return run(argv[2], argv[3]);
  if (argc >= 4 && std::string(argv[1]) == "run-reversed-tags") return run(argv[2], argv[3], true);
  if (argc >= 4 && std::string(argv[1]) == "run-duplicate-tag") return run(argv[2], argv[3], false, true);
  if (argc >= 6 && std::string(argv[1]) == "repeat") return repeat(argv[2], argv[3], argv[4], argv[5]);
  if (argc >= 4 && std::string(argv[1]) == "repeat") return repeat(argv[2], argv[3]);
  if (argc >= 5 && std::string(argv[1]) == "multirank") return multirank(argv[2], argv[3], std::atoi(argv[4]));
  if (argc >= 3 && std::string(argv[1]) == "turbo-parse") return turbo_parse_checks(argv[2]);
  if (argc >= 4 && std::string(argv[1]) == "turbo-run") return turbo_run(argv[2], argv[3]);
  if (argc >= 4 && std::string(argv[1]) == "turbo-refuse") return turbo_refuse(argv[2], argv[3]);
  std::printf("usage: test_pair_shim parse MODEL | run MODEL INPUT | multirank MODEL INPUT NRANKS | turbo-parse MODEL | "
              "turbo-run MODEL INPUT | turbo-refuse MODEL INPUT\n");
  return 2;
}
