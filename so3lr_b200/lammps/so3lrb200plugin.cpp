// LAMMPS plugin entry point: `plugin load so3lrb200plugin.so` registers the
// pair styles so3lr/b200 and so3lr/b200/turbo, the way the reference's plugin
// registers so3lr/native/mpi (plugins/lammps/so3lrnativeplugin.cpp:17-35).
// Build as a shared module against the LAMMPS src/ headers and
// libso3lr_b200.so.
#include "lammpsplugin.h"
#include "version.h"

#include "pair_so3lr_b200.h"
#include "pair_so3lr_b200_turbo.h"

using namespace LAMMPS_NS;

namespace {
Pair *make_so3lr_b200(LAMMPS *lmp) { return new PairSO3LRB200(lmp); }
Pair *make_so3lr_b200_turbo(LAMMPS *lmp) { return new PairSO3LRB200Turbo(lmp); }
}  // namespace

extern "C" void lammpsplugin_init(void *lmp, void *handle, void *regfunc) {
  auto add = reinterpret_cast<lammpsplugin_regfunc>(regfunc);
  lammpsplugin_t entry;
  entry.version = LAMMPS_VERSION;
  entry.style = "pair";
  entry.author = "so3lr-b200";
  entry.handle = handle;

  entry.name = "so3lr/b200";
  entry.info = "SO3LR force field on B200 GPUs (spatial decomposition over MPI ranks)";
  entry.creator.v1 = reinterpret_cast<lammpsplugin_factory1 *>(&make_so3lr_b200);
  (*add)(&entry, lmp);

  entry.name = "so3lr/b200/turbo";
  entry.info = "SO3LR force field on B200 GPUs, one image per one-rank partition";
  entry.creator.v1 = reinterpret_cast<lammpsplugin_factory1 *>(&make_so3lr_b200_turbo);
  (*add)(&entry, lmp);
}
