// LAMMPS pair style so3lr/b200 on top of libso3lr_b200 (see pair_so3lr_b200.h).
// Mirrors the contract of PairSO3LRNativeMPI (reference
// plugins/lammps/pair_so3lr_native_mpi.cpp:1059-1192, 1246-1978): flags,
// pair_style/pair_coeff parsing, newton requirement, charge/multiplicity
// validation against the system composition, and the writes to atom->f,
// eatom, eng_vdwl and virial[6].
#include "pair_so3lr_b200.h"

#include <cstdlib>
#include <cstring>

#include "atom.h"
#include "comm.h"
#include "domain.h"
#include "error.h"
#include "force.h"
#include "memory.h"
#include "so3lr_b200.h"
#include "utils.h"

using namespace LAMMPS_NS;

PairSO3LRB200::PairSO3LRB200(LAMMPS *lmp) : Pair(lmp) {
  manybody_flag = 1;
  one_coeff = 1;
  restartinfo = 0;
  single_enable = 0;
  no_virial_fdotr_compute = 1;
}

PairSO3LRB200::~PairSO3LRB200() {
  release();
  if (allocated) {
    memory->destroy(setflag);
    memory->destroy(cutsq);
  }
}

void PairSO3LRB200::release() {
  if (handle_) so3lr_destroy(handle_);
  handle_ = nullptr;
}

void PairSO3LRB200::allocate() {
  allocated = 1;
  const int n = atom->ntypes;
  memory->create(setflag, n + 1, n + 1, "so3lr/b200:setflag");
  memory->create(cutsq, n + 1, n + 1, "so3lr/b200:cutsq");
  for (int i = 1; i <= n; ++i)
    for (int j = i; j <= n; ++j) setflag[i][j] = 0;
}

void PairSO3LRB200::settings(int narg, char **arg) {
  if (narg < 1 || narg > 3)
    error->all(FLERR, "Illegal pair_style so3lr/b200 command: expected "
                      "'pair_style so3lr/b200 MODEL [charge [multiplicity]]'");
  model_path_ = arg[0];
  total_charge_ = narg > 1 ? std::strtod(arg[1], nullptr) : 0.0;
  multiplicity_ = narg > 2 ? std::strtod(arg[2], nullptr) : 1.0;
  release();
  char err[2048] = {0};
  so3lr_arch_info info{};
  if (so3lr_inspect_model(model_path_.c_str(), &info, err, sizeof(err)) != 0)
    error->all(FLERR, std::string("Cannot initialize SO3LR model: ") + err);
  sr_cutoff_ = info.sr_cutoff;
  lr_cutoff_ = info.lr_cutoff;
  const char *dev = std::getenv("SO3LR_B200_DEVICE");
  if (so3lr_create(model_path_.c_str(), dev ? std::atoi(dev) : 0, &handle_, err, sizeof(err)) != 0)
    error->all(FLERR, std::string("Cannot initialize SO3LR model on the GPU: ") + err);
}

void PairSO3LRB200::coeff(int narg, char **arg) {
  if (!allocated) allocate();
  if (narg != atom->ntypes + 2 || std::strcmp(arg[0], "*") != 0 || std::strcmp(arg[1], "*") != 0)
    error->all(FLERR, "Pair coeff for so3lr/b200 must be '* * E1 ... Entypes' where each E is an element "
                      "symbol or atomic number");
  type_to_z_.assign(static_cast<std::size_t>(atom->ntypes) + 1, 0);
  for (int type = 1; type <= atom->ntypes; ++type) {
    const int z = so3lr_element_from_token(arg[type + 1]);
    if (z == 0)
      error->all(FLERR, std::string("Unknown SO3LR element '") + arg[type + 1] +
                            "'; use a symbol or atomic number from H/1 through Es/99");
    type_to_z_[static_cast<std::size_t>(type)] = z;
  }
  for (int i = 1; i <= atom->ntypes; ++i)
    for (int j = i; j <= atom->ntypes; ++j) setflag[i][j] = 1;
}

double PairSO3LRB200::init_one(int i, int j) {
  if (!setflag[i][j]) error->all(FLERR, "All so3lr/b200 coefficients are not set");
  return sr_cutoff_;
}

void PairSO3LRB200::init_style() {
  if (!force->newton_pair) error->all(FLERR, "Pair style so3lr/b200 requires newton pair on");
  if (!handle_) error->all(FLERR, "Pair style so3lr/b200 model was not initialized");
  if (type_to_z_.size() != static_cast<std::size_t>(atom->ntypes) + 1)
    error->all(FLERR, "Pair style so3lr/b200 coefficients are missing");
  if (comm->nprocs != 1)
    error->all(FLERR, "Pair style so3lr/b200 runs on one MPI rank that owns every atom; use one rank per "
                      "partition (one GPU each)");
  const bool periodic = domain->xperiodic && domain->yperiodic && domain->zperiodic;
  const bool open = !domain->xperiodic && !domain->yperiodic && !domain->zperiodic;
  if (!periodic && !open) error->all(FLERR, "Pair style so3lr/b200 needs 'p p p' or fully open boundaries");
  if (domain->triclinic) error->all(FLERR, "Pair style so3lr/b200 supports orthorhombic boxes only");
  // charge/multiplicity against the composition (pair_so3lr_native_mpi.cpp:1196-1235)
  long long counts[119] = {0};
  for (int i = 0; i < atom->nlocal; ++i) counts[type_to_z_[static_cast<std::size_t>(atom->type[i])]]++;
  char err[512] = {0};
  if (so3lr_validate_charge_spin(counts, total_charge_, multiplicity_, err, sizeof(err)) != 0)
    error->all(FLERR, std::string("SO3LR charge/multiplicity: ") + err);
}

void PairSO3LRB200::compute(int eflag, int vflag) {
  ev_init(eflag, vflag);
  const int n = atom->nlocal;
  x_.resize(3 * static_cast<std::size_t>(n));
  f_.resize(3 * static_cast<std::size_t>(n));
  eatom_.resize(static_cast<std::size_t>(n));
  z_.resize(static_cast<std::size_t>(n));
  for (int i = 0; i < n; ++i) {
    for (int d = 0; d < 3; ++d) x_[3 * i + d] = atom->x[i][d];
    z_[i] = type_to_z_[static_cast<std::size_t>(atom->type[i])];
  }
  so3lr_frame frame{};
  frame.natoms = n;
  frame.x = x_.data();
  frame.z = z_.data();
  frame.periodic = domain->xperiodic ? 1 : 0;
  for (int d = 0; d < 3; ++d) {
    frame.boxlo[d] = domain->boxlo[d];
    frame.boxlen[d] = domain->prd[d];
  }
  frame.total_charge = total_charge_;
  frame.multiplicity = multiplicity_;
  so3lr_result res{};
  res.f = f_.data();
  res.eatom = eatom_.data();
  char err[2048] = {0};
  if (so3lr_compute(handle_, &frame, &res, err, sizeof(err)) != 0)
    error->all(FLERR, std::string("SO3LR evaluation failed: ") + err);
  for (int i = 0; i < n; ++i)
    for (int d = 0; d < 3; ++d) atom->f[i][d] += f_[3 * i + d];
  if (eflag_atom)
    for (int i = 0; i < n; ++i) eatom[i] += eatom_[i];
  if (eflag_global) eng_vdwl += res.energy;
  if (vflag_global)
    for (int k = 0; k < 6; ++k) virial[k] += res.virial[k];
  if (vflag_atom) {
    // per-atom virial (the reference refuses vflag_atom): half of every pair
    // term to each of its atoms, rows summing to the global virial
    va_.resize(6 * static_cast<std::size_t>(n));
    if (so3lr_virial_atom(handle_, va_.data(), err, sizeof(err)) != 0)
      error->all(FLERR, std::string("SO3LR per-atom virial failed: ") + err);
    for (int i = 0; i < n; ++i)
      for (int k = 0; k < 6; ++k) vatom[i][k] += va_[6 * static_cast<std::size_t>(i) + k];
  }
  if (!reported_ && comm->me == 0) {
    reported_ = true;
    utils::logmesg(lmp, "SO3LR_B200_FORCE_PATH=PASS atoms=" + std::to_string(n) +
                           " energy=" + std::to_string(res.energy) + "\n");
  }
}
