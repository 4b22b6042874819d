// LAMMPS pair style so3lr/b200 on top of libso3lr_b200 (see pair_so3lr_b200.h).
// Mirrors the contract of PairSO3LRNativeMPI (reference
// plugins/lammps/pair_so3lr_native_mpi.cpp:1059-1192, 1246-1978): flags,
// pair_style/pair_coeff parsing, newton requirement, charge/multiplicity
// validation against the system composition, and the writes to atom->f,
// eatom, eng_vdwl and virial[6].
#include "pair_so3lr_b200.h"

#include <mpi.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>

#include "atom.h"
#include "comm.h"
#include "domain.h"
#include "error.h"
#include "force.h"
#include "memory.h"
#include "so3lr_b200.h"
#include "so3lr_b200_precision.h"
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
  std::string problem;
  if (so3lr_inspect_model(model_path_.c_str(), &info, err, sizeof(err)) != 0) {
    problem = std::string("Cannot initialize SO3LR model: ") + err;
  } else {
    sr_cutoff_ = info.sr_cutoff;
    lr_cutoff_ = info.lr_cutoff;
    // one GPU per MPI rank: $SO3LR_B200_DEVICE when set, else the rank number
    // (ranks of one node on that node's GPUs)
    const char *dev = std::getenv("SO3LR_B200_DEVICE");
    const int device = dev ? std::atoi(dev) : comm->me;
    if (so3lr_create(model_path_.c_str(), device, &handle_, err, sizeof(err)) != 0)
      problem = std::string("Cannot initialize SO3LR model on the GPU: ") + err;
    // $SO3LR_B200_PRECISION=mixed: pair-filter GEMMs as three-pass TF32
    else if (so3lr_b200_precision_from_env(handle_, err, sizeof(err)) != 0)
      problem = std::string("SO3LR precision: ") + err;
  }
  // a failure on some ranks only (a missing GPU, a file one node cannot read)
  // must not leave the others waiting in the next collective
  int bad = problem.empty() ? 0 : 1, nbad = 0;
  MPI_Allreduce(&bad, &nbad, 1, MPI_INT, MPI_SUM, world);
  if (nbad == comm->nprocs) error->all(FLERR, problem);
  if (bad) error->one(FLERR, problem);
  if (nbad) error->all(FLERR, "SO3LR model initialization failed on another MPI rank");
  comm_ready_ = false;
  profile_every_ = -1;  // the new handle gets profiling switched on again if asked for
  profile_calls_ = 0;
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
  const bool periodic = domain->xperiodic && domain->yperiodic && domain->zperiodic;
  const bool open = !domain->xperiodic && !domain->yperiodic && !domain->zperiodic;
  if (!periodic && !open) error->all(FLERR, "Pair style so3lr/b200 needs 'p p p' or fully open boundaries");
  if (domain->triclinic) error->all(FLERR, "Pair style so3lr/b200 supports orthorhombic boxes only");
  // charge/multiplicity against the composition of all ranks' atoms
  // (pair_so3lr_native_mpi.cpp:1196-1235)
  long long local[119] = {0}, counts[119] = {0};
  for (int i = 0; i < atom->nlocal; ++i) local[type_to_z_[static_cast<std::size_t>(atom->type[i])]]++;
  MPI_Allreduce(local, counts, 119, MPI_LONG_LONG, MPI_SUM, world);
  char err[512] = {0};
  if (so3lr_validate_charge_spin(counts, total_charge_, multiplicity_, err, sizeof(err)) != 0)
    error->all(FLERR, std::string("SO3LR charge/multiplicity: ") + err);
  if (comm->me == 0) {
    char line[160];
    std::snprintf(line, sizeof(line), "SO3LR: total charge %g, spin multiplicity %g\n", total_charge_,
                  multiplicity_);
    utils::logmesg(lmp, line);
    if (total_charge_ != 0.0 && periodic) {
      std::snprintf(line, sizeof(line),
                    "SO3LR: net charge %g in a periodic cell. SO3LR's long range is truncated real-space "
                    "Coulomb, so the energy is defined, but there is no neutralizing background",
                    total_charge_);
      error->warning(FLERR, line);
    }
  }
  // several ranks: one NCCL communicator over the ranks' GPUs, id from rank 0
  if (comm->nprocs > 1 && !comm_ready_) {
    char uid[128] = {0};
    int rc = 0;
    if (comm->me == 0) rc = so3lr_nccl_unique_id(uid, err, sizeof(err));
    MPI_Bcast(&rc, 1, MPI_INT, 0, world);
    if (rc != 0) error->all(FLERR, std::string("SO3LR: cannot create the NCCL id on rank 0: ") + err);
    MPI_Bcast(uid, 128, MPI_BYTE, 0, world);
    if (so3lr_comm_init(handle_, comm->nprocs, comm->me, uid, err, sizeof(err)) != 0)
      fail_collective(std::string("SO3LR: cannot join the GPUs of the other ranks: ") + err);
    comm_ready_ = true;
  }
}

// One JSON object per call: schema so3lr-native-debug-v1, the long-range
// electrostatic and dispersion totals, and per local atom its tag, type and
// energy terms, charge and Hirshfeld ratio.
void PairSO3LRB200::write_debug_dump(const char *path, const so3lr_result &res, int n) {
  FILE *out = std::fopen(path, "w");
  if (out == nullptr) error->all(FLERR, std::string("cannot open SO3LR_NATIVE_DEBUG_DUMP ") + path);
  double elec = 0.0, disp = 0.0;
  for (int k = 0; k < n; ++k) {
    elec += res.e_elec[k];
    disp += res.e_disp[k];
  }
  const int nlocal = atom->nlocal;
  auto array = [&](const char *name, const std::function<double(int)> &value, bool last) {
    std::fprintf(out, "\"%s\":[", name);
    for (int i = 0; i < nlocal; ++i) std::fprintf(out, i ? ",%.17g" : "%.17g", value(i));
    std::fprintf(out, "]%s", last ? "" : ",");
  };
  // the library's arrays are in tag order; local atom i is row tag - 1
  auto row = [&](int i) { return static_cast<std::size_t>(atom->tag[i] - 1); };
  std::fprintf(out, "{\"schema\":\"so3lr-native-debug-v1\",\"natoms\":%d,", nlocal);
  std::fprintf(out, "\"electrostatic_total\":%.17g,\"dispersion_total\":%.17g,", elec, disp);
  array("tag", [&](int i) { return static_cast<double>(atom->tag[i]); }, false);
  array("type", [&](int i) { return static_cast<double>(atom->type[i]); }, false);
  array("learned_energy", [&](int i) { return res.e_learned[row(i)]; }, false);
  array("zbl_energy", [&](int i) { return res.e_zbl[row(i)]; }, false);
  array("physical_energy", [&](int i) { return res.e_lr[row(i)]; }, false);
  array("partial_charges", [&](int i) { return res.charges[row(i)]; }, false);
  array("hirshfeld_ratios", [&](int i) { return res.ratios[row(i)]; }, true);
  std::fprintf(out, "}\n");
  std::fclose(out);
}

// A failure of a library call that all ranks make together (joining the GPUs,
// an evaluation). With several ranks the others may be waiting inside the
// library's collective communication, where error->all's barrier would never
// return, so the failing rank stops the whole job itself (error->one).
void PairSO3LRB200::fail_collective(const std::string &msg) {
  if (comm->nprocs > 1) error->one(FLERR, msg);
  error->all(FLERR, msg);
}

// The opt-in per-atom dump (one rank): the whole system by tag through
// so3lr_compute, which also returns the per-atom terms the dump schema lists.
void PairSO3LRB200::compute_with_dump(const char *dump_path) {
  const int nlocal = atom->nlocal;
  // the whole system ordered by atom tag (one rank: the gathers below are copies)
  const int nprocs = comm->nprocs;
  counts_.assign(nprocs, 0);
  displs_.assign(nprocs, 0);
  MPI_Allgather(&nlocal, 1, MPI_INT, counts_.data(), 1, MPI_INT, world);
  long long total = 0;
  for (int r = 0; r < nprocs; ++r) {
    displs_[r] = static_cast<int>(total);
    total += counts_[r];
  }
  if (total > (1LL << 30)) error->all(FLERR, "Pair style so3lr/b200: too many atoms");
  const int n = static_cast<int>(total);
  loc_tag_.resize(nlocal);
  loc_x_.resize(3 * static_cast<std::size_t>(nlocal));
  loc_z_.resize(nlocal);
  for (int i = 0; i < nlocal; ++i) {
    loc_tag_[i] = static_cast<int>(atom->tag[i]);
    for (int d = 0; d < 3; ++d) loc_x_[3 * i + d] = atom->x[i][d];
    loc_z_[i] = type_to_z_[static_cast<std::size_t>(atom->type[i])];
  }
  all_tag_.resize(n);
  all_x_.resize(3 * static_cast<std::size_t>(n));
  all_z_.resize(n);
  MPI_Allgatherv(loc_tag_.data(), nlocal, MPI_INT, all_tag_.data(), counts_.data(), displs_.data(), MPI_INT, world);
  MPI_Allgatherv(loc_z_.data(), nlocal, MPI_INT, all_z_.data(), counts_.data(), displs_.data(), MPI_INT, world);
  for (int r = 0; r < nprocs; ++r) {
    counts3_.resize(nprocs);
    displs3_.resize(nprocs);
    counts3_[r] = 3 * counts_[r];
    displs3_[r] = 3 * displs_[r];
  }
  MPI_Allgatherv(loc_x_.data(), 3 * nlocal, MPI_DOUBLE, all_x_.data(), counts3_.data(), displs3_.data(), MPI_DOUBLE,
                 world);
  // tags 1..n: gathered slot k holds atom tag all_tag_[k]
  x_.resize(3 * static_cast<std::size_t>(n));
  z_.resize(n);
  seen_.assign(n, 0);
  for (int k = 0; k < n; ++k) {
    const int tg = all_tag_[k];
    if (tg < 1 || tg > n || seen_[tg - 1]) error->all(FLERR, "Pair style so3lr/b200 needs unique atom tags 1..natoms");
    seen_[tg - 1] = 1;
    for (int d = 0; d < 3; ++d) x_[3 * static_cast<std::size_t>(tg - 1) + d] = all_x_[3 * static_cast<std::size_t>(k) + d];
    z_[tg - 1] = all_z_[k];
  }
  f_.resize(3 * static_cast<std::size_t>(n));
  eatom_.resize(n);
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
  {
    terms_.assign(7 * static_cast<std::size_t>(n), 0.0);
    double *tp = terms_.data();
    res.charges = tp;
    res.ratios = tp + n;
    res.e_learned = tp + 2 * static_cast<std::size_t>(n);
    res.e_zbl = tp + 3 * static_cast<std::size_t>(n);
    res.e_lr = tp + 4 * static_cast<std::size_t>(n);
    res.e_elec = tp + 5 * static_cast<std::size_t>(n);
    res.e_disp = tp + 6 * static_cast<std::size_t>(n);
  }
  char err[2048] = {0};
  if (so3lr_compute(handle_, &frame, &res, err, sizeof(err)) != 0)
    fail_collective(std::string("SO3LR evaluation failed: ") + err);
  write_debug_dump(dump_path, res, n);
  // each rank keeps its own atoms' forces and per-atom terms; the global energy
  // and virial (exact sums, identical on every rank) are reported by rank 0 only,
  // so LAMMPS's sum over ranks counts them once
  for (int i = 0; i < nlocal; ++i) {
    const std::size_t k = static_cast<std::size_t>(loc_tag_[i] - 1);
    for (int d = 0; d < 3; ++d) atom->f[i][d] += f_[3 * k + d];
  }
  if (eflag_atom)
    for (int i = 0; i < nlocal; ++i) eatom[i] += eatom_[static_cast<std::size_t>(loc_tag_[i] - 1)];
  if (eflag_global && comm->me == 0) eng_vdwl += res.energy;
  if (vflag_global && comm->me == 0)
    for (int k = 0; k < 6; ++k) virial[k] += res.virial[k];
  if (vflag_atom) {
    // per-atom virial (the reference refuses vflag_atom): half of every pair
    // term to each of its atoms, rows summing to the global virial
    va_.resize(6 * static_cast<std::size_t>(n));
    if (so3lr_virial_atom(handle_, va_.data(), err, sizeof(err)) != 0)
      fail_collective(std::string("SO3LR per-atom virial failed: ") + err);
    for (int i = 0; i < nlocal; ++i) {
      const std::size_t k = static_cast<std::size_t>(loc_tag_[i] - 1);
      for (int c = 0; c < 6; ++c) vatom[i][c] += va_[6 * k + c];
    }
  }
  if (!reported_ && comm->me == 0) {
    reported_ = true;
    utils::logmesg(lmp, "SO3LR_B200_FORCE_PATH=PASS atoms=" + std::to_string(n) +
                           " energy=" + std::to_string(res.energy) + "\n");
  }
}


void PairSO3LRB200::compute(int eflag, int vflag) {
  ev_init(eflag, vflag);
  setup_profile();
  // opt-in per-atom terms for validation against the reference's JAX harness,
  // in the reference's dump schema (pair_so3lr_native_mpi.cpp:1811-1862)
  const char *dump_path = std::getenv("SO3LR_NATIVE_DEBUG_DUMP");
  if (dump_path != nullptr && dump_path[0] != '\0') {
    if (comm->nprocs != 1) error->all(FLERR, "SO3LR_NATIVE_DEBUG_DUMP requires a single MPI rank");
    compute_with_dump(dump_path);
    report_profile();
    return;
  }
  // this rank's own atoms only, identified by their tags, as the reference
  // hands its evaluator the rank's atoms (pair_so3lr_native_mpi.cpp:1267-1280);
  // the library's GPUs exchange the ranks' atoms among themselves and return
  // this rank's forces, per-atom energies and virials
  const int nlocal = atom->nlocal;
  if (atom->natoms > (1LL << 30)) error->all(FLERR, "Pair style so3lr/b200: too many atoms");
  loc_tag64_.resize(nlocal);
  loc_x_.resize(3 * static_cast<std::size_t>(nlocal));
  loc_z_.resize(nlocal);
  for (int i = 0; i < nlocal; ++i) {
    loc_tag64_[i] = static_cast<long long>(atom->tag[i]);
    for (int d = 0; d < 3; ++d) loc_x_[3 * i + d] = atom->x[i][d];
    loc_z_[i] = type_to_z_[static_cast<std::size_t>(atom->type[i])];
  }
  f_.resize(3 * static_cast<std::size_t>(nlocal));
  so3lr_local_frame frame{};
  frame.natoms = static_cast<long long>(atom->natoms);
  frame.nlocal = nlocal;
  frame.tag = loc_tag64_.data();
  frame.x = loc_x_.data();
  frame.z = loc_z_.data();
  frame.periodic = domain->xperiodic ? 1 : 0;
  for (int d = 0; d < 3; ++d) {
    frame.boxlo[d] = domain->boxlo[d];
    frame.boxlen[d] = domain->prd[d];
  }
  frame.total_charge = total_charge_;
  frame.multiplicity = multiplicity_;
  so3lr_local_result res{};
  res.f = f_.data();
  if (eflag_atom) {
    eatom_.resize(nlocal);
    res.eatom = eatom_.data();
  }
  // per-atom virial (the reference refuses vflag_atom): half of every pair
  // term to each of its atoms, rows summing to the global virial
  if (vflag_atom) {
    va_.resize(6 * static_cast<std::size_t>(nlocal));
    res.vatom = va_.data();
  }
  char err[2048] = {0};
  if (so3lr_compute_local(handle_, &frame, &res, err, sizeof(err)) != 0)
    fail_collective(std::string("SO3LR evaluation failed: ") + err);
  for (int i = 0; i < nlocal; ++i)
    for (int d = 0; d < 3; ++d) atom->f[i][d] += f_[3 * static_cast<std::size_t>(i) + d];
  if (eflag_atom)
    for (int i = 0; i < nlocal; ++i) eatom[i] += eatom_[i];
  if (vflag_atom)
    for (int i = 0; i < nlocal; ++i)
      for (int c = 0; c < 6; ++c) vatom[i][c] += va_[6 * static_cast<std::size_t>(i) + c];
  // the global energy and virial (exact sums, identical on every rank) are
  // reported by rank 0 only, so LAMMPS's sum over ranks counts them once
  if (eflag_global && comm->me == 0) eng_vdwl += res.energy;
  if (vflag_global && comm->me == 0)
    for (int k = 0; k < 6; ++k) virial[k] += res.virial[k];
  if (!reported_ && comm->me == 0) {
    reported_ = true;
    utils::logmesg(lmp, "SO3LR_B200_FORCE_PATH=PASS atoms=" + std::to_string(atom->natoms) +
                           " energy=" + std::to_string(res.energy) + "\n");
  }
  report_profile();
}

// Opt-in timing, the counterpart of the reference's SO3_NATIVE_MPI_PROFILE
// lines (pair_so3lr_native_mpi.cpp:1259-1266, 1887-1956): with
// $SO3LR_B200_PROFILE set, every $SO3LR_B200_PROFILE_EVERY calls (default 100)
// rank 0 logs the device time of the pair-filter kernels (CUDA events on the
// library's stream) and their FP64 rate since the previous line.
void PairSO3LRB200::setup_profile() {
  if (profile_every_ >= 0) return;
  const char *on = std::getenv("SO3LR_B200_PROFILE");
  const char *every = std::getenv("SO3LR_B200_PROFILE_EVERY");
  profile_every_ = (on && on[0] != '\0' && std::strcmp(on, "0") != 0) ? (every ? std::atoi(every) : 100) : 0;
  if (profile_every_ > 0) so3lr_profile(handle_, 1);
}

void PairSO3LRB200::report_profile() {
  if (profile_every_ <= 0 || ++profile_calls_ % profile_every_ != 0) return;
  char err[512] = {0};
  double ms[2] = {0, 0}, flops[2] = {0, 0};
  long long launches[2] = {0, 0};
  for (int k = 0; k < 2; ++k)
    if (so3lr_profile_read(handle_, k, &ms[k], &launches[k], &flops[k], err, sizeof(err)) != 0)
      error->all(FLERR, std::string("SO3LR profile read failed: ") + err);
  if (comm->me != 0) return;
  char line[320];
  std::snprintf(line, sizeof(line),
                "SO3LR_B200_PROFILE calls=%lld filter_forward_ms=%.4f launches=%lld tflops=%.2f "
                "filter_reverse_ms=%.4f launches=%lld tflops=%.2f\n",
                profile_calls_, ms[0], launches[0], ms[0] > 0 ? flops[0] / (ms[0] * 1e-3) / 1e12 : 0.0, ms[1],
                launches[1], ms[1] > 0 ? flops[1] / (ms[1] * 1e-3) / 1e12 : 0.0);
  utils::logmesg(lmp, line);
}
