// LAMMPS pair style so3lr/b200/turbo on top of libso3lr_b200 (see
// pair_so3lr_b200_turbo.h). Mirrors the contract of PairSO3LRTurbo (reference
// plugins/lammps/pair_so3lr_turbo.cpp:76-319): one image per one-rank
// partition, the model loaded on universe rank 0 only (:110-153), the
// partition and boundary refusals of init_style (:182-223), and per image the
// forces, per-atom energies and image energy added to atom->f, eatom and
// eng_vdwl, with the global virial from F dot r (:286-296). The reference's
// broker (src/mpi_turbo_replica_broker.cpp:130-307) ships each image's
// neighbour graph; here each image ships only its positions and atomic numbers
// and the GPU builds the neighbour lists of the whole pack.
//
// Sharding over GPUs: with $SO3LR_B200_TURBO_GPUS = G (default 1) the K
// partitions form G groups of consecutive universe ranks (partition k belongs
// to group k G / K). Each group has its own coordinator (the group's lowest
// universe rank) with its own GPU handle on device $SO3LR_B200_DEVICE + g, and
// the gathers, the batch evaluation and the scatters of a step run inside the
// group only: the groups never communicate during a step. With G = 1 this is
// the reference's single coordinator.
#include "pair_so3lr_b200_turbo.h"

#include <mpi.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "atom.h"
#include "comm.h"
#include "domain.h"
#include "error.h"
#include "force.h"
#include "memory.h"
#include "so3lr_b200.h"
#include "so3lr_b200_precision.h"
#include "universe.h"
#include "utils.h"

using namespace LAMMPS_NS;

PairSO3LRB200Turbo::PairSO3LRB200Turbo(LAMMPS *lmp) : Pair(lmp) {
  manybody_flag = 1;
  one_coeff = 1;
  restartinfo = 0;
  single_enable = 0;
  MPI_Comm_rank(universe->uworld, &universe_rank_);
  MPI_Comm_size(universe->uworld, &universe_size_);
  const char *g = std::getenv("SO3LR_B200_TURBO_GPUS");
  groups_ = g ? std::atoi(g) : 1;
  if (groups_ < 1) groups_ = 1;
  if (groups_ > universe_size_) groups_ = universe_size_;
  group_ = static_cast<int>((static_cast<long long>(universe_rank_) * groups_) / universe_size_);
  MPI_Comm_split(universe->uworld, group_, universe_rank_, &group_comm_);
  MPI_Comm_rank(group_comm_, &group_rank_);
  MPI_Comm_size(group_comm_, &group_size_);
}

PairSO3LRB200Turbo::~PairSO3LRB200Turbo() {
  release();
  MPI_Comm_free(&group_comm_);
  if (allocated) {
    memory->destroy(setflag);
    memory->destroy(cutsq);
  }
}

void PairSO3LRB200Turbo::release() {
  if (handle_) so3lr_destroy(handle_);
  handle_ = nullptr;
  model_ready_ = false;
}

void PairSO3LRB200Turbo::allocate() {
  allocated = 1;
  const int n = atom->ntypes;
  memory->create(setflag, n + 1, n + 1, "so3lr/b200/turbo:setflag");
  memory->create(cutsq, n + 1, n + 1, "so3lr/b200/turbo:cutsq");
  for (int i = 1; i <= n; ++i)
    for (int j = i; j <= n; ++j) setflag[i][j] = 0;
}

void PairSO3LRB200Turbo::settings(int narg, char **arg) {
  if (narg < 1 || narg > 3)
    error->universe_all(FLERR, "Illegal pair_style so3lr/b200/turbo command: expected "
                               "'pair_style so3lr/b200/turbo MODEL [charge [multiplicity]]'");
  model_path_ = arg[0];
  // per image: every partition reads its own values (e.g. world variables)
  total_charge_ = narg > 1 ? std::strtod(arg[1], nullptr) : 0.0;
  multiplicity_ = narg > 2 ? std::strtod(arg[2], nullptr) : 1.0;
  release();
  // every group's coordinator loads the model onto its GPU
  // ($SO3LR_B200_DEVICE + group, default 0 + group) and tells its group's images
  // the outcome; all groups then agree, so a failure anywhere stops every image
  char msg[1024] = {0};
  int ok = 1;
  double cut[2] = {0.0, 0.0};
  if (group_rank_ == 0) {
    char err[960] = {0};
    so3lr_arch_info info{};
    if (so3lr_inspect_model(model_path_.c_str(), &info, err, sizeof(err)) != 0) {
      ok = 0;
      std::snprintf(msg, sizeof(msg), ": %s", err);
    } else {
      cut[0] = info.sr_cutoff;
      cut[1] = info.lr_cutoff;
      const char *dev = std::getenv("SO3LR_B200_DEVICE");
      if (so3lr_create(model_path_.c_str(), (dev ? std::atoi(dev) : 0) + group_, &handle_, err, sizeof(err)) != 0) {
        ok = 0;
        std::snprintf(msg, sizeof(msg), " on the GPU: %s", err);
      } else if (so3lr_b200_precision_from_env(handle_, err, sizeof(err)) != 0) {
        ok = 0;
        std::snprintf(msg, sizeof(msg), ": %s", err);
      }
    }
  }
  MPI_Bcast(&ok, 1, MPI_INT, 0, group_comm_);
  MPI_Bcast(msg, sizeof(msg), MPI_BYTE, 0, group_comm_);
  int all_ok = 0;
  MPI_Allreduce(&ok, &all_ok, 1, MPI_INT, MPI_MIN, universe->uworld);
  if (!all_ok)
    error->universe_all(FLERR, ok ? std::string("Cannot initialize the SO3LR model of another group's coordinator")
                                  : std::string("Cannot initialize the coordinator SO3LR model") + msg);
  MPI_Bcast(cut, 2, MPI_DOUBLE, 0, universe->uworld);
  sr_cutoff_ = cut[0];
  lr_cutoff_ = cut[1];
  model_ready_ = true;
}

void PairSO3LRB200Turbo::coeff(int narg, char **arg) {
  if (!allocated) allocate();
  if (narg != atom->ntypes + 2 || std::strcmp(arg[0], "*") != 0 || std::strcmp(arg[1], "*") != 0)
    error->all(FLERR, "Pair coeff for so3lr/b200/turbo must be '* * E1 ... Entypes' where each E is an element "
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

double PairSO3LRB200Turbo::init_one(int i, int j) {
  if (!setflag[i][j]) error->all(FLERR, "All so3lr/b200/turbo coefficients are not set");
  return lr_cutoff_;
}

void PairSO3LRB200Turbo::init_style() {
  // every partition checks its own setup, then all agree, so that one
  // misconfigured image stops the whole universe instead of leaving the other
  // images waiting in the first gather
  std::string problem;
  if (comm->nprocs != 1) {
    problem = "so3lr/b200/turbo requires one MPI rank per LAMMPS partition";
  } else if (universe->nworlds != universe_size_ || universe_size_ < 2) {
    problem = "so3lr/b200/turbo requires multiple one-rank partitions";
  } else if (domain->xperiodic || domain->yperiodic || domain->zperiodic) {
    problem = "so3lr/b200/turbo requires non-periodic boundaries";
  } else if (!force->newton_pair) {
    problem = "Pair style so3lr/b200/turbo requires newton pair on";
  } else if (!model_ready_) {
    problem = "SO3LR turbo coordinator was not initialized";
  } else if (type_to_z_.size() != static_cast<std::size_t>(atom->ntypes) + 1) {
    problem = "Pair style so3lr/b200/turbo coefficients are missing";
  } else {
    // this image's charge and multiplicity against its composition
    // (pair_so3lr_turbo.cpp:207-219)
    long long counts[119] = {0};
    for (int i = 0; i < atom->nlocal; ++i) counts[type_to_z_[static_cast<std::size_t>(atom->type[i])]]++;
    char err[512] = {0};
    if (so3lr_validate_charge_spin(counts, total_charge_, multiplicity_, err, sizeof(err)) != 0) {
      char head[160];
      std::snprintf(head, sizeof(head), "Pair style so3lr/b200/turbo image %d: charge %g with multiplicity %g: ",
                    universe->iworld, total_charge_, multiplicity_);
      problem = std::string(head) + err;
    }
  }
  int bad = problem.empty() ? 0 : 1, any = 0;
  MPI_Allreduce(&bad, &any, 1, MPI_INT, MPI_MAX, universe->uworld);
  if (bad) error->universe_one(FLERR, problem);
  if (any) error->universe_all(FLERR, "so3lr/b200/turbo: another partition refused its setup");
  char line[160];
  std::snprintf(line, sizeof(line), "SO3LR turbo image %d: total charge %g, spin multiplicity %g\n",
                universe->iworld, total_charge_, multiplicity_);
  utils::logmesg(lmp, line);
}

// A failed step, known to every image of the failing group. With one group
// that is the whole universe (error->universe_all, as the reference); with
// several the other groups do not share the step, so the failing group stops
// the universe itself (error->universe_one) instead of waiting for them.
void PairSO3LRB200Turbo::fail_step(const std::string &msg) {
  if (groups_ > 1) error->universe_one(FLERR, msg);
  error->universe_all(FLERR, msg);
}

void PairSO3LRB200Turbo::compute(int eflag, int vflag) {
  ev_init(eflag, vflag);
  const double t0 = MPI_Wtime();
  // every exchange of the step stays inside this image's group
  const MPI_Comm gcomm = group_comm_;
  const bool coordinator = group_rank_ == 0;
  const int nimg = group_size_;
  const int n = atom->nlocal;

  // this image: atom count, whether it wants per-atom virials, charge and
  // multiplicity, then positions and atomic numbers
  int head[2] = {n, vflag_atom};
  double headd[2] = {total_charge_, multiplicity_};
  if (coordinator) {
    head_i_.resize(2 * static_cast<std::size_t>(nimg));
    head_d_.resize(2 * static_cast<std::size_t>(nimg));
  }
  MPI_Gather(head, 2, MPI_INT, head_i_.data(), 2, MPI_INT, 0, gcomm);
  MPI_Gather(headd, 2, MPI_DOUBLE, head_d_.data(), 2, MPI_DOUBLE, 0, gcomm);
  x_.resize(3 * static_cast<std::size_t>(n));
  z_.resize(n);
  for (int i = 0; i < n; ++i) {
    for (int d = 0; d < 3; ++d) x_[3 * static_cast<std::size_t>(i) + d] = atom->x[i][d];
    z_[i] = type_to_z_[static_cast<std::size_t>(atom->type[i])];
  }
  long long total = 0;
  int any_va = 0;
  if (coordinator) {
    counts_.resize(nimg);
    displs_.resize(nimg);
    counts3_.resize(nimg);
    displs3_.resize(nimg);
    counts6_.resize(nimg);
    displs6_.resize(nimg);
    offsets_.resize(static_cast<std::size_t>(nimg) + 1);
    image_q_.resize(nimg);
    image_m_.resize(nimg);
    for (int k = 0; k < nimg; ++k) {
      const int c = head_i_[2 * k];
      offsets_[k] = total;
      // element offsets fit an int: the pack is limited to 2^26 atoms below
      const long long base = total < (1LL << 26) ? total : 0;
      counts_[k] = c;
      displs_[k] = static_cast<int>(base);
      counts3_[k] = 3 * c;
      displs3_[k] = static_cast<int>(3 * base);
      counts6_[k] = 6 * c;
      displs6_[k] = static_cast<int>(6 * base);
      any_va |= head_i_[2 * k + 1];
      image_q_[k] = head_d_[2 * k];
      image_m_[k] = head_d_[2 * k + 1];
      total += c;
    }
    offsets_[nimg] = total;
    const std::size_t cap = total < (1LL << 26) ? static_cast<std::size_t>(total) : 0;
    all_x_.resize(3 * cap);
    all_z_.resize(cap);
  }
  int status[2] = {0, 0};  // library status, per-atom virials wanted by some image
  char err[1024] = {0};
  if (coordinator && total >= (1LL << 26)) {
    status[0] = 1;
    std::snprintf(err, sizeof(err), "the pack of all images holds %lld atoms; at most %lld are supported", total,
                  (1LL << 26) - 1);
  }
  MPI_Bcast(status, 2, MPI_INT, 0, gcomm);
  if (status[0] != 0) {
    MPI_Bcast(err, sizeof(err), MPI_BYTE, 0, gcomm);
    fail_step(std::string("SO3LR turbo LAMMPS evaluation failed: ") + err);
  }
  MPI_Gatherv(x_.data(), 3 * n, MPI_DOUBLE, all_x_.data(), counts3_.data(), displs3_.data(), MPI_DOUBLE, 0, gcomm);
  MPI_Gatherv(z_.data(), n, MPI_INT, all_z_.data(), counts_.data(), displs_.data(), MPI_INT, 0, gcomm);

  if (coordinator) {
    const std::size_t nt = static_cast<std::size_t>(total);
    all_f_.resize(3 * nt);
    all_eatom_.resize(nt);
    image_e_.resize(nimg);
    so3lr_batch batch{};
    batch.natoms = total;
    batch.nimages = nimg;
    batch.x = all_x_.data();
    batch.z = all_z_.data();
    batch.image_offsets = offsets_.data();
    batch.image_charge = image_q_.data();
    batch.image_multiplicity = image_m_.data();
    so3lr_batch_result res{};
    res.f = all_f_.data();
    res.eatom = all_eatom_.data();
    res.image_energy = image_e_.data();
    status[0] = so3lr_compute_batch(handle_, &batch, &res, err, sizeof(err));
    if (status[0] == 0 && any_va) {
      all_va_.resize(6 * nt);
      status[0] = so3lr_virial_atom(handle_, all_va_.data(), err, sizeof(err));
    }
    status[1] = any_va;
  }
  MPI_Bcast(status, 2, MPI_INT, 0, gcomm);
  if (status[0] != 0) {
    MPI_Bcast(err, sizeof(err), MPI_BYTE, 0, gcomm);
    fail_step(std::string("SO3LR turbo LAMMPS evaluation failed: ") + err);
  }
  f_.resize(3 * static_cast<std::size_t>(n));
  eatom_.resize(n);
  double image_energy = 0.0;
  MPI_Scatterv(all_f_.data(), counts3_.data(), displs3_.data(), MPI_DOUBLE, f_.data(), 3 * n, MPI_DOUBLE, 0, gcomm);
  MPI_Scatterv(all_eatom_.data(), counts_.data(), displs_.data(), MPI_DOUBLE, eatom_.data(), n, MPI_DOUBLE, 0,
               gcomm);
  MPI_Scatter(image_e_.data(), 1, MPI_DOUBLE, &image_energy, 1, MPI_DOUBLE, 0, gcomm);
  if (status[1]) {
    va_.resize(6 * static_cast<std::size_t>(n));
    MPI_Scatterv(all_va_.data(), counts6_.data(), displs6_.data(), MPI_DOUBLE, va_.data(), 6 * n, MPI_DOUBLE, 0,
                 gcomm);
  }

  for (int i = 0; i < n; ++i)
    for (int d = 0; d < 3; ++d) atom->f[i][d] += f_[3 * static_cast<std::size_t>(i) + d];
  if (eflag_atom)
    for (int i = 0; i < n; ++i) eatom[i] += eatom_[i];
  if (eflag_global) eng_vdwl += image_energy;
  if (vflag_atom)
    for (int i = 0; i < n; ++i)
      for (int c = 0; c < 6; ++c) vatom[i][c] += va_[6 * static_cast<std::size_t>(i) + c];
  // an isolated image has no ghost atoms: F dot r over its own atoms is its
  // virial (pair_so3lr_turbo.cpp:296)
  if (vflag_fdotr) virial_fdotr_compute();
  ++evaluations_;

  if (!reported_) {
    reported_ = true;
    char line[256];
    std::snprintf(line, sizeof(line),
                  "SO3LR_TURBO_LIVE image=%d universe_rank=%d coordinator=%d images=%d atoms=%d "
                  "energy=%.10g broker_ms=%.6g gpu_group=%d of %d\n",
                  universe->iworld, universe_rank_, coordinator ? 1 : 0, nimg, n, image_energy,
                  (MPI_Wtime() - t0) * 1000.0, group_, groups_);
    utils::logmesg(lmp, line);
  }
}
