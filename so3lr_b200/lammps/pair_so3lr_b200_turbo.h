// LAMMPS pair style `so3lr/b200/turbo`: the packed evaluation of many
// independent open-boundary systems of `so3lr/turbo`
// (plugins/lammps/pair_so3lr_turbo.h in the reference) driven through the C ABI
// of libso3lr_b200 (include/so3lr_b200.h).
//
//   mpirun -np K lmp -partition Kx1 -in in.images
//   pair_style so3lr/b200/turbo MODEL [charge [multiplicity]]
//   pair_coeff * * E1 ... Entypes        (element symbols H..Es or numbers 1..99)
//
// Every one-rank LAMMPS partition holds one image (a molecule or cluster with
// its own charge and multiplicity, read per partition, e.g. from world
// variables). Each compute gathers the images' atoms to their coordinator,
// which owns a GPU and evaluates all its images in one so3lr_compute_batch
// call, then scatters every image's forces, per-atom energies and energy back.
// By default one coordinator (universe rank 0) serves every partition, as in
// the reference; with $SO3LR_B200_TURBO_GPUS = G the partitions form G groups of
// consecutive universe ranks, each with its own coordinator and GPU
// ($SO3LR_B200_DEVICE + group), and the groups never communicate during a step. Same syntax, defaults and
// refusals as the reference style, except that per-atom virials are supported
// (the reference refuses vflag_atom, pair_so3lr_turbo.cpp:238-240).
#ifdef PAIR_CLASS
// clang-format off
PairStyle(so3lr/b200/turbo,PairSO3LRB200Turbo);
// clang-format on
#else

#ifndef LMP_PAIR_SO3LR_B200_TURBO_H
#define LMP_PAIR_SO3LR_B200_TURBO_H

#include <string>
#include <vector>

#include <mpi.h>

#include "pair.h"

struct so3lr_handle;

namespace LAMMPS_NS {

class PairSO3LRB200Turbo : public Pair {
 public:
  explicit PairSO3LRB200Turbo(class LAMMPS *);
  ~PairSO3LRB200Turbo() override;

  void compute(int, int) override;
  void settings(int, char **) override;
  void coeff(int, char **) override;
  void init_style() override;
  double init_one(int, int) override;

  // for tests
  int type_atomic_number(int type) const { return type_to_z_.at(static_cast<std::size_t>(type)); }
  double short_range_cutoff() const { return sr_cutoff_; }
  double long_range_cutoff() const { return lr_cutoff_; }
  long long evaluations() const { return evaluations_; }

 private:
  std::string model_path_;
  double total_charge_ = 0.0;
  double multiplicity_ = 1.0;
  double sr_cutoff_ = 0.0;
  double lr_cutoff_ = 0.0;
  int universe_rank_ = 0, universe_size_ = 1;
  // GPU groups ($SO3LR_B200_TURBO_GPUS): this partition's group, its rank in
  // the group's communicator (0 = the group's coordinator) and the group size
  int groups_ = 1, group_ = 0, group_rank_ = 0, group_size_ = 1;
  MPI_Comm group_comm_;
  bool model_ready_ = false;
  std::vector<int> type_to_z_;
  // this image
  std::vector<double> x_, f_, eatom_, va_;
  std::vector<int> z_;
  // coordinator: the pack of all images
  so3lr_handle *handle_ = nullptr;
  std::vector<double> all_x_, all_f_, all_eatom_, all_va_, image_q_, image_m_, image_e_, head_d_;
  std::vector<int> all_z_, head_i_, counts_, displs_, counts3_, displs3_, counts6_, displs6_;
  std::vector<long long> offsets_;
  long long evaluations_ = 0;
  bool reported_ = false;

  void allocate();
  void release();
  [[noreturn]] void fail_step(const std::string &msg);
};

}  // namespace LAMMPS_NS

#endif
#endif
