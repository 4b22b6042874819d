// LAMMPS pair style `so3lr/b200`: the SO3LR force evaluation of
// `so3lr/native/mpi` (plugins/lammps/pair_so3lr_native_mpi.h in the reference)
// driven through the C ABI of libso3lr_b200 (include/so3lr_b200.h).
//
//   pair_style so3lr/b200 MODEL [charge [multiplicity]]
//   pair_coeff * * E1 ... Entypes        (element symbols H..Es or numbers 1..99)
//
// Same syntax, defaults and refusals as the reference style, except that
// per-atom virials (compute ... stress/atom, vflag_atom) are supported; the
// reference refuses them (pair_so3lr_native_mpi.cpp:1248-1251). The GPU builds
// its own short- and long-range neighbour lists from the positions, so the
// style requests no LAMMPS list and needs no ghost atoms beyond LAMMPS's own
// bookkeeping (periodic orthorhombic or fully open boundaries). On several MPI
// ranks (one GPU each: $SO3LR_B200_DEVICE, else the rank number) every rank
// gathers the atoms of all ranks by tag and the library evaluates them with its
// own spatial decomposition over the ranks' GPUs; each rank keeps its atoms'
// forces, and rank 0 reports the global energy and virial.
#ifdef PAIR_CLASS
// clang-format off
PairStyle(so3lr/b200,PairSO3LRB200);
// clang-format on
#else

#ifndef LMP_PAIR_SO3LR_B200_H
#define LMP_PAIR_SO3LR_B200_H

#include <string>
#include <vector>

#include "pair.h"
#include "so3lr_b200.h"

namespace LAMMPS_NS {

class PairSO3LRB200 : public Pair {
 public:
  explicit PairSO3LRB200(class LAMMPS *);
  ~PairSO3LRB200() override;

  void compute(int, int) override;
  void settings(int, char **) override;
  void coeff(int, char **) override;
  void init_style() override;
  double init_one(int, int) override;

  // atomic number of a LAMMPS type (after coeff); for tests
  int type_atomic_number(int type) const { return type_to_z_.at(static_cast<std::size_t>(type)); }
  double short_range_cutoff() const { return sr_cutoff_; }
  double long_range_cutoff() const { return lr_cutoff_; }

 private:
  std::string model_path_;
  double total_charge_ = 0.0;
  double multiplicity_ = 1.0;
  double sr_cutoff_ = 0.0;
  double lr_cutoff_ = 0.0;
  std::vector<int> type_to_z_;
  std::vector<int> z_;
  std::vector<double> x_, f_, eatom_, va_, loc_x_, all_x_, terms_;
  std::vector<int> loc_tag_, loc_z_, all_tag_, all_z_, counts_, displs_, counts3_, displs3_;
  std::vector<long long> loc_tag64_;
  std::vector<char> seen_;
  bool comm_ready_ = false;
  so3lr_handle *handle_ = nullptr;
  bool reported_ = false;

  void allocate();
  void release();
  void write_debug_dump(const char *path, const so3lr_result &res, int n);
  void compute_with_dump(const char *dump_path);
  [[noreturn]] void fail_collective(const std::string &msg);
  void setup_profile();
  void report_profile();
  int profile_every_ = -1;  // -1: not read yet, 0: off
  long long profile_calls_ = 0;
};

}  // namespace LAMMPS_NS

#endif
#endif
