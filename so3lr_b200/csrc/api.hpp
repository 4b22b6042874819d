// Width-independent view of the SO3LR evaluator: what the C ABI, the local
// frame path and the no-alloc entry point need, with one implementation per
// compiled model width (evaluator.hpp, namespaces so3lr_b200::f128 / f256).
// make_evaluator() loads the model file and picks the implementation that
// matches its invariant width.
#pragma once

#include <array>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "model_host.hpp"

namespace so3lr_b200 {

template <class T>
class DeviceArray {
 public:
  DeviceArray() = default;
  DeviceArray(const DeviceArray &) = delete;
  DeviceArray &operator=(const DeviceArray &) = delete;
  ~DeviceArray() { release(); }
  void release() {
    if (ptr_) cudaFree(ptr_);
    ptr_ = nullptr;
    cap_ = 0;
  }
  // grow-only; contents are not preserved
  T *reserve(std::size_t n, double slack = 1.0) {
    if (n > cap_) {
      release();
      const std::size_t want = std::max<std::size_t>(1, std::size_t(double(n) * slack));
      SO3_CUDA(cudaMalloc(&ptr_, want * sizeof(T)));
      cap_ = want;
    }
    return ptr_;
  }
  T *get() const { return ptr_; }
  std::size_t capacity() const { return cap_; }
  std::size_t bytes() const { return cap_ * sizeof(T); }

 private:
  T *ptr_ = nullptr;
  std::size_t cap_ = 0;
};

// What the caller asks to be evaluated. Atoms of one image are contiguous.
struct SystemSpec {
  int n = 0;
  bool periodic = false;
  double lo[3] = {0, 0, 0};
  double len[3] = {0, 0, 0};
  std::vector<int> z;                 // atomic numbers, 1..99
  std::vector<int> image_start;       // n_images + 1 (one image when not batched)
  std::vector<double> image_charge;   // n_images
  std::vector<double> image_mult;     // n_images
};

struct StepStats {
  long long edges = 0, pairs = 0;
};

// owner rank of every atom: spatial bricks of the periodic box (host-only, the
// same arithmetic on every rank)
std::vector<int> partition_atoms(const SystemSpec &s, const double *x, int nranks);
void brick_dims(int nranks, int dims[3]);

class EvaluatorApi {
 public:
  virtual ~EvaluatorApi() = default;
  virtual const Model &model() const = 0;
  virtual cudaStream_t stream() const = 0;
  virtual int device() const = 0;

  // Validates Z, charges and multiplicities (so3lr_charge_spin.cpp:116-141),
  // builds the charge/spin offset tables, uploads static per-atom data.
  // host_x (N x 3, input order) is needed only to partition atoms over GPUs.
  virtual void prepare(const SystemSpec &spec, const double *host_x = nullptr) = 0;
  // Join a group of nranks GPUs (one evaluator per GPU, same model, same
  // system); unique_id is an ncclUniqueId made by rank 0 and shared by the
  // caller. Atoms are partitioned into spatial bricks of the periodic box.
  virtual void set_comm(int nranks, int rank, const void *unique_id) = 0;
  virtual int nranks() const = 0;
  // true once compute() has run for the current system
  virtual bool has_result() const = 0;
  virtual int owned_atoms() const = 0;
  virtual const SystemSpec &spec() const = 0;

  // Device positions buffer for the prepared system (N x 3). Callers may write
  // it directly (device-resident MD) or through upload_positions().
  virtual double *positions() = 0;
  virtual void upload_positions(const double *host_x) = 0;
  // Run the whole evaluation on stream(); outputs stay on the device.
  virtual void compute() = 0;
  // Copy results to host (after compute(); synchronises the stream).
  struct HostResult {
    double energy = 0;
    std::array<double, 6> virial{};
  };
  virtual HostResult download(double *f, double *eatom, double *charges, double *ratios, double *e_learned,
                              double *e_zbl, double *e_lr, double *e_elec, double *e_disp, double *image_energy) = 0;
  // per-atom virial (natoms x 6, xx yy zz xy xz yz) of the last compute(), input
  // atom order; collective when decomposed (synchronises the stream)
  virtual void download_virial_atom(double *vatom) = 0;
  // Rank-local frame (local_frame.cu): this rank passes its own nlocal atoms
  // (global tags 1..frame.n, positions, atomic numbers; frame.z unused) and gets
  // the forces (nlocal x 3), and optionally per-atom energies and virials, of
  // those atoms back. Collective on a multi-GPU handle.
  virtual HostResult compute_local(const SystemSpec &frame, int nlocal, const long long *tag, const double *x,
                                   const int *z, double *f, double *eatom, double *vatom) = 0;
  virtual const double *forces() const = 0;
  virtual const double *energy_device() const = 0;  // [0] energy, [1..6] virial
  virtual StepStats stats() const = 0;
  // long-range constants and reference tables (device) of the loaded model
  struct LongRangeTables {
    LrDev params;
    const double *alpha_ref, *c6_ref;
    int table_size;
    double cutoff;
  };
  virtual LongRangeTables long_range_tables() const = 0;
  virtual bool has_c6_head() const = 0;
  virtual std::size_t device_bytes() const = 0;

  // Optional CUDA-event timing on stream() of the pair-filter kernels and of the
  // multi-GPU exchange phases (ProfileKind). read_profile() synchronises,
  // returns the summed device time, launch count and algorithmic FLOPs, and resets.
  enum ProfileKind {
    kProfFilterForward = 0,
    kProfFilterReverse = 1,
    kProfPositionGather = 2,   // all-gather of positions after the drift
    kProfHaloLists = 3,        // halo-list rebuild: lists, count all-gather, host check
    kProfFeatureHalo = 4,      // block-feature halo exchanges (forward)
    kProfAdjointHalo = 5,      // block-adjoint halo exchanges (reverse)
    kProfLrGather = 6,         // all-gathers of charges and ratios before the long range
    kProfExactSums = 7,        // exact global sums (integer all-gathers)
    kProfKinds = 8
  };
  virtual void set_profiling(bool on) = 0;
  // Arithmetic of the pair-filter MLPs: float64 (default) or mixed (three-pass
  // TF32 tensor-core GEMMs with float32 accumulation), every other step
  // float64. Takes effect from the next evaluation. The mixed kernels exist for
  // the F = 128 shape; an F = 256 model refuses mixed precision.
  virtual void set_mixed_precision(bool on) = 0;
  virtual bool mixed_precision() const = 0;
  virtual void read_profile(int kernel, double *ms, long long *launches, double *flops) = 0;

  // velocity-Verlet MD on the device (LAMMPS metal units); masses in g/mol
  virtual void md_setup(const double *host_v, const double *host_mass) = 0;
  // Nose-Hoover chain (thermostat.cu) for the following md_steps; t_damp_ps <= 0
  // switches back to NVE
  virtual void md_thermostat(double t_target_k, double t_damp_ps, int chain) = 0;
  // the chain's energy: sum_j Q_j v_j^2 / 2 + N_f kT eta_1 + kT sum_{j>1} eta_j (eV)
  virtual double md_thermostat_energy() = 0;
  virtual void md_steps(int nsteps, double dt_ps) = 0;
  virtual void md_download(double *x, double *v) = 0;
};

// Loads the model file and returns the evaluator of its width on `device`.
std::unique_ptr<EvaluatorApi> make_evaluator(const std::string &model_path, int device);

// the evaluators of the two compiled widths (evaluator.cu built per width)
std::unique_ptr<EvaluatorApi> create_evaluator_f128(Model &&model, int device);
std::unique_ptr<EvaluatorApi> create_evaluator_f256(Model &&model, int device);

}  // namespace so3lr_b200
