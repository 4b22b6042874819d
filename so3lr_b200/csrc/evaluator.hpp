// SO3LR force evaluation on one GPU: owns the device copy of the model and the
// per-system workspace, and runs neighbour build -> geometry -> interaction
// blocks -> heads -> charge conservation -> long range -> reverse pass ->
// forces, energies and virial. Stream-ordered; nothing here calls MPI or NCCL.
//
// Mirrors the per-step sequence of PairSO3LRNativeMPI::compute
// (plugins/lammps/pair_so3lr_native_mpi.cpp:1595-1788) and of the packed turbo
// evaluator (src/kokkos_packed_so3lr_evaluator.cpp:43-149).
#pragma once

#include <array>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "nccl_dyn.hpp"

#include "api.hpp"
#include "kernels.cuh"
#include "model_host.hpp"

SO3LR_SHAPE_BEGIN

class Evaluator final : public EvaluatorApi {
 public:
  Evaluator(Model &&model, int device);
  ~Evaluator() override;
  const Model &model() const override { return model_; }
  cudaStream_t stream() const override { return stream_; }
  int device() const override { return device_; }
  void prepare(const SystemSpec &spec, const double *host_x = nullptr) override;
  void set_comm(int nranks, int rank, const void *unique_id) override;
  int nranks() const override { return nranks_; }
  bool has_result() const override { return computed_; }
  int owned_atoms() const override { return n_own_; }
  const SystemSpec &spec() const override { return spec_; }
  double *positions() override { return x_.get(); }
  void upload_positions(const double *host_x) override;
  void compute() override;
  HostResult download(double *f, double *eatom, double *charges, double *ratios, double *e_learned, double *e_zbl,
                      double *e_lr, double *e_elec, double *e_disp, double *image_energy) override;
  void download_virial_atom(double *vatom) override;
  HostResult compute_local(const SystemSpec &frame, int nlocal, const long long *tag, const double *x, const int *z,
                           double *f, double *eatom, double *vatom) override;
  const double *forces() const override { return force_.get(); }
  const double *energy_device() const override { return totals_.get(); }
  StepStats stats() const override { return stats_; }
  LongRangeTables long_range_tables() const override { return {lr_, alpha_ref_, c6_ref_, ref_table_, lr_cut_}; }
  bool has_c6_head() const override { return heads_.c6_w2 != nullptr; }
  std::size_t device_bytes() const override;
  void set_profiling(bool on) override { profiling_ = on; }
  void set_mixed_precision(bool on) override;
  bool mixed_precision() const override { return mixed_; }
  void read_profile(int kernel, double *ms, long long *launches, double *flops) override;
  void md_setup(const double *host_v, const double *host_mass) override;
  void md_thermostat(double t_target_k, double t_damp_ps, int chain) override;
  double md_thermostat_energy() override;
  void md_steps(int nsteps, double dt_ps) override;
  void md_download(double *x, double *v) override;

 private:
  Model model_;
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  SystemSpec spec_;
  StepStats stats_;

  // weights
  DeviceArray<double> wbuf_;
  DeviceArray<float> wbuf32_;  // TF32-split filter operands (mixed precision)
  std::vector<TcFwdConsts> tc_fwd_consts_;  // per block, kernel parameters of the tcgen05 filters
  std::vector<TcRevConsts> tc_rev_consts_;
  std::vector<BlockW> blocks_;
  HeadsW heads_{};
  RadialW rad_{};
  ZblDev zbl_{};
  LrDev lr_{};
  const double *emb_w_ = nullptr, *alpha_ref_ = nullptr, *c6_ref_ = nullptr;
  int ref_table_ = 0;
  double inv_emb_scale_ = 1.0, norm_ = 1.0, sr_cut_ = 0, lr_cut_ = 0;
  int layers_ = 0;
  // optional block operators of the model (norm kinds kNormLayer / kNormRms /
  // kNormNone, query/key normalisation, residual scalars per block)
  int norm1_ = 0, norm2_ = 0;
  bool qk_norm_ = false, residual_scalars_ = false;
  std::vector<double> resid_, x0s_;
  static constexpr std::size_t kNoParam = ~std::size_t(0);
  static constexpr int kOpenCellsMinAtoms = 512;
  bool open_cells_possible(const SystemSpec &spec, const double *host_x) const;

  // static per-system data
  DeviceArray<int> z_, image_of_, image_start_, table_of_atom_;
  DeviceArray<double> cs_tables_, image_charge_;
  bool any_charge_spin_ = false;

  // neighbour state
  NeighborState nb_{};
  DeviceArray<double> xw_;
  DeviceArray<int> cell_, cell_count_, cell_start_, cell_fill_, cell_atoms_;
  DeviceArray<int> deg_, row_start_, nbr_, img_, primary_, rev_, pair_scan_, edge_pair_;
  DeviceArray<int> pair_a_, pair_b_, pair_img_, pair_edge_, scan_scratch_, small_ints_;
  int *host_small_ = nullptr;  // pinned
  double *host_totals_ = nullptr;

  // per-pair arrays
  DeviceArray<double> geo_, sh_, gv_, gl0_, pair_sc_, g_filt_inv_, g_filt_ev_, drbf_, g_r_, g_y_;
  std::vector<std::unique_ptr<DeviceArray<double>>> f_inv_, f_ev_, sp_;

  // per-atom arrays
  DeviceArray<double> x_, v_, inv_mass_, force_;
  DeviceArray<double> mass_, ke2_, nhc_scalars_, nhc_state_;
  bool md_ready_ = false, nvt_ = false;
  void nhc_half(double dt);
  std::vector<std::unique_ptr<DeviceArray<double>>> xb_, evb_, qkv_, xhat1_, rstd1_, n1_, A_, hp_, gate_, xhat2_, rstd2_;
  std::vector<std::unique_ptr<DeviceArray<double>>> qkr_;  // inverse RMS of q, k, q_ev, k_ev [row][head][4]
  // float32 copies of the rows the attention gathers, mixed precision with
  // the tcgen05 filters: qkv per block, and the block adjoints g_a, g_A
  std::vector<std::unique_ptr<DeviceArray<float>>> qkv32_;
  DeviceArray<float> ga32_, gA32_;
  DeviceArray<double> x0_;                                  // embedding, kept with residual scalars
  DeviceArray<double> d_inv_, d_ev_, act_, cat_, t_, hpre_, hcat_, hk_, e_nn_, raw_q_, q_, ratio_;
  DeviceArray<double> hk6_, ratio6_, dc6_;  // C6 ratio head (models that have one)
  DeviceArray<double> e_lr_, e_elec_, e_disp_, dq_, dh_, f_lr_, w_lr_, img_sums_, dq_mean_, lr_pos4_, lr_par4_;
  DeviceArray<double> g_hcat_, g_x_, g_x2_, g_ev_, g_ev2_, g_t_, g_cat_, g_hp_, g_n1_, g_a_, g_A_, g_qkv_;
  DeviceArray<double> e_atom_, e_zbl_, w_atom_, totals_, image_energy_;

  // decomposition
  int nranks_ = 1, rank_ = 0;
  ncclComm_t comm_ = nullptr;
  int n_rows_ = 0, stride_ = 0, row0_ = 0, n_own_ = 0;
  bool identity_ = true;
  std::vector<int> row_of_, tag_of_row_;
  // rank-local frames: row of every tag, the gathered records, flags
  DeviceArray<int> row_of_tag_, local_seen_;
  DeviceArray<long long> local_counts_;
  DeviceArray<double> rec_send_, rec_all_, local_out_;
  double *host_rec_ = nullptr;  // pinned
  std::size_t host_rec_cap_ = 0;
  bool local_ready_ = false;
  std::vector<double> stage_;
  bool computed_ = false;
  int host_seg_[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  DeviceArray<int> tag_, seg_, pair_canon_;
  // halo lists of the current neighbour lists (multi-GPU only)
  DeviceArray<int> halo_flags_, halo_pos_, halo_send_rows_, halo_recv_rows_, halo_totals_;
  DeviceArray<long long> halo_offsets_, halo_all_offsets_;
  DeviceArray<double> halo_send_buf_, halo_recv_buf_;
  long long *host_halo_ = nullptr;  // pinned: all ranks' offsets
  std::vector<long long> halo_send_off_, halo_recv_off_;
  DeviceArray<long long> parts_;
  void allgather_rows(double *a, int width, int prof = -1);
  // refresh the halo rows (other GPUs' atoms that neighbour this GPU's atoms)
  // of two row arrays at once; the identity layout (one GPU) does nothing
  void halo_exchange(double *a, int wa, double *b, int wb, int prof);
  void exact_sums(const double *v, int stride, int ncol, int nseg, const int *seg, double *out);

  struct KernelProfile {
    std::vector<cudaEvent_t> events;
    int used = 0;
    long long launches = 0;
    double flops = 0;
  };
  bool profiling_ = false;
  bool mixed_ = false;
  bool mixed_tc_ = true;           // mixed filters on tcgen05 (filter_tc.cu), else mma.sync
  int num_sms_ = 148;
  DeviceArray<int> tc_err_arr_;    // error word of the tcgen05 kernel
  int *tc_err_ = nullptr;
  void check_device_flags() const;
  KernelProfile prof_[kProfKinds];
  void prof_begin(int k);
  void prof_end(int k, double flops);

  void upload_weights();
  void alloc_atoms();
  void build_neighbors();
};

SO3LR_SHAPE_END
