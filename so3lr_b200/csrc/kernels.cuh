// Kernel launchers and device-state structures shared by the evaluator.
#pragma once

#include <algorithm>
#include <cmath>

#include "cell_grid.hpp"
#include "common.cuh"

namespace so3lr_b200 {


struct NeighborState {
  CellGrid grid;
  int ncells = 0;
  double *xw = nullptr;  // wrapped positions (N x 3)
  int *cell = nullptr, *cell_count = nullptr, *cell_start = nullptr, *cell_fill = nullptr, *cell_atoms = nullptr;
  int *image_of = nullptr, *image_start = nullptr;  // open boundaries: atom -> image, image CSR
  int *deg = nullptr, *row_start = nullptr, *nbr = nullptr, *img = nullptr, *primary = nullptr, *rev = nullptr;
  int *pair_scan = nullptr, *edge_pair = nullptr;
  int *pair_a = nullptr, *pair_b = nullptr, *pair_img = nullptr, *pair_edge = nullptr;
  int *scan_total = nullptr, *scan_scratch = nullptr, *error_flag = nullptr;
  int *pair_canon = nullptr;  // pair stored in its canonical orientation (smaller tag receives)
  const int *tag = nullptr;   // global tag of every row (-1: padding row); nullptr: tag = row
  int row0 = 0, n_own = 0;    // rows [row0, row0 + n_own) are owned here and get CSR rows
};

void exclusive_scan(const int *in, int *out, int n, int *total, int *scratch, cudaStream_t s);
std::size_t scan_scratch_ints(std::size_t n);
void build_cells(NeighborState &nb, int n, const double *x, cudaStream_t s);
int sr_reach(const CellGrid &g, double rc);
void count_sr(NeighborState &nb, double rc, cudaStream_t s);
void fill_sr(NeighborState &nb, double rc, int E, cudaStream_t s);
void fill_pairs(NeighborState &nb, int E, cudaStream_t s);

// halo rows of the decomposition (halo.cu). Flags and positions: nranks x stride
// ints each; send_rows / recv_rows: owned / foreign global rows grouped by peer;
// offsets[0..nranks] (sends) and offsets[nranks+1..2 nranks+1] (receives) are the
// per-peer starts; totals[0..1]: scratch for the scan totals
void launch_halo_lists(int n_own, int row0, int stride, int nranks, int rank, const int *row_start, const int *nbr,
                       int *send_flag, int *recv_flag, int *send_pos, int *recv_pos, int *send_rows, int *recv_rows,
                       long long *offsets, int *totals, int *scan_scratch, cudaStream_t s);
// buf[k][0..wa+wb) = (a[rows[k]][0..wa), b[rows[k]][0..wb)) and back
void launch_halo_pack(int count, const int *rows, const double *a, int wa, const double *b, int wb, double *buf,
                      cudaStream_t s);
void launch_halo_unpack(int count, const int *rows, const double *buf, double *a, int wa, double *b, int wb,
                        cudaStream_t s);

// exact fixed-point sums (reduce.cu): nblk partial sums per segment and column,
// parts[((blk * nseg + seg) * ncol + col) * 2 + {hi, lo}]
void launch_fixed_segment_sum(int nseg, int nblk, const int *start, const double *v, int stride, int ncol,
                              long long *parts, cudaStream_t s);
// out[k] = sum over nparts consecutive blocks of `count` fixed-point values
void launch_fixed_finish(const long long *parts, int nparts, int count, double *out, cudaStream_t s);

// ---- per-pair geometry -------------------------------------------------------
// geo[p*8 + {0..7}] = r, ux, uy, uz, phi, dphi/dr, zbl directed energy, zbl pair dE/dr
constexpr int kGeo = 8;
// repulsion: kind 0 = learned ZBL (p, d, a, c); kind 1 = NLH pair tables
// nlh_a / nlh_b [cap][cap][3] in device memory
struct ZblDev {
  double ke, cutoff, switch_off, p, d, a[4], c[4];
  int kind, nlh_cap;
  const double *nlh_a, *nlh_b;
};
void launch_pair_geometry(int P, const NeighborState &nb, const int *z, ZblDev zbl, double sr_cutoff,
                          double *geo, double *sh, double *gv, cudaStream_t s);

struct LrDev {
  double ke, sigma, cutoff, elec_cuton, disp_cuton, fine_factor, bohr, hartree, disp_scale, full_scale;
  double shift, fshift;
};
// Long-range Coulomb + dispersion over the full neighbour set of every atom
// (cell stencil or image range). Per-atom outputs (N): energy (total, elec,
// disp), dE/dq, dE/dh, direct force (3), virial (6).
// n: owned rows (nb.row0 ..); n_cells_atoms: atoms in the cell list (all real
// atoms; with open boundaries, every row). pos4 / par4: n_cells_atoms-element
// scratch for the cell-ordered partner data.
// f32: the pair term in float32 arithmetic, summed in float64 (mixed precision).
// c6r: per-atom C6 ratios of a model with a C6 head (C6_i = C6_ref c6r_i,
// alpha_i = alpha_ref h_i; dc6 = dE/dc6r), or nullptr (C6_i = C6_ref h_i^2, dc6
// unused)
void launch_long_range(int n, int n_cells_atoms, const NeighborState &nb, double rc_lr, const int *z,
                       const double *q, const double *h, const double *c6r, const double *alpha_ref,
                       const double *c6_ref, int table_size, LrDev p, double4 *pos4, double4 *par4, double *e_lr,
                       double *e_elec, double *e_disp, double *dq, double *dh, double *dc6, double *f_lr,
                       double *w_lr, cudaStream_t s, bool f32 = false);

// Allocation-free variant of the long-range step for open-boundary systems of
// at most noalloc_max_atoms() atoms (scratch in file-scope device arrays, noalloc.cu).
int noalloc_max_atoms();
void long_range_noalloc(int n, const double *x, const double *q, const double *h, const int *z,
                        const double *alpha_ref, const double *c6_ref, int table_size, const LrDev &p, double rc_lr,
                        double *e_lr, double *e_elec, double *e_disp, double *dq, double *dh, double *f,
                        double *w_atom, cudaStream_t s);

}  // namespace so3lr_b200

SO3LR_SHAPE_BEGIN
// ---- filters (pair tiles, FP64 tensor cores) --------------------------------
// sp: silu' of the rbf-branch hidden layer for the reverse pass, filter_sp_doubles(P) doubles;
// drbf (optional, P x kR): d rbf_k / dr of every pair (it depends on the geometry only)
void launch_filter_forward(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                           const double *cg_att, const FilterW &finv, const FilterW &fev, const RadialW &rad,
                           double *f_inv, double *f_ev, double *sp, double *drbf, cudaStream_t s);
// pairs per tile of the float64 filter kernels: 64 (F = 128), 32 (F = 256)
constexpr int kFilterTile = kF == 128 ? 64 : 32;
inline std::size_t filter_sp_doubles(int P) {
  return std::size_t((P + kFilterTile - 1) / kFilterTile) * 2 * kFilterTile * kF;
}
// g_filt_inv / g_filt_ev: per-pair gradient w.r.t. the two filter outputs (written by
// the attention reverse at each pair's primary edge)
// g_r (P) and g_y (P x kSH): per-pair radial and distinct-harmonic gradients, written
// (accumulate = false) or added to (accumulate = true); launch_pair_tail turns
// their block sums into the Cartesian pair gradient gv (P x 3, +=)
void launch_filter_reverse(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                           const double *cg_att, const FilterW &finv, const FilterW &fev, const RadialW &rad,
                           const double *g_filt_inv, const double *g_filt_ev, const double *sp, const double *drbf,
                           const double *gA, const double *pair_sc, bool need_l0, bool accumulate, double *g_r,
                           double *g_y, double *gl0, cudaStream_t s);
void launch_pair_tail(int P, const double *geo, const double *g_r, const double *g_y, double *gv, cudaStream_t s);
// mixed precision (filter_mixed.cu): the same outputs with the filter GEMMs in
// three TF32 passes (float32 accuracy); sp holds float32 silu' values
// (filter_sp_doubles(P) floats)
void launch_filter_forward_mixed(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                                 const double *cg_att, const FilterW32 &finv, const FilterW32 &fev,
                                 const RadialW &rad, double *f_inv, double *f_ev, float *sp, double *drbf,
                                 cudaStream_t s);
// the same forward on the tcgen05 tensor cores (filter_tc.cu): persistent, one
// CTA per SM (num_sms); err (device int, zeroed by the caller) receives the
// code of a wait that gave up, 0 when none did
// (filters written in float32 for the float32 attention of this path)
void launch_filter_forward_tc(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                              const TcFwdConsts &consts, const FilterW32 &finv, const FilterW32 &fev, float *f_inv,
                              float *f_ev, float *sp, double *drbf, int *err, int num_sms, cudaStream_t s);
// (filter gradients read in float32)
void launch_filter_reverse_tc(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                              const TcRevConsts &consts, const FilterW32 &finv32, const FilterW32 &fev32,
                              const float *g_filt_inv, const float *g_filt_ev,
                              const float *sp, const double *drbf, const double *gA, const double *pair_sc,
                              bool need_l0, bool accumulate, double *g_r, double *g_y, double *gl0, int *err,
                              int num_sms, cudaStream_t s);
void launch_filter_reverse_mixed(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                                 const double *cg_att, const FilterW &finv, const FilterW &fev,
                                 const FilterW32 &finv32, const FilterW32 &fev32, const double *g_filt_inv,
                                 const double *g_filt_ev, const float *sp, const double *drbf, const double *gA,
                                 const double *pair_sc, bool need_l0, bool accumulate, double *g_r, double *g_y,
                                 double *gl0, cudaStream_t s);

// ---- attention (receiver CSR gathers) ----------------------------------------
void launch_attention_forward(int n, const NeighborState &nb, const double *geo, const double *sh,
                              const double *qkv, const double *f_inv, const double *f_ev, double norm,
                              double *d_inv, double *d_ev, cudaStream_t s);
void launch_attention_reverse(int n, const NeighborState &nb, const double *geo, const double *sh,
                              const double *qkv, const double *f_inv, const double *f_ev, const double *g_a,
                              const double *g_A, double norm, double *g_qkv, double *pair_sc, double *g_filt_inv,
                              double *g_filt_ev, cudaStream_t s);
void launch_ev_l0_reverse(int n, const NeighborState &nb, const double *ev, const double *cg_att,
                          const double *gl0, const double *g_A, double *g_ev, cudaStream_t s);
#if SO3LR_FEATURES == 128
// float32 attention of the mixed-precision path (tcgen05 filters): filters,
// qkv rows and adjoint rows in float32, arithmetic in float32; d_inv, d_ev,
// g_qkv and the pair scalars are written in double for the float64 code that
// reads them, the filter gradients in float32
void launch_attention_forward32(int n, const NeighborState &nb, const double *geo, const double *sh,
                                const float *qkv, const float *f_inv, const float *f_ev, double norm,
                                double *d_inv, double *d_ev, cudaStream_t s);
void launch_attention_reverse32(int n, const NeighborState &nb, const double *geo, const double *sh,
                                const float *qkv, const float *f_inv, const float *f_ev, const float *g_a,
                                const float *g_A, double norm, double *g_qkv, double *pair_sc, float *g_filt_inv,
                                float *g_filt_ev, cudaStream_t s);
// dst rows [r0, r0 + n) and rows[0..nlist) = float(src rows); width even
void launch_rows_to_float(int n, int r0, int nlist, const int *rows, int width, const double *src, float *dst,
                          cudaStream_t s);
#endif

SO3LR_SHAPE_END

namespace so3lr_b200 {

// ---- node GEMM (FP64 tensor cores) ------------------------------------------
enum class Epi { None, Bias, BiasSilu, BiasStorePre, AddResidual, SiluPrimeMul, BiasResidual, GateSiluResidual };
// C[M x N] = A[M x K] * B, B(k, n) = transB ? W[n*ldw + k] : W[k*ldw + n].
// Epilogues:
//   Bias:            C = acc + bias[n]
//   BiasSilu:        C = silu(acc + bias[n])
//   BiasStorePre:    pre = acc + bias[n] -> aux[m*ldaux+n]; C = silu(pre)
//   AddResidual:     C = acc + aux[m*ldaux+n]
//   BiasResidual:    C = acc + bias[n] + aux[m*ldaux+n]
//   SiluPrimeMul:    C = acc * silu'(aux[m*ldaux+n])
//   GateSiluResidual:C = aux2[m*ldaux+n] + acc * silu'(aux[m*ldaux+n])
struct GemmArgs {
  int M, N, K;
  const double *A;
  int lda;
  const double *W;
  int ldw;
  bool transB;
  double *C;
  int ldc;
  const double *bias = nullptr;
  const double *aux = nullptr;
  const double *aux2 = nullptr;
  int ldaux = 0;
  double *aux_out = nullptr;
  Epi epi = Epi::None;
  // optional row list: logical row m of A, C and aux is physical row rows[m]
  const int *rows = nullptr;
  // batched over gridDim.z with per-batch strides (elements)
  int batch = 1;
  long long strideA = 0, strideW = 0, strideC = 0, strideAux = 0, strideBias = 0;
};
}  // namespace so3lr_b200

SO3LR_SHAPE_BEGIN
void launch_gemm(const GemmArgs &g, cudaStream_t s);
// aux added only to columns < aux_cols; aux2 row stride ldaux2
void launch_gemm_ex(const GemmArgs &g, int aux_cols, int ldaux2, cudaStream_t s);

// ---- node elementwise / row kernels -----------------------------------------
void launch_embedding(int n, const int *z, const double *emb_w, const double *cs_table, const int *image_of_atom,
                      double inv_scale, double *x, cudaStream_t s);
// Block norms: kNormLayer = affine LayerNorm (lnw, lnb), kNormRms = RMSNorm
// without scale (no parameters), kNormNone = identity (second position only).
// xhat holds the normalised value and rstd the inverse RMS / standard
// deviation for the reverse.
constexpr int kNormLayer = 0, kNormRms = 1, kNormNone = 2;
void launch_post_attn_pre(int n, const double *x, const double *d_inv, const double *ev, const double *d_ev,
                          int norm, const double *lnw, const double *lnb, const double *cg_int, double *xhat1,
                          double *rstd1, double *n1, double *act, double *A, double *cat, cudaStream_t s);
void launch_post_attn_final(int n, const double *cat, const double *t, const double *A, int norm, const double *lnw,
                            const double *lnb, double *xhat2, double *rstd2, double *gate, double *x_out,
                            double *ev_out, cudaStream_t s);
void launch_post_attn_rev_final(int n, const double *g_x, const double *g_ev, const double *xhat2,
                                const double *rstd2, int norm, const double *lnw2, const double *A,
                                const double *gate, double *g_t, double *g_A, cudaStream_t s);
void launch_post_attn_rev_ln1(int n, const double *g_n1, const double *xhat1, const double *rstd1, int norm,
                              const double *lnw1, const double *A, const double *cg_int, const double *g_cat,
                              double *g_a, double *g_A, cudaStream_t s);
// residual scalars: out[i] = a in[i] + c x0[i] over rows [0, n) of width kF
// (out may alias in)
void launch_residual_combine(int n, const double *in, const double *x0, double a, double c, double *out,
                             cudaStream_t s);
// v[i] *= a over rows [0, n) of width kF
void launch_scale_rows(int n, double *v, double a, cudaStream_t s);
// query/key RMS normalisation of qkv rows ([row][head][5][32], slots q, k, v,
// q_ev, k_ev; v untouched), in place, over rows [0, n) or rows[0..n) when rows
// is given; rinv[row][head][4] keeps the inverse RMS of q, k, q_ev, k_ev
void launch_qk_norm(int n, const int *rows, double *qkv, double *rinv, cudaStream_t s);
// reverse: g[row] (same layout, gradient w.r.t. the normalised values) becomes
// the gradient w.r.t. the raw projections: r (g - y mean(g y)) per 32-vector
void launch_qk_norm_reverse(int n, const double *qkv, const double *rinv, double *g, cudaStream_t s);

// heads
// hk6_out / ratio6 (C6 ratio head keys and ratios) are written only when the
// model has that head (hw.c6_w2 != nullptr)
void launch_heads_finalize(int n, const int *z, const double *hcat, const HeadsW &hw, double *hk_out,
                           double *e_nn, double *raw_q, double *ratio, double *hk6_out, double *ratio6,
                           cudaStream_t s);
void launch_heads_seed(int n, const int *z, const double *hpre, const double *hk, const HeadsW &hw,
                       const double *dq, const double *dq_mean, const int *image_of_atom, const double *dh,
                       const double *hk6, const double *dc6, double *g_hcat, cudaStream_t s);

SO3LR_SHAPE_END

namespace so3lr_b200 {

void launch_charge_correct(int n, const double *raw, const double *raw_sum, const double *qtot,
                           const int *image_of_atom, const int *image_start, double *q, double *dq_mean_out,
                           const double *dq_sum, cudaStream_t s);

// final assembly: per-atom forces and energies, per-atom SR virial
void launch_assemble(const NeighborState &nb, const double *geo, const double *gv, const double *e_nn,
                     const double *e_lr, const double *f_lr, const double *w_lr, double *force, double *e_atom,
                     double *e_zbl, double *w_atom, cudaStream_t s);

// MD integration (velocity Verlet, LAMMPS metal units)
// ---- Nose-Hoover chain (thermostat.cu) ----------------------------------------
constexpr int kMaxChain = 10;
struct NhcState {
  int chain;          // thermostats in the chain
  double kt;          // k_B T (eV)
  double ndof;        // degrees of freedom of the particles
  double q[kMaxChain];     // masses (eV ps^2)
  double eta[kMaxChain];   // positions
  double veta[kMaxChain];  // velocities (1/ps)
};
void launch_two_ke(int n, const double *v, const double *mass, double mvv2e, double *out, cudaStream_t s);
void launch_nhc_half(NhcState *st, const double *two_k, double dt, double *scale, cudaStream_t s);
void launch_scale_v(int n, double *v, const double *scale, cudaStream_t s);

void launch_verlet_first(int n, double *x, double *v, const double *f, const double *inv_mass, double dt,
                         double ftm2v, cudaStream_t s);
void launch_verlet_second(int n, double *v, const double *f, const double *inv_mass, double dt, double ftm2v,
                          cudaStream_t s);

}  // namespace so3lr_b200
