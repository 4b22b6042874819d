/*
 * so3lr_b200.h -- C ABI of the B200-native SO3LR force evaluation.
 *
 * This is the boundary the LAMMPS pair styles `so3lr/native/mpi` and
 * `so3lr/turbo` of CPradaL/so3lrxlammps cross on every MD step. Each entry point
 * names the reference interface it replaces (paths relative to
 * source/so3lr-lammps-native/ in the reference repository).
 *
 * Conventions
 *   - Every function returns 0 on success and a nonzero status on failure; on
 *     failure a NUL-terminated message is written to `err` (at most `errlen`
 *     bytes, when `err` is not NULL). No C++ exception crosses this ABI. The
 *     reference converts its C++ exceptions into LAMMPS `error->all`
 *     (plugins/lammps/pair_so3lr_native_mpi.cpp:1133-1136, 1974-1977); a caller
 *     of this ABI does the same with the returned message.
 *   - Units are LAMMPS `metal`: positions in Angstrom, energies in eV, forces in
 *     eV/Angstrom, virial in eV (LAMMPS order xx, yy, zz, xy, xz, yz).
 *   - Host pointers are owned by the caller; all device memory is owned by the
 *     handle and persists (grow-only) between calls.
 *   - One handle per GPU; a handle is not thread-safe. Calls are ordered on the
 *     handle's CUDA stream and synchronous at return unless stated otherwise.
 *   - All arithmetic is IEEE float64. Every per-atom and global sum is computed
 *     in a fixed order, so repeated calls on the same input return identical bits.
 */
#ifndef SO3LR_B200_H
#define SO3LR_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SO3LR_B200_ABI_VERSION 1

typedef struct so3lr_handle so3lr_handle;

/* Architecture record (replaces So3lrArchitecture / ArchDims,
 * include/so3lr/so3lr_architecture.hpp:62-185). The pair style reads the
 * cutoffs from it for init_style/init_one (pair_so3lr_native_mpi.cpp:1162-1192). */
typedef struct {
  int abi_version;
  int layers;           /* interaction blocks */
  int features;         /* invariant width F */
  int heads;            /* attention heads */
  int head_width;
  int degrees;          /* equivariant degrees l = 1..degrees */
  int ev_width;         /* sum (2l+1) */
  int rbf;              /* radial basis functions */
  double sr_cutoff;     /* Angstrom */
  double lr_cutoff;     /* Angstrom */
  double attention_norm;
  double embedding_scale;
  long long parameter_count;
  char summary[512];
} so3lr_arch_info;

/* One system (replaces the atom snapshot + neighbour lists the pair style
 * hands the evaluator, pair_so3lr_native_mpi.cpp:1267-1280). Neighbour lists are
 * built on the GPU from the positions; no LAMMPS list is needed. */
typedef struct {
  long long natoms;
  const double *x;       /* natoms * 3 */
  const int *z;          /* atomic number of every atom, 1..99 (so3lr_element_from_token maps pair_coeff tokens) */
  int periodic;          /* 1: orthorhombic periodic box (boxlo, boxlen); 0: open boundaries (any size
                            with host positions: a non-wrapping cell grid over the bounding box of the
                            first call; at most 20,000 atoms through so3lr_compute_device) */
  double boxlo[3];
  double boxlen[3];
  double total_charge;   /* pair_style ... MODEL [charge [multiplicity]] (pair_so3lr_native_mpi.cpp:1097-1104) */
  double multiplicity;
} so3lr_frame;

/* Outputs of so3lr_compute (replace the writes to atom->f, eatom, eng_vdwl and
 * virial[6], pair_so3lr_native_mpi.cpp:1867-1878, and the per-atom debug terms,
 * :1811-1865). Optional arrays may be NULL. */
typedef struct {
  double *f;             /* natoms * 3, overwritten with the total force */
  double *eatom;         /* natoms: learned + ZBL + long-range energy per atom */
  double *charges;       /* natoms: partial charges after charge conservation */
  double *ratios;        /* natoms: Hirshfeld ratios */
  double *e_learned;     /* natoms: network energy incl. per-element shift */
  double *e_zbl;         /* natoms: repulsion */
  double *e_lr;          /* natoms: electrostatics + dispersion */
  double *e_elec;        /* natoms */
  double *e_disp;        /* natoms */
  double energy;         /* total potential energy */
  double virial[6];      /* xx yy zz xy xz yz */
} so3lr_result;

/* Packed independent open-boundary images (replaces the turbo broker + packed
 * evaluator, src/mpi_turbo_replica_broker.cpp:130-307,
 * src/kokkos_turbo_replica_bridge.cpp:64-179,
 * src/kokkos_packed_so3lr_evaluator.cpp:43-149). Atoms of image k are
 * [image_offsets[k], image_offsets[k+1]). */
typedef struct {
  long long natoms;
  int nimages;
  const double *x;                    /* natoms * 3 */
  const int *z;                       /* natoms */
  const long long *image_offsets;     /* nimages + 1 */
  const double *image_charge;         /* nimages */
  const double *image_multiplicity;   /* nimages */
} so3lr_batch;

typedef struct {
  double *f;             /* natoms * 3 */
  double *eatom;         /* natoms, optional */
  double *charges;       /* natoms, optional */
  double *image_energy;  /* nimages, optional */
} so3lr_batch_result;

/* Load and verify a `.so3lr` v1 model (header, SHA-256 of manifest, payload and
 * every tensor), negotiate capabilities and upload the weights to `cuda_device`.
 * Replaces NativeModel::load (src/native_model.cpp:325-405),
 * describe_architecture (src/so3lr_architecture.cpp:296) and
 * negotiate_capabilities (src/so3lr_capabilities.cpp:276), as called from
 * PairSO3LRNativeMPI::settings (pair_so3lr_native_mpi.cpp:1097-1137).
 * Both released widths load: invariant_features = 128 (4 heads, degrees
 * [1,2,3,4], 32 radial functions) and 256 (8 heads, degrees [1,1,2,2,3,3,4,4],
 * 64 radial functions); the handle runs the kernels compiled for that width. */
int so3lr_create(const char *model_path, int cuda_device, so3lr_handle **out, char *err, size_t errlen);

/* Architecture record of a loaded model (src/so3lr_architecture.cpp:296-450). */
int so3lr_describe(const so3lr_handle *h, so3lr_arch_info *out);

/* Host-only model check: load, verify and capability-negotiate a `.so3lr` file
 * without touching a GPU, filling `out` on success. Replaces the reference's
 * capability probe (tests/so3lr_capability_probe.cpp driven by
 * tests/test_capability_rejection.py): a model this build cannot execute is
 * refused here with the list of unsupported features. */
int so3lr_inspect_model(const char *model_path, so3lr_arch_info *out, char *err, size_t errlen);

/* Validate a (charge, multiplicity) pair against a global element count, as
 * PairSO3LRNativeMPI::setup_charge_spin does after its MPI_Allreduce of the
 * counts (pair_so3lr_native_mpi.cpp:1196-1235; src/so3lr_charge_spin.cpp:116-141).
 * element_counts[z] for z = 1..118 (index 0 unused). */
int so3lr_validate_charge_spin(const long long element_counts[119], double total_charge, double multiplicity,
                               char *err, size_t errlen);

/* pair_coeff token -> atomic number: element symbol H..Es (case-insensitive) or a
 * number 1..99; 0 when the token is not valid (plugins/lammps/so3lr_element_map.h:19-52). */
int so3lr_element_from_token(const char *token);

/* Energy, forces, per-atom energies and the global virial of one system
 * (replaces PairSO3LRNativeMPI::compute, pair_so3lr_native_mpi.cpp:1246-1978,
 * for a single rank that owns every atom). Host buffers; the call copies the
 * positions to the GPU and the results back. */
int so3lr_compute(so3lr_handle *h, const so3lr_frame *in, so3lr_result *out, char *err, size_t errlen);

/* Same, with positions and forces in device memory of the handle's GPU
 * (pointers from cudaMalloc on that device). Only `energy` and `virial` are
 * returned on the host; d_eatom may be NULL. */
int so3lr_compute_device(so3lr_handle *h, const so3lr_frame *in_device_x, double *d_f, double *d_eatom,
                         double *energy, double virial[6], char *err, size_t errlen);

/* Rank-local frame: the atoms one rank owns (LAMMPS atom->nlocal, identified by
 * atom->tag), the input the reference's pair style hands its evaluator
 * (pair_so3lr_native_mpi.cpp:1267-1280). No ghost atoms: the GPUs exchange the
 * ranks' atoms themselves. */
typedef struct {
  long long natoms;       /* atoms of the whole system (the nlocal of all ranks add up to it) */
  long long nlocal;       /* atoms this rank passes (0 allowed) */
  const long long *tag;   /* nlocal global tags in 1..natoms, each on exactly one rank */
  const double *x;        /* nlocal * 3 */
  const int *z;           /* nlocal atomic numbers, 1..99 */
  int periodic;           /* as in so3lr_frame */
  double boxlo[3];
  double boxlen[3];
  double total_charge;
  double multiplicity;
} so3lr_local_frame;

typedef struct {
  double *f;              /* nlocal * 3, overwritten with the total force on this rank's atoms */
  double *eatom;          /* nlocal, optional */
  double *vatom;          /* nlocal * 6, optional: per-atom virial (as so3lr_virial_atom) */
  double energy;          /* whole-system potential energy (identical on every rank) */
  double virial[6];       /* whole-system virial (identical on every rank) */
} so3lr_local_result;

/* Energy, forces, per-atom energies and virials for rank-local frames
 * (replaces PairSO3LRNativeMPI::compute, pair_so3lr_native_mpi.cpp:1246-1978,
 * with its per-rank input and output). On a multi-GPU handle every rank calls
 * it with its own atoms (any split of the tags over the ranks); the GPUs
 * all-gather the ranks' (tag, position, Z) records over NCCL, evaluate the
 * system in their spatial bricks exactly as so3lr_compute does, and each rank
 * gets back the results of its own atoms only. Forces, energies and virials are
 * bit-identical to so3lr_compute's on the same system, for any split and any
 * number of GPUs. A refusal of one rank's input (counts, NULL arrays, tags
 * outside 1..natoms or repeated) is returned on every rank. On a one-GPU handle
 * nlocal must equal natoms (tags in any order). The first call, and any call
 * whose box, charge, multiplicity, atom count or atomic numbers change,
 * prepares the system from the gathered records. */
int so3lr_compute_local(so3lr_handle *h, const so3lr_local_frame *in, so3lr_local_result *out, char *err,
                        size_t errlen);

/* Multi-GPU spatial decomposition (one process and one handle per GPU; replaces
 * the MPI exchange plans and halo exchanges of pair_so3lr_native_mpi.cpp:455-930).
 * Rank 0 makes a 128-byte NCCL unique id with so3lr_nccl_unique_id and the
 * caller shares it (any transport); every rank then calls so3lr_comm_init on
 * its own handle. After that, so3lr_compute and so3lr_md_* are collective: every
 * rank passes the same whole system, the atoms are split into spatial bricks of
 * the periodic box (1x1x2, 1x2x2, 2x2x2, ... for 2, 4, 8 ranks), each GPU computes
 * its own atoms, rows owned by other GPUs are refreshed over NCCL (positions,
 * charges and Hirshfeld ratios by all-gathers; block features and adjoints only
 * for the halo rows that neighbour this GPU's atoms, by send/receive), and
 * every rank returns the whole result. NCCL (libnccl.so.2) is loaded at the
 * first multi-GPU call, not linked. Global sums are exact, so energies and
 * forces are bit-identical for any number of ranks. so3lr_owned_atoms returns
 * the number of atoms this rank computes (after the first collective call). */
int so3lr_nccl_unique_id(char out[128], char *err, size_t errlen);
int so3lr_comm_init(so3lr_handle *h, int nranks, int rank, const char unique_id[128], char *err, size_t errlen);
int so3lr_owned_atoms(const so3lr_handle *h);
/* Host-only: the rank that owns each atom under the brick partition above.
 * Returns 2 for a NULL pointer, natoms outside 1..2^30 or a box that is not
 * finite and positive. */
int so3lr_partition(long long natoms, const double *x, const double boxlo[3], const double boxlen[3], int nranks,
                    int *owner);

/* Packed turbo evaluation: every image is an independent open-boundary system
 * with its own charge and multiplicity (replaces MpiTurboReplicaBroker::evaluate,
 * KokkosPackedSo3lrEvaluator::launch_device and the per-image charge constraint of
 * src/kokkos_image_segments.cpp:49-141). */
int so3lr_compute_batch(so3lr_handle *h, const so3lr_batch *in, so3lr_batch_result *out, char *err, size_t errlen);

/* Device-resident NVE molecular dynamics (velocity Verlet, LAMMPS `fix nve`
 * semantics, metal units). The reference leaves integration to LAMMPS; this
 * harness keeps positions and velocities in HBM so a step costs no host
 * transfer. mass in g/mol per atom. */
int so3lr_md_init(so3lr_handle *h, const so3lr_frame *in, const double *v, const double *mass, char *err,
                  size_t errlen);
int so3lr_md_run(so3lr_handle *h, int nsteps, double dt_ps, char *err, size_t errlen);
/* Nose-Hoover chain thermostat for the following so3lr_md_run calls (NVT, the
 * ensemble of the reference's multi-GPU benchmark; LAMMPS `fix nvt` in the
 * reference's inputs). Martyna-Tuckerman-Klein chain of `chain` thermostats
 * (1..10), target temperature in K, damping time in ps; t_damp_ps <= 0 returns
 * to NVE. Call after so3lr_md_init. The chain's kinetic-energy input is an
 * exact sum, so NVT trajectories are bit-identical for any number of GPUs. */
int so3lr_md_thermostat(so3lr_handle *h, double t_target_k, double t_damp_ps, int chain, char *err, size_t errlen);
/* Energy stored in the chain (eV); with the kinetic and potential energy it
 * forms the conserved quantity of the NVT run. 0 without a thermostat. */
int so3lr_md_thermostat_energy(so3lr_handle *h, double *energy, char *err, size_t errlen);
/* Copies the current state to host buffers (any may be NULL) and returns the
 * potential energy of the last force evaluation. Synchronises the stream. */
int so3lr_md_state(so3lr_handle *h, double *x, double *v, double *f, double *energy, char *err, size_t errlen);

/* Optional timing of the dominant kernels (the pair-filter MLPs) and of the
 * multi-GPU exchange phases with CUDA events on the handle's stream.
 * kernel 0 = filter forward, 1 = filter reverse; on a multi-GPU handle also
 * 2 = position all-gather after the Verlet drift, 3 = halo-list rebuild (lists,
 * count all-gather and the host check, including the stream's wait for it),
 * 4 = block-feature halo exchanges, 5 = block-adjoint halo exchanges,
 * 6 = charge/ratio all-gathers before the long range, 7 = the integer
 * all-gathers of the exact global sums. so3lr_profile_read synchronises,
 * returns the summed device time, the number of timed spans and (filters
 * only) their algorithmic FLOPs, and resets. The reference has per-phase
 * timing behind SO3_NATIVE_MPI_PROFILE (pair_so3lr_native_mpi.cpp:1259-1266,
 * 1887-1956); this is its per-kernel form. */
int so3lr_profile(so3lr_handle *h, int enable);
int so3lr_profile_read(so3lr_handle *h, int kernel, double *total_ms, long long *launches, double *flops, char *err,
                       size_t errlen);

/* Arithmetic of the pair-filter MLPs, the dominant tensor work of every
 * evaluation. SO3LR_PRECISION_FLOAT64 (the default) is the reference's float64
 * arithmetic (src/kokkos_integrated_block0.cpp:194-255 forward,
 * src/kokkos_block2_attention_input_reverse.cpp:186-336 reverse).
 * SO3LR_PRECISION_MIXED runs their GEMMs on the TF32 tensor cores in three
 * passes (each operand split into two TF32 parts) with float32 accumulation and
 * the hidden-layer SiLU in float32, keeps the filters and their gradients in
 * float32, runs the attention message passing in float32 and evaluates the
 * long-range pair term in float32 (summed per atom in float64); everything
 * else stays float64 (geometry, node layers, heads, the exact global sums).
 * Stated tolerance against float64: force MAE <= 1e-4 eV/A (measured 8.8e-6,
 * max 2.5e-5, on water boxes of 192 to 24,000 atoms).
 * The reference has no reduced-precision runtime (float32 is only a storage type
 * of its model file, src/native_model.cpp:266); this mode serves the mixed
 * float32 run of the benchmark configurations. Takes effect from the next
 * evaluation; returns nonzero for an unknown value, and for
 * SO3LR_PRECISION_MIXED on a model with invariant_features = 256 (the
 * mixed-precision kernels exist for the F = 128 width only). */
#define SO3LR_PRECISION_FLOAT64 0
#define SO3LR_PRECISION_MIXED 1
int so3lr_set_precision(so3lr_handle *h, int precision, char *err, size_t errlen);

/* Total number of CUDA kernels this library has launched in the process. */
long long so3lr_launch_count(void);

/* Allocation-free long-range step (no counterpart in the reference).
 * For callers that cannot let a library call cudaMalloc or cudaFree once their
 * run has started -- e.g. an MD engine that owns all device memory through its
 * own pool and only hands out the buffers to be filled. Evaluates the
 * electrostatic + dispersion term of one open-boundary system of at most 16384
 * atoms from its positions, partial charges, Hirshfeld ratios and atomic numbers,
 * exactly as the full evaluation does, writing per-atom energy (total,
 * electrostatic, dispersion), dE/dq, dE/d(ratio), the direct force (3 per atom)
 * and the per-atom virial (6 per atom, xx yy zz xy xz yz). All pointers are device
 * memory of the handle's GPU; `stream` (a cudaStream_t, NULL = the handle's
 * stream) orders the work, which is asynchronous. Larger systems are refused
 * with an error. The scratch is a fixed file-scope device array (about 1 MiB,
 * held by every GPU that loads the library until exit); the first call on a
 * device resolves its address, so make that first call before any stream
 * capture. Calls share the scratch: calls that overlap on the GPU race and must
 * be serialised by the caller. The resolved address is kept for the life of the
 * process: after a cudaDeviceReset (or any other reset of the device's primary
 * context) this entry point must not be called again in that process. */
int so3lr_long_range_noalloc(so3lr_handle *h, long long natoms, const double *x, const double *q,
                             const double *ratios, const int *z, double *e_lr, double *e_elec, double *e_disp,
                             double *dq, double *dh, double *f, double *virial_atom, void *stream, char *err,
                             size_t errlen);

/* Per-atom virial of the last evaluation on this handle (so3lr_compute,
 * so3lr_compute_device, so3lr_compute_batch or the last so3lr_md_run step):
 * vatom[natoms * 6] in LAMMPS order xx, yy, zz, xy, xz, yz, eV, input atom
 * order. Each short-range pair and each long-range pair gives half of its
 * -v (x) dE/dv to each of its two atoms, so the rows sum to the global virial.
 * The reference refuses per-atom virials (pair_so3lr_native_mpi.cpp:1248-1251);
 * this is the LAMMPS `vflag_atom` quantity its global virial (:944-990) splits
 * into. Collective on a multi-GPU handle. */
int so3lr_virial_atom(so3lr_handle *h, double *vatom, char *err, size_t errlen);

/* The handle's CUDA stream (cudaStream_t), for callers that time or order work. */
void *so3lr_stream(so3lr_handle *h);

/* Edge and pair counts of the last evaluation and the device memory held. */
int so3lr_last_stats(const so3lr_handle *h, long long *sr_edges, long long *sr_pairs, long long *device_bytes);

/* Release the handle and all of its device memory (the reference frees its
 * PersistentCache before Kokkos::finalize, pair_so3lr_native_mpi.cpp:1070-1086). */
void so3lr_destroy(so3lr_handle *h);

#ifdef __cplusplus
}
#endif

#endif /* SO3LR_B200_H */
