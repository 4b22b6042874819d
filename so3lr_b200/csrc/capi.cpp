// extern "C" boundary (include/so3lr_b200.h). Converts every C++ exception into
// a status code plus message, like the reference pair style's catch blocks
// (plugins/lammps/pair_so3lr_native_mpi.cpp:1133-1136, 1974-1977).
#include "../../include/so3lr_b200.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <string>

#include "nccl_dyn.hpp"

#include "api.hpp"

using so3lr_b200::Error;
using Evaluator = so3lr_b200::EvaluatorApi;
using so3lr_b200::SystemSpec;

std::atomic<long long> &so3lr_b200::launch_counter() {
  static std::atomic<long long> count{0};
  return count;
}

struct so3lr_handle {
  std::unique_ptr<Evaluator> eval;
  std::string last_error;
};

namespace {

int report(const std::exception &e, char *err, std::size_t errlen, so3lr_handle *h = nullptr) {
  if (h) h->last_error = e.what();
  if (err && errlen > 0) {
    std::strncpy(err, e.what(), errlen - 1);
    err[errlen - 1] = '\0';
  }
  return 1;
}

int report_msg(const char *msg, char *err, std::size_t errlen) {
  if (err && errlen > 0) {
    std::strncpy(err, msg, errlen - 1);
    err[errlen - 1] = '\0';
  }
  return 2;
}

SystemSpec spec_from_frame(const so3lr_frame &f) {
  if (f.natoms <= 0 || f.natoms > (1LL << 30)) throw Error("SO3LR: natoms must be in 1..2^30");
  if (!f.x || !f.z) throw Error("SO3LR: frame positions and atomic numbers are required");
  SystemSpec s;
  s.n = int(f.natoms);
  s.periodic = f.periodic != 0;
  for (int d = 0; d < 3; ++d) {
    s.lo[d] = f.boxlo[d];
    s.len[d] = f.boxlen[d];
  }
  s.z.assign(f.z, f.z + f.natoms);
  s.image_start = {0, s.n};
  s.image_charge = {f.total_charge};
  s.image_mult = {f.multiplicity};
  return s;
}

bool same_system(const SystemSpec &a, const SystemSpec &b) {
  if (a.n != b.n || a.periodic != b.periodic || a.z != b.z || a.image_start != b.image_start ||
      a.image_charge != b.image_charge || a.image_mult != b.image_mult)
    return false;
  for (int d = 0; d < 3; ++d)
    if (a.periodic && (a.lo[d] != b.lo[d] || a.len[d] != b.len[d])) return false;
  return true;
}

void ensure_prepared(Evaluator &ev, const SystemSpec &spec, const double *host_x) {
  if (ev.spec().n == 0 || !same_system(ev.spec(), spec)) ev.prepare(spec, host_x);
}

}  // namespace

extern "C" {

int so3lr_create(const char *model_path, int cuda_device, so3lr_handle **out, char *err, size_t errlen) {
  if (!out) return report_msg("so3lr_create: out is NULL", err, errlen);
  *out = nullptr;
  try {
    auto h = std::make_unique<so3lr_handle>();
    h->eval = so3lr_b200::make_evaluator(model_path ? model_path : "", cuda_device);
    *out = h.release();
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen);
  }
}

namespace {
void fill_info(const so3lr_b200::Model &m, so3lr_arch_info *out) {
  const auto &a = m.arch();
  std::memset(out, 0, sizeof(*out));
  out->abi_version = SO3LR_B200_ABI_VERSION;
  out->layers = a.layers;
  out->features = a.features;
  out->heads = a.heads;
  out->head_width = a.head_width;
  out->degrees = a.max_degree;
  out->ev_width = a.ev_width;
  out->rbf = a.rbf;
  out->sr_cutoff = a.sr_cutoff;
  out->lr_cutoff = a.lr_cutoff;
  out->attention_norm = a.attention_norm;
  out->embedding_scale = a.embedding_scale;
  out->parameter_count = (long long)m.parameter_count();
  std::snprintf(out->summary, sizeof(out->summary), "%s", a.summary().c_str());
}
}  // namespace

int so3lr_inspect_model(const char *model_path, so3lr_arch_info *out, char *err, size_t errlen) {
  if (!model_path || !out) return report_msg("so3lr_inspect_model: NULL argument", err, errlen);
  try {
    const auto m = so3lr_b200::Model::load(model_path);
    fill_info(m, out);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen);
  }
}

int so3lr_describe(const so3lr_handle *h, so3lr_arch_info *out) {
  if (!h || !out) return 2;
  fill_info(h->eval->model(), out);
  return 0;
}

int so3lr_validate_charge_spin(const long long element_counts[119], double total_charge, double multiplicity,
                               char *err, size_t errlen) {
  if (!element_counts) return report_msg("element_counts is NULL", err, errlen);
  std::array<std::int64_t, 119> counts{};
  for (int z = 1; z <= 118; ++z) counts[z] = element_counts[z];
  const std::string problem = so3lr_b200::charge_multiplicity_problem(counts, total_charge, multiplicity);
  if (problem.empty()) return 0;
  return report_msg(problem.c_str(), err, errlen);
}

int so3lr_element_from_token(const char *token) { return token ? so3lr_b200::element_token_to_z(token) : 0; }

int so3lr_compute(so3lr_handle *h, const so3lr_frame *in, so3lr_result *out, char *err, size_t errlen) {
  if (!h || !in || !out) return report_msg("so3lr_compute: NULL argument", err, errlen);
  try {
    Evaluator &ev = *h->eval;
    ensure_prepared(ev, spec_from_frame(*in), in->x);
    ev.upload_positions(in->x);
    ev.compute();
    const auto r = ev.download(out->f, out->eatom, out->charges, out->ratios, out->e_learned, out->e_zbl, out->e_lr,
                               out->e_elec, out->e_disp, nullptr);
    out->energy = r.energy;
    for (int k = 0; k < 6; ++k) out->virial[k] = r.virial[k];
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_compute_local(so3lr_handle *h, const so3lr_local_frame *in, so3lr_local_result *out, char *err,
                        size_t errlen) {
  if (!h || !in || !out) return report_msg("so3lr_compute_local: NULL argument", err, errlen);
  try {
    SystemSpec s;
    // out-of-range counts are refused collectively inside (every rank learns of them)
    s.n = (in->natoms > 0 && in->natoms <= (1LL << 30)) ? int(in->natoms) : 0;
    const int nlocal = (in->nlocal >= 0 && in->nlocal <= (1LL << 30)) ? int(in->nlocal) : -1;
    s.periodic = in->periodic != 0;
    for (int d = 0; d < 3; ++d) {
      s.lo[d] = in->boxlo[d];
      s.len[d] = in->boxlen[d];
    }
    s.image_start = {0, s.n};
    s.image_charge = {in->total_charge};
    s.image_mult = {in->multiplicity};
    const auto r = h->eval->compute_local(s, nlocal, in->tag, in->x, in->z, out->f, out->eatom, out->vatom);
    out->energy = r.energy;
    for (int k = 0; k < 6; ++k) out->virial[k] = r.virial[k];
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_compute_device(so3lr_handle *h, const so3lr_frame *in, double *d_f, double *d_eatom, double *energy,
                         double virial[6], char *err, size_t errlen) {
  if (!h || !in || !d_f) return report_msg("so3lr_compute_device: NULL argument", err, errlen);
  try {
    Evaluator &ev = *h->eval;
    if (ev.nranks() > 1) throw Error("so3lr_compute_device: not available on a multi-GPU handle");
    ensure_prepared(ev, spec_from_frame(*in), nullptr);
    const std::size_t n = std::size_t(in->natoms);
    SO3_CUDA(cudaSetDevice(ev.device()));
    SO3_CUDA(cudaMemcpyAsync(ev.positions(), in->x, sizeof(double) * 3 * n, cudaMemcpyDeviceToDevice, ev.stream()));
    ev.compute();
    SO3_CUDA(cudaMemcpyAsync(d_f, ev.forces(), sizeof(double) * 3 * n, cudaMemcpyDeviceToDevice, ev.stream()));
    const auto r = ev.download(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
    if (d_eatom) {
      std::vector<double> tmp(n);
      ev.download(nullptr, tmp.data(), nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
      SO3_CUDA(cudaMemcpy(d_eatom, tmp.data(), sizeof(double) * n, cudaMemcpyHostToDevice));
    }
    if (energy) *energy = r.energy;
    if (virial)
      for (int k = 0; k < 6; ++k) virial[k] = r.virial[k];
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_compute_batch(so3lr_handle *h, const so3lr_batch *in, so3lr_batch_result *out, char *err, size_t errlen) {
  if (!h || !in || !out) return report_msg("so3lr_compute_batch: NULL argument", err, errlen);
  try {
    if (in->nimages <= 0 || !in->image_offsets || !in->image_charge || !in->image_multiplicity || !in->x || !in->z)
      throw Error("SO3LR batch: images, offsets, charges, multiplicities, positions and Z are required");
    SystemSpec s;
    s.n = int(in->natoms);
    if (in->natoms <= 0 || in->natoms > (1LL << 30)) throw Error("SO3LR batch: natoms must be in 1..2^30");
    s.periodic = false;
    s.z.assign(in->z, in->z + in->natoms);
    s.image_start.resize(in->nimages + 1);
    for (int k = 0; k <= in->nimages; ++k) {
      if (in->image_offsets[k] < 0 || in->image_offsets[k] > in->natoms) throw Error("SO3LR batch: image offset out of range");
      s.image_start[k] = int(in->image_offsets[k]);
    }
    s.image_charge.assign(in->image_charge, in->image_charge + in->nimages);
    s.image_mult.assign(in->image_multiplicity, in->image_multiplicity + in->nimages);
    Evaluator &ev = *h->eval;
    if (ev.nranks() > 1) throw Error("so3lr_compute_batch: turbo packs run one handle per GPU, without a communicator");
    ensure_prepared(ev, s, in->x);
    ev.upload_positions(in->x);
    ev.compute();
    ev.download(out->f, out->eatom, out->charges, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                out->image_energy);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_md_init(so3lr_handle *h, const so3lr_frame *in, const double *v, const double *mass, char *err,
                  size_t errlen) {
  if (!h || !in || !v || !mass) return report_msg("so3lr_md_init: NULL argument", err, errlen);
  try {
    Evaluator &ev = *h->eval;
    ensure_prepared(ev, spec_from_frame(*in), in->x);
    ev.upload_positions(in->x);
    ev.md_setup(v, mass);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_md_run(so3lr_handle *h, int nsteps, double dt_ps, char *err, size_t errlen) {
  if (!h) return report_msg("so3lr_md_run: NULL handle", err, errlen);
  try {
    h->eval->md_steps(nsteps, dt_ps);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_md_thermostat(so3lr_handle *h, double t_target_k, double t_damp_ps, int chain, char *err,
                        size_t errlen) {
  if (!h) return report_msg("so3lr_md_thermostat: NULL handle", err, errlen);
  try {
    h->eval->md_thermostat(t_target_k, t_damp_ps, chain);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_md_thermostat_energy(so3lr_handle *h, double *energy, char *err, size_t errlen) {
  if (!h || !energy) return report_msg("so3lr_md_thermostat_energy: NULL argument", err, errlen);
  try {
    *energy = h->eval->md_thermostat_energy();
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_md_state(so3lr_handle *h, double *x, double *v, double *f, double *energy, char *err, size_t errlen) {
  if (!h) return report_msg("so3lr_md_state: NULL handle", err, errlen);
  try {
    Evaluator &ev = *h->eval;
    ev.md_download(x, v);
    const auto r = ev.download(f, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
    if (energy) *energy = r.energy;
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_nccl_unique_id(char out[128], char *err, size_t errlen) {
  if (!out) return report_msg("so3lr_nccl_unique_id: NULL argument", err, errlen);
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  try {
    ncclUniqueId id;
    const ncclResult_t r = so3lr_b200::nccl().get_unique_id(&id);
    if (r != ncclSuccess) return report_msg(so3lr_b200::nccl().get_error_string(r), err, errlen);
    std::memcpy(out, &id, sizeof(id));
    return 0;
  } catch (const std::exception &e) {
    return report_msg(e.what(), err, errlen);
  }
}

int so3lr_comm_init(so3lr_handle *h, int nranks, int rank, const char unique_id[128], char *err, size_t errlen) {
  if (!h || (nranks > 1 && !unique_id)) return report_msg("so3lr_comm_init: NULL argument", err, errlen);
  try {
    h->eval->set_comm(nranks, rank, unique_id);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_owned_atoms(const so3lr_handle *h) { return h ? h->eval->owned_atoms() : -1; }

int so3lr_partition(long long natoms, const double *x, const double boxlo[3], const double boxlen[3], int nranks,
                    int *owner) {
  if (natoms <= 0 || natoms > (1LL << 30) || !x || !boxlo || !boxlen || nranks < 1 || !owner) return 2;
  SystemSpec s;
  s.n = int(natoms);
  s.periodic = true;
  for (int d = 0; d < 3; ++d) {
    s.lo[d] = boxlo[d];
    s.len[d] = boxlen[d];
    if (!(s.len[d] > 0) || !std::isfinite(s.len[d]) || !std::isfinite(s.lo[d])) return 2;
  }
  try {
    const auto o = so3lr_b200::partition_atoms(s, x, nranks);
    for (long long i = 0; i < natoms; ++i) owner[i] = o[std::size_t(i)];
    return 0;
  } catch (const std::exception &) {
    return 1;
  }
}

int so3lr_profile(so3lr_handle *h, int enable) {
  if (!h) return 2;
  h->eval->set_profiling(enable != 0);
  return 0;
}

int so3lr_profile_read(so3lr_handle *h, int kernel, double *total_ms, long long *launches, double *flops, char *err,
                       size_t errlen) {
  if (!h) return report_msg("so3lr_profile_read: NULL handle", err, errlen);
  try {
    h->eval->read_profile(kernel, total_ms, launches, flops);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_set_precision(so3lr_handle *h, int precision, char *err, size_t errlen) {
  if (!h) return report_msg("so3lr_set_precision: NULL handle", err, errlen);
  if (precision != SO3LR_PRECISION_FLOAT64 && precision != SO3LR_PRECISION_MIXED)
    return report_msg("so3lr_set_precision: precision must be SO3LR_PRECISION_FLOAT64 (0) or "
                      "SO3LR_PRECISION_MIXED (1)",
                      err, errlen);
  try {
    h->eval->set_mixed_precision(precision == SO3LR_PRECISION_MIXED);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

long long so3lr_launch_count(void) { return so3lr_b200::launch_counter().load(); }

int so3lr_long_range_noalloc(so3lr_handle *h, long long natoms, const double *x, const double *q,
                             const double *ratios, const int *z, double *e_lr, double *e_elec, double *e_disp,
                             double *dq, double *dh, double *f, double *virial_atom, void *stream, char *err,
                             size_t errlen) {
  if (!h || !x || !q || !ratios || !z || !e_lr || !e_elec || !e_disp || !dq || !dh || !f || !virial_atom)
    return report_msg("so3lr_long_range_noalloc: NULL argument", err, errlen);
  try {
    if (natoms <= 0 || natoms > so3lr_b200::noalloc_max_atoms())
      throw Error("SO3LR no-alloc long range: natoms = " + std::to_string(natoms) + " is outside 1.." +
                  std::to_string(so3lr_b200::noalloc_max_atoms()));
    Evaluator &ev = *h->eval;
    if (ev.has_c6_head())
      throw Error("SO3LR no-alloc long range: the model has a C6-ratio head; this entry point takes Hirshfeld "
                  "ratios only");
    // the caller's current device is restored on every exit, the error paths included
    struct DeviceRestore {
      int previous = -1;
      ~DeviceRestore() {
        if (previous >= 0) cudaSetDevice(previous);
      }
    } restore;
    int current = 0;
    SO3_CUDA(cudaGetDevice(&current));
    if (current != ev.device()) {
      restore.previous = current;
      SO3_CUDA(cudaSetDevice(ev.device()));
    }
    const auto t = ev.long_range_tables();
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ev.stream();
    so3lr_b200::long_range_noalloc(int(natoms), x, q, ratios, z, t.alpha_ref, t.c6_ref, t.table_size, t.params,
                                   t.cutoff, e_lr, e_elec, e_disp, dq, dh, f, virial_atom, s);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

int so3lr_virial_atom(so3lr_handle *h, double *vatom, char *err, size_t errlen) {
  if (!h || !vatom) return report_msg("so3lr_virial_atom: NULL argument", err, errlen);
  try {
    if (!h->eval->has_result()) throw Error("so3lr_virial_atom: no evaluation has run on this handle");
    h->eval->download_virial_atom(vatom);
    return 0;
  } catch (const std::exception &e) {
    return report(e, err, errlen, h);
  }
}

void *so3lr_stream(so3lr_handle *h) { return h ? static_cast<void *>(h->eval->stream()) : nullptr; }

int so3lr_last_stats(const so3lr_handle *h, long long *sr_edges, long long *sr_pairs, long long *device_bytes) {
  if (!h) return 2;
  const auto st = h->eval->stats();
  if (sr_edges) *sr_edges = st.edges;
  if (sr_pairs) *sr_pairs = st.pairs;
  if (device_bytes) *device_bytes = (long long)h->eval->device_bytes();
  return 0;
}

void so3lr_destroy(so3lr_handle *h) { delete h; }

}  // extern "C"
