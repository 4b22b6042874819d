// CPU stand-in for the parts of the C ABI (include/so3lr_b200.h) the LAMMPS
// pair styles call, for testing their data routing without a GPU. The
// "evaluation" returns values that encode each atom's image and coordinates, so
// a test can check that every partition got back exactly its own atoms:
//   f[i][d]       = (k + 1) * x[i][d]          (k = image of atom i)
//   eatom[i]      = z[i] + 1000 k
//   image_energy  = sum of eatom over the image
//   vatom[i][c]   = x[i][c % 3] + k
// Element tokens and the charge/multiplicity check are the real ones' simple
// cases (symbols H and O or numbers; electron-count parity).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "so3lr_b200.h"

struct so3lr_handle {
  std::vector<double> va;
  int rank = 0;
};

static int fake_fail(const char *msg, char *err, size_t errlen) {
  if (err && errlen) std::snprintf(err, errlen, "%s", msg);
  return 1;
}

extern "C" {

int so3lr_inspect_model(const char *model_path, so3lr_arch_info *out, char *err, size_t errlen) {
  if (!model_path || std::strcmp(model_path, "fake") != 0) return fake_fail("SO3LR model: cannot open it", err, errlen);
  std::memset(out, 0, sizeof(*out));
  out->sr_cutoff = 4.5;
  out->lr_cutoff = 12.0;
  return 0;
}

int so3lr_create(const char *model_path, int, so3lr_handle **out, char *err, size_t errlen) {
  so3lr_arch_info info;
  if (so3lr_inspect_model(model_path, &info, err, errlen) != 0) return 1;
  *out = new so3lr_handle();
  return 0;
}

void so3lr_destroy(so3lr_handle *h) { delete h; }

int so3lr_element_from_token(const char *token) {
  if (!token) return 0;
  if (std::strcmp(token, "H") == 0) return 1;
  if (std::strcmp(token, "O") == 0) return 8;
  const int z = std::atoi(token);
  return z >= 1 && z <= 99 ? z : 0;
}

int so3lr_validate_charge_spin(const long long counts[119], double total_charge, double multiplicity, char *err,
                               size_t errlen) {
  long long electrons = 0;
  for (int z = 1; z < 119; ++z) electrons += z * counts[z];
  const long long e = electrons - std::llround(total_charge);
  const long long unpaired = std::llround(multiplicity) - 1;
  if (e < 0 || unpaired < 0 || (e - unpaired) % 2 != 0) return fake_fail("cannot have multiplicity", err, errlen);
  return 0;
}

int so3lr_compute_batch(so3lr_handle *h, const so3lr_batch *in, so3lr_batch_result *out, char *err, size_t errlen) {
  if (!h || in->nimages <= 0 || in->image_offsets[0] != 0 || in->image_offsets[in->nimages] != in->natoms)
    return fake_fail("SO3LR batch: bad images", err, errlen);
  h->va.assign(6 * static_cast<std::size_t>(in->natoms), 0.0);
  for (int k = 0; k < in->nimages; ++k) {
    if (in->image_offsets[k + 1] <= in->image_offsets[k])
      return fake_fail("SO3LR: every image needs at least one atom", err, errlen);
    double e = 0.0;
    for (long long i = in->image_offsets[k]; i < in->image_offsets[k + 1]; ++i) {
      for (int d = 0; d < 3; ++d) out->f[3 * i + d] = (k + 1) * in->x[3 * i + d];
      const double ea = in->z[i] + 1000.0 * k;
      if (out->eatom) out->eatom[i] = ea;
      if (out->charges) out->charges[i] = 0.0;
      e += ea;
      for (int c = 0; c < 6; ++c) h->va[6 * i + c] = in->x[3 * i + c % 3] + k;
    }
    if (out->image_energy) out->image_energy[k] = e;
  }
  return 0;
}

int so3lr_virial_atom(so3lr_handle *h, double *vatom, char *, size_t) {
  std::memcpy(vatom, h->va.data(), h->va.size() * sizeof(double));
  return 0;
}

// profiling: each so3lr_compute counts as one launch of 1 ms and 1 GFLOP per kernel
static long long g_profile_calls = 0;
static int g_profile_on = 0;
int so3lr_profile(so3lr_handle *, int enable) {
  g_profile_on = enable;
  return 0;
}
int so3lr_profile_read(so3lr_handle *, int kernel, double *ms, long long *launches, double *flops, char *, size_t) {
  *ms = double(g_profile_calls);
  *launches = g_profile_calls;
  *flops = 1e9 * double(g_profile_calls);
  if (kernel == 1) g_profile_calls = 0;
  return 0;
}
// so3lr_compute (one rank): row k of the system (tag k + 1) gets
//   f = -x, eatom = 0.5 z, charges = 0.01 k, ratios = 1 + 0.001 z,
//   e_learned = 0.25 z, e_zbl = 0.125, e_lr = 0.25 z - 0.125,
//   e_elec = e_disp = e_lr / 2; energy = sum of eatom; virial 0
int so3lr_compute(so3lr_handle *h, const so3lr_frame *in, so3lr_result *out, char *err, size_t errlen) {
  if (!h || !in || !out || !out->f) return fake_fail("so3lr_compute: NULL argument", err, errlen);
  const char *fail_rank = std::getenv("FAKE_SO3LR_FAIL_RANK");  // a failure injected on one rank
  if (fail_rank && std::atoi(fail_rank) == h->rank) return fake_fail("injected failure", err, errlen);
  const long long n = in->natoms;
  double e = 0.0;
  h->va.assign(6 * static_cast<std::size_t>(n), 0.0);
  for (long long k = 0; k < n; ++k) {
    const double z = in->z[k];
    for (int d = 0; d < 3; ++d) out->f[3 * k + d] = -in->x[3 * k + d];
    if (out->eatom) out->eatom[k] = 0.5 * z;
    if (out->charges) out->charges[k] = 0.01 * k;
    if (out->ratios) out->ratios[k] = 1.0 + 0.001 * z;
    if (out->e_learned) out->e_learned[k] = 0.25 * z;
    if (out->e_zbl) out->e_zbl[k] = 0.125;
    if (out->e_lr) out->e_lr[k] = 0.25 * z - 0.125;
    if (out->e_elec) out->e_elec[k] = 0.5 * (0.25 * z - 0.125);
    if (out->e_disp) out->e_disp[k] = 0.5 * (0.25 * z - 0.125);
    e += 0.5 * z;
  }
  out->energy = e;
  for (int c = 0; c < 6; ++c) out->virial[c] = 0.0;
  if (g_profile_on) ++g_profile_calls;
  return 0;
}
// so3lr_compute_local (any number of ranks, no communication in the stand-in):
// local atom i gets f = -x, eatom = 0.5 z, vatom[c] = x[c % 3] + tag / 1000;
// energy = natoms + 0.5 (a value every rank knows); virial = (1, 2, 3, 4, 5, 6).
// Tags must be unique within the rank and in 1..natoms.
int so3lr_compute_local(so3lr_handle *h, const so3lr_local_frame *in, so3lr_local_result *out, char *err,
                        size_t errlen) {
  if (!h || !in || !out || (in->nlocal > 0 && !out->f)) return fake_fail("so3lr_compute_local: NULL argument", err, errlen);
  const char *fail_rank = std::getenv("FAKE_SO3LR_FAIL_RANK");  // a failure injected on one rank
  if (fail_rank && std::atoi(fail_rank) == h->rank) return fake_fail("injected failure", err, errlen);
  std::vector<char> seen(static_cast<std::size_t>(in->natoms), 0);
  for (long long i = 0; i < in->nlocal; ++i) {
    const long long t = in->tag[i];
    if (t < 1 || t > in->natoms || seen[t - 1])
      return fake_fail("SO3LR local frame: atom tags must be unique over the ranks and in 1..natoms", err, errlen);
    seen[t - 1] = 1;
    for (int d = 0; d < 3; ++d) out->f[3 * i + d] = -in->x[3 * i + d];
    if (out->eatom) out->eatom[i] = 0.5 * in->z[i];
    if (out->vatom)
      for (int c = 0; c < 6; ++c) out->vatom[6 * i + c] = in->x[3 * i + c % 3] + 0.001 * t;
  }
  out->energy = double(in->natoms) + 0.5;
  for (int c = 0; c < 6; ++c) out->virial[c] = c + 1.0;
  if (g_profile_on) ++g_profile_calls;
  return 0;
}
int so3lr_set_precision(so3lr_handle *h, int precision, char *err, size_t errlen) {
  if (!h || (precision != SO3LR_PRECISION_FLOAT64 && precision != SO3LR_PRECISION_MIXED))
    return fake_fail("so3lr_set_precision: precision must be SO3LR_PRECISION_FLOAT64 (0) or SO3LR_PRECISION_MIXED (1)",
                     err, errlen);
  return 0;
}
// several ranks: no communication in the stand-in, every rank evaluates the
// whole system it is given (as every rank of the real library returns it)
int so3lr_nccl_unique_id(char *out, char *, size_t) {
  std::memset(out, 0, 128);
  return 0;
}
int so3lr_comm_init(so3lr_handle *h, int nranks, int rank, const char *, char *err, size_t errlen) {
  if (!h || rank < 0 || rank >= nranks) return fake_fail("so3lr_comm_init: bad rank", err, errlen);
  h->rank = rank;
  return 0;
}

}  // extern "C"
