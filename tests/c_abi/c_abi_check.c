/* A plain C99 consumer of include/so3lr_b200.h, as a LAMMPS plugin or another
 * host in C would bind it.
 *   c_abi_check host MODEL   host-only entry points (no GPU): model inspection,
 *                            element tokens, charge/multiplicity rule, partition,
 *                            and a clean refusal where a GPU is needed
 *   c_abi_check gpu MODEL    one so3lr_compute of a 2x2x2 water lattice on
 *                            device 0; prints energy and the first force
 * Prints "C ABI OK" when every check passes. */
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "so3lr_b200.h"

static int fails = 0;
#define CHECK(cond, what)                      \
  do {                                         \
    if (!(cond)) {                             \
      printf("FAIL %s\n", what);               \
      ++fails;                                 \
    }                                          \
  } while (0)

static int host_checks(const char *model) {
  char err[1024];
  so3lr_arch_info info;
  long long counts[119];
  double x[6] = {1.0, 1.0, 1.0, 9.0, 9.0, 9.0};
  double lo[3] = {0.0, 0.0, 0.0}, len[3] = {10.0, 10.0, 10.0};
  int owner[2] = {-1, -1};
  so3lr_handle *h = NULL;

  CHECK(so3lr_inspect_model(model, &info, err, sizeof err) == 0, "inspect shipped model");
  CHECK(info.layers == 3 && info.features == 128 && info.rbf == 32, "architecture record");
  CHECK(fabs(info.sr_cutoff - 4.5) < 1e-12 && fabs(info.lr_cutoff - 12.0) < 1e-12, "cutoffs");
  CHECK(so3lr_inspect_model("/nonexistent.so3lr", &info, err, sizeof err) != 0 && strstr(err, "cannot open"),
        "missing model refused with a message");

  CHECK(so3lr_element_from_token("O") == 8, "token O");
  CHECK(so3lr_element_from_token("es") == 99, "token es (case-insensitive)");
  CHECK(so3lr_element_from_token("17") == 17, "numeric token");
  CHECK(so3lr_element_from_token("Xx") == 0 && so3lr_element_from_token("100") == 0, "unknown tokens");

  memset(counts, 0, sizeof counts);
  counts[8] = 1;
  counts[1] = 2; /* H2O: 10 electrons */
  CHECK(so3lr_validate_charge_spin(counts, 0.0, 1.0, err, sizeof err) == 0, "neutral water singlet");
  CHECK(so3lr_validate_charge_spin(counts, 1.0, 1.0, err, sizeof err) != 0, "cation singlet refused");
  CHECK(so3lr_validate_charge_spin(counts, 1.0, 2.0, err, sizeof err) == 0, "cation doublet");

  CHECK(so3lr_partition(2, x, lo, len, 2, owner) == 0 && owner[0] != owner[1], "two bricks split two far atoms");
  {
    const double bad_len[3] = {10.0, HUGE_VAL, 10.0}, flat_len[3] = {10.0, 0.0, 10.0};
    CHECK(so3lr_partition(2, x, lo, bad_len, 2, owner) == 2, "partition refuses an infinite box");
    CHECK(so3lr_partition(2, x, lo, flat_len, 2, owner) == 2, "partition refuses a zero box length");
    CHECK(so3lr_partition(0, x, lo, len, 2, owner) == 2, "partition refuses zero atoms");
  }

  /* NULL arguments come back as an error status with a message, never a crash */
  err[0] = '\0';
  CHECK(so3lr_compute(NULL, NULL, NULL, err, sizeof err) != 0 && strlen(err) > 0, "compute(NULL)");
  err[0] = '\0';
  CHECK(so3lr_compute_batch(NULL, NULL, NULL, err, sizeof err) != 0 && strlen(err) > 0, "compute_batch(NULL)");
  err[0] = '\0';
  CHECK(so3lr_virial_atom(NULL, NULL, err, sizeof err) != 0 && strlen(err) > 0, "virial_atom(NULL)");
  err[0] = '\0';
  CHECK(so3lr_md_run(NULL, 1, 0.0005, err, sizeof err) != 0 && strlen(err) > 0, "md_run(NULL)");
  CHECK(so3lr_create(model, 0, NULL, err, sizeof err) != 0, "create without an output pointer");

  if (so3lr_create(model, 0, &h, err, sizeof err) == 0) {
    so3lr_destroy(h); /* a GPU is present */
  } else {
    CHECK(strlen(err) > 0, "so3lr_create without a GPU fails with a message");
  }
  return fails;
}

static int gpu_check(const char *model) {
  char err[1024];
  so3lr_handle *h = NULL;
  double x[24 * 3], f[24 * 3];
  int z[24];
  so3lr_frame in;
  so3lr_result out;
  int i, j, k, a = 0;
  if (so3lr_create(model, 0, &h, err, sizeof err) != 0) {
    printf("FAIL create: %s\n", err);
    return 1;
  }
  /* 2 x 2 x 2 water molecules on a 3.1 A lattice, box 6.2 A */
  for (i = 0; i < 2; ++i)
    for (j = 0; j < 2; ++j)
      for (k = 0; k < 2; ++k) {
        const double ox = 3.1 * i + 0.5, oy = 3.1 * j + 0.5, oz = 3.1 * k + 0.5;
        x[3 * a] = ox; x[3 * a + 1] = oy; x[3 * a + 2] = oz; z[a++] = 8;
        x[3 * a] = ox + 0.9572; x[3 * a + 1] = oy; x[3 * a + 2] = oz; z[a++] = 1;
        x[3 * a] = ox - 0.2400; x[3 * a + 1] = oy + 0.9266; x[3 * a + 2] = oz; z[a++] = 1;
      }
  memset(&in, 0, sizeof in);
  in.natoms = 24;
  in.x = x;
  in.z = z;
  in.periodic = 1;
  in.boxlen[0] = in.boxlen[1] = in.boxlen[2] = 6.2;
  in.multiplicity = 1.0;
  memset(&out, 0, sizeof out);
  out.f = f;
  CHECK(so3lr_compute(h, &in, &out, err, sizeof err) == 0, "compute");
  printf("energy %.17g force0 %.17g %.17g %.17g\n", out.energy, f[0], f[1], f[2]);
  so3lr_destroy(h);
  return fails;
}

int main(int argc, char **argv) {
  int rc;
  if (argc < 3) {
    printf("usage: c_abi_check host|gpu MODEL\n");
    return 2;
  }
  rc = strcmp(argv[1], "gpu") == 0 ? gpu_check(argv[2]) : host_checks(argv[2]);
  if (rc == 0) printf("C ABI OK\n");
  return rc ? 1 : 0;
}
