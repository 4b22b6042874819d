// Minimal stand-in for the parts of the LAMMPS API a pair style touches
// (LAMMPS_NS::Pair, Atom, Domain, Force, Comm, Error, Memory, utils::logmesg),
// so the so3lr/b200 pair style compiles and runs in tests without LAMMPS.
// Member names and meanings follow LAMMPS; behaviour is reduced to what the
// style uses. Error::all throws std::runtime_error with the message.
#pragma once
#include <mpi.h>

#include <cstddef>
#include <stdexcept>
#include <string>
#include <vector>

#define FLERR __FILE__, __LINE__
#define MPI_LMP_TAGINT MPI_INT

namespace LAMMPS_NS {

typedef int tagint;  // LAMMPS's default (smallbig) tag type

class LAMMPS;

class Error {
 public:
  [[noreturn]] void all(const char *, int, const std::string &msg) { throw std::runtime_error(msg); }
  [[noreturn]] void universe_all(const char *, int, const std::string &msg) { throw std::runtime_error(msg); }
  [[noreturn]] void universe_one(const char *, int, const std::string &msg) { throw std::runtime_error(msg); }
  // LAMMPS's one() aborts every rank from the calling one; the mock marks its message
  [[noreturn]] void one(const char *, int, const std::string &msg) { throw std::runtime_error("ERROR on proc: " + msg); }
  // LAMMPS prints "WARNING: msg" to the screen and log file; the mock keeps it
  void warning(const char *, int, const std::string &msg) { warnings += "WARNING: " + msg + "\n"; }
  std::string warnings;
};

class Memory {
 public:
  template <class T>
  T **create(T **&array, int n1, int n2, const char *) {
    array = new T *[n1];
    T *data = new T[static_cast<std::size_t>(n1) * n2]();
    for (int i = 0; i < n1; ++i) array[i] = data + static_cast<std::size_t>(i) * n2;
    return array;
  }
  template <class T>
  void destroy(T **&array) {
    if (!array) return;
    delete[] array[0];
    delete[] array;
    array = nullptr;
  }
};

class Atom {
 public:
  int ntypes = 0, nlocal = 0, nghost = 0;
  long long natoms = 0;
  std::vector<int> type_storage;
  std::vector<tagint> tag_storage;
  tagint *tag = nullptr;
  std::vector<double *> x_rows, f_rows;
  std::vector<double> x_data, f_data;
  int *type = nullptr;
  double **x = nullptr, **f = nullptr;
  void resize(int n) {
    nlocal = n;
    natoms = n;
    type_storage.assign(n, 1);
    tag_storage.resize(n);
    for (int i = 0; i < n; ++i) tag_storage[i] = i + 1;
    tag = tag_storage.data();
    x_data.assign(3 * static_cast<std::size_t>(n), 0.0);
    f_data.assign(3 * static_cast<std::size_t>(n), 0.0);
    x_rows.resize(n);
    f_rows.resize(n);
    for (int i = 0; i < n; ++i) {
      x_rows[i] = &x_data[3 * static_cast<std::size_t>(i)];
      f_rows[i] = &f_data[3 * static_cast<std::size_t>(i)];
    }
    type = type_storage.data();
    x = x_rows.data();
    f = f_rows.data();
  }
};

class Domain {
 public:
  int xperiodic = 1, yperiodic = 1, zperiodic = 1, triclinic = 0;
  double boxlo[3] = {0, 0, 0}, prd[3] = {0, 0, 0};
};

class Force {
 public:
  int newton_pair = 1;
};

class Comm {
 public:
  int me = 0, nprocs = 1;
};

// LAMMPS partitions: `nworlds` worlds, this process is rank `me` of the
// universe communicator `uworld` and belongs to world `iworld`
class Universe {
 public:
  int me = 0, nprocs = 1, nworlds = 1, iworld = 0;
  MPI_Comm uworld = MPI_COMM_WORLD;
};

class LAMMPS {
 public:
  Universe universe;
  Error error;
  Memory memory;
  Atom atom;
  Domain domain;
  Force force;
  Comm comm;
  std::string log;
};

namespace utils {
inline void logmesg(LAMMPS *lmp, const std::string &msg) { lmp->log += msg; }
}  // namespace utils

class Pair {
 public:
  explicit Pair(LAMMPS *l)
      : lmp(l), error(&l->error), memory(&l->memory), atom(&l->atom), domain(&l->domain), force(&l->force),
        comm(&l->comm), universe(&l->universe) {}
  virtual ~Pair() {
    delete[] eatom;
    release_vatom();
  }
  virtual void compute(int, int) = 0;
  virtual void settings(int, char **) = 0;
  virtual void coeff(int, char **) = 0;
  virtual void init_style() {}
  virtual double init_one(int, int) { return 0.0; }

  LAMMPS *lmp;
  Error *error;
  Memory *memory;
  Atom *atom;
  Domain *domain;
  Force *force;
  Comm *comm;
  Universe *universe;
  MPI_Comm world = MPI_COMM_WORLD;
  int manybody_flag = 0, one_coeff = 0, restartinfo = 1, single_enable = 1, no_virial_fdotr_compute = 0;
  int allocated = 0;
  int **setflag = nullptr;
  double **cutsq = nullptr;
  double eng_vdwl = 0.0, virial[6] = {0, 0, 0, 0, 0, 0};
  double *eatom = nullptr;
  double **vatom = nullptr;  // [nlocal][6], LAMMPS order xx yy zz xy xz yz
  int eflag_global = 0, eflag_atom = 0, vflag_global = 0, vflag_atom = 0, vflag_fdotr = 0;

  // LAMMPS semantics: eflag bit 1 = global energy, bit 2 = per-atom energy;
  // vflag bit 1 = global virial summed by the style, bit 2 = global virial from
  // F dot r (virial_fdotr_compute) when the style allows it, bit 4/8 = per-atom
  // virial
  void ev_init(int eflag, int vflag) {
    eflag_global = eflag & 1;
    eflag_atom = (eflag & 2) ? 1 : 0;
    vflag_global = (vflag & 3) ? 1 : 0;
    vflag_fdotr = 0;
    if ((vflag & 3) == 2 && !no_virial_fdotr_compute) {
      vflag_fdotr = 1;
      vflag_global = 0;
    }
    vflag_atom = (vflag & 12) ? 1 : 0;
    eng_vdwl = 0.0;
    for (double &v : virial) v = 0.0;
    if (eflag_atom) {
      delete[] eatom;
      eatom = new double[atom->nlocal]();
    }
    if (vflag_atom) {
      release_vatom();
      vatom = new double *[atom->nlocal];
      double *rows = new double[6 * static_cast<std::size_t>(atom->nlocal)]();
      for (int i = 0; i < atom->nlocal; ++i) vatom[i] = rows + 6 * static_cast<std::size_t>(i);
    }
  }

  // global virial as the sum over owned and ghost atoms of x (x) f
  void virial_fdotr_compute() {
    const int nall = atom->nlocal + atom->nghost;
    for (int i = 0; i < nall; ++i) {
      const double *x = atom->x[i], *f = atom->f[i];
      virial[0] += f[0] * x[0];
      virial[1] += f[1] * x[1];
      virial[2] += f[2] * x[2];
      virial[3] += f[1] * x[0];
      virial[4] += f[2] * x[0];
      virial[5] += f[2] * x[1];
    }
  }

 private:
  void release_vatom() {
    if (vatom) {
      delete[] vatom[0];
      delete[] vatom;
      vatom = nullptr;
    }
  }
};

}  // namespace LAMMPS_NS
