// Serial stand-in for the few MPI calls the so3lr/b200 pair style makes, in the
// spirit of LAMMPS's own STUBS library for builds without MPI: one rank, and
// every collective copies its send buffer to its receive buffer.
#pragma once
#include <cstring>

typedef int MPI_Comm;
typedef int MPI_Datatype;
typedef int MPI_Op;
#define MPI_COMM_WORLD 0
#define MPI_SUCCESS 0
#define MPI_BYTE 1
#define MPI_INT 4
#define MPI_LONG_LONG 8
#define MPI_DOUBLE 9
#define MPI_SUM 0

inline int mpi_stub_size(MPI_Datatype t) { return t == MPI_BYTE ? 1 : (t == MPI_INT ? 4 : 8); }
inline int MPI_Comm_rank(MPI_Comm, int *r) { *r = 0; return MPI_SUCCESS; }
inline int MPI_Comm_size(MPI_Comm, int *n) { *n = 1; return MPI_SUCCESS; }
inline int MPI_Bcast(void *, int, MPI_Datatype, int, MPI_Comm) { return MPI_SUCCESS; }
inline int MPI_Allreduce(const void *s, void *r, int n, MPI_Datatype t, MPI_Op, MPI_Comm) {
  if (s != r) std::memmove(r, s, static_cast<std::size_t>(n) * mpi_stub_size(t));
  return MPI_SUCCESS;
}
inline int MPI_Allgather(const void *s, int n, MPI_Datatype t, void *r, int, MPI_Datatype, MPI_Comm) {
  std::memmove(r, s, static_cast<std::size_t>(n) * mpi_stub_size(t));
  return MPI_SUCCESS;
}
inline int MPI_Allgatherv(const void *s, int n, MPI_Datatype t, void *r, const int *, const int *displs,
                          MPI_Datatype, MPI_Comm) {
  std::memmove(static_cast<char *>(r) + static_cast<std::size_t>(displs[0]) * mpi_stub_size(t), s,
               static_cast<std::size_t>(n) * mpi_stub_size(t));
  return MPI_SUCCESS;
}
