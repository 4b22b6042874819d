// Stand-in for the few MPI calls the so3lr/b200 pair styles make, in the spirit
// of LAMMPS's own STUBS library for builds without MPI. By default there is one
// rank and every collective copies its send buffer to its receive buffer.
// mpi_stub_run(n, fn) runs fn(rank) on n threads that act as the n ranks of
// MPI_COMM_WORLD (the LAMMPS universe of the tests); MPI_COMM_SELF is each
// thread alone (a one-rank LAMMPS partition). Collectives post their buffers,
// meet at a barrier, pull what they need from the other ranks' buffers and meet
// again, so every buffer stays valid while others read it. A barrier that waits
// longer than two minutes aborts the test program instead of hanging it.
#pragma once
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

typedef int MPI_Comm;
typedef int MPI_Datatype;
typedef int MPI_Op;
#define MPI_COMM_WORLD 0
#define MPI_COMM_SELF 1
#define MPI_SUCCESS 0
#define MPI_BYTE 1
#define MPI_INT 4
#define MPI_LONG_LONG 8
#define MPI_DOUBLE 9
#define MPI_SUM 0
#define MPI_MAX 1

struct MpiStubSlot {
  const void *send = nullptr;
  void *recv = nullptr;
  int count = 0;
  const int *counts = nullptr;
  const int *displs = nullptr;
};

struct MpiStubWorld {
  int size = 1;
  std::vector<MpiStubSlot> slot = std::vector<MpiStubSlot>(1);
  std::mutex m;
  std::condition_variable cv;
  int arrived = 0;
  long long generation = 0;
};

inline MpiStubWorld &mpi_stub_world() {
  static MpiStubWorld w;
  return w;
}
inline int &mpi_stub_rank() {
  thread_local int r = 0;
  return r;
}

inline void mpi_stub_barrier() {
  MpiStubWorld &w = mpi_stub_world();
  if (w.size == 1) return;
  std::unique_lock<std::mutex> lk(w.m);
  const long long gen = w.generation;
  if (++w.arrived == w.size) {
    w.arrived = 0;
    ++w.generation;
    w.cv.notify_all();
    return;
  }
  if (!w.cv.wait_for(lk, std::chrono::seconds(120), [&] { return w.generation != gen; })) {
    std::fprintf(stderr, "mpi stub: rank %d waited two minutes at a collective\n", mpi_stub_rank());
    std::abort();
  }
}

// runs fn(rank) on n threads acting as the ranks of MPI_COMM_WORLD; an
// exception on a rank is stored and returned for that rank (empty if none)
inline std::vector<std::exception_ptr> mpi_stub_run(int n, const std::function<void(int)> &fn) {
  MpiStubWorld &w = mpi_stub_world();
  w.size = n;
  w.slot.assign(n, MpiStubSlot{});
  std::vector<std::exception_ptr> errors(n);
  std::vector<std::thread> threads;
  for (int r = 0; r < n; ++r)
    threads.emplace_back([&, r] {
      mpi_stub_rank() = r;
      try {
        fn(r);
      } catch (...) {
        errors[r] = std::current_exception();
      }
    });
  for (std::thread &t : threads) t.join();
  w.size = 1;
  w.slot.assign(1, MpiStubSlot{});
  return errors;
}

inline std::size_t mpi_stub_size(MPI_Datatype t) { return t == MPI_BYTE ? 1 : (t == MPI_INT ? 4 : 8); }
inline bool mpi_stub_alone(MPI_Comm c) { return c == MPI_COMM_SELF || mpi_stub_world().size == 1; }
inline MpiStubSlot &mpi_stub_post() { return mpi_stub_world().slot[mpi_stub_rank()]; }

inline int MPI_Comm_rank(MPI_Comm c, int *r) {
  *r = mpi_stub_alone(c) ? 0 : mpi_stub_rank();
  return MPI_SUCCESS;
}
inline int MPI_Comm_size(MPI_Comm c, int *n) {
  *n = mpi_stub_alone(c) ? 1 : mpi_stub_world().size;
  return MPI_SUCCESS;
}

inline int MPI_Bcast(void *buf, int n, MPI_Datatype t, int root, MPI_Comm c) {
  if (mpi_stub_alone(c)) return MPI_SUCCESS;
  MpiStubWorld &w = mpi_stub_world();
  mpi_stub_post().send = buf;
  mpi_stub_barrier();
  if (mpi_stub_rank() != root) std::memcpy(buf, w.slot[root].send, n * mpi_stub_size(t));
  mpi_stub_barrier();
  return MPI_SUCCESS;
}

template <class T>
inline void mpi_stub_reduce(const void *s, void *r, int n, MPI_Op op, MPI_Comm c) {
  std::vector<T> acc(static_cast<const T *>(s), static_cast<const T *>(s) + n);
  if (!mpi_stub_alone(c)) {
    MpiStubWorld &w = mpi_stub_world();
    mpi_stub_post().send = s;
    mpi_stub_barrier();
    for (int q = 0; q < w.size; ++q) {
      if (q == mpi_stub_rank()) continue;
      const T *src = static_cast<const T *>(w.slot[q].send);
      for (int i = 0; i < n; ++i) acc[i] = op == MPI_MAX ? (src[i] > acc[i] ? src[i] : acc[i]) : acc[i] + src[i];
    }
    mpi_stub_barrier();
  }
  std::memcpy(r, acc.data(), n * sizeof(T));
}

inline int MPI_Allreduce(const void *s, void *r, int n, MPI_Datatype t, MPI_Op op, MPI_Comm c) {
  if (t == MPI_INT)
    mpi_stub_reduce<int>(s, r, n, op, c);
  else if (t == MPI_LONG_LONG)
    mpi_stub_reduce<long long>(s, r, n, op, c);
  else
    mpi_stub_reduce<double>(s, r, n, op, c);
  return MPI_SUCCESS;
}

// gather family: rank q's `count` items land at displacement displs[q] (or q * n)
inline void mpi_stub_gather(const void *s, int n, MPI_Datatype t, void *r, const int *displs, bool all, int root,
                            MPI_Comm c) {
  const std::size_t es = mpi_stub_size(t);
  if (mpi_stub_alone(c)) {
    std::memmove(static_cast<char *>(r) + (displs ? displs[0] : 0) * es, s, n * es);
    return;
  }
  MpiStubWorld &w = mpi_stub_world();
  mpi_stub_post().send = s;
  mpi_stub_post().count = n;
  mpi_stub_barrier();
  if (all || mpi_stub_rank() == root)
    for (int q = 0; q < w.size; ++q) {
      const std::size_t off = displs ? static_cast<std::size_t>(displs[q]) : static_cast<std::size_t>(q) * n;
      std::memcpy(static_cast<char *>(r) + off * es, w.slot[q].send, w.slot[q].count * es);
    }
  mpi_stub_barrier();
}

inline int MPI_Allgather(const void *s, int n, MPI_Datatype t, void *r, int, MPI_Datatype, MPI_Comm c) {
  mpi_stub_gather(s, n, t, r, nullptr, true, 0, c);
  return MPI_SUCCESS;
}
inline int MPI_Allgatherv(const void *s, int n, MPI_Datatype t, void *r, const int *, const int *displs,
                          MPI_Datatype, MPI_Comm c) {
  mpi_stub_gather(s, n, t, r, displs, true, 0, c);
  return MPI_SUCCESS;
}
inline int MPI_Gather(const void *s, int n, MPI_Datatype t, void *r, int, MPI_Datatype, int root, MPI_Comm c) {
  mpi_stub_gather(s, n, t, r, nullptr, false, root, c);
  return MPI_SUCCESS;
}
inline int MPI_Gatherv(const void *s, int n, MPI_Datatype t, void *r, const int *, const int *displs, MPI_Datatype,
                       int root, MPI_Comm c) {
  mpi_stub_gather(s, n, t, r, displs, false, root, c);
  return MPI_SUCCESS;
}

// scatter family: rank q receives n items from displacement displs[q] (or q * n)
// of the root's send buffer
inline void mpi_stub_scatter(const void *s, const int *displs, MPI_Datatype t, void *r, int n, int root,
                             MPI_Comm c) {
  const std::size_t es = mpi_stub_size(t);
  if (mpi_stub_alone(c)) {
    std::memmove(r, static_cast<const char *>(s) + (displs ? displs[0] : 0) * es, n * es);
    return;
  }
  MpiStubWorld &w = mpi_stub_world();
  mpi_stub_post().send = s;
  mpi_stub_post().displs = displs;
  mpi_stub_barrier();
  const int me = mpi_stub_rank();
  const MpiStubSlot &rs = w.slot[root];
  const std::size_t off = rs.displs ? static_cast<std::size_t>(rs.displs[me]) : static_cast<std::size_t>(me) * n;
  std::memcpy(r, static_cast<const char *>(rs.send) + off * es, n * es);
  mpi_stub_barrier();
}

inline int MPI_Scatter(const void *s, int, MPI_Datatype t, void *r, int n, MPI_Datatype, int root, MPI_Comm c) {
  mpi_stub_scatter(s, nullptr, t, r, n, root, c);
  return MPI_SUCCESS;
}
inline int MPI_Scatterv(const void *s, const int *, const int *displs, MPI_Datatype t, void *r, int n, MPI_Datatype,
                        int root, MPI_Comm c) {
  mpi_stub_scatter(s, displs, t, r, n, root, c);
  return MPI_SUCCESS;
}

inline double MPI_Wtime() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}
