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
#include <algorithm>
#include <functional>
#include <memory>
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
#define MPI_MIN 2

struct MpiStubSlot {
  const void *send = nullptr;
  void *recv = nullptr;
  int count = 0;
  const int *counts = nullptr;
  const int *displs = nullptr;
};

// One communicator: its members (world ranks, in communicator-rank order), a
// barrier of its own and one posting slot per member.
struct MpiStubComm {
  std::vector<int> members;
  std::vector<MpiStubSlot> slot;
  std::mutex m;
  std::condition_variable cv;
  int arrived = 0;
  long long generation = 0;
  int size() const { return static_cast<int>(members.size()); }
  int rank_of(int world_rank) const {
    for (int k = 0; k < size(); ++k)
      if (members[k] == world_rank) return k;
    return -1;
  }
};

struct MpiStubWorld {
  int size = 1;
  MpiStubComm world;  // MPI_COMM_WORLD
  // communicators made by MPI_Comm_split: handle 2 + color
  std::mutex reg_m;
  std::vector<std::unique_ptr<MpiStubComm>> split;
  MpiStubWorld() {
    world.members = {0};
    world.slot.assign(1, MpiStubSlot{});
  }
};

inline MpiStubWorld &mpi_stub_world() {
  static MpiStubWorld w;
  return w;
}
inline int &mpi_stub_rank() {
  thread_local int r = 0;
  return r;
}

inline MpiStubComm &mpi_stub_comm(MPI_Comm c) {
  MpiStubWorld &w = mpi_stub_world();
  if (c < 2) return w.world;
  std::lock_guard<std::mutex> lk(w.reg_m);
  return *w.split.at(static_cast<std::size_t>(c - 2));
}

inline void mpi_stub_barrier(MpiStubComm &cm) {
  if (cm.size() == 1) return;
  std::unique_lock<std::mutex> lk(cm.m);
  const long long gen = cm.generation;
  if (++cm.arrived == cm.size()) {
    cm.arrived = 0;
    ++cm.generation;
    cm.cv.notify_all();
    return;
  }
  if (!cm.cv.wait_for(lk, std::chrono::seconds(120), [&] { return cm.generation != gen; })) {
    std::fprintf(stderr, "mpi stub: rank %d waited two minutes at a collective\n", mpi_stub_rank());
    std::abort();
  }
}
inline void mpi_stub_barrier() { mpi_stub_barrier(mpi_stub_world().world); }

// runs fn(rank) on n threads acting as the ranks of MPI_COMM_WORLD; an
// exception on a rank is stored and returned for that rank (empty if none)
inline std::vector<std::exception_ptr> mpi_stub_run(int n, const std::function<void(int)> &fn) {
  MpiStubWorld &w = mpi_stub_world();
  w.size = n;
  w.world.members.resize(n);
  for (int r = 0; r < n; ++r) w.world.members[r] = r;
  w.world.slot.assign(n, MpiStubSlot{});
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
  w.world.members = {0};
  w.world.slot.assign(1, MpiStubSlot{});
  w.split.clear();
  return errors;
}

inline std::size_t mpi_stub_size(MPI_Datatype t) { return t == MPI_BYTE ? 1 : (t == MPI_INT ? 4 : 8); }
inline bool mpi_stub_alone(MPI_Comm c) { return c == MPI_COMM_SELF || mpi_stub_comm(c).size() == 1; }
// this thread's rank in communicator c
inline int mpi_stub_me(MpiStubComm &cm) { return cm.rank_of(mpi_stub_rank()); }
inline MpiStubSlot &mpi_stub_post(MpiStubComm &cm) { return cm.slot[mpi_stub_me(cm)]; }

inline int MPI_Comm_rank(MPI_Comm c, int *r) {
  *r = mpi_stub_alone(c) ? 0 : mpi_stub_me(mpi_stub_comm(c));
  return MPI_SUCCESS;
}
inline int MPI_Comm_size(MPI_Comm c, int *n) {
  *n = mpi_stub_alone(c) ? 1 : mpi_stub_comm(c).size();
  return MPI_SUCCESS;
}

inline int MPI_Bcast(void *buf, int n, MPI_Datatype t, int root, MPI_Comm c) {
  if (mpi_stub_alone(c)) return MPI_SUCCESS;
  MpiStubComm &cm = mpi_stub_comm(c);
  mpi_stub_post(cm).send = buf;
  mpi_stub_barrier(cm);
  if (mpi_stub_me(cm) != root) std::memcpy(buf, cm.slot[root].send, n * mpi_stub_size(t));
  mpi_stub_barrier(cm);
  return MPI_SUCCESS;
}

template <class T>
inline void mpi_stub_reduce(const void *s, void *r, int n, MPI_Op op, MPI_Comm c) {
  std::vector<T> acc(static_cast<const T *>(s), static_cast<const T *>(s) + n);
  if (!mpi_stub_alone(c)) {
    MpiStubComm &cm = mpi_stub_comm(c);
    mpi_stub_post(cm).send = s;
    mpi_stub_barrier(cm);
    for (int q = 0; q < cm.size(); ++q) {
      if (q == mpi_stub_me(cm)) continue;
      const T *src = static_cast<const T *>(cm.slot[q].send);
      for (int i = 0; i < n; ++i)
        acc[i] = op == MPI_MAX   ? (src[i] > acc[i] ? src[i] : acc[i])
                 : op == MPI_MIN ? (src[i] < acc[i] ? src[i] : acc[i])
                                 : acc[i] + src[i];
    }
    mpi_stub_barrier(cm);
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
  MpiStubComm &cm = mpi_stub_comm(c);
  mpi_stub_post(cm).send = s;
  mpi_stub_post(cm).count = n;
  mpi_stub_barrier(cm);
  if (all || mpi_stub_me(cm) == root)
    for (int q = 0; q < cm.size(); ++q) {
      const std::size_t off = displs ? static_cast<std::size_t>(displs[q]) : static_cast<std::size_t>(q) * n;
      std::memcpy(static_cast<char *>(r) + off * es, cm.slot[q].send, cm.slot[q].count * es);
    }
  mpi_stub_barrier(cm);
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
  MpiStubComm &cm = mpi_stub_comm(c);
  mpi_stub_post(cm).send = s;
  mpi_stub_post(cm).displs = displs;
  mpi_stub_barrier(cm);
  const int me = mpi_stub_me(cm);
  const MpiStubSlot &rs = cm.slot[root];
  const std::size_t off = rs.displs ? static_cast<std::size_t>(rs.displs[me]) : static_cast<std::size_t>(me) * n;
  std::memcpy(r, static_cast<const char *>(rs.send) + off * es, n * es);
  mpi_stub_barrier(cm);
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

// Split a communicator by color (all members call it); members of one color
// are ordered by (key, rank). The new communicator's handle is 2 + color, the
// same on every member of that color.
inline int MPI_Comm_split(MPI_Comm c, int color, int key, MPI_Comm *out) {
  MpiStubComm &cm = mpi_stub_comm(c);
  const int n = mpi_stub_alone(c) ? 1 : cm.size();
  std::vector<int> mine = {color, key, mpi_stub_rank()};
  std::vector<int> all(3 * static_cast<std::size_t>(n));
  mpi_stub_gather(mine.data(), 3, MPI_INT, all.data(), nullptr, true, 0, c);
  std::vector<std::pair<std::pair<int, int>, int>> group;
  for (int q = 0; q < n; ++q)
    if (all[3 * q] == color) group.push_back({{all[3 * q + 1], q}, all[3 * q + 2]});
  std::sort(group.begin(), group.end());
  MpiStubWorld &w = mpi_stub_world();
  {
    std::lock_guard<std::mutex> lk(w.reg_m);
    const std::size_t id = static_cast<std::size_t>(color);
    if (w.split.size() <= id) w.split.resize(id + 1);
    if (!w.split[id]) {
      w.split[id].reset(new MpiStubComm());
      for (auto &g : group) w.split[id]->members.push_back(g.second);
      w.split[id]->slot.assign(group.size(), MpiStubSlot{});
    }
  }
  if (!mpi_stub_alone(c)) mpi_stub_barrier(cm);  // every member sees the new communicator
  *out = 2 + color;
  return MPI_SUCCESS;
}
inline int MPI_Comm_free(MPI_Comm *c) {
  *c = -1;
  return MPI_SUCCESS;
}

inline double MPI_Wtime() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}
