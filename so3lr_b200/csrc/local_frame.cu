// Rank-local frames: every rank passes only the atoms it owns, with their
// global tags, and receives the forces, per-atom energies and per-atom virials
// of exactly those atoms.
//
// This is the input the reference's pair style hands its evaluator: the rank's
// own atoms (atom->nlocal) plus ghosts, identified by atom->tag
// (plugins/lammps/pair_so3lr_native_mpi.cpp:1267-1280). Ghost atoms are not
// needed here: the GPUs exchange the owned records among themselves over NCCL
// (one all-gather of tag, position and atomic number per atom, 40 bytes), so no
// rank gathers the whole system on the host and no host copies more than its
// own atoms to or from its GPU.
//
// Per call: the ranks' atom counts are all-gathered (8 bytes per rank, one host
// wait), the records of every rank are all-gathered into a padded
// [nranks][max count] table, and a scatter kernel writes each position into the
// row of its tag (row_of_tag: tag - 1 -> row of the brick layout). The kernel
// also counts tags that are out of range or seen twice and atomic numbers that
// differ from the prepared system; an atomic-number change prepares the system
// again from the gathered records, a bad tag is an error on every rank (every
// rank scatters the same table, so every rank reaches the same verdict).
// Results: the rows other GPUs own are all-gathered (as the whole-system path
// does before its host copy), and a gather kernel picks this rank's atoms by
// tag into a compact device buffer that is copied to the caller.
#include <cmath>

#include "evaluator.hpp"

SO3LR_SHAPE_BEGIN
namespace {

constexpr int kRec = 5;  // tag, x, y, z, Z (tags and Z are exact in a double)

__global__ void k_scatter_local(int nrec, const double *__restrict__ rec, int natoms,
                                const int *__restrict__ row_of_tag, const int *__restrict__ z_rows,
                                double *__restrict__ x_rows, int *__restrict__ seen, int *__restrict__ flags) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= nrec) return;
  const double *r = rec + std::size_t(k) * kRec;
  const double t = r[0];
  if (t == 0.0) return;  // padding record
  if (!(t >= 1.0 && t <= double(natoms)) || t != floor(t)) {
    atomicAdd(flags, 1);
    return;
  }
  const int tag = int(t);
  if (atomicAdd(seen + tag - 1, 1) != 0) {
    atomicAdd(flags, 1);
    return;
  }
  const int row = row_of_tag[tag - 1];
  x_rows[3 * std::size_t(row)] = r[1];
  x_rows[3 * std::size_t(row) + 1] = r[2];
  x_rows[3 * std::size_t(row) + 2] = r[3];
  if (double(z_rows[row]) != r[4]) atomicAdd(flags + 1, 1);
}

// dst[i][0..width) = src[row_of_tag[tag_i - 1]][0..width) for this rank's records
__global__ void k_gather_local(int nlocal, const double *__restrict__ rec, const int *__restrict__ row_of_tag,
                               const double *__restrict__ src, int width, double *__restrict__ dst) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= nlocal * width) return;
  const int i = k / width, c = k - i * width;
  const int tag = int(rec[std::size_t(i) * kRec]);
  dst[k] = src[std::size_t(row_of_tag[tag - 1]) * width + c];
}

bool same_frame(const SystemSpec &a, const SystemSpec &b) {
  if (a.n != b.n || a.periodic != b.periodic || a.image_charge != b.image_charge || a.image_mult != b.image_mult)
    return false;
  for (int d = 0; d < 3; ++d)
    if (a.periodic && (a.lo[d] != b.lo[d] || a.len[d] != b.len[d])) return false;
  return true;
}

}  // namespace

Evaluator::HostResult Evaluator::compute_local(const SystemSpec &frame, int nlocal, const long long *tag,
                                               const double *x, const int *z, double *f, double *eatom,
                                               double *vatom) {
  SO3_CUDA(cudaSetDevice(device_));
  const int natoms = frame.n;
  cudaStream_t s = stream_;
  // this rank's input checks travel with its atom count, so that a refusal on
  // one rank is a refusal on every rank (no rank is left in a collective)
  const bool bad = natoms <= 0 || nlocal < 0 || nlocal > natoms || (nlocal > 0 && (!tag || !x || !z || !f));
  constexpr long long kWantE = 1LL << 40, kWantV = 1LL << 41, kBad = 1LL << 42, kCount = (1LL << 40) - 1;
  const long long word = (bad ? kBad : (long long)nlocal) | (eatom ? kWantE : 0) | (vatom ? kWantV : 0);

  // ---- atom counts (and requests) of all ranks -----------------------------------
  std::vector<long long> words(nranks_, word);
  if (nranks_ > 1) {
    long long *d = local_counts_.reserve(std::size_t(nranks_) + 1);
    host_totals_[15] = 0.0;
    long long *mine = reinterpret_cast<long long *>(host_totals_ + 15);  // pinned
    *mine = word;
    SO3_CUDA(cudaMemcpyAsync(d + nranks_, mine, sizeof(long long), cudaMemcpyHostToDevice, s));
    const ncclResult_t r = nccl().all_gather(d + nranks_, d, 1, ncclInt64, comm_, s);
    if (r != ncclSuccess) throw Error(std::string("SO3LR: ncclAllGather failed: ") + nccl().get_error_string(r));
    SO3_CUDA(cudaMemcpyAsync(words.data(), d, sizeof(long long) * nranks_, cudaMemcpyDeviceToHost, s));
    SO3_CUDA(cudaStreamSynchronize(s));
  }
  long long total = 0, most = 1;
  bool any_bad = false, want_e = false, want_v = false;
  for (long long w : words) {
    any_bad = any_bad || (w & kBad);
    want_e = want_e || (w & kWantE);
    want_v = want_v || (w & kWantV);
    total += w & kCount;
    most = std::max(most, w & kCount);
  }
  if (any_bad)
    throw Error("SO3LR local frame: a rank passed natoms outside 1..2^30, nlocal outside 0..natoms, or no tags, "
                "positions, atomic numbers or force array");
  if (total != natoms)
    throw Error("SO3LR local frame: the ranks pass " + std::to_string(total) + " atoms in all, not natoms = " +
                std::to_string(natoms));
  const std::size_t M = std::size_t(most);

  // ---- this rank's records, all-gathered --------------------------------------
  if (host_rec_cap_ < M * kRec) {
    if (host_rec_) cudaFreeHost(host_rec_);
    host_rec_ = nullptr;
    host_rec_cap_ = 0;
    SO3_CUDA(cudaMallocHost(&host_rec_, sizeof(double) * M * kRec));
    host_rec_cap_ = M * kRec;
  }
  for (int i = 0; i < nlocal; ++i) {
    double *r = host_rec_ + std::size_t(i) * kRec;
    r[0] = double(tag[i]);
    r[1] = x[3 * std::size_t(i)];
    r[2] = x[3 * std::size_t(i) + 1];
    r[3] = x[3 * std::size_t(i) + 2];
    r[4] = double(z[i]);
  }
  std::fill(host_rec_ + std::size_t(nlocal) * kRec, host_rec_ + M * kRec, 0.0);
  double *send = rec_send_.reserve(M * kRec);
  SO3_CUDA(cudaMemcpyAsync(send, host_rec_, sizeof(double) * M * kRec, cudaMemcpyHostToDevice, s));
  const double *all = send;
  if (nranks_ > 1) {
    double *recv = rec_all_.reserve(M * kRec * nranks_);
    prof_begin(kProfPositionGather);
    const ncclResult_t r = nccl().all_gather(send, recv, M * kRec, ncclDouble, comm_, s);
    if (r != ncclSuccess) throw Error(std::string("SO3LR: ncclAllGather failed: ") + nccl().get_error_string(r));
    prof_end(kProfPositionGather, 0.0);
    all = recv;
  }
  const int nrec = int(M * nranks_);

  // ---- positions into the rows of their tags (or a new preparation) ---------
  SystemSpec spec = frame;
  bool need = !local_ready_ || !same_frame(spec_, spec);
  if (!need) {
    int *seen = local_seen_.reserve(std::size_t(natoms) + 2);
    int *flags = seen + natoms;
    SO3_CUDA(cudaMemsetAsync(seen, 0, sizeof(int) * (std::size_t(natoms) + 2), s));
    k_scatter_local<<<(nrec + 255) / 256, 256, 0, s>>>(nrec, all, natoms, row_of_tag_.get(), z_.get(), x_.get(), seen,
                                                       flags);
    SO3_LAUNCH("scatter_local");
    SO3_CUDA(cudaMemcpyAsync(host_small_ + 12, flags, 2 * sizeof(int), cudaMemcpyDeviceToHost, s));
    SO3_CUDA(cudaStreamSynchronize(s));
    if (host_small_[12] != 0) throw Error("SO3LR local frame: atom tags must be unique over the ranks and in 1..natoms");
    need = host_small_[13] != 0;  // atomic numbers changed: prepare again
  }
  if (need) {
    std::vector<double> recs(std::size_t(nrec) * kRec);
    SO3_CUDA(cudaMemcpyAsync(recs.data(), all, sizeof(double) * recs.size(), cudaMemcpyDeviceToHost, s));
    SO3_CUDA(cudaStreamSynchronize(s));
    std::vector<double> xt(3 * std::size_t(natoms), 0.0);
    std::vector<int> zt(natoms, 0);
    std::vector<char> seen(natoms, 0);
    for (int k = 0; k < nrec; ++k) {
      const double *r = recs.data() + std::size_t(k) * kRec;
      if (r[0] == 0.0) continue;
      if (!(r[0] >= 1.0 && r[0] <= double(natoms)) || r[0] != std::floor(r[0]) || seen[std::size_t(r[0]) - 1])
        throw Error("SO3LR local frame: atom tags must be unique over the ranks and in 1..natoms");
      const std::size_t t = std::size_t(r[0]) - 1;
      seen[t] = 1;
      for (int d = 0; d < 3; ++d) xt[3 * t + d] = r[1 + d];
      zt[t] = int(r[4]);
    }
    spec.z = zt;
    prepare(spec, xt.data());
    upload_positions(xt.data());
    SO3_CUDA(cudaMemcpyAsync(row_of_tag_.reserve(std::size_t(natoms)), row_of_.data(), sizeof(int) * natoms,
                             cudaMemcpyHostToDevice, s));
    local_ready_ = true;
  }

  compute();

  // ---- this rank's results ------------------------------------------------------
  // the other GPUs' rows of every array some rank asked for (the same
  // collectives on every rank), then this rank's atoms
  auto pick = [&](double *dst, double *src, int width, bool any_rank) {
    if (nranks_ > 1 && any_rank) allgather_rows(src, width);
    if (!dst || nlocal == 0) return;
    double *out = local_out_.reserve(std::size_t(nlocal) * 6);
    const int cnt = nlocal * width;
    k_gather_local<<<(cnt + 255) / 256, 256, 0, s>>>(nlocal, send, row_of_tag_.get(), src, width, out);
    SO3_LAUNCH("gather_local");
    SO3_CUDA(cudaMemcpyAsync(dst, out, sizeof(double) * cnt, cudaMemcpyDeviceToHost, s));
    SO3_CUDA(cudaStreamSynchronize(s));  // `out` is reused by the next pick
  };
  pick(f, force_.get(), 3, true);
  pick(eatom, e_atom_.get(), 1, want_e);
  pick(vatom, w_atom_.get(), 6, want_v);
  SO3_CUDA(cudaMemcpyAsync(host_totals_, totals_.get(), sizeof(double) * 7, cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaMemcpyAsync(host_small_ + 8, nb_.error_flag, sizeof(int), cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaMemcpyAsync(host_small_ + 9, tc_err_, sizeof(int), cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaStreamSynchronize(s));
  check_device_flags();
  HostResult res;
  res.energy = host_totals_[0];
  for (int k = 0; k < 6; ++k) res.virial[k] = host_totals_[1 + k];
  return res;
}

SO3LR_SHAPE_END
