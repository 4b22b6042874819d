#include "evaluator.hpp"

#include <cmath>
#include <cstring>
#include <numeric>
#include <sstream>

namespace so3lr_b200 {

Evaluator::Evaluator(const std::string &model_path, int device) : model_(Model::load(model_path)), device_(device) {
  int count = 0;
  SO3_CUDA(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count) throw Error("SO3LR: CUDA device " + std::to_string(device) + " not available");
  SO3_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop{};
  SO3_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major < 10)
    throw Error(std::string("SO3LR: this library is built for sm_100a (B200); device is ") + prop.name);
  SO3_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  SO3_CUDA(cudaMallocHost(&host_small_, 16 * sizeof(int)));
  SO3_CUDA(cudaMallocHost(&host_totals_, 16 * sizeof(double)));
  upload_weights();
}

Evaluator::~Evaluator() {
  if (stream_) {
    cudaSetDevice(device_);
    cudaStreamSynchronize(stream_);
    for (auto &p : prof_)
      for (auto ev : p.events) cudaEventDestroy(ev);
    cudaStreamDestroy(stream_);
  }
  if (host_small_) cudaFreeHost(host_small_);
  if (host_totals_) cudaFreeHost(host_totals_);
}

// ---------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------
void Evaluator::upload_weights() {
  const Architecture &a = model_.arch();
  layers_ = a.layers;
  norm_ = a.attention_norm;
  sr_cut_ = a.sr_cutoff;
  lr_cut_ = a.lr_cutoff;
  inv_emb_scale_ = 1.0 / a.embedding_scale;
  std::vector<double> host;
  std::vector<std::pair<std::size_t *, std::size_t>> fixups;  // not used; offsets recorded below
  auto push = [&](const std::vector<double> &v) {
    while (host.size() % 8) host.push_back(0.0);  // 64-byte alignment
    const std::size_t off = host.size();
    host.insert(host.end(), v.begin(), v.end());
    return off;
  };
  const std::size_t F = kF, R = kR, H = kEH;
  struct FOff { std::size_t w0, b0, w1, b1, v0, c0, v1, c1; };
  struct BOff {
    FOff finv, fev;
    std::size_t cg_att, cg_int, qf, qr, ln1w, ln1b, ln2w, ln2b, m1w, m1b, m2w, m2b, iw, ib;
  };
  std::vector<BOff> boff(layers_);
  auto filt = [&](const std::string &prefix) {
    FOff o;
    o.w0 = push(model_.f64(prefix + ".mlp_rbf.0.weight", {F, R}));
    o.b0 = push(model_.f64(prefix + ".mlp_rbf.0.bias", {F}));
    o.w1 = push(model_.f64(prefix + ".mlp_rbf.mlp_rbf_layer_1.0.weight", {F, F}));
    o.b1 = push(model_.f64(prefix + ".mlp_rbf.mlp_rbf_layer_1.0.bias", {F}));
    o.v0 = push(model_.f64(prefix + ".mlp_ev.0.weight", {H, 4}));
    o.c0 = push(model_.f64(prefix + ".mlp_ev.0.bias", {H}));
    o.v1 = push(model_.f64(prefix + ".mlp_ev.mlp_ev_layer_1.0.weight", {F, H}));
    o.c1 = push(model_.f64(prefix + ".mlp_ev.mlp_ev_layer_1.0.bias", {F}));
    return o;
  };
  for (int b = 0; b < layers_; ++b) {
    const std::string blk = "model.euclidean_transformers." + std::to_string(b);
    const std::string att = blk + ".euclidean_attention_block.";
    BOff &o = boff[b];
    // the attention block carries byte-identical copies of the block's filters;
    // the block-level tensors are the ones the reference kernels load
    o.finv = filt(blk + ".filter_net_inv");
    o.fev = filt(blk + ".filter_net_ev");
    o.cg_att = push(model_.f64(att + "so3_conv_invariants.cg_rep", {kEV}));
    o.cg_int = push(model_.f64(blk + ".interaction_block.so3_conv_invariants.cg_rep", {kEV}));
    static const char *names[5] = {"W_q_inv", "W_k_inv", "W_v_inv", "W_q_ev", "W_k_ev"};
    std::vector<std::vector<double>> w(5);
    for (int p = 0; p < 5; ++p) w[p] = model_.f64(att + names[p], {4, 32, 32});  // [head][in][out]
    std::vector<double> qf(4 * 160 * 32), qr(4 * 32 * 160);
    for (int h = 0; h < 4; ++h)
      for (int p = 0; p < 5; ++p)
        for (int i = 0; i < 32; ++i)
          for (int oo = 0; oo < 32; ++oo) {
            const double v = w[p][(h * 32 + i) * 32 + oo];
            qf[(h * 160 + p * 32 + oo) * 32 + i] = v;
            qr[(h * 32 + i) * 160 + p * 32 + oo] = v;
          }
    o.qf = push(qf);
    o.qr = push(qr);
    o.ln1w = push(model_.f64(blk + ".layer_norm_inv_1.weight", {F}));
    o.ln1b = push(model_.f64(blk + ".layer_norm_inv_1.bias", {F}));
    o.ln2w = push(model_.f64(blk + ".layer_norm_inv_2.weight", {F}));
    o.ln2b = push(model_.f64(blk + ".layer_norm_inv_2.bias", {F}));
    o.m1w = push(model_.f64(blk + ".mlp_1.1.weight", {F, F}));
    o.m1b = push(model_.f64(blk + ".mlp_1.1.bias", {F}));
    o.m2w = push(model_.f64(blk + ".mlp_1.3.weight", {F, F}));
    o.m2b = push(model_.f64(blk + ".mlp_1.3.bias", {F}));
    const auto iw = model_.f64(blk + ".interaction_block.linear_layer.weight", {132, 132});
    const auto ib = model_.f64(blk + ".interaction_block.linear_layer.bias", {132});
    std::vector<double> iwp(kIntW * kIntW, 0.0), ibp(kIntW, 0.0);
    for (int r = 0; r < 132; ++r) {
      ibp[r] = ib[r];
      for (int c = 0; c < 132; ++c) iwp[r * kIntW + c] = iw[r * 132 + c];
    }
    o.iw = push(iwp);
    o.ib = push(ibp);
  }
  // heads
  const std::string eo = "model.atomic_energy_output_block.", co = "model.partial_charges_output_block.",
                    ho = "model.hirshfeld_output_block.";
  std::vector<double> w1cat, b1cat;
  for (auto &part : {model_.f64(eo + "layers.0.weight", {128, F}), model_.f64(co + "transform_inv_features.0.weight", {128, F}),
                     model_.f64(ho + "transform_features.0.weight", {64, F})})
    w1cat.insert(w1cat.end(), part.begin(), part.end());
  for (auto &part : {model_.f64(eo + "layers.0.bias", {128}), model_.f64(co + "transform_inv_features.0.bias", {128}),
                     model_.f64(ho + "transform_features.0.bias", {64})})
    b1cat.insert(b1cat.end(), part.begin(), part.end());
  const std::size_t o_w1cat = push(w1cat), o_b1cat = push(b1cat);
  const std::size_t o_ew2 = push(model_.f64(eo + "final_layer.weight", {1, 128}));
  const double e_b2 = model_.f64(eo + "final_layer.bias", {1})[0];
  const std::size_t o_escale = push(model_.f64(eo + "energy_scales.weight", {1, 118}));
  const std::size_t o_eshift = push(model_.f64(eo + "energy_shifts", {118}));
  const std::size_t o_cw2 = push(model_.f64(co + "transform_inv_features.2.weight", {1, 128}));
  const double c_b2 = model_.f64(co + "transform_inv_features.2.bias", {1})[0];
  const std::size_t o_cemb = push(model_.f64(co + "atomic_embedding.weight", {100, 1}));
  const std::size_t o_hw2 = push(model_.f64(ho + "transform_features.2.weight", {64, 64}));
  const std::size_t o_hb2 = push(model_.f64(ho + "transform_features.2.bias", {64}));
  const std::size_t o_hq = push(model_.f64(ho + "q_embedding.weight", {100, 64}));
  const std::size_t o_hv = push(model_.f64(ho + "v_shift_embedding.weight", {100, 1}));
  const std::size_t o_emb = push(model_.f64("model.inv_feature_embedding.embedding.weight", {F, 118}));
  const std::size_t o_rb = push(model_.f64("model.radial_embedding.radial_basis_fn.b", {R}));
  std::vector<double> kd, krd;
  for (auto v : model_.i64("model.radial_embedding.radial_basis_fn.k")) kd.push_back(double(v));
  for (auto v : model_.i64("model.radial_embedding.radial_basis_fn.k_rev")) krd.push_back(double(v));
  if (kd.size() != R || krd.size() != R) throw Error("SO3LR model: Bernstein order tensors have the wrong size");
  const std::size_t o_rk = push(kd), o_rkr = push(krd);
  const auto &ta = model_.tensor("physical.reference_alphas");
  if (ta.shape.size() != 1 || ta.shape[0] < 8) throw Error("SO3LR model: physical reference tables changed");
  ref_table_ = int(ta.shape[0]);
  const std::size_t o_alpha = push(model_.f64("physical.reference_alphas", {std::size_t(ref_table_)}));
  const std::size_t o_c6 = push(model_.f64("physical.reference_c6", {std::size_t(ref_table_)}));

  double *d = wbuf_.reserve(host.size());
  SO3_CUDA(cudaMemcpy(d, host.data(), host.size() * sizeof(double), cudaMemcpyHostToDevice));
  auto P = [&](std::size_t off) { return static_cast<const double *>(d + off); };
  blocks_.resize(layers_);
  for (int b = 0; b < layers_; ++b) {
    const BOff &o = boff[b];
    BlockW &w = blocks_[b];
    auto fw = [&](const FOff &f) {
      return FilterW{P(f.w0), P(f.b0), P(f.w1), P(f.b1), P(f.v0), P(f.c0), P(f.v1), P(f.c1)};
    };
    w.finv = fw(o.finv);
    w.fev = fw(o.fev);
    w.cg_att = P(o.cg_att);
    w.cg_int = P(o.cg_int);
    w.qkv_fwd = P(o.qf);
    w.qkv_rev = P(o.qr);
    w.ln1w = P(o.ln1w); w.ln1b = P(o.ln1b); w.ln2w = P(o.ln2w); w.ln2b = P(o.ln2b);
    w.mlp1w = P(o.m1w); w.mlp1b = P(o.m1b); w.mlp2w = P(o.m2w); w.mlp2b = P(o.m2b);
    w.intw = P(o.iw); w.intb = P(o.ib);
  }
  heads_.w1cat = P(o_w1cat);
  heads_.b1cat = P(o_b1cat);
  heads_.e_w2 = P(o_ew2);
  heads_.e_b2 = e_b2;
  heads_.e_scale = P(o_escale);
  heads_.e_shift = P(o_eshift);
  heads_.c_w2 = P(o_cw2);
  heads_.c_b2 = c_b2;
  heads_.c_emb = P(o_cemb);
  heads_.h_w2 = P(o_hw2);
  heads_.h_b2 = P(o_hb2);
  heads_.h_qemb = P(o_hq);
  heads_.h_vshift = P(o_hv);
  emb_w_ = P(o_emb);
  rad_.b = P(o_rb);
  rad_.k = P(o_rk);
  rad_.kr = P(o_rkr);
  rad_.gamma = model_.f64("model.radial_embedding.radial_basis_fn.gamma", {})[0];
  alpha_ref_ = P(o_alpha);
  c6_ref_ = P(o_c6);
  const ZblParams z = model_.zbl();
  zbl_.ke = z.ke; zbl_.cutoff = z.cutoff; zbl_.switch_off = z.switch_off; zbl_.p = z.p; zbl_.d = z.d;
  for (int k = 0; k < 4; ++k) { zbl_.a[k] = z.a[k]; zbl_.c[k] = z.c[k]; }
  const LongRangeParams l = model_.long_range();
  lr_.ke = l.ke; lr_.sigma = l.sigma; lr_.cutoff = l.cutoff; lr_.elec_cuton = l.elec_cuton;
  lr_.disp_cuton = l.disp_cuton; lr_.bohr = l.bohr; lr_.hartree = l.hartree; lr_.disp_scale = l.disp_scale;
  lr_.full_scale = 2.0 * l.pair_scale;
  lr_.fine_factor = std::pow(l.fine_structure, -4.0 / 21.0);
  const double ratio = l.cutoff / l.sigma;
  const double cerf = std::erf(ratio), cexp = std::exp(-(ratio * ratio));
  constexpr double inv_sqrt_pi = 0.56418958354775628695;
  lr_.shift = cerf / l.cutoff;
  lr_.fshift = (2.0 * l.cutoff * cexp * inv_sqrt_pi / l.sigma - cerf) / (l.cutoff * l.cutoff);
}

// ---------------------------------------------------------------------------
// system preparation
// ---------------------------------------------------------------------------
void Evaluator::prepare(const SystemSpec &spec_in) {
  SO3_CUDA(cudaSetDevice(device_));
  SystemSpec spec = spec_in;
  const int n = spec.n;
  if (n <= 0) throw Error("SO3LR: the system has no atoms");
  if (int(spec.z.size()) != n) throw Error("SO3LR: atomic-number array has the wrong length");
  for (int zz : spec.z)
    if (zz < 1 || zz > 99) throw Error("SO3LR: atomic number " + std::to_string(zz) + " outside 1..99");
  if (spec.image_start.empty()) spec.image_start = {0, n};
  const int nimg = int(spec.image_start.size()) - 1;
  if (spec.image_start.front() != 0 || spec.image_start.back() != n) throw Error("SO3LR: image offsets must span 0..N");
  for (int i = 0; i < nimg; ++i)
    if (spec.image_start[i + 1] <= spec.image_start[i]) throw Error("SO3LR: every image needs at least one atom");
  if (spec.image_charge.empty()) spec.image_charge.assign(nimg, 0.0);
  if (spec.image_mult.empty()) spec.image_mult.assign(nimg, 1.0);
  if (int(spec.image_charge.size()) != nimg || int(spec.image_mult.size()) != nimg)
    throw Error("SO3LR: per-image charge/multiplicity arrays have the wrong length");
  if (spec.periodic) {
    if (nimg != 1) throw Error("SO3LR: batched images must be non-periodic");
    for (int d = 0; d < 3; ++d)
      if (!(spec.len[d] > 0.0)) throw Error("SO3LR: periodic box lengths must be positive");
  } else {
    for (int i = 0; i < nimg; ++i)
      if (spec.image_start[i + 1] - spec.image_start[i] > 20000)
        throw Error("SO3LR: open-boundary images are limited to 20000 atoms; use a periodic box with vacuum");
  }

  // charge / spin tables, cached by (composition, Q, M)
  std::vector<int> table_of_atom(n, -1), image_of(n);
  std::vector<double> tables;
  std::map<std::vector<std::int64_t>, int> cache;
  any_charge_spin_ = false;
  for (int im = 0; im < nimg; ++im) {
    std::array<std::int64_t, 119> counts{};
    for (int i = spec.image_start[im]; i < spec.image_start[im + 1]; ++i) {
      counts[spec.z[i]]++;
      image_of[i] = im;
    }
    const double Q = spec.image_charge[im], M = spec.image_mult[im];
    const std::string problem = charge_multiplicity_problem(counts, Q, M);
    if (!problem.empty()) throw Error("SO3LR charge/multiplicity: " + problem);
    if (Q == 0.0 && M == 1.0) continue;
    std::vector<std::int64_t> key(counts.begin(), counts.end());
    key.push_back(std::int64_t(Q));
    key.push_back(std::int64_t(M));
    int tab;
    auto it = cache.find(key);
    if (it == cache.end()) {
      const auto t = charge_spin_table(model_, counts, Q, M - 1.0);
      tab = int(cache.size());
      cache.emplace(key, tab);
      tables.insert(tables.end(), t.begin(), t.end());
    } else {
      tab = it->second;
    }
    for (int i = spec.image_start[im]; i < spec.image_start[im + 1]; ++i) table_of_atom[i] = tab;
    any_charge_spin_ = true;
  }
  spec_ = spec;
  alloc_atoms();
  SO3_CUDA(cudaMemcpyAsync(z_.reserve(n), spec.z.data(), sizeof(int) * n, cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(image_of_.reserve(n), image_of.data(), sizeof(int) * n, cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(image_start_.reserve(nimg + 1), spec.image_start.data(), sizeof(int) * (nimg + 1),
                           cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(image_charge_.reserve(nimg), spec.image_charge.data(), sizeof(double) * nimg,
                           cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(table_of_atom_.reserve(n), table_of_atom.data(), sizeof(int) * n, cudaMemcpyHostToDevice,
                           stream_));
  if (any_charge_spin_) {
    SO3_CUDA(cudaMemcpyAsync(cs_tables_.reserve(tables.size()), tables.data(), sizeof(double) * tables.size(),
                             cudaMemcpyHostToDevice, stream_));
  }
  // cell grid: cells no smaller than the short-range cutoff
  CellGrid g;
  g.periodic = spec.periodic ? 1 : 0;
  for (int d = 0; d < 3; ++d) {
    g.lo[d] = spec.lo[d];
    g.len[d] = spec.periodic ? spec.len[d] : 1.0;
    g.ncell[d] = spec.periodic ? std::max(1, int(std::floor(spec.len[d] / sr_cut_))) : 1;
  }
  const long long ncells = (long long)g.ncell[0] * g.ncell[1] * g.ncell[2];
  if (ncells > (1 << 26)) throw Error("SO3LR: periodic box is too large for the cell grid");
  nb_.grid = g;
  nb_.xw = xw_.reserve(3 * std::size_t(n));
  nb_.cell = cell_.reserve(n);
  nb_.cell_count = cell_count_.reserve(ncells);
  nb_.cell_start = cell_start_.reserve(ncells + 1);
  nb_.cell_fill = cell_fill_.reserve(ncells);
  nb_.cell_atoms = cell_atoms_.reserve(n);
  nb_.image_of = image_of_.get();
  nb_.image_start = image_start_.get();
  nb_.deg = deg_.reserve(n);
  nb_.row_start = row_start_.reserve(n + 1);
  nb_.scan_scratch = scan_scratch_.reserve(scan_scratch_ints(std::max<long long>(ncells, 64LL * n)));
  nb_.scan_total = small_ints_.reserve(16);
  nb_.error_flag = nb_.scan_total + 4;
  {
    const int seg[4] = {0, nimg, 0, n};  // [6..7]: image-energy segment, [8..9]: atom segment
    SO3_CUDA(cudaMemcpyAsync(nb_.scan_total + 6, seg, sizeof(seg), cudaMemcpyHostToDevice, stream_));
  }
  SO3_CUDA(cudaStreamSynchronize(stream_));
}

void Evaluator::alloc_atoms() {
  const std::size_t n = std::size_t(spec_.n);
  const int nimg = int(spec_.image_start.size()) - 1;
  auto ensure_vec = [&](std::vector<std::unique_ptr<DeviceArray<double>>> &v, int count, std::size_t elems) {
    while (int(v.size()) < count) v.emplace_back(new DeviceArray<double>());
    for (int i = 0; i < count; ++i) v[i]->reserve(elems);
  };
  x_.reserve(3 * n);
  force_.reserve(3 * n);
  ensure_vec(xb_, layers_ + 1, n * kF);
  ensure_vec(evb_, layers_ + 1, n * kEV);
  ensure_vec(qkv_, layers_, n * kQKV);
  ensure_vec(xhat1_, layers_, n * kF);
  ensure_vec(rstd1_, layers_, n);
  ensure_vec(n1_, layers_, n * kF);
  ensure_vec(A_, layers_, n * kEV);
  ensure_vec(hp_, layers_, n * kF);
  ensure_vec(gate_, layers_, n * 4);
  ensure_vec(xhat2_, layers_, n * kF);
  ensure_vec(rstd2_, layers_, n);
  d_inv_.reserve(n * kF);
  d_ev_.reserve(n * kEV);
  act_.reserve(n * kF);
  cat_.reserve(n * kIntW);
  t_.reserve(n * kIntW);
  hpre_.reserve(n * kHeadCat);
  hcat_.reserve(n * kHeadCat);
  hk_.reserve(n * kHirsh);
  e_nn_.reserve(n);
  raw_q_.reserve(n);
  q_.reserve(n);
  ratio_.reserve(n);
  e_lr_.reserve(n);
  e_elec_.reserve(n);
  e_disp_.reserve(n);
  dq_.reserve(n);
  dh_.reserve(n);
  f_lr_.reserve(3 * n);
  lr_pos4_.reserve(4 * n);
  lr_par4_.reserve(4 * n);
  w_lr_.reserve(6 * n);
  img_sums_.reserve(nimg + 1);
  dq_mean_.reserve(nimg + 1);
  g_hcat_.reserve(n * kHeadCat);
  g_x_.reserve(n * kF);
  g_x2_.reserve(n * kF);
  g_ev_.reserve(n * kEV);
  g_ev2_.reserve(n * kEV);
  g_t_.reserve(n * kIntW);
  g_cat_.reserve(n * kIntW);
  g_hp_.reserve(n * kF);
  g_n1_.reserve(n * kF);
  g_a_.reserve(n * kF);
  g_A_.reserve(n * kEV);
  g_qkv_.reserve(n * kQKV);
  e_atom_.reserve(n);
  e_zbl_.reserve(n);
  w_atom_.reserve(6 * n);
  totals_.reserve(8);
  image_energy_.reserve(nimg);
}

void Evaluator::upload_positions(const double *host_x) {
  SO3_CUDA(cudaSetDevice(device_));
  SO3_CUDA(cudaMemcpyAsync(x_.get(), host_x, sizeof(double) * 3 * spec_.n, cudaMemcpyHostToDevice, stream_));
}

std::size_t Evaluator::device_bytes() const {
  std::size_t total = wbuf_.bytes() + geo_.bytes() + sh_.bytes() + gv_.bytes() + gl0_.bytes() + pair_sc_.bytes();
  for (auto &v : f_inv_) total += v->bytes();
  for (auto &v : f_ev_) total += v->bytes();
  for (auto *vec : {&xb_, &evb_, &qkv_, &xhat1_, &rstd1_, &n1_, &A_, &hp_, &gate_, &xhat2_, &rstd2_})
    for (auto &v : *vec) total += v->bytes();
  total += nbr_.bytes() * 8;
  return total;
}

// ---------------------------------------------------------------------------
// kernel timing (CUDA events on the launching stream)
// ---------------------------------------------------------------------------
void Evaluator::prof_begin(int k) {
  if (!profiling_) return;
  KernelProfile &p = prof_[k];
  if (p.used + 2 > int(p.events.size())) {
    for (int i = 0; i < 64; ++i) {
      cudaEvent_t ev;
      SO3_CUDA(cudaEventCreate(&ev));
      p.events.push_back(ev);
    }
  }
  SO3_CUDA(cudaEventRecord(p.events[p.used], stream_));
}
void Evaluator::prof_end(int k, double flops) {
  if (!profiling_) return;
  KernelProfile &p = prof_[k];
  SO3_CUDA(cudaEventRecord(p.events[p.used + 1], stream_));
  p.used += 2;
  p.launches += 1;
  p.flops += flops;
}
void Evaluator::read_profile(int k, double *ms, long long *launches, double *flops) {
  if (k < 0 || k > 1) throw Error("SO3LR: unknown profiled kernel");
  SO3_CUDA(cudaStreamSynchronize(stream_));
  KernelProfile &p = prof_[k];
  double total = 0;
  for (int i = 0; i < p.used; i += 2) {
    float t = 0;
    SO3_CUDA(cudaEventElapsedTime(&t, p.events[i], p.events[i + 1]));
    total += t;
  }
  if (ms) *ms = total;
  if (launches) *launches = p.launches;
  if (flops) *flops = p.flops;
  p.used = 0;
  p.launches = 0;
  p.flops = 0;
}

// ---------------------------------------------------------------------------
// neighbour lists
// ---------------------------------------------------------------------------
void Evaluator::build_neighbors() {
  const int n = spec_.n;
  build_cells(nb_, n, x_.get(), stream_);
  count_sr(nb_, n, sr_cut_, stream_);
  SO3_CUDA(cudaMemcpyAsync(host_small_, nb_.row_start + n, sizeof(int), cudaMemcpyDeviceToHost, stream_));
  SO3_CUDA(cudaStreamSynchronize(stream_));
  const int E = host_small_[0];
  if (E < 0) throw Error("SO3LR: edge count overflow");
  if (E % 2 != 0) throw Error("SO3LR: short-range list is not symmetric");
  const int P = E / 2;
  stats_.edges = E;
  stats_.pairs = P;
  nb_.nbr = nbr_.reserve(E, 1.25);
  nb_.img = img_.reserve(E, 1.25);
  nb_.primary = primary_.reserve(E, 1.25);
  nb_.rev = rev_.reserve(E, 1.25);
  nb_.pair_scan = pair_scan_.reserve(E, 1.25);
  nb_.edge_pair = edge_pair_.reserve(E, 1.25);
  nb_.pair_a = pair_a_.reserve(P, 1.25);
  nb_.pair_b = pair_b_.reserve(P, 1.25);
  nb_.pair_img = pair_img_.reserve(P, 1.25);
  nb_.pair_edge = pair_edge_.reserve(P, 1.25);
  if (scan_scratch_.capacity() < scan_scratch_ints(std::size_t(E) + 1)) {
    nb_.scan_scratch = scan_scratch_.reserve(scan_scratch_ints(std::size_t(E) * 2 + 1));
  }
  SO3_CUDA(cudaMemsetAsync(nb_.error_flag, 0, sizeof(int), stream_));
  fill_sr(nb_, n, sr_cut_, E, stream_);
  fill_pairs(nb_, n, E, stream_);
  // per-pair storage
  geo_.reserve(std::size_t(P) * kGeo, 1.25);
  sh_.reserve(std::size_t(P) * kEV, 1.25);
  gv_.reserve(std::size_t(P) * 3, 1.25);
  gl0_.reserve(std::size_t(P) * 4, 1.25);
  pair_sc_.reserve(std::size_t(P) * kPairScalars, 1.25);
  g_filt_inv_.reserve(std::size_t(P) * kF, 1.25);
  g_filt_ev_.reserve(std::size_t(P) * kF, 1.25);
  while (int(f_inv_.size()) < layers_) {
    f_inv_.emplace_back(new DeviceArray<double>());
    f_ev_.emplace_back(new DeviceArray<double>());
  }
  for (int b = 0; b < layers_; ++b) {
    f_inv_[b]->reserve(std::size_t(P) * kF, 1.25);
    f_ev_[b]->reserve(std::size_t(P) * kF, 1.25);
  }
}

// ---------------------------------------------------------------------------
// the evaluation
// ---------------------------------------------------------------------------
void Evaluator::compute() {
  SO3_CUDA(cudaSetDevice(device_));
  const int n = spec_.n;
  const int nimg = int(spec_.image_start.size()) - 1;
  cudaStream_t s = stream_;
  build_neighbors();
  const int P = int(stats_.pairs);
  launch_pair_geometry(P, nb_, z_.get(), zbl_, sr_cut_, geo_.get(), sh_.get(), gv_.get(), s);
  launch_embedding(n, z_.get(), emb_w_, any_charge_spin_ ? cs_tables_.get() : nullptr, table_of_atom_.get(),
                   inv_emb_scale_, xb_[0]->get(), s);
  SO3_CUDA(cudaMemsetAsync(evb_[0]->get(), 0, sizeof(double) * n * kEV, s));

  for (int b = 0; b < layers_; ++b) {
    const BlockW &w = blocks_[b];
    prof_begin(0);
    launch_filter_forward(P, geo_.get(), nb_.pair_a, nb_.pair_b, b == 0 ? nullptr : evb_[b]->get(), w.cg_att, w.finv,
                          w.fev, rad_, f_inv_[b]->get(), f_ev_[b]->get(), s);
    prof_end(0, kFilterFlopsPerPair * double(P));
    {  // per-head projections: qkv[n][h][5][32] = x[n][h*32:(h+1)*32] W_h
      GemmArgs g{};
      g.M = n; g.N = 160; g.K = 32;
      g.A = xb_[b]->get(); g.lda = kF; g.strideA = 32;
      g.W = w.qkv_fwd; g.ldw = 32; g.transB = true; g.strideW = 160 * 32;
      g.C = qkv_[b]->get(); g.ldc = kQKV; g.strideC = 160;
      g.batch = 4;
      launch_gemm(g, s);
    }
    launch_attention_forward(n, nb_, geo_.get(), sh_.get(), qkv_[b]->get(), f_inv_[b]->get(), f_ev_[b]->get(), norm_,
                             d_inv_.get(), d_ev_.get(), s);
    launch_post_attn_pre(n, xb_[b]->get(), d_inv_.get(), evb_[b]->get(), d_ev_.get(), w.ln1w, w.ln1b, w.cg_int,
                         xhat1_[b]->get(), rstd1_[b]->get(), n1_[b]->get(), act_.get(), A_[b]->get(), cat_.get(), s);
    {  // hidden = silu(act W1^T + b1), pre-activation kept for the reverse
      GemmArgs g{};
      g.M = n; g.N = kF; g.K = kF;
      g.A = act_.get(); g.lda = kF;
      g.W = w.mlp1w; g.ldw = kF; g.transB = true;
      g.C = d_inv_.get(); g.ldc = kF;  // reuse d_inv as the hidden activation
      g.bias = w.mlp1b; g.aux_out = hp_[b]->get(); g.ldaux = kF;
      g.epi = Epi::BiasStorePre;
      launch_gemm(g, s);
    }
    {  // post = n1 + hidden W2^T + b2  -> cat[:, :128]
      GemmArgs g{};
      g.M = n; g.N = kF; g.K = kF;
      g.A = d_inv_.get(); g.lda = kF;
      g.W = w.mlp2w; g.ldw = kF; g.transB = true;
      g.C = cat_.get(); g.ldc = kIntW;
      g.bias = w.mlp2b; g.aux = n1_[b]->get(); g.ldaux = kF;
      g.epi = Epi::BiasResidual;
      launch_gemm(g, s);
    }
    {  // t = [post, L0'] W_int^T + b_int
      GemmArgs g{};
      g.M = n; g.N = kIntW; g.K = kIntW;
      g.A = cat_.get(); g.lda = kIntW;
      g.W = w.intw; g.ldw = kIntW; g.transB = true;
      g.C = t_.get(); g.ldc = kIntW;
      g.bias = w.intb;
      g.epi = Epi::Bias;
      launch_gemm(g, s);
    }
    launch_post_attn_final(n, cat_.get(), t_.get(), A_[b]->get(), w.ln2w, w.ln2b, xhat2_[b]->get(), rstd2_[b]->get(),
                           gate_[b]->get(), xb_[b + 1]->get(), evb_[b + 1]->get(), s);
  }

  // ---- output heads --------------------------------------------------------
  {
    GemmArgs g{};
    g.M = n; g.N = kHeadCat; g.K = kF;
    g.A = xb_[layers_]->get(); g.lda = kF;
    g.W = heads_.w1cat; g.ldw = kF; g.transB = true;
    g.C = hcat_.get(); g.ldc = kHeadCat;
    g.bias = heads_.b1cat; g.aux_out = hpre_.get(); g.ldaux = kHeadCat;
    g.epi = Epi::BiasStorePre;
    launch_gemm(g, s);
  }
  launch_heads_finalize(n, z_.get(), hcat_.get(), heads_, hk_.get(), e_nn_.get(), raw_q_.get(), ratio_.get(), s);
  launch_segment_sum(nimg, image_start_.get(), raw_q_.get(), 1, 1, img_sums_.get(), s);
  launch_charge_correct(n, raw_q_.get(), img_sums_.get(), image_charge_.get(), image_of_.get(), image_start_.get(),
                        q_.get(), nullptr, nullptr, s);

  // ---- long range ----------------------------------------------------------
  launch_long_range(n, nb_, lr_cut_, z_.get(), q_.get(), ratio_.get(), alpha_ref_, c6_ref_, ref_table_, lr_,
                    reinterpret_cast<double4 *>(lr_pos4_.get()), reinterpret_cast<double4 *>(lr_par4_.get()),
                    e_lr_.get(), e_elec_.get(), e_disp_.get(), dq_.get(), dh_.get(), f_lr_.get(), w_lr_.get(), s);
  launch_segment_sum(nimg, image_start_.get(), dq_.get(), 1, 1, img_sums_.get(), s);
  launch_charge_correct(nimg, nullptr, nullptr, nullptr, nullptr, image_start_.get(), nullptr, dq_mean_.get(),
                        img_sums_.get(), s);

  // ---- reverse ---------------------------------------------------------------
  launch_heads_seed(n, z_.get(), hpre_.get(), hk_.get(), heads_, dq_.get(), dq_mean_.get(), image_of_.get(),
                    dh_.get(), g_hcat_.get(), s);
  {
    GemmArgs g{};
    g.M = n; g.N = kF; g.K = kHeadCat;
    g.A = g_hcat_.get(); g.lda = kHeadCat;
    g.W = heads_.w1cat; g.ldw = kF; g.transB = false;
    g.C = g_x_.get(); g.ldc = kF;
    launch_gemm(g, s);
  }
  double *gx = g_x_.get(), *gx_next = g_x2_.get();
  double *gev = nullptr, *gev_next = g_ev_.get();
  for (int b = layers_ - 1; b >= 0; --b) {
    const BlockW &w = blocks_[b];
    launch_post_attn_rev_final(n, gx, gev, xhat2_[b]->get(), rstd2_[b]->get(), w.ln2w, A_[b]->get(), gate_[b]->get(),
                               g_t_.get(), g_A_.get(), s);
    {  // g_cat = g_t W_int; g_post = g_cat[:, :128] + g_t[:, :128]
      GemmArgs g{};
      g.M = n; g.N = kIntW; g.K = kIntW;
      g.A = g_t_.get(); g.lda = kIntW;
      g.W = w.intw; g.ldw = kIntW; g.transB = false;
      g.C = g_cat_.get(); g.ldc = kIntW;
      g.aux = g_t_.get(); g.ldaux = kIntW;
      g.epi = Epi::AddResidual;
      launch_gemm_ex(g, kF, 0, s);
    }
    {  // g_hp = (g_post W2) * silu'(hp)
      GemmArgs g{};
      g.M = n; g.N = kF; g.K = kF;
      g.A = g_cat_.get(); g.lda = kIntW;
      g.W = w.mlp2w; g.ldw = kF; g.transB = false;
      g.C = g_hp_.get(); g.ldc = kF;
      g.aux = hp_[b]->get(); g.ldaux = kF;
      g.epi = Epi::SiluPrimeMul;
      launch_gemm(g, s);
    }
    {  // g_n1 = g_post + (g_hp W1) * silu'(n1)
      GemmArgs g{};
      g.M = n; g.N = kF; g.K = kF;
      g.A = g_hp_.get(); g.lda = kF;
      g.W = w.mlp1w; g.ldw = kF; g.transB = false;
      g.C = g_n1_.get(); g.ldc = kF;
      g.aux = n1_[b]->get(); g.ldaux = kF;
      g.aux2 = g_cat_.get();
      g.epi = Epi::GateSiluResidual;
      launch_gemm_ex(g, kF, kIntW, s);
    }
    launch_post_attn_rev_ln1(n, g_n1_.get(), xhat1_[b]->get(), rstd1_[b]->get(), w.ln1w, A_[b]->get(), w.cg_int,
                             g_cat_.get(), g_a_.get(), g_A_.get(), s);
    launch_attention_reverse(n, nb_, geo_.get(), sh_.get(), qkv_[b]->get(), f_inv_[b]->get(), f_ev_[b]->get(),
                             g_a_.get(), g_A_.get(), norm_, b > 0 ? g_qkv_.get() : nullptr, pair_sc_.get(),
                             g_filt_inv_.get(), g_filt_ev_.get(), s);
    prof_begin(1);
    launch_filter_reverse(P, geo_.get(), nb_.pair_a, nb_.pair_b, b > 0 ? evb_[b]->get() : nullptr, w.cg_att, w.finv,
                          w.fev, rad_, g_filt_inv_.get(), g_filt_ev_.get(), g_A_.get(), pair_sc_.get(), b > 0,
                          gv_.get(), gl0_.get(), s);
    prof_end(1, kFilterFlopsPerPair * double(P));
    if (b > 0) {
      GemmArgs g{};  // g_x_in = g_a + per-head (g_qkv W^T)
      g.M = n; g.N = 32; g.K = 160;
      g.A = g_qkv_.get(); g.lda = kQKV; g.strideA = 160;
      g.W = w.qkv_rev; g.ldw = 160; g.transB = true; g.strideW = 32 * 160;
      g.C = gx_next; g.ldc = kF; g.strideC = 32;
      g.aux = g_a_.get(); g.ldaux = kF; g.strideAux = 32;
      g.epi = Epi::AddResidual;
      g.batch = 4;
      launch_gemm(g, s);
      launch_ev_l0_reverse(n, nb_, evb_[b]->get(), w.cg_att, gl0_.get(), g_A_.get(), gev_next, s);
      std::swap(gx, gx_next);
      gev = gev_next;
      gev_next = (gev == g_ev_.get()) ? g_ev2_.get() : g_ev_.get();
    }
  }

  // ---- assembly --------------------------------------------------------------
  launch_assemble(n, nb_, geo_.get(), gv_.get(), e_nn_.get(), e_lr_.get(), f_lr_.get(), w_lr_.get(), force_.get(),
                  e_atom_.get(), e_zbl_.get(), w_atom_.get(), s);
  launch_segment_sum(nimg, image_start_.get(), e_atom_.get(), 1, 1, image_energy_.get(), s);
  // virial: one segment [0, n) over atoms; energy: one segment [0, nimg) over image energies
  launch_segment_sum(1, small_ints_.get() + 8, w_atom_.get(), 6, 6, totals_.get() + 1, s);
  launch_segment_sum(1, small_ints_.get() + 6, image_energy_.get(), 1, 1, totals_.get(), s);
}

Evaluator::HostResult Evaluator::download(double *f, double *eatom, double *charges, double *ratios,
                                          double *e_learned, double *e_zbl, double *e_lr, double *e_elec,
                                          double *e_disp, double *image_energy) {
  SO3_CUDA(cudaSetDevice(device_));
  const int n = spec_.n;
  const int nimg = int(spec_.image_start.size()) - 1;
  cudaStream_t s = stream_;
  auto d2h = [&](double *dst, const double *src, std::size_t count) {
    if (dst) SO3_CUDA(cudaMemcpyAsync(dst, src, sizeof(double) * count, cudaMemcpyDeviceToHost, s));
  };
  d2h(f, force_.get(), 3 * std::size_t(n));
  d2h(eatom, e_atom_.get(), n);
  d2h(charges, q_.get(), n);
  d2h(ratios, ratio_.get(), n);
  d2h(e_learned, e_nn_.get(), n);
  d2h(e_zbl, e_zbl_.get(), n);
  d2h(e_lr, e_lr_.get(), n);
  d2h(e_elec, e_elec_.get(), n);
  d2h(e_disp, e_disp_.get(), n);
  d2h(image_energy, image_energy_.get(), nimg);
  SO3_CUDA(cudaMemcpyAsync(host_totals_, totals_.get(), sizeof(double) * 7, cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaMemcpyAsync(host_small_ + 8, nb_.error_flag, sizeof(int), cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaStreamSynchronize(s));
  if (host_small_[8] != 0) throw Error("SO3LR: short-range list has an edge without its reverse");
  HostResult r;
  r.energy = host_totals_[0];
  for (int k = 0; k < 6; ++k) r.virial[k] = host_totals_[1 + k];
  return r;
}

// ---------------------------------------------------------------------------
// device-resident MD (velocity Verlet, LAMMPS metal units: ftm2v = 1/1.0364269e-4)
// ---------------------------------------------------------------------------
void Evaluator::md_setup(const double *host_v, const double *host_mass) {
  SO3_CUDA(cudaSetDevice(device_));
  const int n = spec_.n;
  std::vector<double> inv(n);
  for (int i = 0; i < n; ++i) {
    if (!(host_mass[i] > 0)) throw Error("SO3LR MD: masses must be positive");
    inv[i] = 1.0 / host_mass[i];
  }
  SO3_CUDA(cudaMemcpyAsync(v_.reserve(3 * std::size_t(n)), host_v, sizeof(double) * 3 * n, cudaMemcpyHostToDevice,
                           stream_));
  SO3_CUDA(cudaMemcpyAsync(inv_mass_.reserve(n), inv.data(), sizeof(double) * n, cudaMemcpyHostToDevice, stream_));
  compute();  // forces at the starting positions
  SO3_CUDA(cudaStreamSynchronize(stream_));
}

void Evaluator::md_steps(int nsteps, double dt) {
  constexpr double ftm2v = 1.0 / 1.0364269e-4;
  const int n = spec_.n;
  for (int step = 0; step < nsteps; ++step) {
    launch_verlet_first(n, x_.get(), v_.get(), force_.get(), inv_mass_.get(), dt, ftm2v, stream_);
    compute();
    launch_verlet_second(n, v_.get(), force_.get(), inv_mass_.get(), dt, ftm2v, stream_);
  }
}

void Evaluator::md_download(double *x, double *v) {
  const int n = spec_.n;
  if (x) SO3_CUDA(cudaMemcpyAsync(x, x_.get(), sizeof(double) * 3 * n, cudaMemcpyDeviceToHost, stream_));
  if (v) SO3_CUDA(cudaMemcpyAsync(v, v_.get(), sizeof(double) * 3 * n, cudaMemcpyDeviceToHost, stream_));
  SO3_CUDA(cudaStreamSynchronize(stream_));
}

}  // namespace so3lr_b200
