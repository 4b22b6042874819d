#include "evaluator.hpp"

#include "nccl_dyn.hpp"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <numeric>
#include <sstream>

SO3LR_SHAPE_BEGIN

Evaluator::Evaluator(Model &&model, int device) : model_(std::move(model)), device_(device) {
  int count = 0;
  SO3_CUDA(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count) throw Error("SO3LR: CUDA device " + std::to_string(device) + " not available");
  SO3_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop{};
  SO3_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major < 10)
    throw Error(std::string("SO3LR: this library is built for sm_100a (B200); device is ") + prop.name);
  num_sms_ = prop.multiProcessorCount;
  // the mixed-precision filter kernels run on the tcgen05 tensor cores unless
  // SO3LR_B200_MIXED_FORWARD=mma selects the mma.sync kernels (for comparisons)
  const char *fwd = std::getenv("SO3LR_B200_MIXED_FORWARD");
  mixed_tc_ = !(fwd && std::string(fwd) == "mma");
  SO3_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  tc_err_ = tc_err_arr_.reserve(1);
  SO3_CUDA(cudaMemset(tc_err_, 0, sizeof(int)));
  SO3_CUDA(cudaMallocHost(&host_small_, 16 * sizeof(int)));
  SO3_CUDA(cudaMallocHost(&host_totals_, 16 * sizeof(double)));
  upload_weights();
}

Evaluator::~Evaluator() {
  if (stream_) {
    cudaSetDevice(device_);
    cudaStreamSynchronize(stream_);
    if (comm_) nccl().comm_destroy(comm_);
    for (auto &p : prof_)
      for (auto ev : p.events) cudaEventDestroy(ev);
    cudaStreamDestroy(stream_);
  }
  if (host_small_) cudaFreeHost(host_small_);
  if (host_halo_) cudaFreeHost(host_halo_);
  if (host_totals_) cudaFreeHost(host_totals_);
  if (host_rec_) cudaFreeHost(host_rec_);
}

// ---------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------
// A K x N matrix B(k, n) laid out as the B operand of m16n8k8 DMMA tiles 32
// columns wide. The kernels read the MMA's k slots t and t + 4 of k-step ks
// from columns 8 ks + 2t and 8 ks + 2t + 1 of their activation tiles, so lane
// (g = lane / 4, t = lane % 4) needs, for column slab s and column block ni,
// {B(8 ks + 2t, n), B(8 ks + 2t + 1, n)} with n = 32 s + 8 ni + g; its eight
// values of one k-step and slab are stored contiguously (one warp reads 2 KB of
// consecutive memory).
static std::vector<double> fragment_major(int K, int N, const std::function<double(int, int)> &B) {
  if (K % 8 != 0 || N % 32 != 0) throw Error("SO3LR: fragment-major operand needs K % 8 == 0 and N % 32 == 0");
  std::vector<double> out(std::size_t(K) * N);
  for (int k = 0; k < K; ++k)
    for (int n = 0; n < N; ++n) {
      const int ks = k / 8, t = (k % 8) / 2, h = k % 2, slab = n / 32, ni = (n % 32) / 8, g = n % 8;
      out[(((std::size_t(ks) * (N / 32) + slab) * 32 + (4 * g + t)) * 4 + ni) * 2 + h] = B(k, n);
    }
  return out;
}

// x rounded to TF32 (10 explicit mantissa bits), to nearest with ties away from
// zero, as cvt.rna.tf32.f32 rounds on the device
static float tf32_round(float x) {
  std::uint32_t u;
  std::memcpy(&u, &x, sizeof(u));
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
  std::memcpy(&x, &u, sizeof(u));
  return x;
}

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
  struct FOff { std::size_t w0, b0, w1, b1, v0, c0, v1, c1, bc1, w0t_f, w1t_f, v1t_f, w1_f, v1_f, w0_f; };
  // float copies for the mixed-precision filter kernels (FilterW32)
  std::vector<float> host32;
  auto push32 = [&](const std::vector<double> &v) {
    while (host32.size() % 16) host32.push_back(0.0f);  // 64-byte alignment
    const std::size_t off = host32.size();
    for (double x : v) host32.push_back(float(x));
    return off;
  };
  // a fragment-major operand as its TF32 high and low parts
  auto push_split = [&](const std::vector<double> &v) {
    std::vector<double> hi(v.size()), lo(v.size());
    for (std::size_t i = 0; i < v.size(); ++i) {
      const float h = tf32_round(float(v[i]));
      hi[i] = h;
      lo[i] = tf32_round(float(v[i] - double(h)));
    }
    const std::size_t a = push32(hi);
    const std::size_t b = push32(lo);
    return std::make_pair(a, b);
  };
  struct FOff32 {
    std::size_t b0, bc1, v0, c0;
    std::pair<std::size_t, std::size_t> w0t, w1t, v1t, w1, v1, w0;
    std::size_t tc_fwd, tc_rev;
  };
  // [128 x 32] K-chunk c of a row-major [128 x K] matrix as TF32 hi and lo tiles
  // in the 128-byte-swizzled K-major layout (row n, column k at byte
  // 1024 (n / 8) + 128 (n % 8) + 16 ((k / 4) xor (n % 8)) + 4 (k % 4))
  struct TcChunk {
    const std::vector<double> *m;  // row-major [rows x K]
    int rows, c;                   // rows (128 or 32) and K-chunk index
  };
  auto push_tc_chunks = [&](const std::vector<TcChunk> &chunks) {
    std::vector<double> all;
    for (const auto &ch : chunks) {
      const std::vector<double> &m = *ch.m;
      const int rows = ch.rows, K = int(m.size() / std::size_t(rows)), c = ch.c;
      std::vector<double> hi(std::size_t(rows) * 32), lo(std::size_t(rows) * 32);
      for (int n = 0; n < rows; ++n)
        for (int k = 0; k < 32; ++k) {
          const double v = m[std::size_t(n) * K + 32 * c + k];
          const float h = tf32_round(float(v));
          const std::size_t off = (n / 8) * 256 + (n % 8) * 32 + (((k / 4) ^ (n % 8)) * 4) + (k % 4);
          hi[off] = h;
          lo[off] = tf32_round(float(v - double(h)));
        }
      all.insert(all.end(), hi.begin(), hi.end());
      all.insert(all.end(), lo.begin(), lo.end());
    }
    while (host32.size() % 256) host32.push_back(0.0f);  // 1024-byte alignment
    const std::size_t off = host32.size();
    for (double x : all) host32.push_back(float(x));
    return off;
  };
  struct BOff {
    FOff finv, fev;
    std::size_t cg_att, cg_int, qf, qr, ln1w, ln1b, ln2w, ln2b, m1w, m1b, m2w, m2b, iw, ib;
  };
  std::vector<BOff> boff(layers_);
  std::vector<FOff32> foff32(2 * std::size_t(layers_));
  std::size_t filt_count = 0;  // filters in upload order: block 0 inv, ev, block 1 inv, ...
  struct FiltHost {
    std::vector<double> b0, bc1, v0, c0;
  };
  std::vector<FiltHost> filt_host(2 * std::size_t(layers_));
  auto filt = [&](const std::string &prefix) {
    FOff o;
    const auto w0 = model_.f64(prefix + ".mlp_rbf.0.weight", {F, R});                  // [j][r]
    const auto w1 = model_.f64(prefix + ".mlp_rbf.mlp_rbf_layer_1.0.weight", {F, F});  // [o][j]
    const auto v1 = model_.f64(prefix + ".mlp_ev.mlp_ev_layer_1.0.weight", {F, H});    // [o][h]
    o.w0 = push(w0);
    o.b0 = push(model_.f64(prefix + ".mlp_rbf.0.bias", {F}));
    o.w1 = push(w1);
    o.b1 = push(model_.f64(prefix + ".mlp_rbf.mlp_rbf_layer_1.0.bias", {F}));
    o.v0 = push(model_.f64(prefix + ".mlp_ev.0.weight", {H, std::size_t(kHeads)}));
    o.c0 = push(model_.f64(prefix + ".mlp_ev.0.bias", {H}));
    o.v1 = push(v1);
    const auto b1 = model_.f64(prefix + ".mlp_rbf.mlp_rbf_layer_1.0.bias", {F});
    const auto c1 = model_.f64(prefix + ".mlp_ev.mlp_ev_layer_1.0.bias", {F});
    o.c1 = push(c1);
    std::vector<double> bc1(F);
    for (std::size_t k = 0; k < F; ++k) bc1[k] = b1[k] + c1[k];
    o.bc1 = push(bc1);
    const int iF = int(F), iR = int(R), iH = int(H);
    o.w0t_f = push(fragment_major(iR, iF, [&](int r, int j) { return w0[std::size_t(j) * R + r]; }));
    o.w1t_f = push(fragment_major(iF, iF, [&](int j, int oo) { return w1[std::size_t(oo) * F + j]; }));
    o.v1t_f = push(fragment_major(iH, iF, [&](int h, int oo) { return v1[std::size_t(oo) * H + h]; }));
    o.w1_f = push(fragment_major(iF, iF, [&](int oo, int j) { return w1[std::size_t(oo) * F + j]; }));
    o.v1_f = push(fragment_major(iF, iH, [&](int oo, int h) { return v1[std::size_t(oo) * H + h]; }));
    o.w0_f = push(fragment_major(iF, iR, [&](int j, int r) { return w0[std::size_t(j) * R + r]; }));
    filt_host[filt_count] = {model_.f64(prefix + ".mlp_rbf.0.bias", {F}), bc1, model_.f64(prefix + ".mlp_ev.0.weight", {H, std::size_t(kHeads)}),
                             model_.f64(prefix + ".mlp_ev.0.bias", {H})};
    FOff32 &o32 = foff32[filt_count++];
    if (kF != 128) return o;  // the mixed-precision operands exist for F = 128 only
    o32.b0 = push32(model_.f64(prefix + ".mlp_rbf.0.bias", {F}));
    o32.bc1 = push32(bc1);
    o32.v0 = push32(model_.f64(prefix + ".mlp_ev.0.weight", {H, std::size_t(kHeads)}));
    o32.c0 = push32(model_.f64(prefix + ".mlp_ev.0.bias", {H}));
    o32.w0t = push_split(fragment_major(iR, iF, [&](int r, int j) { return w0[std::size_t(j) * R + r]; }));
    o32.w1t = push_split(fragment_major(iF, iF, [&](int j, int oo) { return w1[std::size_t(oo) * F + j]; }));
    o32.v1t = push_split(fragment_major(iH, iF, [&](int h, int oo) { return v1[std::size_t(oo) * H + h]; }));
    o32.w1 = push_split(fragment_major(iF, iF, [&](int oo, int j) { return w1[std::size_t(oo) * F + j]; }));
    o32.v1 = push_split(fragment_major(iF, iH, [&](int oo, int h) { return v1[std::size_t(oo) * H + h]; }));
    o32.w0 = push_split(fragment_major(iF, iR, [&](int j, int r) { return w0[std::size_t(j) * R + r]; }));
    o32.tc_fwd = push_tc_chunks({{&w0, 128, 0}, {&w1, 128, 0}, {&w1, 128, 1}, {&w1, 128, 2}, {&w1, 128, 3},
                                 {&v1, 128, 0}});
    // reverse operands: W1^T [j][o], V1^T [h][o], W0^T [r][j]
    std::vector<double> w1t(F * F), v1t(H * F), w0t(R * F);
    for (std::size_t o = 0; o < F; ++o)
      for (std::size_t j = 0; j < F; ++j) w1t[j * F + o] = w1[o * F + j];
    for (std::size_t o = 0; o < F; ++o)
      for (std::size_t h = 0; h < H; ++h) v1t[h * F + o] = v1[o * H + h];
    for (std::size_t j = 0; j < F; ++j)
      for (std::size_t r = 0; r < R; ++r) w0t[r * F + j] = w0[j * R + r];
    o32.tc_rev = push_tc_chunks({{&w1t, 128, 0}, {&v1t, 32, 0}, {&w1t, 128, 1}, {&v1t, 32, 1},
                                 {&w1t, 128, 2}, {&v1t, 32, 2}, {&w1t, 128, 3}, {&v1t, 32, 3},
                                 {&w0t, 32, 0}, {&w0t, 32, 1}, {&w0t, 32, 2}, {&w0t, 32, 3}});
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
    for (int p = 0; p < 5; ++p) w[p] = model_.f64(att + names[p], {std::size_t(kHeads), 32, 32});  // [head][in][out]
    std::vector<double> qf(kHeads * 160 * 32), qr(kHeads * 32 * 160);
    for (int h = 0; h < kHeads; ++h)
      for (int p = 0; p < 5; ++p)
        for (int i = 0; i < 32; ++i)
          for (int oo = 0; oo < 32; ++oo) {
            const double v = w[p][(h * 32 + i) * 32 + oo];
            qf[(h * 160 + p * 32 + oo) * 32 + i] = v;
            qr[(h * 32 + i) * 160 + p * 32 + oo] = v;
          }
    o.qf = push(qf);
    o.qr = push(qr);
    // only an affine LayerNorm has parameters (post_attention_block0.cpp:395-424)
    o.ln1w = o.ln1b = o.ln2w = o.ln2b = kNoParam;
    if (a.norm1 == kNormLayer) {
      o.ln1w = push(model_.f64(blk + ".layer_norm_inv_1.weight", {F}));
      o.ln1b = push(model_.f64(blk + ".layer_norm_inv_1.bias", {F}));
    }
    if (a.norm2 == kNormLayer) {
      o.ln2w = push(model_.f64(blk + ".layer_norm_inv_2.weight", {F}));
      o.ln2b = push(model_.f64(blk + ".layer_norm_inv_2.bias", {F}));
    }
    o.m1w = push(model_.f64(blk + ".mlp_1.1.weight", {F, F}));
    o.m1b = push(model_.f64(blk + ".mlp_1.1.bias", {F}));
    o.m2w = push(model_.f64(blk + ".mlp_1.3.weight", {F, F}));
    o.m2b = push(model_.f64(blk + ".mlp_1.3.bias", {F}));
    constexpr std::size_t kIw = kF + kHeads;  // interaction layer: F features and one L0 invariant per slot
    const auto iw = model_.f64(blk + ".interaction_block.linear_layer.weight", {kIw, kIw});
    const auto ib = model_.f64(blk + ".interaction_block.linear_layer.bias", {kIw});
    std::vector<double> iwp(kIntW * kIntW, 0.0), ibp(kIntW, 0.0);
    for (std::size_t r = 0; r < kIw; ++r) {
      ibp[r] = ib[r];
      for (std::size_t c = 0; c < kIw; ++c) iwp[r * kIntW + c] = iw[r * kIw + c];
    }
    o.iw = push(iwp);
    o.ib = push(ibp);
  }
  // heads
  const std::string eo = "model.atomic_energy_output_block.", co = "model.partial_charges_output_block.",
                    ho = "model.hirshfeld_output_block.";
  const std::string c6o = "model.c6_ratios_output_block.";
  std::vector<double> w1cat, b1cat;
  for (auto &part : {model_.f64(eo + "layers.0.weight", {128, F}), model_.f64(co + "transform_inv_features.0.weight", {128, F}),
                     model_.f64(ho + "transform_features.0.weight", {64, F})})
    w1cat.insert(w1cat.end(), part.begin(), part.end());
  for (auto &part : {model_.f64(eo + "layers.0.bias", {128}), model_.f64(co + "transform_inv_features.0.bias", {128}),
                     model_.f64(ho + "transform_features.0.bias", {64})})
    b1cat.insert(b1cat.end(), part.begin(), part.end());
  if (a.has_c6) {  // the C6 ratio head's first layer joins the fused GEMM
    const auto w = model_.f64(c6o + "transform_features.0.weight", {64, F});
    const auto b = model_.f64(c6o + "transform_features.0.bias", {64});
    w1cat.insert(w1cat.end(), w.begin(), w.end());
    b1cat.insert(b1cat.end(), b.begin(), b.end());
  }
  // a ratio head with K keys, zero-padded to 64 keys: the padded keys are 0 and
  // their embeddings 0, so they add nothing (output_heads.cpp:105-133)
  struct RatioOff { std::size_t w2, w2t, b2, qemb, vshift; double sqrt_k; };
  auto ratio_head = [&](const std::string &prefix, int K) {
    const std::size_t k = std::size_t(K);
    const auto w2 = model_.f64(prefix + "transform_features.2.weight", {k, 64});
    const auto b2 = model_.f64(prefix + "transform_features.2.bias", {k});
    const auto qe = model_.f64(prefix + "q_embedding.weight", {100, k});
    std::vector<double> w2p(64 * 64, 0.0), w2tp(64 * 64, 0.0), b2p(64, 0.0), qep(100 * 64, 0.0);
    for (std::size_t r = 0; r < k; ++r) {
      b2p[r] = b2[r];
      for (std::size_t j = 0; j < 64; ++j) {
        w2p[r * 64 + j] = w2[r * 64 + j];
        w2tp[j * 64 + r] = w2[r * 64 + j];
      }
    }
    for (std::size_t zz = 0; zz < 100; ++zz)
      for (std::size_t r = 0; r < k; ++r) qep[zz * 64 + r] = qe[zz * k + r];
    RatioOff o;
    o.w2 = push(w2p);
    o.w2t = push(w2tp);
    o.b2 = push(b2p);
    o.qemb = push(qep);
    o.vshift = push(model_.f64(prefix + "v_shift_embedding.weight", {100, 1}));
    o.sqrt_k = std::sqrt(double(K));
    return o;
  };
  const std::size_t o_w1cat = push(w1cat), o_b1cat = push(b1cat);
  const std::size_t o_ew2 = push(model_.f64(eo + "final_layer.weight", {1, 128}));
  const double e_b2 = model_.f64(eo + "final_layer.bias", {1})[0];
  const std::size_t o_escale = push(model_.f64(eo + "energy_scales.weight", {1, 118}));
  const std::size_t o_eshift = push(model_.f64(eo + "energy_shifts", {118}));
  const std::size_t o_cw2 = push(model_.f64(co + "transform_inv_features.2.weight", {1, 128}));
  const double c_b2 = model_.f64(co + "transform_inv_features.2.bias", {1})[0];
  const std::size_t o_cemb = push(model_.f64(co + "atomic_embedding.weight", {100, 1}));
  const RatioOff o_h = ratio_head(ho, a.hirshfeld_keys);
  RatioOff o_r6{kNoParam, kNoParam, kNoParam, kNoParam, kNoParam, 1.0};
  if (a.has_c6) o_r6 = ratio_head(c6o, a.c6_keys);
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
  const ZblParams z = model_.zbl();
  std::size_t o_nlh_a = kNoParam, o_nlh_b = kNoParam;
  if (z.kind == 1) {
    const std::size_t cap = std::size_t(z.nlh_cap);
    o_nlh_a = push(model_.f64("physical.nlh_a", {cap, cap, 3}));
    o_nlh_b = push(model_.f64("physical.nlh_b", {cap, cap, 3}));
  }
  norm1_ = a.norm1;
  norm2_ = a.norm2;
  qk_norm_ = a.qk_norm;
  resid_.assign(layers_, 1.0);
  x0s_.assign(layers_, 0.0);
  if (a.residual_scalars) {
    resid_ = model_.f64("model.resid_lambdas", {std::size_t(layers_)});
    x0s_ = model_.f64("model.x0_lambdas", {std::size_t(layers_)});
  }
  residual_scalars_ = a.residual_scalars;

  double *d = wbuf_.reserve(host.size());
  SO3_CUDA(cudaMemcpy(d, host.data(), host.size() * sizeof(double), cudaMemcpyHostToDevice));
  auto P = [&](std::size_t off) { return off == kNoParam ? nullptr : static_cast<const double *>(d + off); };
  float *d32 = wbuf32_.reserve(host32.size());
  SO3_CUDA(cudaMemcpy(d32, host32.data(), host32.size() * sizeof(float), cudaMemcpyHostToDevice));
  auto P32 = [&](std::size_t off) { return static_cast<const float *>(d32 + off); };
  auto fw32 = [&](const FOff32 &f) {
    return FilterW32{P32(f.b0),         P32(f.bc1),         P32(f.v0),          P32(f.c0),
                     P32(f.w0t.first),  P32(f.w0t.second),  P32(f.w1t.first),   P32(f.w1t.second),
                     P32(f.v1t.first),  P32(f.v1t.second),  P32(f.w1.first),    P32(f.w1.second),
                     P32(f.v1.first),   P32(f.v1.second),   P32(f.w0.first),    P32(f.w0.second),
                     P32(f.tc_fwd),     P32(f.tc_rev)};
  };
  blocks_.resize(layers_);
  for (int b = 0; b < layers_; ++b) {
    const BOff &o = boff[b];
    BlockW &w = blocks_[b];
    auto fw = [&](const FOff &f) {
      return FilterW{P(f.w0),  P(f.b0),    P(f.w1),    P(f.b1),    P(f.v0),   P(f.c0),   P(f.v1),  P(f.c1),
                     P(f.bc1), P(f.w0t_f), P(f.w1t_f), P(f.v1t_f), P(f.w1_f), P(f.v1_f), P(f.w0_f)};
    };
    w.finv = fw(o.finv);
    w.fev = fw(o.fev);
    if (kF == 128) {
      w.finv32 = fw32(foff32[2 * std::size_t(b)]);
      w.fev32 = fw32(foff32[2 * std::size_t(b) + 1]);
    }
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
  heads_.h_w2 = P(o_h.w2);
  heads_.h_w2t = P(o_h.w2t);
  heads_.h_b2 = P(o_h.b2);
  heads_.h_qemb = P(o_h.qemb);
  heads_.h_vshift = P(o_h.vshift);
  heads_.h_sqrt_k = o_h.sqrt_k;
  heads_.c6_w2 = P(o_r6.w2);
  heads_.c6_w2t = P(o_r6.w2t);
  heads_.c6_b2 = P(o_r6.b2);
  heads_.c6_qemb = P(o_r6.qemb);
  heads_.c6_vshift = P(o_r6.vshift);
  heads_.c6_sqrt_k = o_r6.sqrt_k;
  heads_.ldh = a.has_c6 ? kHeadCatC6 : kHeadCat;
  emb_w_ = P(o_emb);
  rad_.b = P(o_rb);
  rad_.k = P(o_rk);
  rad_.kr = P(o_rkr);
  rad_.gamma = model_.f64("model.radial_embedding.radial_basis_fn.gamma", {})[0];
  if (kF == 128) {  // kernel-parameter constants of the tcgen05 filter kernels, per block
    const auto rb = model_.f64("model.radial_embedding.radial_basis_fn.b", {R});
    const auto rk = model_.i64("model.radial_embedding.radial_basis_fn.k");
    const auto rkr = model_.i64("model.radial_embedding.radial_basis_fn.k_rev");
    tc_fwd_consts_.assign(layers_, TcFwdConsts{});
    tc_rev_consts_.assign(layers_, TcRevConsts{});
    for (int b = 0; b < layers_; ++b) {
      TcFwdConsts &cf = tc_fwd_consts_[b];
      TcRevConsts &cr = tc_rev_consts_[b];
      for (int f = 0; f < 2; ++f) {
        const FiltHost &fh = filt_host[2 * std::size_t(b) + f];
        for (int j = 0; j < kF; ++j) {
          cf.b0[f][j] = float(fh.b0[j]);
          cf.bc1[f][j] = float(fh.bc1[j]);
          cf.v0[f][j] = float(fh.v0[j]);
          cr.v0[f][j] = fh.v0[j];
        }
        for (int j = 0; j < kEH; ++j) {
          cf.c0[f][j] = float(fh.c0[j]);
          cr.c0[f][j] = fh.c0[j];
        }
      }
      for (int k = 0; k < kR; ++k) {
        cf.rb[k] = rb[k];
        cf.rk[k] = double(rk[k]);
        cf.rkr[k] = double(rkr[k]);
      }
      cf.gamma = rad_.gamma;
      const std::string att = "model.euclidean_transformers." + std::to_string(b) + ".euclidean_attention_block.";
      const auto cg = model_.f64(att + "so3_conv_invariants.cg_rep", {kEV});
      for (int m = 0; m < kEV; ++m) cf.cg[m] = cr.cg[m] = cg[m];
    }
  }
  alpha_ref_ = P(o_alpha);
  c6_ref_ = P(o_c6);
  zbl_.ke = z.ke; zbl_.cutoff = z.cutoff; zbl_.switch_off = z.switch_off; zbl_.p = z.p; zbl_.d = z.d;
  for (int k = 0; k < 4; ++k) { zbl_.a[k] = z.a[k]; zbl_.c[k] = z.c[k]; }
  zbl_.kind = z.kind;
  zbl_.nlh_cap = z.nlh_cap;
  zbl_.nlh_a = P(o_nlh_a);
  zbl_.nlh_b = P(o_nlh_b);
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
// ---------------------------------------------------------------------------
// multi-GPU
// ---------------------------------------------------------------------------
void Evaluator::set_comm(int nranks, int rank, const void *unique_id) {
  if (nranks < 1 || rank < 0 || rank >= nranks) throw Error("SO3LR: invalid rank / rank count");
  if (nranks > 63) throw Error("SO3LR: at most 63 GPUs per decomposition");
  SO3_CUDA(cudaSetDevice(device_));
  if (comm_) {
    nccl().comm_destroy(comm_);
    comm_ = nullptr;
  }
  nranks_ = nranks;
  rank_ = rank;
  spec_ = SystemSpec();  // force a new partition on the next prepare
  if (nranks == 1) return;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  const ncclResult_t r = nccl().comm_init_rank(&comm_, nranks, id, rank);
  if (r != ncclSuccess) throw Error(std::string("SO3LR: ncclCommInitRank failed: ") + nccl().get_error_string(r));
}

void Evaluator::allgather_rows(double *a, int width, int prof) {
  if (nranks_ == 1) return;
  if (prof >= 0) prof_begin(prof);
  const std::size_t count = std::size_t(stride_) * width;
  const ncclResult_t r = nccl().all_gather(a + std::size_t(rank_) * count, a, count, ncclDouble, comm_, stream_);
  if (r != ncclSuccess) throw Error(std::string("SO3LR: ncclAllGather failed: ") + nccl().get_error_string(r));
  if (prof >= 0) prof_end(prof, 0.0);
}

void Evaluator::halo_exchange(double *a, int wa, double *b, int wb, int prof) {
  if (nranks_ == 1) return;
  prof_begin(prof);
  const int w = wa + wb;
  const long long nsend = halo_send_off_[nranks_], nrecv = halo_recv_off_[nranks_];
  double *sbuf = halo_send_buf_.reserve(std::size_t(std::max(1LL, nsend)) * w, 1.25);
  double *rbuf = halo_recv_buf_.reserve(std::size_t(std::max(1LL, nrecv)) * w, 1.25);
  launch_halo_pack(int(nsend), halo_send_rows_.get(), a, wa, b, wb, sbuf, stream_);
  const NcclApi &api = nccl();
  auto check = [&](ncclResult_t r, const char *what) {
    if (r != ncclSuccess) throw Error(std::string("SO3LR: ") + what + " failed: " + api.get_error_string(r));
  };
  check(api.group_start(), "ncclGroupStart");
  for (int p = 0; p < nranks_; ++p) {
    if (p == rank_) continue;
    const long long cs = halo_send_off_[p + 1] - halo_send_off_[p];
    const long long cr = halo_recv_off_[p + 1] - halo_recv_off_[p];
    if (cs > 0) check(api.send(sbuf + halo_send_off_[p] * w, std::size_t(cs) * w, ncclDouble, p, comm_, stream_), "ncclSend");
    if (cr > 0) check(api.recv(rbuf + halo_recv_off_[p] * w, std::size_t(cr) * w, ncclDouble, p, comm_, stream_), "ncclRecv");
  }
  check(api.group_end(), "ncclGroupEnd");
  launch_halo_unpack(int(nrecv), halo_recv_rows_.get(), rbuf, a, wa, b, wb, stream_);
  prof_end(prof, 0.0);
}

// exact sums over segments of the owned rows (global over ranks when decomposed);
// seg: device [nseg + 1] row offsets; out: device [nseg * ncol]
void Evaluator::exact_sums(const double *v, int stride, int ncol, int nseg, const int *seg, double *out) {
  const int count = nseg * ncol;
  // one segment (a global sum over this GPU's atoms): spread it over many blocks;
  // the block count depends only on the rank stride, so every rank sends the
  // same number of partial sums
  const int nblk = nseg == 1 ? std::max(1, std::min(64, (stride_ + 2047) / 2048)) : 1;
  const std::size_t per_rank = std::size_t(count) * 2 * nblk;
  long long *local = parts_.reserve(per_rank * (nranks_ + 1));
  long long *all = local + per_rank;
  launch_fixed_segment_sum(nseg, nblk, seg, v, stride, ncol, local, stream_);
  if (nranks_ > 1) {
    prof_begin(kProfExactSums);
    const ncclResult_t r = nccl().all_gather(local, all, per_rank, ncclInt64, comm_, stream_);
    if (r != ncclSuccess) throw Error(std::string("SO3LR: ncclAllGather failed: ") + nccl().get_error_string(r));
    prof_end(kProfExactSums, 0.0);
    launch_fixed_finish(all, nranks_ * nblk, count, out, stream_);
  } else {
    launch_fixed_finish(local, nblk, count, out, stream_);
  }
}

// brick index of a position (the same arithmetic on every rank)
// ---------------------------------------------------------------------------
// system preparation
// ---------------------------------------------------------------------------
void Evaluator::prepare(const SystemSpec &spec_in, const double *host_x) {
  SO3_CUDA(cudaSetDevice(device_));
  computed_ = false;
  md_ready_ = false;
  nvt_ = false;
  local_ready_ = false;
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
    for (int d = 0; d < 3; ++d) {
      if (!(spec.len[d] > 0.0)) throw Error("SO3LR: periodic box lengths must be positive");
      if (!std::isfinite(spec.len[d]) || !std::isfinite(spec.lo[d]))
        throw Error("SO3LR: periodic box bounds must be finite");
    }
  } else if (!open_cells_possible(spec, host_x)) {
    for (int i = 0; i < nimg; ++i)
      if (spec.image_start[i + 1] - spec.image_start[i] > 20000)
        throw Error("SO3LR: open-boundary images are limited to 20000 atoms when positions are not given on the "
                    "host (so3lr_compute_device) or the system is a pack of images");
  }
  if (nranks_ > 1) {
    if (!spec.periodic) throw Error("SO3LR: multi-GPU decomposition needs a periodic box");
    if (host_x == nullptr) throw Error("SO3LR: multi-GPU decomposition needs positions to partition");
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

  // row layout: rank-major bricks of `stride` rows; input atom i -> row_of_[i]
  const std::vector<int> owner = partition_atoms(spec, host_x, nranks_);
  std::vector<int> per_rank(nranks_, 0);
  for (int i = 0; i < n; ++i) per_rank[owner[i]]++;
  stride_ = nranks_ == 1 ? n : *std::max_element(per_rank.begin(), per_rank.end());
  if (stride_ == 0) stride_ = 1;
  n_rows_ = nranks_ * stride_;
  row0_ = rank_ * stride_;
  n_own_ = per_rank[rank_];
  identity_ = nranks_ == 1;
  row_of_.assign(n, 0);
  tag_of_row_.assign(n_rows_, -1);
  {
    std::vector<int> fill(nranks_, 0);
    for (int i = 0; i < n; ++i) {
      const int row = owner[i] * stride_ + fill[owner[i]]++;
      row_of_[i] = row;
      tag_of_row_[row] = i;
    }
  }
  std::vector<int> z_rows(n_rows_, 1), image_rows(n_rows_, 0), table_rows(n_rows_, -1);
  for (int i = 0; i < n; ++i) {
    z_rows[row_of_[i]] = spec.z[i];
    image_rows[row_of_[i]] = image_of[i];
    table_rows[row_of_[i]] = table_of_atom[i];
  }
  spec_ = spec;
  alloc_atoms();
  const int nr = n_rows_;
  SO3_CUDA(cudaMemcpyAsync(z_.reserve(nr), z_rows.data(), sizeof(int) * nr, cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(image_of_.reserve(nr), image_rows.data(), sizeof(int) * nr, cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(table_of_atom_.reserve(nr), table_rows.data(), sizeof(int) * nr, cudaMemcpyHostToDevice,
                           stream_));
  SO3_CUDA(cudaMemcpyAsync(tag_.reserve(nr), tag_of_row_.data(), sizeof(int) * nr, cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(image_start_.reserve(nimg + 1), spec.image_start.data(), sizeof(int) * (nimg + 1),
                           cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(image_charge_.reserve(nimg), spec.image_charge.data(), sizeof(double) * nimg,
                           cudaMemcpyHostToDevice, stream_));
  if (any_charge_spin_) {
    SO3_CUDA(cudaMemcpyAsync(cs_tables_.reserve(tables.size()), tables.data(), sizeof(double) * tables.size(),
                             cudaMemcpyHostToDevice, stream_));
  }
  // segments: [0..1] owned rows, [2..3] image count of the (single, global) image,
  // [4..5] image-energy segment over images
  {
    const int seg[6] = {row0_, row0_ + n_own_, 0, n, 0, nimg};
    std::memcpy(host_seg_, seg, sizeof(seg));
    SO3_CUDA(cudaMemcpyAsync(seg_.reserve(8), host_seg_, sizeof(seg), cudaMemcpyHostToDevice, stream_));
  }
  // cell grid: cells no smaller than the short-range cutoff (cell_grid.cpp)
  const CellGrid g = plan_cell_grid(spec.periodic, spec.lo, spec.len, sr_cut_, open_cells_possible(spec, host_x), n,
                                    host_x);
  const long long ncells = (long long)g.ncell[0] * g.ncell[1] * g.ncell[2];
  nb_.grid = g;
  nb_.tag = identity_ ? nullptr : tag_.get();
  nb_.row0 = row0_;
  nb_.n_own = n_own_;
  nb_.xw = xw_.reserve(3 * std::size_t(nr));
  nb_.cell = cell_.reserve(nr);
  nb_.cell_count = cell_count_.reserve(ncells);
  nb_.cell_start = cell_start_.reserve(ncells + 1);
  nb_.cell_fill = cell_fill_.reserve(ncells);
  nb_.cell_atoms = cell_atoms_.reserve(nr);
  nb_.image_of = image_of_.get();
  nb_.image_start = image_start_.get();
  nb_.deg = deg_.reserve(nr);
  nb_.row_start = row_start_.reserve(nr + 1);
  nb_.scan_scratch = scan_scratch_.reserve(scan_scratch_ints(std::max<long long>(ncells, 64LL * nr)));
  nb_.scan_total = small_ints_.reserve(16);
  nb_.error_flag = nb_.scan_total + 4;
  SO3_CUDA(cudaStreamSynchronize(stream_));
}

// A single open-boundary system with host positions and more than a few
// hundred atoms gets a cell grid; smaller systems and packs of images scan
// their image's index range.
bool Evaluator::open_cells_possible(const SystemSpec &spec, const double *host_x) const {
  const int nimg = spec.image_start.empty() ? 1 : int(spec.image_start.size()) - 1;
  return !spec.periodic && nimg == 1 && host_x != nullptr && spec.n > kOpenCellsMinAtoms;
}

void Evaluator::alloc_atoms() {
  const std::size_t n = std::size_t(n_rows_);
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
  ensure_vec(gate_, layers_, n * kHeads);
  ensure_vec(xhat2_, layers_, n * kF);
  ensure_vec(rstd2_, layers_, n);
  if (qk_norm_) ensure_vec(qkr_, layers_, n * 4 * kHeads);
  if (residual_scalars_) x0_.reserve(n * kF);
  d_inv_.reserve(n * kF);
  d_ev_.reserve(n * kEV);
  act_.reserve(n * kF);
  cat_.reserve(n * kIntW);
  t_.reserve(n * kIntW);
  hpre_.reserve(n * heads_.ldh);
  hcat_.reserve(n * heads_.ldh);
  hk_.reserve(n * kHirsh);
  if (heads_.c6_w2 != nullptr) {
    hk6_.reserve(n * kHirsh);
    ratio6_.reserve(n);
    dc6_.reserve(n);
  }
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
  g_hcat_.reserve(n * heads_.ldh);
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
  stage_.resize(std::size_t(n) * 6);
}

// flags the kernels of the last evaluation left (copied to host_small_[8..9])
void Evaluator::check_device_flags() const {
  if (host_small_[8] != 0) throw Error("SO3LR: short-range list has an edge without its reverse");
  if (host_small_[9] != 0)
    throw Error("SO3LR: the tensor-core filter kernel gave up waiting for its pipeline (stage " +
                std::to_string(host_small_[9]) + "); its results are not valid");
}

void Evaluator::upload_positions(const double *host_x) {
  SO3_CUDA(cudaSetDevice(device_));
  if (identity_) {
    SO3_CUDA(cudaMemcpyAsync(x_.get(), host_x, sizeof(double) * 3 * spec_.n, cudaMemcpyHostToDevice, stream_));
    return;
  }
  std::fill(stage_.begin(), stage_.begin() + 3 * std::size_t(n_rows_), 0.0);
  for (int i = 0; i < spec_.n; ++i)
    for (int d = 0; d < 3; ++d) stage_[3 * std::size_t(row_of_[i]) + d] = host_x[3 * std::size_t(i) + d];
  SO3_CUDA(cudaMemcpyAsync(x_.get(), stage_.data(), sizeof(double) * 3 * n_rows_, cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaStreamSynchronize(stream_));  // stage_ is reused
}

std::size_t Evaluator::device_bytes() const {
  std::size_t total = wbuf_.bytes() + geo_.bytes() + sh_.bytes() + gv_.bytes() + gl0_.bytes() + pair_sc_.bytes();
  for (auto &v : f_inv_) total += v->bytes();
  for (auto &v : f_ev_) total += v->bytes();
  for (auto &v : sp_) total += v->bytes();
  for (auto &v : qkv32_) total += v->bytes();
  total += ga32_.bytes() + gA32_.bytes();
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
  if (k < 0 || k >= kProfKinds) throw Error("SO3LR: unknown profiled kernel");
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
  build_cells(nb_, n_rows_, x_.get(), stream_);
  count_sr(nb_, sr_cut_, stream_);
  SO3_CUDA(cudaMemcpyAsync(host_small_, nb_.row_start + n_own_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
  SO3_CUDA(cudaStreamSynchronize(stream_));
  const int E = host_small_[0];
  if (E < 0) throw Error("SO3LR: edge count overflow");
  stats_.edges = E;
  nb_.nbr = nbr_.reserve(E, 1.25);
  nb_.img = img_.reserve(E, 1.25);
  nb_.primary = primary_.reserve(E, 1.25);
  nb_.rev = rev_.reserve(E, 1.25);
  nb_.pair_scan = pair_scan_.reserve(E, 1.25);
  nb_.edge_pair = edge_pair_.reserve(E, 1.25);
  if (scan_scratch_.capacity() < scan_scratch_ints(std::size_t(E) + 1)) {
    nb_.scan_scratch = scan_scratch_.reserve(scan_scratch_ints(std::size_t(E) * 2 + 1));
  }
  SO3_CUDA(cudaMemsetAsync(nb_.error_flag, 0, sizeof(int), stream_));
  fill_sr(nb_, sr_cut_, E, stream_);
  SO3_CUDA(cudaMemcpyAsync(host_small_ + 1, nb_.scan_total, sizeof(int), cudaMemcpyDeviceToHost, stream_));
  if (!identity_) {
    // halo lists from this GPU's (symmetric) neighbour lists; every rank's
    // per-peer counts are gathered so that all ranks can check them together
    prof_begin(kProfHaloLists);
    const int cnt = nranks_ * stride_;
    int *flags = halo_flags_.reserve(2 * std::size_t(cnt));
    int *pos = halo_pos_.reserve(2 * std::size_t(cnt));
    const std::size_t nscratch = scan_scratch_ints(std::size_t(cnt) + 1);
    if (scan_scratch_.capacity() < nscratch) nb_.scan_scratch = scan_scratch_.reserve(nscratch);
    nb_.scan_scratch = scan_scratch_.get();
    const int lo = 2 * (nranks_ + 1);
    long long *off = halo_offsets_.reserve(lo);
    long long *all = halo_all_offsets_.reserve(std::size_t(lo) * nranks_);
    launch_halo_lists(n_own_, row0_, stride_, nranks_, rank_, nb_.row_start, nb_.nbr, flags, flags + cnt, pos,
                      pos + cnt, halo_send_rows_.reserve(cnt), halo_recv_rows_.reserve(cnt), off,
                      halo_totals_.reserve(2), nb_.scan_scratch, stream_);
    const ncclResult_t r = nccl().all_gather(off, all, std::size_t(lo), ncclInt64, comm_, stream_);
    if (r != ncclSuccess) throw Error(std::string("SO3LR: ncclAllGather failed: ") + nccl().get_error_string(r));
    if (!host_halo_) SO3_CUDA(cudaMallocHost(&host_halo_, sizeof(long long) * 2 * 64 * 64));
    SO3_CUDA(cudaMemcpyAsync(host_halo_, all, sizeof(long long) * lo * nranks_, cudaMemcpyDeviceToHost, stream_));
  }
  SO3_CUDA(cudaStreamSynchronize(stream_));
  if (!identity_) {
    const int lo = 2 * (nranks_ + 1);
    auto sends = [&](int s, int p) { return host_halo_[s * lo + p + 1] - host_halo_[s * lo + p]; };
    auto recvs = [&](int r, int p) { return host_halo_[r * lo + nranks_ + 2 + p] - host_halo_[r * lo + nranks_ + 1 + p]; };
    for (int s = 0; s < nranks_; ++s)  // the same verdict on every rank
      for (int p = 0; p < nranks_; ++p)
        if (s != p && sends(s, p) != recvs(p, s))
          throw Error("SO3LR: halo lists of GPUs " + std::to_string(s) + " and " + std::to_string(p) + " disagree");
    halo_send_off_.assign(host_halo_ + rank_ * lo, host_halo_ + rank_ * lo + nranks_ + 1);
    halo_recv_off_.assign(host_halo_ + rank_ * lo + nranks_ + 1, host_halo_ + rank_ * lo + lo);
    // recorded after the host check: the span includes the stream's wait for it
    prof_end(kProfHaloLists, 0.0);
  }
  const int P = host_small_[1];
  if (identity_ && 2 * P != E) throw Error("SO3LR: short-range list is not symmetric");
  stats_.pairs = P;
  nb_.pair_a = pair_a_.reserve(P, 1.25);
  nb_.pair_b = pair_b_.reserve(P, 1.25);
  nb_.pair_img = pair_img_.reserve(P, 1.25);
  nb_.pair_edge = pair_edge_.reserve(P, 1.25);
  nb_.pair_canon = pair_canon_.reserve(P, 1.25);
  fill_pairs(nb_, E, stream_);
  // per-pair storage
  geo_.reserve(std::size_t(P) * kGeo, 1.25);
  sh_.reserve(std::size_t(P) * kSH, 1.25);
  gv_.reserve(std::size_t(P) * 3, 1.25);
  gl0_.reserve(std::size_t(P) * kHeads, 1.25);
  pair_sc_.reserve(std::size_t(P) * kPairScalars, 1.25);
  g_filt_inv_.reserve(std::size_t(P) * kF, 1.25);
  g_filt_ev_.reserve(std::size_t(P) * kF, 1.25);
  drbf_.reserve(std::size_t(P) * kR, 1.25);
  g_r_.reserve(std::size_t(P), 1.25);
  g_y_.reserve(std::size_t(P) * kSH, 1.25);
  while (int(f_inv_.size()) < layers_) {
    f_inv_.emplace_back(new DeviceArray<double>());
    f_ev_.emplace_back(new DeviceArray<double>());
    sp_.emplace_back(new DeviceArray<double>());
  }
  for (int b = 0; b < layers_; ++b) {
    f_inv_[b]->reserve(std::size_t(P) * kF, 1.25);
    f_ev_[b]->reserve(std::size_t(P) * kF, 1.25);
    sp_[b]->reserve(filter_sp_doubles(P), 1.25);
  }
}

// ---------------------------------------------------------------------------
// the evaluation
//
// Rows [row0, row0 + n_own) are this GPU's atoms; every other row is a copy of
// another GPU's atom, refreshed right after its owner computed it: positions,
// charges and Hirshfeld ratios by all-gathers, block features and adjoints only
// for the halo rows (the other GPUs' short-range neighbours of this GPU's atoms,
// halo.cu). Everything an owned atom sums over (its CSR row, its cell stencil)
// is complete locally, so no partial sum ever crosses GPUs; the only global sums
// (charge, charge seeds, energy, virial, kinetic energy) are exact.
// ---------------------------------------------------------------------------
void Evaluator::compute() {
  SO3_CUDA(cudaSetDevice(device_));
  const int N = n_rows_;          // all rows
  const int n = n_own_;           // owned rows
  const std::size_t r0 = std::size_t(row0_);
  const int nimg = int(spec_.image_start.size()) - 1;
  cudaStream_t s = stream_;
  const int *own_seg = seg_.get();
  const int *count_seg = identity_ ? image_start_.get() : seg_.get() + 2;
  if (mixed_ && mixed_tc_) SO3_CUDA(cudaMemsetAsync(tc_err_, 0, sizeof(int), s));
  // mixed precision with the tcgen05 filters: filters, filter gradients and the
  // attention in float32 (the stated tolerance holds; the float64 path and the
  // mma.sync mixed path keep the float64 attention)
  const bool att32 = kF == 128 && mixed_ && mixed_tc_;
  (void)att32;
  if (att32 && qkv32_.size() != std::size_t(layers_)) {
    qkv32_.clear();
    for (int b = 0; b < layers_; ++b) qkv32_.push_back(std::make_unique<DeviceArray<float>>());
  }
  build_neighbors();
  const int P = int(stats_.pairs);
  launch_pair_geometry(P, nb_, z_.get(), zbl_, sr_cut_, geo_.get(), sh_.get(), gv_.get(), s);
  // with residual scalars the embedding x0 is kept apart: every block's input
  // is resid[b] x + x0[b] x0
  launch_embedding(N, z_.get(), emb_w_, any_charge_spin_ ? cs_tables_.get() : nullptr, table_of_atom_.get(),
                   inv_emb_scale_, residual_scalars_ ? x0_.get() : xb_[0]->get(), s);
  if (residual_scalars_) launch_residual_combine(N, x0_.get(), x0_.get(), resid_[0], x0s_[0], xb_[0]->get(), s);
  SO3_CUDA(cudaMemsetAsync(evb_[0]->get(), 0, sizeof(double) * N * kEV, s));

  for (int b = 0; b < layers_; ++b) {
    const BlockW &w = blocks_[b];
    prof_begin(kProfFilterForward);
#if SO3LR_FEATURES == 128
    if (mixed_ && mixed_tc_)
      launch_filter_forward_tc(P, geo_.get(), nb_.pair_a, nb_.pair_b, b == 0 ? nullptr : evb_[b]->get(),
                               tc_fwd_consts_[b], w.finv32, w.fev32, reinterpret_cast<float *>(f_inv_[b]->get()),
                               reinterpret_cast<float *>(f_ev_[b]->get()),
                               reinterpret_cast<float *>(sp_[b]->get()), b == 0 ? drbf_.get() : nullptr, tc_err_,
                               num_sms_, s);
    else if (mixed_)
      launch_filter_forward_mixed(P, geo_.get(), nb_.pair_a, nb_.pair_b, b == 0 ? nullptr : evb_[b]->get(), w.cg_att,
                                  w.finv32, w.fev32, rad_, f_inv_[b]->get(), f_ev_[b]->get(),
                                  reinterpret_cast<float *>(sp_[b]->get()), b == 0 ? drbf_.get() : nullptr, s);
    else
#endif
      launch_filter_forward(P, geo_.get(), nb_.pair_a, nb_.pair_b, b == 0 ? nullptr : evb_[b]->get(), w.cg_att,
                            w.finv, w.fev, rad_, f_inv_[b]->get(), f_ev_[b]->get(), sp_[b]->get(),
                            b == 0 ? drbf_.get() : nullptr, s);
    prof_end(kProfFilterForward, kFilterFlopsPerPair * double(P));
    {  // per-head projections qkv[row][h][5][32] = x[row][h*32:(h+1)*32] W_h of every
       // row the attention reads: the owned rows and (decomposed) their halo
      GemmArgs g{};
      g.M = identity_ ? N : n; g.N = 160; g.K = 32;
      g.A = xb_[b]->get() + (identity_ ? 0 : r0 * kF); g.lda = kF; g.strideA = 32;
      g.W = w.qkv_fwd; g.ldw = 32; g.transB = true; g.strideW = 160 * 32;
      g.C = qkv_[b]->get() + (identity_ ? 0 : r0 * kQKV); g.ldc = kQKV; g.strideC = 160;
      g.batch = kHeads;
      launch_gemm(g, s);
      if (!identity_ && halo_recv_off_[nranks_] > 0) {
        g.M = int(halo_recv_off_[nranks_]);
        g.A = xb_[b]->get();
        g.C = qkv_[b]->get();
        g.rows = halo_recv_rows_.get();
        launch_gemm(g, s);
      }
      if (qk_norm_) {
        launch_qk_norm(identity_ ? N : n, nullptr, qkv_[b]->get() + (identity_ ? 0 : r0 * kQKV),
                       qkr_[b]->get() + (identity_ ? 0 : r0 * 4 * kHeads), s);
        if (!identity_ && halo_recv_off_[nranks_] > 0)
          launch_qk_norm(int(halo_recv_off_[nranks_]), halo_recv_rows_.get(), qkv_[b]->get(), qkr_[b]->get(), s);
      }
    }
#if SO3LR_FEATURES == 128
    if (att32) {  // float32 attention: float32 copies of the rows the QKV GEMM computed
      float *q32 = qkv32_[b]->reserve(std::size_t(N) * kQKV);
      launch_rows_to_float(identity_ ? N : n, identity_ ? 0 : int(r0), identity_ ? 0 : int(halo_recv_off_[nranks_]),
                           halo_recv_rows_.get(), kQKV, qkv_[b]->get(), q32, s);
      launch_attention_forward32(n, nb_, geo_.get(), sh_.get(), q32, reinterpret_cast<const float *>(f_inv_[b]->get()),
                                 reinterpret_cast<const float *>(f_ev_[b]->get()), norm_, d_inv_.get(), d_ev_.get(),
                                 s);
    } else
#endif
      launch_attention_forward(n, nb_, geo_.get(), sh_.get(), qkv_[b]->get(), f_inv_[b]->get(), f_ev_[b]->get(),
                               norm_, d_inv_.get(), d_ev_.get(), s);
    launch_post_attn_pre(n, xb_[b]->get() + r0 * kF, d_inv_.get() + r0 * kF, evb_[b]->get() + r0 * kEV,
                         d_ev_.get() + r0 * kEV, norm1_, w.ln1w, w.ln1b, w.cg_int, xhat1_[b]->get() + r0 * kF,
                         rstd1_[b]->get() + r0, n1_[b]->get() + r0 * kF, act_.get() + r0 * kF,
                         A_[b]->get() + r0 * kEV, cat_.get() + r0 * kIntW, s);
    {  // hidden = silu(act W1^T + b1), pre-activation kept for the reverse
      GemmArgs g{};
      g.M = n; g.N = kF; g.K = kF;
      g.A = act_.get() + r0 * kF; g.lda = kF;
      g.W = w.mlp1w; g.ldw = kF; g.transB = true;
      g.C = d_inv_.get() + r0 * kF; g.ldc = kF;  // reuse d_inv as the hidden activation
      g.bias = w.mlp1b; g.aux_out = hp_[b]->get() + r0 * kF; g.ldaux = kF;
      g.epi = Epi::BiasStorePre;
      launch_gemm(g, s);
    }
    {  // post = n1 + hidden W2^T + b2  -> cat[:, :128]
      GemmArgs g{};
      g.M = n; g.N = kF; g.K = kF;
      g.A = d_inv_.get() + r0 * kF; g.lda = kF;
      g.W = w.mlp2w; g.ldw = kF; g.transB = true;
      g.C = cat_.get() + r0 * kIntW; g.ldc = kIntW;
      g.bias = w.mlp2b; g.aux = n1_[b]->get() + r0 * kF; g.ldaux = kF;
      g.epi = Epi::BiasResidual;
      launch_gemm(g, s);
    }
    {  // t = [post, L0'] W_int^T + b_int
      GemmArgs g{};
      g.M = n; g.N = kIntW; g.K = kIntW;
      g.A = cat_.get() + r0 * kIntW; g.lda = kIntW;
      g.W = w.intw; g.ldw = kIntW; g.transB = true;
      g.C = t_.get() + r0 * kIntW; g.ldc = kIntW;
      g.bias = w.intb;
      g.epi = Epi::Bias;
      launch_gemm(g, s);
    }
    launch_post_attn_final(n, cat_.get() + r0 * kIntW, t_.get() + r0 * kIntW, A_[b]->get() + r0 * kEV, norm2_,
                           w.ln2w, w.ln2b, xhat2_[b]->get() + r0 * kF, rstd2_[b]->get() + r0,
                           gate_[b]->get() + r0 * kHeads, xb_[b + 1]->get() + r0 * kF, evb_[b + 1]->get() + r0 * kEV, s);
    if (b + 1 < layers_) {
      if (residual_scalars_)  // the next block's input, on this GPU's rows
        launch_residual_combine(n, xb_[b + 1]->get() + r0 * kF, x0_.get() + r0 * kF, resid_[b + 1], x0s_[b + 1],
                                xb_[b + 1]->get() + r0 * kF, s);
      // the halo rows of the next block's input
      halo_exchange(xb_[b + 1]->get(), kF, evb_[b + 1]->get(), kEV, kProfFeatureHalo);
    }
  }

  // ---- output heads (owned rows) --------------------------------------------
  {
    GemmArgs g{};
    const int ldh = heads_.ldh;
    g.M = n; g.N = ldh; g.K = kF;
    g.A = xb_[layers_]->get() + r0 * kF; g.lda = kF;
    g.W = heads_.w1cat; g.ldw = kF; g.transB = true;
    g.C = hcat_.get() + r0 * ldh; g.ldc = ldh;
    g.bias = heads_.b1cat; g.aux_out = hpre_.get() + r0 * ldh; g.ldaux = ldh;
    g.epi = Epi::BiasStorePre;
    launch_gemm(g, s);
  }
  const bool c6 = heads_.c6_w2 != nullptr;
  launch_heads_finalize(n, z_.get() + r0, hcat_.get() + r0 * heads_.ldh, heads_, hk_.get() + r0 * kHirsh,
                        e_nn_.get() + r0, raw_q_.get() + r0, ratio_.get() + r0, c6 ? hk6_.get() + r0 * kHirsh : nullptr,
                        c6 ? ratio6_.get() + r0 : nullptr, s);
  // charge conservation: exact sum of the raw charges per image (over all GPUs)
  if (identity_) {
    exact_sums(raw_q_.get(), 1, 1, nimg, image_start_.get(), img_sums_.get());
  } else {
    exact_sums(raw_q_.get(), 1, 1, 1, own_seg, img_sums_.get());
  }
  launch_charge_correct(n, raw_q_.get() + r0, img_sums_.get(), image_charge_.get(), image_of_.get() + r0, count_seg,
                        q_.get() + r0, nullptr, nullptr, s);
  allgather_rows(q_.get(), 1, kProfLrGather);
  allgather_rows(ratio_.get(), 1, kProfLrGather);
  if (c6) allgather_rows(ratio6_.get(), 1, kProfLrGather);

  // ---- long range (owned rows) ------------------------------------------------
  launch_long_range(n, spec_.n, nb_, lr_cut_, z_.get(), q_.get(), ratio_.get(), c6 ? ratio6_.get() : nullptr,
                    alpha_ref_, c6_ref_, ref_table_, lr_,
                    reinterpret_cast<double4 *>(lr_pos4_.get()), reinterpret_cast<double4 *>(lr_par4_.get()),
                    e_lr_.get(), e_elec_.get(), e_disp_.get(), dq_.get(), dh_.get(), c6 ? dc6_.get() : nullptr,
                    f_lr_.get(), w_lr_.get(), s, att32);  // float32 pair term with the float32 attention
  if (identity_) {
    exact_sums(dq_.get(), 1, 1, nimg, image_start_.get(), img_sums_.get());
  } else {
    exact_sums(dq_.get(), 1, 1, 1, own_seg, img_sums_.get());
  }
  launch_charge_correct(identity_ ? nimg : 1, nullptr, nullptr, nullptr, nullptr, count_seg, nullptr, dq_mean_.get(),
                        img_sums_.get(), s);

  // ---- reverse ---------------------------------------------------------------
  launch_heads_seed(n, z_.get() + r0, hpre_.get() + r0 * heads_.ldh, hk_.get() + r0 * kHirsh, heads_, dq_.get() + r0,
                    dq_mean_.get(), image_of_.get() + r0, dh_.get() + r0, c6 ? hk6_.get() + r0 * kHirsh : nullptr,
                    c6 ? dc6_.get() + r0 : nullptr, g_hcat_.get() + r0 * heads_.ldh, s);
  {
    GemmArgs g{};
    g.M = n; g.N = kF; g.K = heads_.ldh;
    g.A = g_hcat_.get() + r0 * heads_.ldh; g.lda = heads_.ldh;
    g.W = heads_.w1cat; g.ldw = kF; g.transB = false;
    g.C = g_x_.get() + r0 * kF; g.ldc = kF;
    launch_gemm(g, s);
  }
  double *gx = g_x_.get(), *gx_next = g_x2_.get();
  double *gev = nullptr, *gev_next = g_ev_.get();
  for (int b = layers_ - 1; b >= 0; --b) {
    const BlockW &w = blocks_[b];
    launch_post_attn_rev_final(n, gx + r0 * kF, gev ? gev + r0 * kEV : nullptr, xhat2_[b]->get() + r0 * kF,
                               rstd2_[b]->get() + r0, norm2_, w.ln2w, A_[b]->get() + r0 * kEV,
                               gate_[b]->get() + r0 * kHeads, g_t_.get() + r0 * kIntW, g_A_.get() + r0 * kEV, s);
    {  // g_cat = g_t W_int; g_post = g_cat[:, :128] + g_t[:, :128]
      GemmArgs g{};
      g.M = n; g.N = kIntW; g.K = kIntW;
      g.A = g_t_.get() + r0 * kIntW; g.lda = kIntW;
      g.W = w.intw; g.ldw = kIntW; g.transB = false;
      g.C = g_cat_.get() + r0 * kIntW; g.ldc = kIntW;
      g.aux = g_t_.get() + r0 * kIntW; g.ldaux = kIntW;
      g.epi = Epi::AddResidual;
      launch_gemm_ex(g, kF, 0, s);
    }
    {  // g_hp = (g_post W2) * silu'(hp)
      GemmArgs g{};
      g.M = n; g.N = kF; g.K = kF;
      g.A = g_cat_.get() + r0 * kIntW; g.lda = kIntW;
      g.W = w.mlp2w; g.ldw = kF; g.transB = false;
      g.C = g_hp_.get() + r0 * kF; g.ldc = kF;
      g.aux = hp_[b]->get() + r0 * kF; g.ldaux = kF;
      g.epi = Epi::SiluPrimeMul;
      launch_gemm(g, s);
    }
    {  // g_n1 = g_post + (g_hp W1) * silu'(n1)
      GemmArgs g{};
      g.M = n; g.N = kF; g.K = kF;
      g.A = g_hp_.get() + r0 * kF; g.lda = kF;
      g.W = w.mlp1w; g.ldw = kF; g.transB = false;
      g.C = g_n1_.get() + r0 * kF; g.ldc = kF;
      g.aux = n1_[b]->get() + r0 * kF; g.ldaux = kF;
      g.aux2 = g_cat_.get() + r0 * kIntW;
      g.epi = Epi::GateSiluResidual;
      launch_gemm_ex(g, kF, kIntW, s);
    }
    launch_post_attn_rev_ln1(n, g_n1_.get() + r0 * kF, xhat1_[b]->get() + r0 * kF, rstd1_[b]->get() + r0, norm1_,
                             w.ln1w, A_[b]->get() + r0 * kEV, w.cg_int, g_cat_.get() + r0 * kIntW,
                             g_a_.get() + r0 * kF, g_A_.get() + r0 * kEV, s);
    // the sender role of the attention reverse reads the neighbours' adjoints
    halo_exchange(g_a_.get(), kF, g_A_.get(), kEV, kProfAdjointHalo);
#if SO3LR_FEATURES == 128
    if (att32) {  // float32 copies of the adjoint rows the reverse gathers (owned and halo)
      const int nh = identity_ ? 0 : int(halo_recv_off_[nranks_]);
      float *ga32 = ga32_.reserve(std::size_t(N) * kF), *gA32 = gA32_.reserve(std::size_t(N) * kEV);
      launch_rows_to_float(identity_ ? N : n, identity_ ? 0 : int(r0), nh, halo_recv_rows_.get(), kF, g_a_.get(), ga32,
                           s);
      launch_rows_to_float(identity_ ? N : n, identity_ ? 0 : int(r0), nh, halo_recv_rows_.get(), kEV, g_A_.get(),
                           gA32, s);
      launch_attention_reverse32(n, nb_, geo_.get(), sh_.get(), qkv32_[b]->get(),
                                 reinterpret_cast<const float *>(f_inv_[b]->get()),
                                 reinterpret_cast<const float *>(f_ev_[b]->get()), ga32, gA32, norm_,
                                 b > 0 ? g_qkv_.get() : nullptr, pair_sc_.get(),
                                 reinterpret_cast<float *>(g_filt_inv_.get()), reinterpret_cast<float *>(g_filt_ev_.get()),
                                 s);
    } else
#endif
      launch_attention_reverse(n, nb_, geo_.get(), sh_.get(), qkv_[b]->get(), f_inv_[b]->get(), f_ev_[b]->get(),
                               g_a_.get(), g_A_.get(), norm_, b > 0 ? g_qkv_.get() : nullptr, pair_sc_.get(),
                               g_filt_inv_.get(), g_filt_ev_.get(), s);
    prof_begin(kProfFilterReverse);
#if SO3LR_FEATURES == 128
    if (mixed_ && mixed_tc_)
      launch_filter_reverse_tc(P, geo_.get(), nb_.pair_a, nb_.pair_b, b > 0 ? evb_[b]->get() : nullptr,
                               tc_rev_consts_[b], w.finv32, w.fev32, reinterpret_cast<const float *>(g_filt_inv_.get()),
                               reinterpret_cast<const float *>(g_filt_ev_.get()),
                               reinterpret_cast<const float *>(sp_[b]->get()), drbf_.get(), g_A_.get(),
                               pair_sc_.get(), b > 0, b < layers_ - 1, g_r_.get(), g_y_.get(), gl0_.get(), tc_err_,
                               num_sms_, s);
    else if (mixed_)
      launch_filter_reverse_mixed(P, geo_.get(), nb_.pair_a, nb_.pair_b, b > 0 ? evb_[b]->get() : nullptr, w.cg_att,
                                  w.finv, w.fev, w.finv32, w.fev32, g_filt_inv_.get(), g_filt_ev_.get(),
                                  reinterpret_cast<const float *>(sp_[b]->get()), drbf_.get(), g_A_.get(),
                                  pair_sc_.get(), b > 0, b < layers_ - 1, g_r_.get(), g_y_.get(), gl0_.get(), s);
    else
#endif
      launch_filter_reverse(P, geo_.get(), nb_.pair_a, nb_.pair_b, b > 0 ? evb_[b]->get() : nullptr, w.cg_att,
                            w.finv, w.fev, rad_, g_filt_inv_.get(), g_filt_ev_.get(), sp_[b]->get(), drbf_.get(),
                            g_A_.get(), pair_sc_.get(), b > 0, b < layers_ - 1, g_r_.get(), g_y_.get(),
                            gl0_.get(), s);
    prof_end(kProfFilterReverse, kFilterFlopsPerPair * double(P));
    if (b > 0) {
      if (qk_norm_)  // gradient w.r.t. the projections before their normalisation
        launch_qk_norm_reverse(n, qkv_[b]->get() + r0 * kQKV, qkr_[b]->get() + r0 * 4 * kHeads, g_qkv_.get() + r0 * kQKV, s);
      GemmArgs g{};  // g_x_in = g_a + per-head (g_qkv W^T)
      g.M = n; g.N = 32; g.K = 160;
      g.A = g_qkv_.get() + r0 * kQKV; g.lda = kQKV; g.strideA = 160;
      g.W = w.qkv_rev; g.ldw = 160; g.transB = true; g.strideW = 32 * 160;
      g.C = gx_next + r0 * kF; g.ldc = kF; g.strideC = 32;
      g.aux = g_a_.get() + r0 * kF; g.ldaux = kF; g.strideAux = 32;
      g.epi = Epi::AddResidual;
      g.batch = kHeads;
      launch_gemm(g, s);
      // block b's input is resid[b] y + x0[b] x0: the previous output y gets resid[b] of it
      if (residual_scalars_) launch_scale_rows(n, gx_next + r0 * kF, resid_[b], s);
      launch_ev_l0_reverse(n, nb_, evb_[b]->get(), w.cg_att, gl0_.get(), g_A_.get(), gev_next, s);
      std::swap(gx, gx_next);
      gev = gev_next;
      gev_next = (gev == g_ev_.get()) ? g_ev2_.get() : g_ev_.get();
    }
  }

  launch_pair_tail(P, geo_.get(), g_r_.get(), g_y_.get(), gv_.get(), s);

  // ---- assembly (owned rows) ----------------------------------------------------
  launch_assemble(nb_, geo_.get(), gv_.get(), e_nn_.get(), e_lr_.get(), f_lr_.get(), w_lr_.get(), force_.get(),
                  e_atom_.get(), e_zbl_.get(), w_atom_.get(), s);
  if (identity_) {
    exact_sums(e_atom_.get(), 1, 1, nimg, image_start_.get(), image_energy_.get());
    exact_sums(e_atom_.get(), 1, 1, 1, own_seg, totals_.get());
  } else {
    exact_sums(e_atom_.get(), 1, 1, 1, own_seg, image_energy_.get());
    exact_sums(e_atom_.get(), 1, 1, 1, own_seg, totals_.get());
  }
  exact_sums(w_atom_.get(), 6, 6, 1, own_seg, totals_.get() + 1);
  computed_ = true;
}

void Evaluator::download_virial_atom(double *vatom) {
  SO3_CUDA(cudaSetDevice(device_));
  const int n = spec_.n;
  if (identity_) {
    SO3_CUDA(cudaMemcpyAsync(vatom, w_atom_.get(), sizeof(double) * 6 * std::size_t(n), cudaMemcpyDeviceToHost,
                             stream_));
    SO3_CUDA(cudaStreamSynchronize(stream_));
    return;
  }
  allgather_rows(w_atom_.get(), 6);
  SO3_CUDA(cudaMemcpyAsync(stage_.data(), w_atom_.get(), sizeof(double) * 6 * std::size_t(n_rows_),
                           cudaMemcpyDeviceToHost, stream_));
  SO3_CUDA(cudaStreamSynchronize(stream_));
  for (int i = 0; i < n; ++i)
    for (int k = 0; k < 6; ++k) vatom[std::size_t(i) * 6 + k] = stage_[std::size_t(row_of_[i]) * 6 + k];
}

Evaluator::HostResult Evaluator::download(double *f, double *eatom, double *charges, double *ratios,
                                          double *e_learned, double *e_zbl, double *e_lr, double *e_elec,
                                          double *e_disp, double *image_energy) {
  SO3_CUDA(cudaSetDevice(device_));
  const int n = spec_.n;
  const int nimg = int(spec_.image_start.size()) - 1;
  cudaStream_t s = stream_;
  // every rank returns the whole system: gather the other GPUs' rows first
  auto fetch = [&](double *dst, double *src, int width) {
    if (!dst) return;
    if (identity_) {
      SO3_CUDA(cudaMemcpyAsync(dst, src, sizeof(double) * width * std::size_t(n), cudaMemcpyDeviceToHost, s));
      return;
    }
    allgather_rows(src, width);
    SO3_CUDA(cudaMemcpyAsync(stage_.data(), src, sizeof(double) * width * std::size_t(n_rows_), cudaMemcpyDeviceToHost,
                             s));
    SO3_CUDA(cudaStreamSynchronize(s));
    for (int i = 0; i < n; ++i)
      for (int k = 0; k < width; ++k) dst[std::size_t(i) * width + k] = stage_[std::size_t(row_of_[i]) * width + k];
  };
  fetch(f, force_.get(), 3);
  fetch(eatom, e_atom_.get(), 1);
  fetch(charges, q_.get(), 1);
  fetch(ratios, ratio_.get(), 1);
  fetch(e_learned, e_nn_.get(), 1);
  fetch(e_zbl, e_zbl_.get(), 1);
  fetch(e_lr, e_lr_.get(), 1);
  fetch(e_elec, e_elec_.get(), 1);
  fetch(e_disp, e_disp_.get(), 1);
  if (image_energy) SO3_CUDA(cudaMemcpyAsync(image_energy, image_energy_.get(), sizeof(double) * nimg, cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaMemcpyAsync(host_totals_, totals_.get(), sizeof(double) * 7, cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaMemcpyAsync(host_small_ + 8, nb_.error_flag, sizeof(int), cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaMemcpyAsync(host_small_ + 9, tc_err_, sizeof(int), cudaMemcpyDeviceToHost, s));
  SO3_CUDA(cudaStreamSynchronize(s));
  check_device_flags();
  HostResult r;
  r.energy = host_totals_[0];
  for (int k = 0; k < 6; ++k) r.virial[k] = host_totals_[1 + k];
  return r;
}

// ---------------------------------------------------------------------------
// device-resident MD (velocity Verlet, LAMMPS metal units: ftm2v = 1/1.0364269e-4);
// each GPU integrates its own atoms and the new positions are all-gathered
// ---------------------------------------------------------------------------
void Evaluator::md_setup(const double *host_v, const double *host_mass) {
  SO3_CUDA(cudaSetDevice(device_));
  const int n = spec_.n;
  std::vector<double> v_rows(3 * std::size_t(n_rows_), 0.0), inv_rows(n_rows_, 0.0);
  for (int i = 0; i < n; ++i) {
    if (!(host_mass[i] > 0)) throw Error("SO3LR MD: masses must be positive");
    inv_rows[row_of_[i]] = 1.0 / host_mass[i];
    for (int d = 0; d < 3; ++d) v_rows[3 * std::size_t(row_of_[i]) + d] = host_v[3 * std::size_t(i) + d];
  }
  SO3_CUDA(cudaMemcpyAsync(v_.reserve(3 * std::size_t(n_rows_)), v_rows.data(), sizeof(double) * 3 * n_rows_,
                           cudaMemcpyHostToDevice, stream_));
  SO3_CUDA(cudaMemcpyAsync(inv_mass_.reserve(n_rows_), inv_rows.data(), sizeof(double) * n_rows_,
                           cudaMemcpyHostToDevice, stream_));
  std::vector<double> mass_rows(n_rows_, 0.0);
  for (int i = 0; i < n; ++i) mass_rows[row_of_[i]] = host_mass[i];
  SO3_CUDA(cudaMemcpyAsync(mass_.reserve(n_rows_), mass_rows.data(), sizeof(double) * n_rows_,
                           cudaMemcpyHostToDevice, stream_));
  ke2_.reserve(n_rows_);
  nvt_ = false;
  compute();  // forces at the starting positions
  SO3_CUDA(cudaStreamSynchronize(stream_));
  md_ready_ = true;
}

void Evaluator::md_thermostat(double t_target_k, double t_damp_ps, int chain) {
  SO3_CUDA(cudaSetDevice(device_));
  if (!md_ready_) throw Error("SO3LR MD: call so3lr_md_init before setting a thermostat");
  if (!(t_damp_ps > 0.0)) {
    nvt_ = false;
    return;
  }
  if (!(t_target_k > 0.0)) throw Error("SO3LR MD: the thermostat target temperature must be positive");
  if (chain < 1 || chain > kMaxChain)
    throw Error("SO3LR MD: Nose-Hoover chain length must be in 1.." + std::to_string(kMaxChain));
  constexpr double kBoltzMetal = 8.617343e-5;  // eV / K
  NhcState st{};
  st.chain = chain;
  st.kt = kBoltzMetal * t_target_k;
  st.ndof = 3.0 * spec_.n - 3.0;
  if (st.ndof < 1.0) throw Error("SO3LR MD: a thermostat needs at least two atoms");
  const double tau2 = t_damp_ps * t_damp_ps;
  for (int j = 0; j < chain; ++j) st.q[j] = (j == 0 ? st.ndof : 1.0) * st.kt * tau2;
  constexpr std::size_t words = (sizeof(NhcState) + sizeof(double) - 1) / sizeof(double);
  double *d = nhc_state_.reserve(words);
  SO3_CUDA(cudaMemcpyAsync(d, &st, sizeof(NhcState), cudaMemcpyHostToDevice, stream_));
  nhc_scalars_.reserve(2);
  SO3_CUDA(cudaStreamSynchronize(stream_));
  nvt_ = true;
}

double Evaluator::md_thermostat_energy() {
  SO3_CUDA(cudaSetDevice(device_));
  if (!nvt_) return 0.0;
  NhcState st{};
  SO3_CUDA(cudaMemcpyAsync(&st, nhc_state_.get(), sizeof(NhcState), cudaMemcpyDeviceToHost, stream_));
  SO3_CUDA(cudaStreamSynchronize(stream_));
  double e = 0.0;
  for (int j = 0; j < st.chain; ++j) {
    e += 0.5 * st.q[j] * st.veta[j] * st.veta[j];
    e += (j == 0 ? st.ndof : 1.0) * st.kt * st.eta[j];
  }
  return e;
}

// half step of the chain: exact 2K over all GPUs, chain update, velocity scaling
void Evaluator::nhc_half(double dt) {
  constexpr double mvv2e = 1.0364269e-4;
  const std::size_t r0 = std::size_t(row0_);
  double *two_k = nhc_scalars_.get(), *scale = two_k + 1;
  launch_two_ke(n_own_, v_.get() + 3 * r0, mass_.get() + r0, mvv2e, ke2_.get() + r0, stream_);
  exact_sums(ke2_.get(), 1, 1, 1, seg_.get(), two_k);
  launch_nhc_half(reinterpret_cast<NhcState *>(nhc_state_.get()), two_k, dt, scale, stream_);
  launch_scale_v(n_own_, v_.get() + 3 * r0, scale, stream_);
}

void Evaluator::md_steps(int nsteps, double dt) {
  constexpr double ftm2v = 1.0 / 1.0364269e-4;
  const std::size_t r0 = std::size_t(row0_);
  if (!md_ready_) throw Error("SO3LR MD: call so3lr_md_init first");
  if (nsteps < 0) throw Error("SO3LR MD: the step count must not be negative");
  if (!std::isfinite(dt)) throw Error("SO3LR MD: the timestep must be finite");
  for (int step = 0; step < nsteps; ++step) {
    if (nvt_) nhc_half(dt);
    launch_verlet_first(n_own_, x_.get() + 3 * r0, v_.get() + 3 * r0, force_.get() + 3 * r0, inv_mass_.get() + r0, dt,
                        ftm2v, stream_);
    allgather_rows(x_.get(), 3, kProfPositionGather);
    compute();
    launch_verlet_second(n_own_, v_.get() + 3 * r0, force_.get() + 3 * r0, inv_mass_.get() + r0, dt, ftm2v, stream_);
    if (nvt_) nhc_half(dt);
  }
}

void Evaluator::md_download(double *x, double *v) {
  const int n = spec_.n;
  auto fetch = [&](double *dst, double *src) {
    if (!dst) return;
    if (identity_) {
      SO3_CUDA(cudaMemcpyAsync(dst, src, sizeof(double) * 3 * n, cudaMemcpyDeviceToHost, stream_));
      SO3_CUDA(cudaStreamSynchronize(stream_));
      return;
    }
    allgather_rows(src, 3);
    SO3_CUDA(cudaMemcpyAsync(stage_.data(), src, sizeof(double) * 3 * n_rows_, cudaMemcpyDeviceToHost, stream_));
    SO3_CUDA(cudaStreamSynchronize(stream_));
    for (int i = 0; i < n; ++i)
      for (int d = 0; d < 3; ++d) dst[3 * std::size_t(i) + d] = stage_[3 * std::size_t(row_of_[i]) + d];
  };
  fetch(x, x_.get());
  fetch(v, v_.get());
}

void Evaluator::set_mixed_precision(bool on) {
  if (on && kF != 128)
    throw Error("SO3LR: mixed precision is implemented for F = 128 models only; this model has F = " +
                std::to_string(kF));
  mixed_ = on;
}

SO3LR_SHAPE_END

namespace so3lr_b200 {
#if SO3LR_FEATURES == 128
std::unique_ptr<EvaluatorApi> create_evaluator_f128(Model &&model, int device) {
  return std::make_unique<Evaluator>(std::move(model), device);
}
#else
std::unique_ptr<EvaluatorApi> create_evaluator_f256(Model &&model, int device) {
  return std::make_unique<Evaluator>(std::move(model), device);
}
#endif
}  // namespace so3lr_b200
