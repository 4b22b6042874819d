// Equivariant attention message passing over the receiver CSR, forward and
// reverse, one warp per receiver atom, no atomics.
//
// Reference: src/kokkos_integrated_block0.cpp:330-385 (forward: per head
// alpha = sum_c q_r k_s f / norm, no softmax; d_inv[r] += phi alpha v_s,
// d_ev[r] += phi alpha_ev Y), src/kokkos_attention_scatter_reverse.cpp:280-502 and
// src/kokkos_block2_attention_input_reverse.cpp:267-299 (reverse). The reference
// scatters sender-side gradients with float atomics; here every atom gathers
// both roles over its own row: as receiver of edge b->a and as sender of the
// reverse edge a->b, which visits each outgoing edge exactly once.
//
// Lane layout: lane owns invariant channels kPL lane .. kPL lane + kPL - 1
// (kPL = F / 32: 4 for F = 128, 8 for F = 256; head = lane / kLPH, kLPH = 32 /
// heads lanes per head) and equivariant channels lane + 32 j (j < kEVL).
// qkv rows are head-major: [head][q, k, v, q_ev, k_ev][32].
//
// Both kernels are templates on the real type T of the per-pair filters, the
// per-atom rows they gather (qkv, and g_a, g_A in the reverse) and their
// arithmetic: double for the float64 path, float for the mixed-precision path
// with the tcgen05 filters (the filters are stored in float32 there and the
// rows are float32 copies; outputs that float64 code consumes stay double).
#include "kernels.cuh"

SO3LR_SHAPE_BEGIN
namespace {

constexpr int kPL = kF / 32;          // invariant channels per lane
constexpr int kLPH = 32 / kHeads;     // lanes per head
constexpr int kEVL = (kEV + 31) / 32; // equivariant channels per lane

template <typename T>
__device__ inline T head_sum(T v) {  // sum over the kLPH lanes of a head
#pragma unroll
  for (int off = 1; off < kLPH; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}
// explicitly rounded product and sum (no FMA contraction)
__device__ inline double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ inline float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ inline double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ inline float add_rn(float a, float b) { return __fadd_rn(a, b); }

// kPL consecutive doubles (32-byte aligned, read-only during the kernel) with
// 256-bit loads
__device__ inline void load4(const double *p, double (&v)[kPL]) {
#pragma unroll
  for (int q = 0; q < kPL; q += 4)
    asm("ld.global.nc.v4.f64 {%0,%1,%2,%3}, [%4];"
        : "=d"(v[q]), "=d"(v[q + 1]), "=d"(v[q + 2]), "=d"(v[q + 3])
        : "l"(p + q));
}
__device__ inline void store4(double *p, const double (&v)[kPL]) {
#pragma unroll
  for (int q = 0; q < kPL; q += 2) *reinterpret_cast<double2 *>(p + q) = make_double2(v[q], v[q + 1]);
}
// the same for float32 rows (16-byte aligned): 128-bit loads and stores
__device__ inline void load4(const float *p, float (&v)[kPL]) {
#pragma unroll
  for (int q = 0; q < kPL; q += 4)
    asm("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v[q]), "=f"(v[q + 1]), "=f"(v[q + 2]), "=f"(v[q + 3])
        : "l"(p + q));
}
__device__ inline void store4(float *p, const float (&v)[kPL]) {
#pragma unroll
  for (int q = 0; q < kPL; q += 4) *reinterpret_cast<float4 *>(p + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
}
__device__ inline void store4(double *p, const float (&v)[kPL]) {  // widened for float64 consumers
#pragma unroll
  for (int q = 0; q < kPL; q += 2) *reinterpret_cast<double2 *>(p + q) = make_double2(v[q], v[q + 1]);
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(256) k_attention_forward(int n, int row0, const int *__restrict__ row_start,
                                                           const int *__restrict__ nbr,
                                                           const int *__restrict__ edge_pair,
                                                           const double *__restrict__ geo,
                                                           const double *__restrict__ sh,
                                                           const T *__restrict__ qkv,
                                                           const T *__restrict__ f_inv,
                                                           const T *__restrict__ f_ev, double norm,
                                                           double *__restrict__ d_inv, double *__restrict__ d_ev) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const int a = row0 + r;
  const int h = lane / kLPH, o = (lane % kLPH) * kPL;
  const size_t head_off = size_t(h) * 160 + o;
  T qa[kPL], qea[kPL];
  load4(qkv + (size_t)a * kQKV + head_off + 0 * 32, qa);
  load4(qkv + (size_t)a * kQKV + head_off + 3 * 32, qea);
  T acc[kPL];
#pragma unroll
  for (int j = 0; j < kPL; ++j) acc[j] = T(0);
  T acc_ev[kEVL];
  int my_deg[kEVL], my_sh[kEVL];
  T my_par[kEVL];
#pragma unroll
  for (int j = 0; j < kEVL; ++j) {
    const int m = lane + 32 * j;
    acc_ev[j] = T(0);
    my_deg[j] = m < kEV ? degree_of_channel(m) : 0;
    my_sh[j] = m < kEV ? sh_of_channel(m) : 0;
    my_par[j] = T(parity_sign(my_deg[j]));
  }
  const T inv_norm = T(1.0 / norm);  // one division per atom instead of two per edge
  const int e0 = row_start[r], e1 = row_start[r + 1];
  // pull an edge's rows into L1 ahead of its use: the k, v and k_ev lines of
  // each head (double: lines 2-5 and 8-9 of the head's ten 128-byte lines;
  // float: lines 1, 2 and 4 of five), both filters and the harmonics (two
  // 96-byte halves)
  auto prefetch_edge = [&](int e) {
    const int bb = nbr[e], cc = edge_pair[e];
    const int pp = cc >= 0 ? cc : ~cc;
    constexpr int kLq = sizeof(T) == 8 ? 6 : 3;  // lines per head
    constexpr int kQl = kLq * kHeads, kFl = kF * int(sizeof(T)) / 128;
    for (int c = lane; c < kQl + 2 * kFl + 2; c += 32) {
      const char *addr;
      if (c < kQl) {
        const int j = c % kLq;
        const int line = sizeof(T) == 8 ? (c / 6) * 10 + (j < 4 ? 2 + j : 4 + j) : (c / 3) * 5 + (j < 2 ? 1 + j : 4);
        addr = reinterpret_cast<const char *>(qkv + (size_t)bb * kQKV) + 128 * line;
      } else if (c < kQl + kFl) {
        addr = reinterpret_cast<const char *>(f_inv + (size_t)pp * kF) + 128 * (c - kQl);
      } else if (c < kQl + 2 * kFl) {
        addr = reinterpret_cast<const char *>(f_ev + (size_t)pp * kF) + 128 * (c - kQl - kFl);
      } else {
        addr = reinterpret_cast<const char *>(sh + (size_t)pp * kSH) + 96 * (c - kQl - 2 * kFl);
      }
      asm volatile("prefetch.global.L1 [%0];\n" ::"l"(addr));
    }
  };
  // one edge's attention coefficients (alpha of both attentions, already
  // divided by the norm) and the rows its messages need
  struct EdgeTerms {
    T phi, ai, ae, vb[kPL], y[kEVL];
  };
  auto edge_terms = [&](int e, EdgeTerms &t) {
    const int bb = nbr[e], code = edge_pair[e];
    const int p = code >= 0 ? code : ~code;
    t.phi = T(geo[(size_t)p * kGeo + 4]);
    T kb[kPL], keb[kPL], fi[kPL], fe[kPL];
    load4(qkv + (size_t)bb * kQKV + head_off + 1 * 32, kb);
    load4(qkv + (size_t)bb * kQKV + head_off + 2 * 32, t.vb);
    load4(qkv + (size_t)bb * kQKV + head_off + 4 * 32, keb);
    load4(f_inv + (size_t)p * kF + lane * kPL, fi);
    load4(f_ev + (size_t)p * kF + lane * kPL, fe);
#pragma unroll
    for (int j = 0; j < kEVL; ++j) {
      T y = lane + 32 * j < kEV ? T(sh[(size_t)p * kSH + my_sh[j]]) : T(0);
      if (code < 0) y *= my_par[j];
      t.y[j] = y;
    }
    T ai = T(0), ae = T(0);
#pragma unroll
    for (int j = 0; j < kPL; ++j) {
      ai += qa[j] * kb[j] * fi[j];
      ae += qea[j] * keb[j] * fe[j];
    }
    t.ai = ai;
    t.ae = ae;
  };
  // the messages of one edge, added in edge order
  auto accumulate = [&](const EdgeTerms &t, T ai, T ae) {
    const T wi = t.phi * ai;
#pragma unroll
    for (int j = 0; j < kPL; ++j) acc[j] += wi * t.vb[j];
#pragma unroll
    for (int j = 0; j < kEVL; ++j) {
      const T ae_m = __shfl_sync(0xffffffffu, ae, my_deg[j] * kLPH);
      if (lane + 32 * j < kEV) acc_ev[j] += t.phi * ae_m * t.y[j];
    }
  };
  // two edges per iteration: their loads and head reductions interleave
  int e = e0;
  for (; e + 1 < e1; e += 2) {
    if (e + 2 < e1) prefetch_edge(e + 2);
    if (e + 3 < e1) prefetch_edge(e + 3);
    EdgeTerms t0, t1;
    edge_terms(e, t0);
    edge_terms(e + 1, t1);
    const T ai0 = head_sum(t0.ai) * inv_norm, ai1 = head_sum(t1.ai) * inv_norm;
    const T ae0 = head_sum(t0.ae) * inv_norm, ae1 = head_sum(t1.ae) * inv_norm;
    accumulate(t0, ai0, ae0);
    accumulate(t1, ai1, ae1);
  }
  if (e < e1) {
    EdgeTerms t0;
    edge_terms(e, t0);
    accumulate(t0, head_sum(t0.ai) * inv_norm, head_sum(t0.ae) * inv_norm);
  }
  store4(d_inv + (size_t)a * kF + lane * kPL, acc);
#pragma unroll
  for (int j = 0; j < kEVL; ++j)
    if (lane + 32 * j < kEV) d_ev[(size_t)a * kEV + lane + 32 * j] = double(acc_ev[j]);
}

void launch_attention_forward(int n, const NeighborState &nb, const double *geo, const double *sh,
                              const double *qkv, const double *f_inv, const double *f_ev, double norm,
                              double *d_inv, double *d_ev, cudaStream_t s) {
  if (n == 0) return;
  k_attention_forward<double><<<(n * 32 + 255) / 256, 256, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair,
                                                                   geo, sh, qkv, f_inv, f_ev, norm, d_inv, d_ev);
  SO3_LAUNCH("attention_forward");
}
#if SO3LR_FEATURES == 128
void launch_attention_forward32(int n, const NeighborState &nb, const double *geo, const double *sh,
                                const float *qkv, const float *f_inv, const float *f_ev, double norm,
                                double *d_inv, double *d_ev, cudaStream_t s) {
  if (n == 0) return;
  k_attention_forward<float><<<(n * 32 + 255) / 256, 256, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair,
                                                                  geo, sh, qkv, f_inv, f_ev, norm, d_inv, d_ev);
  SO3_LAUNCH("attention_forward32");
}
#endif

// Reverse: given g_a = dL/d(d_inv) (= dL/da) and g_A = dL/d(d_ev) for every atom,
// produce dL/d{q,k,v,q_ev,k_ev} per atom and, for the primary edge of every pair,
// the scalars the filter reverse needs.
template <typename T>
__global__ void __launch_bounds__(32) k_attention_reverse(
    int n, int row0, const int *__restrict__ row_start, const int *__restrict__ nbr, const int *__restrict__ edge_pair,
    const double *__restrict__ geo, const double *__restrict__ sh, const T *__restrict__ qkv,
    const T *__restrict__ f_inv, const T *__restrict__ f_ev, const T *__restrict__ g_a,
    const T *__restrict__ g_A, double norm, double *__restrict__ g_qkv, double *__restrict__ pair_sc,
    T *__restrict__ g_filt_inv, T *__restrict__ g_filt_ev) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const int a = row0 + r;
  const int h = lane / kLPH, o = (lane % kLPH) * kPL;
  const size_t head_off = size_t(h) * 160 + o;
  const T *qa_row = qkv + (size_t)a * kQKV + head_off;
  T qa[kPL], ka[kPL], va[kPL], qea[kPL], kea[kPL], ga[kPL];
  load4(qa_row + 0 * 32, qa);
  load4(qa_row + 1 * 32, ka);
  load4(qa_row + 2 * 32, va);
  load4(qa_row + 3 * 32, qea);
  load4(qa_row + 4 * 32, kea);
  load4(g_a + (size_t)a * kF + lane * kPL, ga);
  // Equivariant channels by degree group: the kLPH lanes of head h hold the
  // channels of degree slot h (2 l + 1 of them; lane j of the group holds
  // channels j, j + kLPH, ...), so a reduction inside the group gives every
  // lane the degree sum its head uses. F = 128: 8 lanes for 3, 5, 7 and 9
  // channels (the group's first lane holds the ninth channel of l = 4 as well).
  constexpr int kCPL = (9 + kLPH - 1) / kLPH;  // channels per lane
  int ch[kCPL], shc[kCPL];
  T gAa[kCPL];
#pragma unroll
  for (int k = 0; k < kCPL; ++k) {
    const int j = lane % kLPH + kLPH * k;
    ch[k] = j < slot_width(h) ? slot_offset(h) + j : -1;
    shc[k] = ch[k] >= 0 ? sh_of_channel(ch[k]) : 0;
    gAa[k] = ch[k] >= 0 ? g_A[(size_t)a * kEV + ch[k]] : T(0);
  }
  const T par = T(parity_sign(h));
  T gq[kPL], gk[kPL], gv[kPL], gqe[kPL], gke[kPL];
#pragma unroll
  for (int j = 0; j < kPL; ++j) gq[j] = gk[j] = gv[j] = gqe[j] = gke[j] = T(0);
  const T inv_norm = T(1.0 / norm);
  const int e0 = row_start[r], e1 = row_start[r + 1];
  int b_nx = 0, code_nx = 0;
  if (e0 < e1) { b_nx = nbr[e0]; code_nx = edge_pair[e0]; }
  for (int e = e0; e < e1; ++e) {
    const int b = b_nx;
    const int code = code_nx;
    if (e + 1 < e1) { b_nx = nbr[e + 1]; code_nx = edge_pair[e + 1]; }
    const int p = code >= 0 ? code : ~code;
    if (e + 1 < e1) {
      // pull the next edge's rows into L1 while this one is processed: the qkv
      // row (5 kF / 16 lines of 128 B), g_a, f_inv and f_ev (kF / 16 lines
      // each), the 96-byte pieces of g_A and the two of the harmonics
      const int p_nx = code_nx >= 0 ? code_nx : ~code_nx;
      constexpr int kQl = 5 * kF * int(sizeof(T)) / 128, kFl = kF * int(sizeof(T)) / 128;
      constexpr int kAp = kEV * int(sizeof(T)) / 96;
      const char *qrow = reinterpret_cast<const char *>(qkv + (size_t)b_nx * kQKV);
#pragma unroll
      for (int c = lane; c < kQl + 3 * kFl + kAp + 2; c += 32) {
        const char *addr = c < kQl            ? qrow + 128 * c
                           : c < kQl + kFl     ? reinterpret_cast<const char *>(g_a + (size_t)b_nx * kF) + 128 * (c - kQl)
                           : c < kQl + 2 * kFl ? reinterpret_cast<const char *>(f_inv + (size_t)p_nx * kF) + 128 * (c - kQl - kFl)
                           : c < kQl + 3 * kFl ? reinterpret_cast<const char *>(f_ev + (size_t)p_nx * kF) + 128 * (c - kQl - 2 * kFl)
                           : c < kQl + 3 * kFl + kAp
                               ? reinterpret_cast<const char *>(g_A + (size_t)b_nx * kEV) + 96 * (c - kQl - 3 * kFl)
                               : reinterpret_cast<const char *>(sh + (size_t)p_nx * kSH) + 96 * (c - kQl - 3 * kFl - kAp);
        asm volatile("prefetch.global.L1 [%0];\n" ::"l"(addr));
      }
    }
    const T phi = T(geo[(size_t)p * kGeo + 4]);
    const T *b_row = qkv + (size_t)b * kQKV + head_off;
    T qb[kPL], kb[kPL], vb[kPL], qeb[kPL], keb[kPL], gb[kPL], fi[kPL], fe[kPL];
    load4(b_row + 0 * 32, qb);
    load4(b_row + 1 * 32, kb);
    load4(b_row + 2 * 32, vb);
    load4(b_row + 3 * 32, qeb);
    load4(b_row + 4 * 32, keb);
    load4(g_a + (size_t)b * kF + lane * kPL, gb);
    load4(f_inv + (size_t)p * kF + lane * kPL, fi);
    load4(f_ev + (size_t)p * kF + lane * kPL, fe);
    // harmonic-weighted adjoint sums per degree, for edge b->a ("in": y of the
    // edge into a) and a->b ("out": parity times that)
    T s_in, s_out;
    {
      const T pin = code < 0 ? par : T(1);  // harmonics are stored for the primary orientation
      T y[kCPL], gAb[kCPL];
#pragma unroll
      for (int k = 0; k < kCPL; ++k) {
        y[k] = ch[k] >= 0 ? T(sh[(size_t)p * kSH + shc[k]]) * pin : T(0);
        gAb[k] = ch[k] >= 0 ? g_A[(size_t)b * kEV + ch[k]] : T(0);
      }
      if constexpr (kCPL == 2) {
        s_in = gAa[0] * y[0] + gAa[1] * y[1];
        s_out = (gAb[0] * y[0] + gAb[1] * y[1]) * par;
      } else {
        s_in = gAa[0] * y[0];
        s_out = gAb[0] * y[0];
#pragma unroll
        for (int k = 1; k < kCPL; ++k) {
          s_in += gAa[k] * y[k];
          s_out += gAb[k] * y[k];
        }
        s_out *= par;
      }
      s_in = head_sum(s_in);
      s_out = head_sum(s_out);
    }
    T ai_out = 0, si_in = 0, si_out = 0;
#pragma unroll
    for (int j = 0; j < kPL; ++j) {
      ai_out += qb[j] * ka[j] * fi[j];
      si_in += ga[j] * vb[j];
      si_out += gb[j] * va[j];
    }
    ai_out = head_sum(ai_out) * inv_norm;
    si_in = head_sum(si_in);
    si_out = head_sum(si_out);
    const T c_q = phi * si_in * inv_norm, c_qe = phi * s_in * inv_norm;
    const T c_v = phi * ai_out, c_k = phi * si_out * inv_norm, c_ke = phi * s_out * inv_norm;
#pragma unroll
    for (int j = 0; j < kPL; ++j) {
      gq[j] += c_q * (kb[j] * fi[j]);
      gqe[j] += c_qe * (keb[j] * fe[j]);
      gv[j] += c_v * gb[j];
      gk[j] += c_k * (qb[j] * fi[j]);
      gke[j] += c_ke * (qeb[j] * fe[j]);
    }
    if (code >= 0) {
      // primary edge: the pair's filter gradient and its per-head scalars
      if (g_filt_inv != nullptr) {
        // g_f_inv[c] = phi/norm (s_in[h] q_a[c] k_b[c] + s_out[h] q_b[c] k_a[c]), same for ev;
        // explicitly rounded products and sum (no FMA contraction): the two
        // directions' terms swap when the pair is held from its other endpoint,
        // and a rounded sum is exactly commutative
        T gi[kPL], ge[kPL];
#pragma unroll
        for (int j = 0; j < kPL; ++j) {
          gi[j] = add_rn(mul_rn(c_q, mul_rn(qa[j], kb[j])), mul_rn(c_k, mul_rn(qb[j], ka[j])));
          ge[j] = add_rn(mul_rn(c_qe, mul_rn(qea[j], keb[j])), mul_rn(c_ke, mul_rn(qeb[j], kea[j])));
        }
        store4(g_filt_inv + (size_t)p * kF + lane * kPL, gi);
        store4(g_filt_ev + (size_t)p * kF + lane * kPL, ge);
      }
      T ai_in = 0, ae_in = 0, ae_out = 0;
#pragma unroll
      for (int j = 0; j < kPL; ++j) {
        ai_in += qa[j] * kb[j] * fi[j];
        ae_in += qea[j] * keb[j] * fe[j];
        ae_out += qeb[j] * kea[j] * fe[j];
      }
      ai_in = head_sum(ai_in) * inv_norm;
      ae_in = head_sum(ae_in) * inv_norm;
      ae_out = head_sum(ae_out) * inv_norm;
      // pair scalars for the filter reverse: the cutoff-gradient weight
      // sum_h (a_in s_in + a_out s_out) of the invariant and the ev attention,
      // and the ev coefficients of both directions per head. The two
      // directions' products are added with explicitly rounded (commutative)
      // sums and the heads in a symmetric tree, so the values do not depend on
      // which endpoint holds the pair.
      T t = add_rn(add_rn(mul_rn(ai_in, si_in), mul_rn(ai_out, si_out)),
                   add_rn(mul_rn(ae_in, s_in), mul_rn(ae_out, s_out)));
#pragma unroll
      for (int off = kLPH; off < 32; off <<= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
      double *ps = pair_sc + (size_t)p * kPairScalars;
      if (lane == 0) ps[0] = double(t);
      if (lane == 1) ps[kPairScalars - 1] = 0.0;
      if (lane % kLPH == 0) {
        ps[1 + h] = double(ae_in);
        ps[1 + kHeads + h] = double(ae_out);
      }
    }
  }
  if (g_qkv != nullptr) {
    double *out = g_qkv + (size_t)a * kQKV + head_off;
    store4(out + 0 * 32, gq);
    store4(out + 1 * 32, gk);
    store4(out + 2 * 32, gv);
    store4(out + 3 * 32, gqe);
    store4(out + 4 * 32, gke);
  }
}

void launch_attention_reverse(int n, const NeighborState &nb, const double *geo, const double *sh,
                              const double *qkv, const double *f_inv, const double *f_ev, const double *g_a,
                              const double *g_A, double norm, double *g_qkv, double *pair_sc, double *g_filt_inv,
                              double *g_filt_ev, cudaStream_t s) {
  if (n == 0) return;
  // one warp per CTA: at ~190 registers per thread a CTA's registers are freed
  // as soon as its own atom is done, instead of waiting for the slowest of eight
  k_attention_reverse<double><<<n, 32, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair, geo, sh, qkv, f_inv,
                                               f_ev, g_a, g_A, norm, g_qkv, pair_sc, g_filt_inv, g_filt_ev);
  SO3_LAUNCH("attention_reverse");
}
#if SO3LR_FEATURES == 128
void launch_attention_reverse32(int n, const NeighborState &nb, const double *geo, const double *sh,
                                const float *qkv, const float *f_inv, const float *f_ev, const float *g_a,
                                const float *g_A, double norm, double *g_qkv, double *pair_sc, float *g_filt_inv,
                                float *g_filt_ev, cudaStream_t s) {
  if (n == 0) return;
  k_attention_reverse<float><<<n, 32, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair, geo, sh, qkv, f_inv,
                                              f_ev, g_a, g_A, norm, g_qkv, pair_sc, g_filt_inv, g_filt_ev);
  SO3_LAUNCH("attention_reverse32");
}

// float32 copies of rows [r0, r0 + n) and of the listed rows of a row-major
// double array of the given width (the rows the attention kernels gather)
__global__ void k_rows_to_float(int n, int r0, int nlist, const int *__restrict__ rows, int width,
                                const double *__restrict__ src, float *__restrict__ dst) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)(n + nlist) * (width / 2);
  if (i >= total) return;
  const int k = int(i / (width / 2)), c = int(i % (width / 2)) * 2;
  const long long row = k < n ? (long long)r0 + k : (long long)rows[k - n];
  const double2 v = *reinterpret_cast<const double2 *>(src + row * width + c);
  *reinterpret_cast<float2 *>(dst + row * width + c) = make_float2(float(v.x), float(v.y));
}
void launch_rows_to_float(int n, int r0, int nlist, const int *rows, int width, const double *src, float *dst,
                          cudaStream_t s) {
  const long long total = (long long)(n + nlist) * (width / 2);
  if (total == 0) return;
  k_rows_to_float<<<unsigned((total + 255) / 256), 256, 0, s>>>(n, r0, nlist, rows, width, src, dst);
  SO3_LAUNCH("rows_to_float");
}
#endif

// g_ev[a][m] = g_A[a][m] + sum over a's pairs of 2 (ev_a - ev_b)[m] cg[m] gl0[p][slot of m]
__global__ void k_ev_l0_reverse(int n, int row0, const int *__restrict__ row_start, const int *__restrict__ nbr,
                                const int *__restrict__ edge_pair, const double *__restrict__ ev,
                                const double *__restrict__ cg, const double *__restrict__ gl0,
                                const double *__restrict__ g_A, double *__restrict__ g_ev) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const int a = row0 + r;
#pragma unroll
  for (int j = 0; j < kEVL; ++j) {
    const int m = lane + 32 * j;
    if (m >= kEV) break;
    const int d = degree_of_channel(m);
    const double eva = ev[(size_t)a * kEV + m];
    const double c = 2.0 * cg[m];
    double acc = 0.0;
    for (int e = row_start[r]; e < row_start[r + 1]; ++e) {
      const int b = nbr[e];
      const int code = edge_pair[e];
      const int p = code >= 0 ? code : ~code;
      acc += (eva - ev[(size_t)b * kEV + m]) * c * gl0[(size_t)p * kHeads + d];
    }
    g_ev[(size_t)a * kEV + m] = g_A[(size_t)a * kEV + m] + acc;
  }
}

void launch_ev_l0_reverse(int n, const NeighborState &nb, const double *ev, const double *cg_att,
                          const double *gl0, const double *g_A, double *g_ev, cudaStream_t s) {
  if (n == 0) return;
  k_ev_l0_reverse<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair, ev, cg_att,
                                                       gl0, g_A, g_ev);
  SO3_LAUNCH("ev_l0_reverse");
}

SO3LR_SHAPE_END
