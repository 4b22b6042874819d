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
// Lane layout: lane owns channels 4*lane .. 4*lane+3 of the 128 invariant
// channels (head = lane / 8); lanes 0..23 own the 24 equivariant channels.
// qkv rows are head-major: [head][q, k, v, q_ev, k_ev][32].
#include "kernels.cuh"

namespace so3lr_b200 {
namespace {

__device__ inline double head_sum(double v) {  // sum over the 8 lanes of a head
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  return v;
}

// four consecutive doubles (32-byte aligned, read-only during the kernel) with
// one 256-bit load
__device__ inline void load4(const double *p, double (&v)[4]) {
  asm("ld.global.nc.v4.f64 {%0,%1,%2,%3}, [%4];"
               : "=d"(v[0]), "=d"(v[1]), "=d"(v[2]), "=d"(v[3])
               : "l"(p));
}
__device__ inline void store4(double *p, const double (&v)[4]) {
  *reinterpret_cast<double2 *>(p) = make_double2(v[0], v[1]);
  *reinterpret_cast<double2 *>(p + 2) = make_double2(v[2], v[3]);
}

}  // namespace

__global__ void __launch_bounds__(256) k_attention_forward(int n, int row0, const int *__restrict__ row_start,
                                                           const int *__restrict__ nbr,
                                                           const int *__restrict__ edge_pair,
                                                           const double *__restrict__ geo,
                                                           const double *__restrict__ sh,
                                                           const double *__restrict__ qkv,
                                                           const double *__restrict__ f_inv,
                                                           const double *__restrict__ f_ev, double norm,
                                                           double *__restrict__ d_inv, double *__restrict__ d_ev) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const int a = row0 + r;
  const int h = lane >> 3, o = (lane & 7) * 4;
  const size_t head_off = size_t(h) * 160 + o;
  double qa[4], qea[4];
  load4(qkv + (size_t)a * kQKV + head_off + 0 * 32, qa);
  load4(qkv + (size_t)a * kQKV + head_off + 3 * 32, qea);
  double acc[4] = {0, 0, 0, 0};
  double acc_ev = 0.0;
  const double inv_norm = 1.0 / norm;  // one division per atom instead of two per edge
  const int my_deg = lane < kEV ? degree_of_channel(lane) : 0;
  const double my_par = parity_sign(my_deg);
  const int e0 = row_start[r], e1 = row_start[r + 1];
  int b_nx = 0, code_nx = 0;  // indices of the next edge, loaded one iteration ahead
  if (e0 < e1) {
    b_nx = nbr[e0];
    code_nx = edge_pair[e0];
  }
  for (int e = e0; e < e1; ++e) {
    const int b = b_nx;
    const int code = code_nx;
    if (e + 1 < e1) {
      b_nx = nbr[e + 1];
      code_nx = edge_pair[e + 1];
      // pull the next edge's rows into L1 while this one is processed: the k, v
      // and k_ev lines of each head (lines 2-5 and 8-9 of the head's ten 128-byte
      // lines), both filters (8 lines each) and the harmonics (two 96-byte halves)
      const int p_nx = code_nx >= 0 ? code_nx : ~code_nx;
      for (int c = lane; c < 42; c += 32) {
        const char *addr;
        if (c < 24) {
          const int j = c % 6;
          addr = reinterpret_cast<const char *>(qkv + (size_t)b_nx * kQKV) + 128 * ((c / 6) * 10 + (j < 4 ? 2 + j : 4 + j));
        } else if (c < 32) {
          addr = reinterpret_cast<const char *>(f_inv + (size_t)p_nx * kF) + 128 * (c - 24);
        } else if (c < 40) {
          addr = reinterpret_cast<const char *>(f_ev + (size_t)p_nx * kF) + 128 * (c - 32);
        } else {
          addr = reinterpret_cast<const char *>(sh + (size_t)p_nx * kEV) + 96 * (c - 40);
        }
        asm volatile("prefetch.global.L1 [%0];\n" ::"l"(addr));
      }
    }
    const int p = code >= 0 ? code : ~code;
    const double phi = geo[(size_t)p * kGeo + 4];
    double kb[4], vb[4], keb[4], fi[4], fe[4];
    load4(qkv + (size_t)b * kQKV + head_off + 1 * 32, kb);
    load4(qkv + (size_t)b * kQKV + head_off + 2 * 32, vb);
    load4(qkv + (size_t)b * kQKV + head_off + 4 * 32, keb);
    load4(f_inv + (size_t)p * kF + lane * 4, fi);
    load4(f_ev + (size_t)p * kF + lane * 4, fe);
    double ai = 0.0, ae = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ai += qa[j] * kb[j] * fi[j];
      ae += qea[j] * keb[j] * fe[j];
    }
    ai = head_sum(ai) * inv_norm;
    ae = head_sum(ae) * inv_norm;
    const double wi = phi * ai;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] += wi * vb[j];
    const double ae_m = __shfl_sync(0xffffffffu, ae, my_deg * 8);
    if (lane < kEV) {
      double y = sh[(size_t)p * kEV + lane];
      if (code < 0) y *= my_par;
      acc_ev += phi * ae_m * y;
    }
  }
  store4(d_inv + (size_t)a * kF + lane * 4, acc);
  if (lane < kEV) d_ev[(size_t)a * kEV + lane] = acc_ev;
}

void launch_attention_forward(int n, const NeighborState &nb, const double *geo, const double *sh,
                              const double *qkv, const double *f_inv, const double *f_ev, double norm,
                              double *d_inv, double *d_ev, cudaStream_t s) {
  if (n == 0) return;
  k_attention_forward<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair, geo, sh,
                                                           qkv, f_inv, f_ev, norm, d_inv, d_ev);
  SO3_LAUNCH("attention_forward");
}

// Reverse: given g_a = dL/d(d_inv) (= dL/da) and g_A = dL/d(d_ev) for every atom,
// produce dL/d{q,k,v,q_ev,k_ev} per atom and, for the primary edge of every pair,
// the scalars the filter reverse needs.
__global__ void __launch_bounds__(32) k_attention_reverse(
    int n, int row0, const int *__restrict__ row_start, const int *__restrict__ nbr, const int *__restrict__ edge_pair,
    const double *__restrict__ geo, const double *__restrict__ sh, const double *__restrict__ qkv,
    const double *__restrict__ f_inv, const double *__restrict__ f_ev, const double *__restrict__ g_a,
    const double *__restrict__ g_A, double norm, double *__restrict__ g_qkv, double *__restrict__ pair_sc,
    double *__restrict__ g_filt_inv, double *__restrict__ g_filt_ev) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const int a = row0 + r;
  const int h = lane >> 3, o = (lane & 7) * 4;
  const size_t head_off = size_t(h) * 160 + o;
  const double *qa_row = qkv + (size_t)a * kQKV + head_off;
  double qa[4], ka[4], va[4], qea[4], kea[4], ga[4];
  load4(qa_row + 0 * 32, qa);
  load4(qa_row + 1 * 32, ka);
  load4(qa_row + 2 * 32, va);
  load4(qa_row + 3 * 32, qea);
  load4(qa_row + 4 * 32, kea);
  load4(g_a + (size_t)a * kF + lane * 4, ga);
  // Equivariant channels by degree group: the 8 lanes of head h hold the
  // channels of degree slot h (3, 5, 7 and 9 channels; lane 24 holds the ninth
  // channel of the last degree as well), so a 3-step reduction inside the group
  // gives every lane the degree sum its head uses.
  const int dbase = h == 0 ? 0 : (h == 1 ? 3 : (h == 2 ? 8 : 15));
  const int dcount = h == 0 ? 3 : (h == 1 ? 5 : (h == 2 ? 7 : 8));
  const int ch0 = (lane & 7) < dcount ? dbase + (lane & 7) : -1;
  const int ch1 = lane == 24 ? 23 : -1;
  const double par = parity_sign(h);
  const double gAa0 = ch0 >= 0 ? g_A[(size_t)a * kEV + ch0] : 0.0;
  const double gAa1 = ch1 >= 0 ? g_A[(size_t)a * kEV + ch1] : 0.0;
  double gq[4] = {0, 0, 0, 0}, gk[4] = {0, 0, 0, 0}, gv[4] = {0, 0, 0, 0}, gqe[4] = {0, 0, 0, 0},
         gke[4] = {0, 0, 0, 0};
  const double inv_norm = 1.0 / norm;
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
      // row (40 lines of 128 B), g_a, f_inv and f_ev (8 lines each), and the
      // two 96-byte halves of g_A and of the harmonics
      const int p_nx = code_nx >= 0 ? code_nx : ~code_nx;
      const char *qrow = reinterpret_cast<const char *>(qkv + (size_t)b_nx * kQKV);
      const char *l1 = lane < 8 ? qrow + 128 * (32 + lane)
                     : lane < 16 ? reinterpret_cast<const char *>(g_a + (size_t)b_nx * kF) + 128 * (lane - 8)
                     : lane < 24 ? reinterpret_cast<const char *>(f_inv + (size_t)p_nx * kF) + 128 * (lane - 16)
                                 : reinterpret_cast<const char *>(f_ev + (size_t)p_nx * kF) + 128 * (lane - 24);
      asm volatile("prefetch.global.L1 [%0];\n" ::"l"(qrow + 128 * lane));
      asm volatile("prefetch.global.L1 [%0];\n" ::"l"(l1));
      if (lane < 4) {
        const char *l2 = lane < 2 ? reinterpret_cast<const char *>(g_A + (size_t)b_nx * kEV) + 96 * lane
                                  : reinterpret_cast<const char *>(sh + (size_t)p_nx * kEV) + 96 * (lane - 2);
        asm volatile("prefetch.global.L1 [%0];\n" ::"l"(l2));
      }
    }
    const double phi = geo[(size_t)p * kGeo + 4];
    const double *b_row = qkv + (size_t)b * kQKV + head_off;
    double qb[4], kb[4], vb[4], qeb[4], keb[4], gb[4], fi[4], fe[4];
    load4(b_row + 0 * 32, qb);
    load4(b_row + 1 * 32, kb);
    load4(b_row + 2 * 32, vb);
    load4(b_row + 3 * 32, qeb);
    load4(b_row + 4 * 32, keb);
    load4(g_a + (size_t)b * kF + lane * 4, gb);
    load4(f_inv + (size_t)p * kF + lane * 4, fi);
    load4(f_ev + (size_t)p * kF + lane * 4, fe);
    // harmonic-weighted adjoint sums per degree, for edge b->a ("in": y of the
    // edge into a) and a->b ("out": parity times that)
    double s_in, s_out;
    {
      const double pin = code < 0 ? par : 1.0;  // harmonics are stored for the primary orientation
      const double y0 = ch0 >= 0 ? sh[(size_t)p * kEV + ch0] * pin : 0.0;
      const double y1 = ch1 >= 0 ? sh[(size_t)p * kEV + ch1] * pin : 0.0;
      const double gAb0 = ch0 >= 0 ? g_A[(size_t)b * kEV + ch0] : 0.0;
      const double gAb1 = ch1 >= 0 ? g_A[(size_t)b * kEV + ch1] : 0.0;
      s_in = gAa0 * y0 + gAa1 * y1;
      s_out = (gAb0 * y0 + gAb1 * y1) * par;
      s_in = head_sum(s_in);
      s_out = head_sum(s_out);
    }
    double ai_out = 0, si_in = 0, si_out = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ai_out += qb[j] * ka[j] * fi[j];
      si_in += ga[j] * vb[j];
      si_out += gb[j] * va[j];
    }
    ai_out = head_sum(ai_out) * inv_norm;
    si_in = head_sum(si_in);
    si_out = head_sum(si_out);
    const double c_q = phi * si_in * inv_norm, c_qe = phi * s_in * inv_norm;
    const double c_v = phi * ai_out, c_k = phi * si_out * inv_norm, c_ke = phi * s_out * inv_norm;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
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
        double gi[4], ge[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          gi[j] = __dadd_rn(__dmul_rn(c_q, __dmul_rn(qa[j], kb[j])), __dmul_rn(c_k, __dmul_rn(qb[j], ka[j])));
          ge[j] = __dadd_rn(__dmul_rn(c_qe, __dmul_rn(qea[j], keb[j])), __dmul_rn(c_ke, __dmul_rn(qeb[j], kea[j])));
        }
        store4(g_filt_inv + (size_t)p * kF + lane * 4, gi);
        store4(g_filt_ev + (size_t)p * kF + lane * 4, ge);
      }
      double ai_in = 0, ae_in = 0, ae_out = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
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
      double t = __dadd_rn(__dadd_rn(__dmul_rn(ai_in, si_in), __dmul_rn(ai_out, si_out)),
                           __dadd_rn(__dmul_rn(ae_in, s_in), __dmul_rn(ae_out, s_out)));
      t += __shfl_xor_sync(0xffffffffu, t, 8);
      t += __shfl_xor_sync(0xffffffffu, t, 16);
      double *ps = pair_sc + (size_t)p * kPairScalars;
      if (lane == 0) ps[0] = t;
      if (lane == 1) ps[9] = 0.0;
      if ((lane & 7) == 0) {
        ps[1 + h] = ae_in;
        ps[5 + h] = ae_out;
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
  k_attention_reverse<<<n, 32, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair, geo, sh,
                                                           qkv, f_inv, f_ev, g_a, g_A, norm, g_qkv, pair_sc,
                                                           g_filt_inv, g_filt_ev);
  SO3_LAUNCH("attention_reverse");
}

// g_ev[a][m] = g_A[a][m] + sum over a's pairs of 2 (ev_a - ev_b)[m] cg[m] gl0[p][deg m]
__global__ void k_ev_l0_reverse(int n, int row0, const int *__restrict__ row_start, const int *__restrict__ nbr,
                                const int *__restrict__ edge_pair, const double *__restrict__ ev,
                                const double *__restrict__ cg, const double *__restrict__ gl0,
                                const double *__restrict__ g_A, double *__restrict__ g_ev) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= n || lane >= kEV) return;
  const int a = row0 + r;
  const int d = degree_of_channel(lane);
  const double eva = ev[(size_t)a * kEV + lane];
  const double c = 2.0 * cg[lane];
  double acc = 0.0;
  for (int e = row_start[r]; e < row_start[r + 1]; ++e) {
    const int b = nbr[e];
    const int code = edge_pair[e];
    const int p = code >= 0 ? code : ~code;
    acc += (eva - ev[(size_t)b * kEV + lane]) * c * gl0[(size_t)p * 4 + d];
  }
  g_ev[(size_t)a * kEV + lane] = g_A[(size_t)a * kEV + lane] + acc;
}

void launch_ev_l0_reverse(int n, const NeighborState &nb, const double *ev, const double *cg_att,
                          const double *gl0, const double *g_A, double *g_ev, cudaStream_t s) {
  if (n == 0) return;
  k_ev_l0_reverse<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair, ev, cg_att,
                                                       gl0, g_A, g_ev);
  SO3_LAUNCH("ev_l0_reverse");
}

}  // namespace so3lr_b200
