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

// per-degree sums of a value held by lanes 0..23; returns the sum for degree `want`
__device__ inline void degree_sums(double v, double out[4]) {
  const int lane = threadIdx.x & 31;
  const int d = lane < kEV ? degree_of_channel(lane) : -1;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    double s = d == k ? v : 0.0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    out[k] = s;
  }
}

// v[i] for a runtime index without dynamic register-array indexing
__device__ inline double pick4(const double (&v)[4], int i) {
  return i == 0 ? v[0] : (i == 1 ? v[1] : (i == 2 ? v[2] : v[3]));
}

__device__ inline void load4(const double *p, double (&v)[4]) {
  const double2 a = *reinterpret_cast<const double2 *>(p);
  const double2 b = *reinterpret_cast<const double2 *>(p + 2);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
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
    ai = head_sum(ai) / norm;
    ae = head_sum(ae) / norm;
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
__global__ void __launch_bounds__(256) k_attention_reverse(
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
  const double gAa = lane < kEV ? g_A[(size_t)a * kEV + lane] : 0.0;
  const int my_deg = lane < kEV ? degree_of_channel(lane) : 0;
  const double my_par = parity_sign(my_deg);
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
    if (e + 1 < e1) {  // pull the next edge's rows into L1 while this one is processed
      const int p_nx = code_nx >= 0 ? code_nx : ~code_nx;
      // 68 prefetches: qkv row (40 lines of 128 B), g_a, f_inv, f_ev (8 each), g_A and sh (two 96-byte halves each)
      for (int c = lane; c < 68; c += 32) {
        const char *addr;
        if (c < 40) addr = reinterpret_cast<const char *>(qkv + (size_t)b_nx * kQKV) + 128 * c;
        else if (c < 48) addr = reinterpret_cast<const char *>(g_a + (size_t)b_nx * kF) + 128 * (c - 40);
        else if (c < 56) addr = reinterpret_cast<const char *>(f_inv + (size_t)p_nx * kF) + 128 * (c - 48);
        else if (c < 64) addr = reinterpret_cast<const char *>(f_ev + (size_t)p_nx * kF) + 128 * (c - 56);
        else if (c < 66) addr = reinterpret_cast<const char *>(g_A + (size_t)b_nx * kEV) + 96 * (c - 64);
        else addr = reinterpret_cast<const char *>(sh + (size_t)p_nx * kEV) + 96 * (c - 66);
        asm volatile("prefetch.global.L1 [%0];\n" ::"l"(addr));
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
    const double gAb = lane < kEV ? g_A[(size_t)b * kEV + lane] : 0.0;
    double y = lane < kEV ? sh[(size_t)p * kEV + lane] : 0.0;
    const double y_in = code < 0 ? y * my_par : y;
    const double y_out = y_in * my_par;
    double ai_in = 0, ae_in = 0, ai_out = 0, ae_out = 0, si_in = 0, si_out = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ai_in += qa[j] * kb[j] * fi[j];
      ae_in += qea[j] * keb[j] * fe[j];
      ai_out += qb[j] * ka[j] * fi[j];
      ae_out += qeb[j] * kea[j] * fe[j];
      si_in += ga[j] * vb[j];
      si_out += gb[j] * va[j];
    }
    ai_in = head_sum(ai_in) / norm;
    ae_in = head_sum(ae_in) / norm;
    ai_out = head_sum(ai_out) / norm;
    ae_out = head_sum(ae_out) / norm;
    si_in = head_sum(si_in);
    si_out = head_sum(si_out);
    double se_in, se_out, se_in_q, se_out_q;
    const int qsel = lane >> 2, hh = lane & 3;
    double se_in_d[4], se_out_d[4];
    degree_sums(gAa * y_in, se_in_d);
    degree_sums(gAb * y_out, se_out_d);
    se_in = pick4(se_in_d, h);
    se_out = pick4(se_out_d, h);
    se_in_q = pick4(se_in_d, hh);
    se_out_q = pick4(se_out_d, hh);
    const double c_q = phi * si_in * inv_norm, c_qe = phi * se_in * inv_norm;
    const double c_v = phi * ai_out, c_k = phi * si_out * inv_norm, c_ke = phi * se_out * inv_norm;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      gq[j] += c_q * (kb[j] * fi[j]);
      gqe[j] += c_qe * (keb[j] * fe[j]);
      gv[j] += c_v * gb[j];
      gk[j] += c_k * (qb[j] * fi[j]);
      gke[j] += c_ke * (qeb[j] * fe[j]);
    }
    if (code >= 0 && g_filt_inv != nullptr) {
      double gi[4], ge[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        gi[j] = __dadd_rn(__dmul_rn(c_q, __dmul_rn(qa[j], kb[j])), __dmul_rn(c_k, __dmul_rn(qb[j], ka[j])));
        ge[j] = __dadd_rn(__dmul_rn(c_qe, __dmul_rn(qea[j], keb[j])), __dmul_rn(c_ke, __dmul_rn(qeb[j], kea[j])));
      }
      store4(g_filt_inv + (size_t)p * kF + lane * 4, gi);
      store4(g_filt_ev + (size_t)p * kF + lane * 4, ge);
    }
    if (code >= 0) {
      const double v_ai_in = __shfl_sync(0xffffffffu, ai_in, hh * 8);
      const double v_ae_in = __shfl_sync(0xffffffffu, ae_in, hh * 8);
      const double v_si_in = __shfl_sync(0xffffffffu, si_in, hh * 8);
      const double v_ai_out = __shfl_sync(0xffffffffu, ai_out, hh * 8);
      const double v_ae_out = __shfl_sync(0xffffffffu, ae_out, hh * 8);
      const double v_si_out = __shfl_sync(0xffffffffu, si_out, hh * 8);
      double val;
      switch (qsel) {
        case 0: val = v_ai_in; break;
        case 1: val = v_ae_in; break;
        case 2: val = v_si_in; break;
        case 3: val = se_in_q; break;
        case 4: val = v_ai_out; break;
        case 5: val = v_ae_out; break;
        case 6: val = v_si_out; break;
        default: val = se_out_q; break;
      }
      pair_sc[(size_t)p * kPairScalars + lane] = val;
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
  k_attention_reverse<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, nb.row0, nb.row_start, nb.nbr, nb.edge_pair, geo, sh,
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
