// Per-atom ("node") work: dense layers over atoms on FP64 tensor cores with
// fused epilogues, plus the row kernels (residuals, LayerNorm forward/backward,
// degree gate, L0 contraction, output heads).
//
// Reference: src/kokkos_post_attention_block0.cpp:97-300 (post-attention forward),
// src/kokkos_post_attention_reverse.cpp:107-449 (its reverse),
// src/kokkos_integrated_block0.cpp:257-286 (per-head QKV projections),
// src/kokkos_output_heads.cpp:137-222, 341-581 (energy, charge and Hirshfeld heads
// and their reverse), src/kokkos_local_energy_reverse.cpp:192-218 (embedding).
// The reference runs each dense layer as a cuBLAS DGEMM followed by separate
// elementwise kernels; here the bias/activation/residual work is fused into the
// GEMM epilogue.
#include <cstdint>
#include <initializer_list>
#include <type_traits>

#include "kernels.cuh"

SO3LR_SHAPE_BEGIN
namespace {

// 32 x 64 (or 64 x 32) output tile per CTA, 4 warps of 32 x 16 (2 x 2 m16n8k8
// blocks), K in steps of 16 through a two-stage cp.async pipeline. (The node GEMMs have
// M = atoms and N, K = 32..320: at 24,000 atoms 64-row tiles gave 1.27 waves of
// CTAs on 148 SMs; 32-row tiles at about 70 registers run 6 CTAs per SM and
// measured 0.23 ms per MD step faster.) A is staged as [m][k] and
// B as [n][k] (transposed weights) or [k][n]; the shared-memory row strides keep
// the fragment loads free of bank conflicts (24 = 8 mod 16 doubles for 16-byte
// loads of two rows, 66 or 34 = 2 mod 16 for 8-byte loads of four k rows).
constexpr int BK = 16;
constexpr int LDA_S = BK + 8, LDBT_S = BK + 8;
constexpr int kGemmThreads = 128;
template <bool TRANSB, int BMT, int BNT>
constexpr int gemm_smem_doubles() {
  return 2 * BMT * LDA_S + 2 * (TRANSB ? BNT * LDBT_S : BK * (BNT + 2));
}

// BMT x BNT output tile: 32 x 64, or 64 x 32 for N that 64-column tiles would
// pad by more (N = 32, 160, 136: the per-head QKV projections and the
// interaction layer); either way a warp computes 32 x 16.
template <bool TRANSB, Epi EPI, int BMT, int BNT>
__global__ void __launch_bounds__(kGemmThreads) k_gemm(GemmArgs g, int aux_cols, int ldaux2, bool vec) {
  extern __shared__ double gsm[];
  constexpr int BM = BMT, BN = BNT;
  constexpr int LDBN_S = BN + 2;
  constexpr int WN = BMT == 64 ? 2 : 4;  // warps along N (warp tiles of 32 rows)
  constexpr int NI = BN / WN / 8;        // n8 blocks per warp
  constexpr int ASTAGE = BM * LDA_S;
  constexpr int BSTAGE = TRANSB ? BN * LDBT_S : BK * LDBN_S;
  double *As = gsm;
  double *Bs = gsm + 2 * ASTAGE;
  const int z = blockIdx.z;
  const double *A = g.A + z * g.strideA;
  const double *W = g.W + z * g.strideW;
  double *C = g.C + z * g.strideC;
  const double *aux = g.aux ? g.aux + z * g.strideAux : nullptr;
  const double *bias = g.bias ? g.bias + z * g.strideBias : nullptr;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
  const int wm = warp / WN, wn = warp % WN;
  auto load_stage = [&](int stage, int k0) {
    double *as = As + stage * ASTAGE;
    for (int c = tid; c < BM * BK / 2; c += kGemmThreads) {
      const int row = c / (BK / 2), col = (c % (BK / 2)) * 2;
      const int gm = m0 + row, gk = k0 + col;
      double *dst = as + row * LDA_S + col;
      if (gm < g.M && gk < g.K) {
        cp_async16(dst, A + (size_t)(g.rows ? g.rows[gm] : gm) * g.lda + gk);
      } else {
        dst[0] = 0.0;
        dst[1] = 0.0;
      }
    }
    double *bs = Bs + stage * BSTAGE;
    if (TRANSB) {  // W[n][k]
      for (int c = tid; c < BN * BK / 2; c += kGemmThreads) {
        const int nn = c / (BK / 2), col = (c % (BK / 2)) * 2;
        const int gn = n0 + nn, gk = k0 + col;
        double *dst = bs + nn * LDBT_S + col;
        if (gn < g.N && gk < g.K) {
          cp_async16(dst, W + (size_t)gn * g.ldw + gk);
        } else {
          dst[0] = 0.0;
          dst[1] = 0.0;
        }
      }
    } else {  // W[k][n]
      for (int c = tid; c < BK * BN / 2; c += kGemmThreads) {
        const int kk = c / (BN / 2), col = (c % (BN / 2)) * 2;
        const int gk = k0 + kk, gn = n0 + col;
        double *dst = bs + kk * LDBN_S + col;
        if (gk < g.K && gn < g.N) {
          cp_async16(dst, W + (size_t)gk * g.ldw + gn);
        } else {
          dst[0] = 0.0;
          dst[1] = 0.0;
        }
      }
    }
  };
  double acc[2][NI][4];
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int ni = 0; ni < NI; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = acc[mi][ni][2] = acc[mi][ni][3] = 0.0;
  const int nk = (g.K + BK - 1) / BK;
  load_stage(0, 0);
  cp_async_commit();
  for (int kt = 0; kt < nk; ++kt) {
    if (kt + 1 < nk) load_stage((kt + 1) & 1, (kt + 1) * BK);
    cp_async_commit();
    cp_async_wait<1>();  // stage kt has landed
    __syncthreads();
    const double *as = As + (kt & 1) * ASTAGE;
    const double *bs = Bs + (kt & 1) * BSTAGE;
#pragma unroll
    for (int ks = 0; ks < BK / 8; ++ks) {
      double a[2][4], b[NI][2];
      load_afrag(as, LDA_S, wm * 32, ks, gq, tq, a[0]);
      load_afrag(as, LDA_S, wm * 32 + 16, ks, gq, tq, a[1]);
#pragma unroll
      for (int ni = 0; ni < NI; ++ni) {
        const int nn = wn * (BN / WN) + ni * 8 + gq;
        if (TRANSB) {
          const double2 v = *reinterpret_cast<const double2 *>(bs + nn * LDBT_S + 8 * ks + 2 * tq);
          b[ni][0] = v.x;
          b[ni][1] = v.y;
        } else {
          b[ni][0] = bs[(8 * ks + 2 * tq) * LDBN_S + nn];
          b[ni][1] = bs[(8 * ks + 2 * tq + 1) * LDBN_S + nn];
        }
      }
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < NI; ++ni) dmma16(acc[mi][ni], a[mi], b[ni]);
    }
    __syncthreads();  // the stage is refilled two iterations later
  }
  // epilogue: each lane holds two adjacent columns of a row; with vec (every
  // array 16-byte aligned, every row stride even) they move as one 16-byte
  // load or store
  auto epilogue = [&](int row, int col, double v, const double *aux_p, const double *aux2_p) {
    if (EPI == Epi::Bias) {
      v += bias[col];
    } else if (EPI == Epi::BiasSilu) {
      v = silu(v + bias[col]);
    } else if (EPI == Epi::BiasStorePre) {
      const double pre = v + bias[col];
      g.aux_out[(size_t)row * g.ldaux + col] = pre;
      v = silu(pre);
    } else if (EPI == Epi::AddResidual) {
      if (col < aux_cols) v += *aux_p;
    } else if (EPI == Epi::BiasResidual) {
      v = v + bias[col] + *aux_p;
    } else if (EPI == Epi::SiluPrimeMul) {
      v *= silu_prime(*aux_p);
    } else if (EPI == Epi::GateSiluResidual) {
      v = *aux2_p + v * silu_prime(*aux_p);
    }
    return v;
  };
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int lrow = m0 + wm * 32 + mi * 16 + hf * 8 + gq;
      if (lrow >= g.M) continue;
      const int row = g.rows ? g.rows[lrow] : lrow;
#pragma unroll
      for (int ni = 0; ni < NI; ++ni) {
        const int col = n0 + wn * (BN / WN) + ni * 8 + 2 * tq;
        const double *aux_p = aux ? aux + (size_t)row * g.ldaux + col : nullptr;
        const double *aux2_p = g.aux2 ? g.aux2 + (size_t)row * ldaux2 + col : nullptr;
        if (vec && col + 1 < g.N) {
          double2 a2 = make_double2(0.0, 0.0), b2 = make_double2(0.0, 0.0);
          if (EPI == Epi::AddResidual) {
            if (col + 1 < aux_cols) a2 = *reinterpret_cast<const double2 *>(aux_p);
            else if (col < aux_cols) a2.x = aux_p[0];
          } else if (EPI == Epi::BiasResidual || EPI == Epi::SiluPrimeMul || EPI == Epi::GateSiluResidual) {
            a2 = *reinterpret_cast<const double2 *>(aux_p);
          }
          if (EPI == Epi::GateSiluResidual) b2 = *reinterpret_cast<const double2 *>(aux2_p);
          double2 out;
          if (EPI == Epi::BiasStorePre) {
            const double2 bb = *reinterpret_cast<const double2 *>(bias + col);
            const double2 pre = make_double2(acc[mi][ni][2 * hf] + bb.x, acc[mi][ni][2 * hf + 1] + bb.y);
            *reinterpret_cast<double2 *>(g.aux_out + (size_t)row * g.ldaux + col) = pre;
            out = make_double2(silu(pre.x), silu(pre.y));
          } else {
            out.x = epilogue(row, col, acc[mi][ni][2 * hf], &a2.x, &b2.x);
            out.y = epilogue(row, col + 1, acc[mi][ni][2 * hf + 1], &a2.y, &b2.y);
          }
          *reinterpret_cast<double2 *>(C + (size_t)row * g.ldc + col) = out;
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (col + h >= g.N) continue;
            const double v = epilogue(row, col + h, acc[mi][ni][2 * hf + h], aux_p ? aux_p + h : nullptr,
                                      aux2_p ? aux2_p + h : nullptr);
            C[(size_t)row * g.ldc + col + h] = v;
          }
        }
      }
    }
}

template <bool T, Epi E>
void launch_gemm_kernel(const GemmArgs &g, cudaStream_t s, int aux_cols, int ldaux2) {
  auto al = [](const void *p) { return (reinterpret_cast<std::uintptr_t>(p) & 15) == 0; };
  auto ev = [](long long x) { return (x & 1) == 0; };
  const bool vec = al(g.C) && al(g.bias) && al(g.aux) && al(g.aux2) && al(g.aux_out) && ev(g.ldc) &&
                   ev(g.ldaux) && ev(ldaux2) && ev(g.strideC) && ev(g.strideAux) && ev(g.strideBias);
  auto go = [&](auto bm, auto bn) {
    constexpr int BMT = decltype(bm)::value, BNT = decltype(bn)::value;
    constexpr size_t smem = sizeof(double) * gemm_smem_doubles<T, BMT, BNT>();
    allow_dynamic_smem(reinterpret_cast<const void *>(k_gemm<T, E, BMT, BNT>), smem);
    const dim3 grid((g.N + BNT - 1) / BNT, (g.M + BMT - 1) / BMT, g.batch);
    k_gemm<T, E, BMT, BNT><<<grid, kGemmThreads, smem, s>>>(g, aux_cols, ldaux2, vec);
  };
  // the tile shape that pads N least (64 columns on a tie)
  const int pad64 = (g.N + 63) / 64 * 64 - g.N, pad32 = (g.N + 31) / 32 * 32 - g.N;
  if (pad32 < pad64) go(std::integral_constant<int, 64>{}, std::integral_constant<int, 32>{});
  else go(std::integral_constant<int, 32>{}, std::integral_constant<int, 64>{});
}

template <bool T>
void dispatch_epi(const GemmArgs &g, cudaStream_t s, int aux_cols, int ldaux2) {
  switch (g.epi) {
    case Epi::None: launch_gemm_kernel<T, Epi::None>(g, s, aux_cols, ldaux2); break;
    case Epi::Bias: launch_gemm_kernel<T, Epi::Bias>(g, s, aux_cols, ldaux2); break;
    case Epi::BiasSilu: launch_gemm_kernel<T, Epi::BiasSilu>(g, s, aux_cols, ldaux2); break;
    case Epi::BiasStorePre: launch_gemm_kernel<T, Epi::BiasStorePre>(g, s, aux_cols, ldaux2); break;
    case Epi::AddResidual: launch_gemm_kernel<T, Epi::AddResidual>(g, s, aux_cols, ldaux2); break;
    case Epi::BiasResidual: launch_gemm_kernel<T, Epi::BiasResidual>(g, s, aux_cols, ldaux2); break;
    case Epi::SiluPrimeMul: launch_gemm_kernel<T, Epi::SiluPrimeMul>(g, s, aux_cols, ldaux2); break;
    case Epi::GateSiluResidual: launch_gemm_kernel<T, Epi::GateSiluResidual>(g, s, aux_cols, ldaux2); break;
  }
}

}  // namespace

void launch_gemm_ex(const GemmArgs &g, int aux_cols, int ldaux2, cudaStream_t s) {
  if (g.M == 0) return;
  if (g.transB) dispatch_epi<true>(g, s, aux_cols, ldaux2);
  else dispatch_epi<false>(g, s, aux_cols, ldaux2);
  SO3_LAUNCH("gemm");
}
void launch_gemm(const GemmArgs &g, cudaStream_t s) { launch_gemm_ex(g, g.N, g.ldaux, s); }

// ---------------------------------------------------------------------------
// embedding: x0 = W_emb[:, Z-1] / s + offset_table[image][Z-1] / s
// ---------------------------------------------------------------------------
__global__ void k_embedding(int n, const int *__restrict__ z, const double *__restrict__ w,
                            const double *__restrict__ table, const int *__restrict__ table_of_atom,
                            double inv_scale, double *__restrict__ x) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * kF) return;
  const int i = idx / kF, c = idx % kF;
  const int zz = z[i];
  double v = (zz > 0 && zz <= 118) ? w[c * 118 + zz - 1] * inv_scale : 0.0;
  if (table != nullptr) {
    const int tab = table_of_atom[i];
    if (tab >= 0 && zz > 0 && zz <= 118) v += table[((size_t)tab * 118 + zz - 1) * kF + c] * inv_scale;
  }
  x[idx] = v;
}
void launch_embedding(int n, const int *z, const double *emb_w, const double *cs_table, const int *table_of_atom,
                      double inv_scale, double *x, cudaStream_t s) {
  if (n == 0) return;
  k_embedding<<<(n * kF + 255) / 256, 256, 0, s>>>(n, z, emb_w, cs_table, table_of_atom, inv_scale, x);
  SO3_LAUNCH("embedding");
}

namespace {
__device__ inline double warp_sum(double v) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Row kernels: one warp per atom, lane owns invariant channels kPL lane ..
// kPL lane + kPL - 1 and equivariant channels lane + 32 j (j < kEVL).
constexpr int kPL = kF / 32;
constexpr int kEVL = (kEV + 31) / 32;

// A lane's kPL consecutive channels of a row (row strides kF and kIntW are
// multiples of 4 doubles): 256-bit loads and 128-bit stores when the launch's
// row arrays are 32-byte aligned (vec, checked on the host), else 8-byte ones.
__device__ inline void ld_lane(bool vec, const double *p, double (&v)[kPL]) {
  if (vec) {
#pragma unroll
    for (int q = 0; q < kPL; q += 4)
      asm("ld.global.v4.f64 {%0,%1,%2,%3}, [%4];"
          : "=d"(v[q]), "=d"(v[q + 1]), "=d"(v[q + 2]), "=d"(v[q + 3])
          : "l"(p + q));
  } else {
#pragma unroll
    for (int q = 0; q < kPL; ++q) v[q] = p[q];
  }
}
__device__ inline void st_lane(bool vec, double *p, const double (&v)[kPL]) {
  if (vec) {
#pragma unroll
    for (int q = 0; q < kPL; q += 2) *reinterpret_cast<double2 *>(p + q) = make_double2(v[q], v[q + 1]);
  } else {
#pragma unroll
    for (int q = 0; q < kPL; ++q) p[q] = v[q];
  }
}
inline bool aligned32(std::initializer_list<const void *> ptrs) {
  for (const void *p : ptrs)
    if ((reinterpret_cast<std::uintptr_t>(p) & 31) != 0) return false;
  return true;
}

// sum over the warp of the per-lane terms t[j] of the channels of degree slot k
// (ch[j] = slot of the lane's j-th equivariant channel, -1 when it has none)
__device__ inline double slot_sum(int k, const int (&ch)[kEVL], const double (&t)[kEVL]) {
  double v = ch[0] == k ? t[0] : 0.0;
#pragma unroll
  for (int j = 1; j < kEVL; ++j) v += ch[j] == k ? t[j] : 0.0;
  return warp_sum(v);
}

// Block norm of one kF-wide row held as kPL values per lane: xh = normalised
// row, returns the inverse standard deviation (LayerNorm) or inverse RMS
// (RMSNorm without scale, post_attention_block0.cpp:124-146); identity for
// kNormNone. eps = 1e-6 (the only value the model contract admits).
__device__ inline double row_norm(int norm, const double (&v)[kPL], double (&xh)[kPL]) {
  if (norm == kNormNone) {
#pragma unroll
    for (int j = 0; j < kPL; ++j) xh[j] = v[j];
    return 1.0;
  }
  double mean = 0.0;
  if (norm == kNormLayer) {
    double s = v[0];
#pragma unroll
    for (int j = 1; j < kPL; ++j) s += v[j];
    mean = warp_sum(s) / double(kF);
  }
  double var = 0.0;
#pragma unroll
  for (int j = 0; j < kPL; ++j) {
    const double d = v[j] - mean;
    var += d * d;
  }
  var = warp_sum(var) / double(kF);
  const double rs = 1.0 / sqrt(var + 1.0e-6);
#pragma unroll
  for (int j = 0; j < kPL; ++j) xh[j] = (v[j] - mean) * rs;
  return rs;
}
}  // namespace

// a = x + d_inv; A = ev + d_ev; n1 = LN1(a); act = silu(n1);
// cat[:, F:F+H] = L0'(A) (interaction cg), cat[:, F+H:kIntW] = 0. One warp per atom.
__global__ void k_post_attn_pre(int n, const double *__restrict__ x, const double *__restrict__ d_inv,
                                const double *__restrict__ ev, const double *__restrict__ d_ev, int norm,
                                const double *__restrict__ lnw, const double *__restrict__ lnb,
                                const double *__restrict__ cg_int, double *__restrict__ xhat1,
                                double *__restrict__ rstd1, double *__restrict__ n1_out, double *__restrict__ act,
                                double *__restrict__ A_out, double *__restrict__ cat, bool vec) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const size_t o = (size_t)i * kF + lane * kPL;
  double a[kPL], xh[kPL], dv[kPL];
  ld_lane(vec, x + o, a);
  ld_lane(vec, d_inv + o, dv);
#pragma unroll
  for (int j = 0; j < kPL; ++j) a[j] += dv[j];
  const double rs = row_norm(norm, a, xh);
  double y[kPL], sy[kPL];
#pragma unroll
  for (int j = 0; j < kPL; ++j) {
    const int c = lane * kPL + j;
    y[j] = norm == kNormLayer ? xh[j] * lnw[c] + lnb[c] : xh[j];
    sy[j] = silu(y[j]);
  }
  st_lane(vec, xhat1 + o, xh);
  st_lane(vec, n1_out + o, y);
  st_lane(vec, act + o, sy);
  if (lane == 0) rstd1[i] = rs;
  int d[kEVL];
  double term[kEVL];
#pragma unroll
  for (int j = 0; j < kEVL; ++j) {
    const int m = lane + 32 * j;
    d[j] = m < kEV ? degree_of_channel(m) : -1;
    term[j] = 0.0;
    if (m < kEV) {
      const double Am = ev[(size_t)i * kEV + m] + d_ev[(size_t)i * kEV + m];
      A_out[(size_t)i * kEV + m] = Am;
      term[j] = Am * Am * cg_int[m];
    }
  }
#pragma unroll
  for (int k = 0; k < kHeads; ++k) {
    const double sk = slot_sum(k, d, term);
    if (lane == 0) cat[(size_t)i * kIntW + kF + k] = sk;
  }
  if (lane < kIntW - kF - kHeads) cat[(size_t)i * kIntW + kF + kHeads + lane] = 0.0;
}

void launch_post_attn_pre(int n, const double *x, const double *d_inv, const double *ev, const double *d_ev,
                          int norm, const double *lnw, const double *lnb, const double *cg_int, double *xhat1,
                          double *rstd1, double *n1, double *act, double *A, double *cat, cudaStream_t s) {
  const bool vec = aligned32({x, d_inv, xhat1, n1, act});
  k_post_attn_pre<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, x, d_inv, ev, d_ev, norm, lnw, lnb, cg_int, xhat1, rstd1,
                                                       n1, act, A, cat, vec);
  SO3_LAUNCH("post_attn_pre");
}

// pre2 = post + t[:F]; x' = LN2(pre2); ev' = A (1 + t_gate). One warp per atom.
__global__ void k_post_attn_final(int n, const double *__restrict__ cat, const double *__restrict__ t,
                                  const double *__restrict__ A, int norm, const double *__restrict__ lnw,
                                  const double *__restrict__ lnb, double *__restrict__ xhat2,
                                  double *__restrict__ rstd2, double *__restrict__ gate,
                                  double *__restrict__ x_out, double *__restrict__ ev_out, bool vec) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const size_t oi = (size_t)i * kIntW + lane * kPL, o = (size_t)i * kF + lane * kPL;
  double v[kPL], tv[kPL], xh[kPL];
  ld_lane(vec, cat + oi, v);
  ld_lane(vec, t + oi, tv);
#pragma unroll
  for (int j = 0; j < kPL; ++j) v[j] += tv[j];
  const double rs = row_norm(norm, v, xh);
  double y[kPL];
#pragma unroll
  for (int j = 0; j < kPL; ++j) {
    const int c = lane * kPL + j;
    y[j] = norm == kNormLayer ? xh[j] * lnw[c] + lnb[c] : xh[j];
  }
  st_lane(vec, xhat2 + o, xh);
  st_lane(vec, x_out + o, y);
  if (lane == 0) rstd2[i] = rs;
  if (lane < kHeads) gate[(size_t)i * kHeads + lane] = t[(size_t)i * kIntW + kF + lane];
#pragma unroll
  for (int j = 0; j < kEVL; ++j) {
    const int m = lane + 32 * j;
    if (m < kEV) {
      const int d = degree_of_channel(m);
      ev_out[(size_t)i * kEV + m] = A[(size_t)i * kEV + m] * (1.0 + t[(size_t)i * kIntW + kF + d]);
    }
  }
}

void launch_post_attn_final(int n, const double *cat, const double *t, const double *A, int norm, const double *lnw,
                            const double *lnb, double *xhat2, double *rstd2, double *gate, double *x_out,
                            double *ev_out, cudaStream_t s) {
  const bool vec = aligned32({cat, t, xhat2, x_out});
  k_post_attn_final<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, cat, t, A, norm, lnw, lnb, xhat2, rstd2, gate, x_out,
                                                         ev_out, vec);
  SO3_LAUNCH("post_attn_final");
}

// Block-norm backward. LayerNorm (affine): g_x = rstd (g_xh - mean(g_xh) -
// xh mean(g_xh xh)), g_xh = g_y w. RMSNorm without scale: g_x = rrms (g_y -
// xh mean(g_y xh)). Identity: g_x = g_y.
__device__ inline void norm_backward(int norm, const double (&gy)[kPL], const double (&xh)[kPL], const double *w,
                                     int lane, double rs, double (&gx)[kPL]) {
  if (norm == kNormNone) {
#pragma unroll
    for (int j = 0; j < kPL; ++j) gx[j] = gy[j];
    return;
  }
  double gxh[kPL], s1 = 0.0, s2 = 0.0;
#pragma unroll
  for (int j = 0; j < kPL; ++j) {
    gxh[j] = norm == kNormLayer ? gy[j] * w[lane * kPL + j] : gy[j];
    s1 += gxh[j];
    s2 += gxh[j] * xh[j];
  }
  s1 = norm == kNormLayer ? warp_sum(s1) / double(kF) : 0.0;
  s2 = warp_sum(s2) / double(kF);
#pragma unroll
  for (int j = 0; j < kPL; ++j) gx[j] = rs * (gxh[j] - s1 - xh[j] * s2);
}

// reverse of k_post_attn_final: g_t[:F] = LN2^T(g_x), g_t[F+d] = sum g_ev A, g_A = g_ev (1 + gate)
__global__ void k_post_attn_rev_final(int n, const double *__restrict__ g_x, const double *__restrict__ g_ev,
                                      const double *__restrict__ xhat2, const double *__restrict__ rstd2, int norm,
                                      const double *__restrict__ lnw2, const double *__restrict__ A,
                                      const double *__restrict__ gate, double *__restrict__ g_t,
                                      double *__restrict__ g_A, bool vec) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  double gy[kPL], xh[kPL], gx[kPL];
  ld_lane(vec, g_x + (size_t)i * kF + lane * kPL, gy);
  ld_lane(vec, xhat2 + (size_t)i * kF + lane * kPL, xh);
  norm_backward(norm, gy, xh, lnw2, lane, rstd2[i], gx);
  st_lane(vec, g_t + (size_t)i * kIntW + lane * kPL, gx);
  double ge[kEVL], gA[kEVL];
  int d[kEVL];
#pragma unroll
  for (int j = 0; j < kEVL; ++j) {
    const int m = lane + 32 * j;
    ge[j] = 0.0;
    gA[j] = 0.0;
    d[j] = -1;
    if (m < kEV && g_ev != nullptr) {
      ge[j] = g_ev[(size_t)i * kEV + m];
      gA[j] = ge[j] * A[(size_t)i * kEV + m];
      d[j] = degree_of_channel(m);
    }
  }
#pragma unroll
  for (int k = 0; k < kHeads; ++k) {
    const double sk = slot_sum(k, d, gA);
    if (lane == 0) g_t[(size_t)i * kIntW + kF + k] = sk;
  }
  if (lane < kIntW - kF - kHeads) g_t[(size_t)i * kIntW + kF + kHeads + lane] = 0.0;
#pragma unroll
  for (int j = 0; j < kEVL; ++j) {
    const int m = lane + 32 * j;
    if (m < kEV) g_A[(size_t)i * kEV + m] = d[j] >= 0 ? ge[j] * (1.0 + gate[(size_t)i * kHeads + d[j]]) : 0.0;
  }
}

void launch_post_attn_rev_final(int n, const double *g_x, const double *g_ev, const double *xhat2,
                                const double *rstd2, int norm, const double *lnw2, const double *A,
                                const double *gate, double *g_t, double *g_A, cudaStream_t s) {
  const bool vec = aligned32({g_x, xhat2, g_t});
  k_post_attn_rev_final<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, g_x, g_ev, xhat2, rstd2, norm, lnw2, A, gate, g_t,
                                                             g_A, vec);
  SO3_LAUNCH("post_attn_rev_final");
}

// g_a = LN1^T(g_n1); g_A += 2 A cg_int g_l0'[deg]
__global__ void k_post_attn_rev_ln1(int n, const double *__restrict__ g_n1, const double *__restrict__ xhat1,
                                    const double *__restrict__ rstd1, int norm, const double *__restrict__ lnw1,
                                    const double *__restrict__ A, const double *__restrict__ cg_int,
                                    const double *__restrict__ g_cat, double *__restrict__ g_a,
                                    double *__restrict__ g_A, bool vec) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  double gy[kPL], xh[kPL], gx[kPL];
  ld_lane(vec, g_n1 + (size_t)i * kF + lane * kPL, gy);
  ld_lane(vec, xhat1 + (size_t)i * kF + lane * kPL, xh);
  norm_backward(norm, gy, xh, lnw1, lane, rstd1[i], gx);
  st_lane(vec, g_a + (size_t)i * kF + lane * kPL, gx);
#pragma unroll
  for (int j = 0; j < kEVL; ++j) {
    const int m = lane + 32 * j;
    if (m < kEV) {
      const int d = degree_of_channel(m);
      const double Am = A[(size_t)i * kEV + m];
      g_A[(size_t)i * kEV + m] += 2.0 * Am * cg_int[m] * g_cat[(size_t)i * kIntW + kF + d];
    }
  }
}

void launch_post_attn_rev_ln1(int n, const double *g_n1, const double *xhat1, const double *rstd1, int norm,
                              const double *lnw1, const double *A, const double *cg_int, const double *g_cat,
                              double *g_a, double *g_A, cudaStream_t s) {
  const bool vec = aligned32({g_n1, xhat1, g_a});
  k_post_attn_rev_ln1<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, g_n1, xhat1, rstd1, norm, lnw1, A, cg_int, g_cat, g_a,
                                                           g_A, vec);
  SO3_LAUNCH("post_attn_rev_ln1");
}

// ---------------------------------------------------------------------------
// residual scalars (local_energy_reverse.cpp:121-170): the input of block b is
// resid[b] x + x0[b] x0, x0 = the embedding; the reverse scales the gradient
// reaching the previous block's output by resid[b]
// ---------------------------------------------------------------------------
__global__ void k_residual_combine(long long count, const double *__restrict__ in, const double *__restrict__ x0,
                                   double a, double c, double *__restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) out[i] = a * in[i] + c * x0[i];
}
void launch_residual_combine(int n, const double *in, const double *x0, double a, double c, double *out,
                             cudaStream_t s) {
  const long long count = (long long)n * kF;
  if (count == 0) return;
  k_residual_combine<<<unsigned((count + 255) / 256), 256, 0, s>>>(count, in, x0, a, c, out);
  SO3_LAUNCH("residual_combine");
}

__global__ void k_scale_rows(long long count, double *__restrict__ v, double a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) v[i] *= a;
}
void launch_scale_rows(int n, double *v, double a, cudaStream_t s) {
  const long long count = (long long)n * kF;
  if (count == 0) return;
  k_scale_rows<<<unsigned((count + 255) / 256), 256, 0, s>>>(count, v, a);
  SO3_LAUNCH("scale_rows");
}

// ---------------------------------------------------------------------------
// query/key RMS normalisation (integrated_block0.cpp:288-328): every 32-wide q,
// k, q_ev, k_ev vector of a row is divided by sqrt(mean(v^2) + 1e-6). One warp
// per (row, head, slot), lane = channel.
// ---------------------------------------------------------------------------
__device__ inline int qk_slot_offset(int slot) { return slot < 2 ? slot * 32 : (slot + 1) * 32; }  // q k | q_ev k_ev
constexpr int kQkPerRow = 4 * kHeads;  // normalised vectors per row

__global__ void k_qk_norm(int n, const int *__restrict__ rows, double *__restrict__ qkv, double *__restrict__ rinv) {
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)n * kQkPerRow) return;
  const int slot = int(w & 3), head = int((w >> 2) % kHeads);
  const long long m = w / kQkPerRow;
  const long long row = rows ? rows[m] : m;
  double *v = qkv + row * kQKV + head * 160 + qk_slot_offset(slot);
  const double x = v[lane];
  const double r = 1.0 / sqrt(warp_sum(x * x) / 32.0 + 1.0e-6);
  v[lane] = x * r;
  if (lane == 0) rinv[row * kQkPerRow + head * 4 + slot] = r;
}
void launch_qk_norm(int n, const int *rows, double *qkv, double *rinv, cudaStream_t s) {
  if (n == 0) return;
  const long long threads = (long long)n * kQkPerRow * 32;
  k_qk_norm<<<unsigned((threads + 255) / 256), 256, 0, s>>>(n, rows, qkv, rinv);
  SO3_LAUNCH("qk_norm");
}

__global__ void k_qk_norm_reverse(int n, const double *__restrict__ qkv, const double *__restrict__ rinv,
                                  double *__restrict__ g) {
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)n * kQkPerRow) return;
  const int slot = int(w & 3), head = int((w >> 2) % kHeads);
  const long long row = w / kQkPerRow;
  const long long off = row * kQKV + head * 160 + qk_slot_offset(slot);
  const double y = qkv[off + lane], gy = g[off + lane];
  const double mean_gy = warp_sum(gy * y) / 32.0;
  g[off + lane] = rinv[row * kQkPerRow + head * 4 + slot] * (gy - y * mean_gy);
}
void launch_qk_norm_reverse(int n, const double *qkv, const double *rinv, double *g, cudaStream_t s) {
  if (n == 0) return;
  const long long threads = (long long)n * kQkPerRow * 32;
  k_qk_norm_reverse<<<unsigned((threads + 255) / 256), 256, 0, s>>>(n, qkv, rinv, g);
  SO3_LAUNCH("qk_norm_reverse");
}


// ---------------------------------------------------------------------------
// output heads (output_heads.cpp:137-176, 341-451): hcat = silu(x W1cat^T + b1cat)
// energy  = (hcat[0:128] . w2 + b2) * scale[Z-1] + shift[Z-1]
// raw q   =  hcat[128:256] . w2c + b2c + emb[Z]
// ratio   = | v_shift[Z] + q_emb[Z] . (hcat[256:320] Wh2^T + bh2) / 8 |
// ---------------------------------------------------------------------------
// One ratio head (Hirshfeld / a0 or C6; 64 hidden units, keys zero-padded to
// 64) of one atom: keys k = h1 W2^T + b2 (lane owns keys 2 lane, 2 lane + 1),
// ratio = |v_shift[Z] + q_emb[Z] . k / sqrt(K)| (output_heads.cpp:135-176).
// The ratio heads (Hirshfeld, C6) of kHA atoms per warp: every weight row is
// loaded once for all of them. Per atom and output the 64-term dot product runs
// as four interleaved chains added in a fixed order.
constexpr int kHA = 4;
__device__ inline void ratio_head(const double *const (&hh)[kHA], const double *__restrict__ w2t,
                                  const double *__restrict__ b2, const double *__restrict__ qemb,
                                  const double *__restrict__ vshift, double sqrt_k, const int (&zz)[kHA], int na,
                                  int lane, double *const (&k_out)[kHA], double (&res)[kHA]) {
  double s0[kHA][4], s1[kHA][4];
#pragma unroll
  for (int a = 0; a < kHA; ++a)
#pragma unroll
    for (int u = 0; u < 4; ++u) s0[a][u] = s1[a][u] = 0.0;
#pragma unroll 2
  for (int j = 0; j < kHirsh; j += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const double2 w = *reinterpret_cast<const double2 *>(w2t + (j + u) * kHirsh + 2 * lane);  // coalesced
#pragma unroll
      for (int a = 0; a < kHA; ++a) {
        const double hv = hh[a][j + u];
        s0[a][u] += hv * w.x;
        s1[a][u] += hv * w.y;
      }
    }
  }
#pragma unroll
  for (int a = 0; a < kHA; ++a) {
    if (a >= na) break;
    double k0 = b2[2 * lane], k1 = b2[2 * lane + 1];
    k0 += (s0[a][0] + s0[a][1]) + (s0[a][2] + s0[a][3]);
    k1 += (s1[a][0] + s1[a][1]) + (s1[a][2] + s1[a][3]);
    k_out[a][2 * lane] = k0;
    k_out[a][2 * lane + 1] = k1;
    double qk = qemb[zz[a] * kHirsh + 2 * lane] * k0 + qemb[zz[a] * kHirsh + 2 * lane + 1] * k1;
    qk = warp_sum(qk);
    res[a] = fabs(vshift[zz[a]] + qk / sqrt_k);
  }
}

// Output heads of kHA atoms per warp: energy and charge (128-wide dot products)
// and the ratio heads.
__global__ void k_heads_finalize(int n, const int *__restrict__ z, const double *__restrict__ hcat, HeadsW hw,
                                 double *__restrict__ hk_out, double *__restrict__ e_nn, double *__restrict__ raw_q,
                                 double *__restrict__ ratio, double *__restrict__ hk6_out,
                                 double *__restrict__ ratio6) {
  const int i0 = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * kHA;
  const int lane = threadIdx.x & 31;
  if (i0 >= n) return;
  const int na = min(kHA, n - i0);
  const double *hh[kHA], *hh6[kHA];
  double *ko[kHA], *ko6[kHA];
  int zz[kHA];
#pragma unroll
  for (int a = 0; a < kHA; ++a) {
    const int i = i0 + (a < na ? a : 0);  // surplus slots repeat the first atom; their results are dropped
    const double *h = hcat + (size_t)i * hw.ldh;
    hh[a] = h + 2 * kHeadHidden;
    hh6[a] = h + kHeadCat;
    ko[a] = hk_out + (size_t)i * kHirsh;
    ko6[a] = hk6_out + (size_t)i * kHirsh;
    zz[a] = z[i];
  }
  for (int a = 0; a < na; ++a) {
    const int i = i0 + a;
    const double *h = hcat + (size_t)i * hw.ldh;
    double se = 0.0, sq = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      se += h[lane * 4 + j] * hw.e_w2[lane * 4 + j];
      sq += h[kHeadHidden + lane * 4 + j] * hw.c_w2[lane * 4 + j];
    }
    se = warp_sum(se);
    sq = warp_sum(sq);
    if (lane == 0) {
      e_nn[i] = (se + hw.e_b2) * hw.e_scale[zz[a] - 1] + hw.e_shift[zz[a] - 1];
      raw_q[i] = sq + hw.c_b2 + hw.c_emb[zz[a]];
    }
  }
  double rh[kHA];
  ratio_head(hh, hw.h_w2t, hw.h_b2, hw.h_qemb, hw.h_vshift, hw.h_sqrt_k, zz, na, lane, ko, rh);
  if (lane == 0)
    for (int a = 0; a < na; ++a) ratio[i0 + a] = rh[a];
  if (hw.c6_w2 != nullptr) {
    ratio_head(hh6, hw.c6_w2t, hw.c6_b2, hw.c6_qemb, hw.c6_vshift, hw.c6_sqrt_k, zz, na, lane, ko6, rh);
    if (lane == 0)
      for (int a = 0; a < na; ++a) ratio6[i0 + a] = rh[a];
  }
}

void launch_heads_finalize(int n, const int *z, const double *hcat, const HeadsW &hw, double *hk_out,
                           double *e_nn, double *raw_q, double *ratio, double *hk6_out, double *ratio6,
                           cudaStream_t s) {
  if (n == 0) return;
  const int warps = (n + kHA - 1) / kHA;
  k_heads_finalize<<<(warps * 32 + 255) / 256, 256, 0, s>>>(n, z, hcat, hw, hk_out, e_nn, raw_q, ratio, hk6_out,
                                                            ratio6);
  SO3_LAUNCH("heads_finalize");
}

// Reverse of one ratio head for one atom, seeded with d = dE/d(ratio):
// g[j] = (sum_k g_k[k] W2[k][j]) silu'(pre[j]), g_k = d sign(eff) q_emb[Z] / sqrt(K);
// lane owns hidden units j = 2 lane, 2 lane + 1. gk is this warp's 64-double scratch.
__device__ inline void ratio_head_seed(const double *__restrict__ hk, const double *__restrict__ pre,
                                       const double *__restrict__ w2, const double *__restrict__ qemb,
                                       const double *__restrict__ vshift, double sqrt_k, double d, int zz, int lane,
                                       double *gk, double *__restrict__ g) {
  const double k0 = hk[2 * lane], k1 = hk[2 * lane + 1];
  const double qe0 = qemb[zz * kHirsh + 2 * lane], qe1 = qemb[zz * kHirsh + 2 * lane + 1];
  double eff = qe0 * k0 / sqrt_k + qe1 * k1 / sqrt_k;
  eff = warp_sum(eff) + vshift[zz];
  const double sign = eff > 0.0 ? 1.0 : (eff < 0.0 ? -1.0 : 0.0);
  const double seed = d * sign / sqrt_k;
  __syncwarp();
  gk[2 * lane] = seed * qe0;
  gk[2 * lane + 1] = seed * qe1;
  __syncwarp();
  // both of the lane's outputs from one 16-byte load of each weight row; per
  // output four interleaved chains, added in a fixed order
  double s[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll 4
  for (int k = 0; k < kHirsh; k += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const double2 w = *reinterpret_cast<const double2 *>(w2 + (k + u) * kHirsh + 2 * lane);
      s[0][u] += gk[k + u] * w.x;
      s[1][u] += gk[k + u] * w.y;
    }
  }
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const int j = 2 * lane + jj;
    g[j] = ((s[jj][0] + s[jj][1]) + (s[jj][2] + s[jj][3])) * silu_prime(pre[j]);
  }
}

// seeds of the heads' reverse: energy seed 1, charge seed dE/dq - image mean,
// Hirshfeld seed dE/dh, C6 seed dE/dc6 (output_heads.cpp:493-581). Writes
// g_hcat = dL/d(pre-activation).
__global__ void k_heads_seed(int n, const int *__restrict__ z, const double *__restrict__ hpre,
                             const double *__restrict__ hk, HeadsW hw, const double *__restrict__ dq,
                             const double *__restrict__ dq_mean, const int *__restrict__ image_of,
                             const double *__restrict__ dh, const double *__restrict__ hk6,
                             const double *__restrict__ dc6, double *__restrict__ g_hcat) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int zz = z[i];
  const double *pre = hpre + (size_t)i * hw.ldh;
  double *g = g_hcat + (size_t)i * hw.ldh;
  const double scale = hw.e_scale[zz - 1];
  const double qseed = dq[i] - dq_mean[image_of[i]];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane * 4 + j;
    g[c] = scale * hw.e_w2[c] * silu_prime(pre[c]);
    g[kHeadHidden + c] = qseed * hw.c_w2[c] * silu_prime(pre[kHeadHidden + c]);
  }
  __shared__ double gk_s[8][kHirsh];
  const int w = (threadIdx.x >> 5);
  ratio_head_seed(hk + (size_t)i * kHirsh, pre + 2 * kHeadHidden, hw.h_w2, hw.h_qemb, hw.h_vshift, hw.h_sqrt_k,
                  dh[i], zz, lane, gk_s[w], g + 2 * kHeadHidden);
  if (hw.c6_w2 != nullptr)
    ratio_head_seed(hk6 + (size_t)i * kHirsh, pre + kHeadCat, hw.c6_w2, hw.c6_qemb, hw.c6_vshift, hw.c6_sqrt_k,
                    dc6[i], zz, lane, gk_s[w], g + kHeadCat);
}

void launch_heads_seed(int n, const int *z, const double *hpre, const double *hk, const HeadsW &hw,
                       const double *dq, const double *dq_mean, const int *image_of_atom, const double *dh,
                       const double *hk6, const double *dc6, double *g_hcat, cudaStream_t s) {
  if (n == 0) return;
  k_heads_seed<<<(n * 32 + 255) / 256, 256, 0, s>>>(n, z, hpre, hk, hw, dq, dq_mean, image_of_atom, dh, hk6, dc6,
                                                    g_hcat);
  SO3_LAUNCH("heads_seed");
}

SO3LR_SHAPE_END
