// Per-pair geometry (distance, real spherical harmonics, PhysNet cutoff, learned
// ZBL), the long-range physics kernel, force/energy/virial assembly, the
// deterministic segment sums and the velocity-Verlet integrator.
//
// Reference arithmetic restated here:
//   real SH l=1..4 and their input VJP: src/kokkos_learned_energy_forces.cpp:14-139
//   PhysNet cutoff: src/kokkos_integrated_block0.cpp:145-155 (derivative: block2_attention_input_reverse.cpp:314-321)
//   learned ZBL: src/kokkos_physical_zbl.cpp:81-178
//   long range (erf Coulomb, shifted force + switch; QDO dispersion): src/kokkos_physical_long_range.cpp:11-380
//   virial: plugins/lammps/pair_so3lr_native_mpi.cpp:944-990
// The reference accumulates atoms with float atomics; here every per-atom sum is
// a gather over the atom's own CSR row or cell stencil in a fixed order.
#include <type_traits>

#include "cells.cuh"
#include "sh.cuh"

namespace so3lr_b200 {

// ---------------------------------------------------------------------------
// geometry of every undirected short-range pair
// ---------------------------------------------------------------------------
__global__ void k_pair_geometry(int P, const int *__restrict__ pa, const int *__restrict__ pb,
                                const int *__restrict__ pimg, const int *__restrict__ pcanon,
                                const double *__restrict__ xw, CellGrid g, const int *__restrict__ z, ZblDev zbl,
                                double rc, double *__restrict__ geo, double *__restrict__ sh,
                                double *__restrict__ gv) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= P) return;
  const int a = pa[p], b = pb[p];
  int sx, sy, sz;
  unpack_image(pimg[p], sx, sy, sz);
  // The vector is always formed in the pair's canonical orientation (smaller
  // tag receives) and negated otherwise, so a pair that two GPUs both hold,
  // each in its own orientation, gets bitwise opposite vectors.
  double vx, vy, vz;
  // explicitly rounded (no FMA contraction) so both branches round alike
  if (pcanon == nullptr || pcanon[p]) {
    vx = __dsub_rn(xw[3 * a], __dadd_rn(xw[3 * b], __dmul_rn(double(sx), g.len[0])));
    vy = __dsub_rn(xw[3 * a + 1], __dadd_rn(xw[3 * b + 1], __dmul_rn(double(sy), g.len[1])));
    vz = __dsub_rn(xw[3 * a + 2], __dadd_rn(xw[3 * b + 2], __dmul_rn(double(sz), g.len[2])));
  } else {
    vx = -__dsub_rn(xw[3 * b], __dadd_rn(xw[3 * a], __dmul_rn(double(-sx), g.len[0])));
    vy = -__dsub_rn(xw[3 * b + 1], __dadd_rn(xw[3 * a + 1], __dmul_rn(double(-sy), g.len[1])));
    vz = -__dsub_rn(xw[3 * b + 2], __dadd_rn(xw[3 * a + 2], __dmul_rn(double(-sz), g.len[2])));
  }
  const double r = sqrt(vx * vx + vy * vy + vz * vz);
  const double inv = r > 1.0e-14 ? 1.0 / r : 0.0;
  const double ux = vx * inv, uy = vy * inv, uz = vz * inv;
  double y[kSH];
  real_sh(ux, uy, uz, y);
#pragma unroll
  for (int m = 0; m < kSH; m += 2)  // 16-byte stores (a pair's row is 192 bytes)
    *reinterpret_cast<double2 *>(sh + (size_t)p * kSH + m) = make_double2(y[m], y[m + 1]);
  // PhysNet cutoff 1 - 10x^3 + 15x^4 - 6x^5 and its derivative
  double phi = 0.0, dphi = 0.0;
  if (r < rc) {
    const double x = r / rc, x2 = x * x, x3 = x2 * x;
    phi = 1.0 - 10.0 * x3 + 15.0 * x3 * x - 6.0 * x3 * x2;
    const double om = 1.0 - x;
    dphi = -30.0 * x * x * om * om / rc;
  }
  // repulsion (learned ZBL or NLH), directed edge b -> a (identical value for a -> b)
  double e_dir = 0.0, de_pair = 0.0;
  if (r > 0.0 && !(r > zbl.cutoff * (1.0 + 1.0e-12))) {
    const double zi = double(z[a]), zj = double(z[b]), zz = zi * zj;
    const double xn = r / zbl.cutoff, x2 = xn * xn, x3 = x2 * xn;
    const double cut = r < zbl.cutoff ? 1.0 - 10.0 * x3 + 15.0 * x3 * xn - 6.0 * x3 * x2 : 0.0;
    const double dcut = r < zbl.cutoff ? (-30.0 * x2 + 60.0 * x3 - 30.0 * x3 * xn) / zbl.cutoff : 0.0;
    const double c = r / zbl.switch_off;
    const double left = 1.0 - c, right = c;
    const double sl_ = left > 1.0e-12 ? left : 1.0e-12, sr_ = right > 1.0e-12 ? right : 1.0e-12;
    const double sig_l = left > 0.0 ? exp(-1.0 / sl_) : 0.0;
    const double sig_r = right > 0.0 ? exp(-1.0 / sr_) : 0.0;
    const double den = sig_l + sig_r + 1.0e-12;
    const double dl = left > 0.0 ? -sig_l / (sl_ * sl_) : 0.0;
    const double dr = right > 0.0 ? sig_r / (sr_ * sr_) : 0.0;
    const double sw = sig_l / den;
    const double dsw = ((dl * den - sig_l * (dl + dr)) / (den * den)) / zbl.switch_off;
    const double safe_r = r > 1.0e-6 ? r : 1.0e-6;
    const double ir = 1.0 / safe_r;
    const double dir = r > 1.0e-6 ? -1.0 / (r * r) : 0.0;
    const double xx = zbl.ke * cut * zz * ir;
    const double dxx = zbl.ke * zz * (dcut * ir + cut * dir);
    double yy = 0.0, dyy = 0.0;
    if (zbl.kind == 1) {
      // NLH: three exponentials from the pair tables, indexed (min Z, max Z)
      // from 1; pairs beyond the table capacity have no screening term
      const int za = min(z[a], z[b]), zb = max(z[a], z[b]);
      if (za >= 1 && zb <= zbl.nlh_cap) {
        const size_t base = ((size_t)(za - 1) * zbl.nlh_cap + (zb - 1)) * 3;
        for (int k = 0; k < 3; ++k) {
          const double amp = zbl.nlh_a[base + k], rate = zbl.nlh_b[base + k];
          const double ex = exp(-rate * r);
          yy += amp * ex;
          dyy -= rate * amp * ex;
        }
      }
    } else {
      const double rate = (pow(zi, zbl.p) + pow(zj, zbl.p)) * zbl.d;
      const double rzd = r * rate;
      for (int k = 0; k < 4; ++k) {
        const double ex = exp(-zbl.a[k] * rzd);
        yy += zbl.c[k] * ex;
        dyy -= zbl.c[k] * zbl.a[k] * rate * ex;
      }
    }
    e_dir = 0.5 * sw * xx * yy;
    de_pair = 2.0 * (0.5 * (dsw * xx * yy + sw * dxx * yy + sw * xx * dyy));
  }
  double2 *gp = reinterpret_cast<double2 *>(geo + (size_t)p * kGeo);
  gp[0] = make_double2(r, ux);
  gp[1] = make_double2(uy, uz);
  gp[2] = make_double2(phi, dphi);
  gp[3] = make_double2(e_dir, de_pair);
  gv[3 * p] = de_pair * ux;
  gv[3 * p + 1] = de_pair * uy;
  gv[3 * p + 2] = de_pair * uz;
}

void launch_pair_geometry(int P, const NeighborState &nb, const int *z, ZblDev zbl, double sr_cutoff,
                          double *geo, double *sh, double *gv, cudaStream_t s) {
  if (P == 0) return;
  k_pair_geometry<<<(P + 127) / 128, 128, 0, s>>>(P, nb.pair_a, nb.pair_b, nb.pair_img, nb.pair_canon, nb.xw,
                                                   nb.grid, z, zbl, sr_cutoff, geo, sh, gv);
  SO3_LAUNCH("pair_geometry");
}

// ---------------------------------------------------------------------------
// long range: erf-screened shifted-force Coulomb + QDO dispersion
// ---------------------------------------------------------------------------
// Smooth switch of physical_long_range.cpp: v = s_l / (s_l + s_r + 1e-12) with
// s_l = exp(-1/left), s_r = exp(-1/right), c = (r - cuton) / width, left = 1 - c,
// right = c (each clamped below at 1e-12 inside the exponent), and its derivative
// dv/dr, for both switches of a pair (electrostatic and dispersion: the same
// cutoff, different cutons). The divisions of the textbook form are folded into
// reciprocals shared by the two switches: 1/(sl sr) of both from one division,
// 1/den of both from another.
__device__ inline void smooth_switch2(double r, double cutoff, double cuton_e, double inv_we, double cuton_d,
                                      double inv_wd, double &ve, double &dve, double &vd, double &dvd) {
  if (r >= cutoff) {
    ve = dve = vd = dvd = 0.0;
    return;
  }
  const double ce = (r - cuton_e) * inv_we, cd = (r - cuton_d) * inv_wd;
  const double le = 1.0 - ce, re = ce, ld = 1.0 - cd, rd = cd;
  const double sle = le > 1.0e-12 ? le : 1.0e-12, sre = re > 1.0e-12 ? re : 1.0e-12;
  const double sld = ld > 1.0e-12 ? ld : 1.0e-12, srd = rd > 1.0e-12 ? rd : 1.0e-12;
  const double pe = sle * sre, pd = sld * srd;  // each >= ~1e-12: the product stays normal
  const double ip = 1.0 / (pe * pd);
  const double inv_e = pd * ip, inv_d = pe * ip;
  const double isle = sre * inv_e, isre = sle * inv_e, isld = srd * inv_d, isrd = sld * inv_d;
  // exp_tang clamps its argument: computed for every lane, then selected
  const double xle = exp_tang(-isle), xre = exp_tang(-isre), xld = exp_tang(-isld), xrd = exp_tang(-isrd);
  const double sig_le = le > 0.0 ? xle : 0.0, sig_re = re > 0.0 ? xre : 0.0;
  const double sig_ld = ld > 0.0 ? xld : 0.0, sig_rd = rd > 0.0 ? xrd : 0.0;
  const double dene = sig_le + sig_re + 1.0e-12, dend = sig_ld + sig_rd + 1.0e-12;
  const double iq = 1.0 / (dene * dend);
  const double idene = dend * iq, idend = dene * iq;
  ve = sig_le * idene;
  vd = sig_ld * idend;
  const double dle = le > 0.0 ? -sig_le * isle * isle : 0.0, dre = re > 0.0 ? sig_re * isre * isre : 0.0;
  const double dld = ld > 0.0 ? -sig_ld * isld * isld : 0.0, drd = rd > 0.0 ? sig_rd * isrd * isrd : 0.0;
  dve = (dle - ve * (dle + dre)) * idene * inv_we;
  dvd = (dld - vd * (dld + drd)) * idend * inv_wd;
}

struct LrPair {
  double e_elec, e_disp, dq, dh, dc;
  double radial;  // float64 pair term: dE/dr divided by r; float32 pair term: dE/dr
};

// per-launch constants of the pair term, computed once per thread
struct LrConst {
  double inv_sigma, inv_elec_width, inv_disp_width, inv_bohr;
};
__device__ inline LrConst lr_const(const LrDev &p) {
  LrConst c;
  c.inv_sigma = 1.0 / p.sigma;
  c.inv_elec_width = 1.0 / (p.cutoff - p.elec_cuton);
  c.inv_disp_width = 1.0 / (p.cutoff - p.disp_cuton);
  c.inv_bohr = 1.0 / p.bohr;
  return c;
}

// One unordered pair seen from atom i (its partner j); r > 0 and r < cutoff.
// ai0/aj0, ci0/cj0: reference polarisabilities and C6 of the two elements
// (aj0 < 0 marks an element without reference data: no dispersion).
// Arithmetic of physical_long_range.cpp:11-380 (erf-screened shifted-force
// Coulomb with its switch; QDO dispersion with C6 mixing, the fitted sigma(R_vdW)
// polynomial and its switch), with shared reciprocals instead of repeated
// divisions (about 10 divisions per pair instead of 49).
// kSepC6: the model has a C6 ratio head; si, sj are the two atoms' C6 ratios,
// C6 = C6_ref s instead of C6_ref h^2, and dc = dE/ds_i (physical_long_range.cpp:118-262).
template <bool kSepC6>
__device__ inline LrPair lr_pair_tab(const LrDev &p, const LrConst &k, double r, double qi, double qj, double hi,
                                     double hj, double ai0, double aj0, double ci0, double cj0, double si,
                                     double sj) {
  constexpr double inv_sqrt_pi = 0.56418958354775628695;
  constexpr double inv7 = 1.0 / 7.0;
  LrPair o{0, 0, 0, 0, 0, 0};
  double esw, desw, dsw, ddsw;
  smooth_switch2(r, p.cutoff, p.elec_cuton, k.inv_elec_width, p.disp_cuton, k.inv_disp_width, esw, desw, dsw, ddsw);
  const double inv_r = 1.0 / r;
  const double ratio = r * k.inv_sigma;
  const double erf_t = erf(ratio);
  const double exp_t = exp_tang(-(ratio * ratio));
  const double pot = erf_t * inv_r;
  const double dpot = (2.0 * r * exp_t * inv_sqrt_pi * k.inv_sigma - erf_t) * (inv_r * inv_r);
  const double disp = r - p.cutoff;
  const double shifted = pot - p.shift - p.fshift * disp;
  const double kernel = esw * (pot - p.shift) + (1.0 - esw) * shifted;
  const double rkernel = dpot - (1.0 - esw) * p.fshift + desw * p.fshift * disp;
  o.e_elec = p.full_scale * p.ke * qi * qj * kernel;
  o.dq = p.full_scale * p.ke * kernel * qj;
  const double erad = p.full_scale * p.ke * qi * qj * rkernel;
  double drad = 0.0;
  {
    // computed without branches, so that the dispersion chain interleaves with
    // the electrostatic one; a pair without dispersion (no reference data, or
    // alpha or the C6 denominator not positive) runs on stand-in values and its
    // results are dropped at the end
    const bool has = ai0 >= 0.0 && aj0 >= 0.0;
    const double ai = ai0 * hi, aj = aj0 * hj;
    const double c6i = kSepC6 ? ci0 * si : ci0 * hi * hi, c6j = kSepC6 ? cj0 * sj : cj0 * hj * hj;
    const double alpha_v = 0.5 * (ai + aj);
    const double num = 2.0 * c6i * c6j * aj * ai;
    const double den_v = ai * ai * c6j + aj * aj * c6i;
    const bool ok = has && alpha_v > 0.0 && den_v > 1.0e-30;
    const double alpha = ok ? alpha_v : 1.0, den = ok ? den_v : 1.0;
    {
      const double iad = 1.0 / (alpha * den);  // 1/(alpha den): both positive, product far inside the normal range
      const double iden = alpha * iad;
      const double c6 = num * iden;
      double dc6_dhi, dc6_dsi = 0.0;
      if (!kSepC6) {  // h_i drives both alpha_i and C6_i
        const double dc6i = 2.0 * ci0 * hi;
        const double dn_dhi = 2.0 * (dc6i * c6j * aj * ai + c6i * c6j * aj * ai0);
        const double dd_dhi = 2.0 * ai * ai0 * c6j + aj * aj * dc6i;
        dc6_dhi = (dn_dhi * den - num * dd_dhi) * (iden * iden);
      } else {  // h_i through alpha_i only, s_i through C6_i only
        const double dn_dai = 2.0 * c6i * c6j * aj * ai0;
        const double dd_dai = 2.0 * ai * ai0 * c6j;
        dc6_dhi = (dn_dai * den - num * dd_dai) * (iden * iden);
        const double dn_dsi = 2.0 * ci0 * c6j * aj * ai;
        const double dd_dsi = aj * aj * ci0;
        dc6_dsi = (dn_dsi * den - num * dd_dsi) * (iden * iden);
      }
      const double ialpha7 = inv7 * (den * iad);  // 1 / (7 alpha)
      const double a7 = exp_tang(log(alpha) * inv7);
      const double rv = p.fine_factor * a7;
      constexpr double b0 = -0.00433008, b1 = 0.24428889, b2 = 0.04125273, b3 = -0.00078893;
      const double sig = b3 * rv * rv * rv + b2 * rv * rv + b1 * rv + b0;
      const double isig = 1.0 / sig;
      const double gam = 0.5 * isig * isig;
      const double igam = 2.0 * sig * sig;  // 1 / gam
      const double drv = rv * ialpha7;
      const double dsig = (3.0 * b3 * rv * rv + 2.0 * b2 * rv + b1) * drv;
      const double dgam = -2.0 * gam * dsig * isig;
      const double c8 = 5.0 * c6 * igam;
      const double c10 = 245.0 * c6 * (igam * igam) * 0.125;
      const double damp = p.disp_scale * 2.0 * 2.54 * a7;
      const double ddamp = damp * ialpha7;
      const double ra = r * k.inv_bohr;
      const double r2 = ra * ra, r4 = r2 * r2, r6 = r4 * r2, r8 = r4 * r4, r10 = r8 * r2;
      const double p2 = damp * damp, p4 = p2 * p2, p6 = p4 * p2, p8 = p4 * p4, p10 = p8 * p2;
      const double d6 = r6 + p6, d8 = r8 + p8, d10 = r10 + p10;
      // one division for the three denominators r^n + damp^n (n = 6, 8, 10):
      // their product is at least damp^24 and overflows only beyond r ~ 1e12 bohr
      const double id = 1.0 / (d6 * d8 * d10);
      const double id6 = d8 * d10 * id, id8 = d6 * d10 * id, id10 = d6 * d8 * id;
      const double qdo = -c6 * id6 - c8 * id8 - c10 * id10;
      const double rad_au =
          (6.0 * c6 * r4 * id6 * id6 + 8.0 * c8 * r6 * id8 * id8 + 10.0 * c10 * r8 * id10 * id10) * ra;
      const double dc8 = -c8 * dgam * igam;
      const double dc10 = -2.0 * c10 * dgam * igam;
      const double dd6 = 6.0 * p4 * damp * ddamp;
      const double dd8 = 8.0 * p6 * damp * ddamp;
      const double dd10 = 10.0 * p8 * damp * ddamp;
      const double dpot_da = c6 * dd6 * id6 * id6 - dc8 * id8 + c8 * dd8 * id8 * id8 - dc10 * id10 +
                             c10 * dd10 * id10 * id10;
      const double dpot_dc6 = -id6 - 5.0 * igam * id8 - 245.0 * 0.125 * (igam * igam) * id10;
      const double dpot_dhi = dpot_dc6 * dc6_dhi + dpot_da * 0.5 * ai0;
      o.e_disp = ok ? p.full_scale * p.hartree * qdo * dsw : 0.0;
      drad = ok ? p.full_scale * p.hartree * (rad_au * dsw * k.inv_bohr + qdo * ddsw) : 0.0;
      o.dh = ok ? p.full_scale * p.hartree * dsw * dpot_dhi : 0.0;
      if (kSepC6) o.dc = ok ? p.full_scale * p.hartree * dsw * dpot_dc6 * dc6_dsi : 0.0;
    }
  }
  o.radial = (erad + drad) * inv_r;
  return o;
}


// The same pair term in float32 arithmetic, for the mixed-precision mode: the
// caller passes the float32 distance and per-atom values and adds the float32
// results into float64 sums. Same formulas and switch as lr_pair_tab, with
// CUDA's float32 erf/exp/log and IEEE float32 division.
struct LrConst32 {
  float ke_s, hartree_s, inv_sigma, inv_elec_width, inv_disp_width, inv_bohr, cutoff, elec_cuton, disp_cuton, shift,
      fshift, fine_factor, disp_scale;
};
__device__ inline LrConst32 lr_const32(const LrDev &p) {
  LrConst32 c;
  c.ke_s = float(p.full_scale * p.ke);
  c.hartree_s = float(p.full_scale * p.hartree);
  c.inv_sigma = float(1.0 / p.sigma);
  c.inv_elec_width = float(1.0 / (p.cutoff - p.elec_cuton));
  c.inv_disp_width = float(1.0 / (p.cutoff - p.disp_cuton));
  c.inv_bohr = float(1.0 / p.bohr);
  c.cutoff = float(p.cutoff);
  c.elec_cuton = float(p.elec_cuton);
  c.disp_cuton = float(p.disp_cuton);
  c.shift = float(p.shift);
  c.fshift = float(p.fshift);
  c.fine_factor = float(p.fine_factor);
  c.disp_scale = float(p.disp_scale);
  return c;
}
__device__ inline void smooth_switch32(float r, float cuton, float cutoff, float inv_width, float &v, float &dv) {
  if (r >= cutoff) {
    v = 0.0f;
    dv = 0.0f;
    return;
  }
  const float c = (r - cuton) * inv_width;
  const float left = 1.0f - c, right = c;
  const float sl = left > 1.0e-12f ? left : 1.0e-12f, sr = right > 1.0e-12f ? right : 1.0e-12f;
  const float isl = 1.0f / sl, isr = 1.0f / sr;
  const float xl = expf(-isl), xr = expf(-isr);  // for every lane, then selected
  const float sig_l = left > 0.0f ? xl : 0.0f;
  const float sig_r = right > 0.0f ? xr : 0.0f;
  const float iden = 1.0f / (sig_l + sig_r + 1.0e-12f);
  v = sig_l * iden;
  const float dl = left > 0.0f ? -sig_l * isl * isl : 0.0f;
  const float dr = right > 0.0f ? sig_r * isr * isr : 0.0f;
  dv = (dl - v * (dl + dr)) * iden * inv_width;
}
template <bool kSepC6>
__device__ inline LrPair lr_pair_f32(const LrConst32 &k, float r, float qi, float qj, float hi, float hj, float ai0,
                                     float aj0, float ci0, float cj0, float si, float sj) {
  constexpr float inv_sqrt_pi = 0.56418958354775628695f;
  constexpr float inv7 = 1.0f / 7.0f;
  LrPair o{0, 0, 0, 0, 0, 0};
  float esw, desw;
  smooth_switch32(r, k.elec_cuton, k.cutoff, k.inv_elec_width, esw, desw);
  const float inv_r = 1.0f / r;
  const float ratio = r * k.inv_sigma;
  const float erf_t = erff(ratio);
  const float exp_t = expf(-(ratio * ratio));
  const float pot = erf_t * inv_r;
  const float dpot = (2.0f * r * exp_t * inv_sqrt_pi * k.inv_sigma - erf_t) * (inv_r * inv_r);
  const float disp = r - k.cutoff;
  const float shifted = pot - k.shift - k.fshift * disp;
  const float kernel = esw * (pot - k.shift) + (1.0f - esw) * shifted;
  const float rkernel = dpot - (1.0f - esw) * k.fshift + desw * k.fshift * disp;
  o.e_elec = k.ke_s * qi * qj * kernel;
  o.dq = k.ke_s * kernel * qj;
  const float erad = k.ke_s * qi * qj * rkernel;
  float drad = 0.0f;
  {
    // without branches, as in the float64 term: stand-in values where a pair
    // has no dispersion, results dropped at the end
    const bool has = ai0 >= 0.0f && aj0 >= 0.0f;
    const float ai = ai0 * hi, aj = aj0 * hj;
    const float c6i = kSepC6 ? ci0 * si : ci0 * hi * hi, c6j = kSepC6 ? cj0 * sj : cj0 * hj * hj;
    const float alpha_v = 0.5f * (ai + aj);
    const float num = 2.0f * c6i * c6j * aj * ai;
    const float den_v = ai * ai * c6j + aj * aj * c6i;
    const bool ok = has && alpha_v > 0.0f && den_v > 1.0e-30f;
    const float alpha = ok ? alpha_v : 1.0f, den = ok ? den_v : 1.0f;
    {
      const float iden = 1.0f / den;
      const float c6 = num * iden;
      float dc6_dhi, dc6_dsi = 0.0f;
      if (!kSepC6) {
        const float dc6i = 2.0f * ci0 * hi;
        const float dn_dhi = 2.0f * (dc6i * c6j * aj * ai + c6i * c6j * aj * ai0);
        const float dd_dhi = 2.0f * ai * ai0 * c6j + aj * aj * dc6i;
        dc6_dhi = (dn_dhi * den - num * dd_dhi) * (iden * iden);
      } else {
        const float dn_dai = 2.0f * c6i * c6j * aj * ai0;
        const float dd_dai = 2.0f * ai * ai0 * c6j;
        dc6_dhi = (dn_dai * den - num * dd_dai) * (iden * iden);
        const float dn_dsi = 2.0f * ci0 * c6j * aj * ai;
        const float dd_dsi = aj * aj * ci0;
        dc6_dsi = (dn_dsi * den - num * dd_dsi) * (iden * iden);
      }
      const float ialpha7 = inv7 / alpha;
      const float a7 = expf(logf(alpha) * inv7);
      const float rv = k.fine_factor * a7;
      constexpr float b0 = -0.00433008f, b1 = 0.24428889f, b2 = 0.04125273f, b3 = -0.00078893f;
      const float sig = b3 * rv * rv * rv + b2 * rv * rv + b1 * rv + b0;
      const float isig = 1.0f / sig;
      const float gam = 0.5f * isig * isig;
      const float igam = 2.0f * sig * sig;
      const float drv = rv * ialpha7;
      const float dsig = (3.0f * b3 * rv * rv + 2.0f * b2 * rv + b1) * drv;
      const float dgam = -2.0f * gam * dsig * isig;
      const float c8 = 5.0f * c6 * igam;
      const float c10 = 245.0f * c6 * (igam * igam) * 0.125f;
      const float damp = k.disp_scale * 2.0f * 2.54f * a7;
      const float ddamp = damp * ialpha7;
      const float ra = r * k.inv_bohr;
      const float r2 = ra * ra, r4 = r2 * r2, r6 = r4 * r2, r8 = r4 * r4, r10 = r8 * r2;
      const float p2 = damp * damp, p4 = p2 * p2, p6 = p4 * p2, p8 = p4 * p4, p10 = p8 * p2;
      const float id6 = 1.0f / (r6 + p6), id8 = 1.0f / (r8 + p8), id10 = 1.0f / (r10 + p10);
      const float qdo = -c6 * id6 - c8 * id8 - c10 * id10;
      const float rad_au =
          (6.0f * c6 * r4 * id6 * id6 + 8.0f * c8 * r6 * id8 * id8 + 10.0f * c10 * r8 * id10 * id10) * ra;
      const float dc8 = -c8 * dgam * igam;
      const float dc10 = -2.0f * c10 * dgam * igam;
      const float dd6 = 6.0f * p4 * damp * ddamp;
      const float dd8 = 8.0f * p6 * damp * ddamp;
      const float dd10 = 10.0f * p8 * damp * ddamp;
      const float dpot_da = c6 * dd6 * id6 * id6 - dc8 * id8 + c8 * dd8 * id8 * id8 - dc10 * id10 +
                            c10 * dd10 * id10 * id10;
      const float dpot_dc6 = -id6 - 5.0f * igam * id8 - 245.0f * 0.125f * (igam * igam) * id10;
      const float dpot_dhi = dpot_dc6 * dc6_dhi + dpot_da * 0.5f * ai0;
      float dsw, ddsw;
      smooth_switch32(r, k.disp_cuton, k.cutoff, k.inv_disp_width, dsw, ddsw);
      o.e_disp = ok ? k.hartree_s * qdo * dsw : 0.0f;
      drad = ok ? k.hartree_s * (rad_au * dsw * k.inv_bohr + qdo * ddsw) : 0.0f;
      o.dh = ok ? k.hartree_s * dsw * dpot_dhi : 0.0f;
      if (kSepC6) o.dc = ok ? k.hartree_s * dsw * dpot_dc6 * dc6_dsi : 0.0f;
    }
  }
  o.radial = erad + drad;
  return o;
}

// one 256-bit read-only load of a 32-byte aligned double4
__device__ inline double4 ld4(const double4 *p) {
  double4 v;
  asm("ld.global.nc.v4.f64 {%0,%1,%2,%3}, [%4];" : "=d"(v.x), "=d"(v.y), "=d"(v.z), "=d"(v.w) : "l"(p));
  return v;
}

__device__ inline double warp_sum(double v) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Cell-ordered copy of what the long-range pair term reads from a partner atom:
// pos4[k] = (x, y, z, q) and par4[k] = (h, alpha_ref, C6_ref, C6 ratio or 0)
// of atom cell_atoms[k] (atom k itself for open boundaries), so that every
// stencil row of cells is one contiguous, coalesced range of candidates.
__global__ void k_lr_gather(int n, int cell_ordered, const int *__restrict__ cell_atoms, const double *__restrict__ xw,
                            const double *__restrict__ q, const double *__restrict__ h,
                            const double *__restrict__ c6r, const int *__restrict__ z,
                            const double *__restrict__ aref, const double *__restrict__ cref, int table,
                            double4 *__restrict__ pos4, double4 *__restrict__ par4) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const int j = cell_ordered ? cell_atoms[k] : k;
  const int zj = z[j] - 1;
  const bool known = zj >= 0 && zj < table;
  pos4[k] = make_double4(xw[3 * j], xw[3 * j + 1], xw[3 * j + 2], q[j]);
  par4[k] = make_double4(h[j], known ? aref[zj] : -1.0, known ? cref[zj] : 0.0, c6r ? c6r[j] : 0.0);
}

// One warp per atom. The candidate ranges of the atom's cell stencil (x runs of
// cells, contiguous in the cell-ordered arrays) are listed lane-parallel, 32
// stencil rows at a time, into a per-warp table in shared memory; the lanes then
// walk the concatenation of those ranges 32 candidates at a time, across range
// boundaries. Candidates inside the cutoff are compacted (ballot + prefix) into
// a per-warp queue (candidate index and periodic shift), and the pair math runs
// only on full batches of 32 queued pairs. The queue receives the pairs in the
// stencil's serial order (rows by z then y, runs by x shift) and every lane
// accumulates its queue slots in a fixed order, so the result is deterministic.
constexpr int kLrWarps = 8;
constexpr int kLrMaxReach = 8;
// per (|oy|, |oz|) of the cell stencil: the x reach of the cells that can hold
// a neighbour within the cutoff (-1: none)
struct LrStencil {
  signed char rx[kLrMaxReach + 1][kLrMaxReach + 1];
};
constexpr int kLrQueue = 64;
constexpr int kLrSegs = 64;  // candidate ranges per table fill (two per lane)
// periodic shift (sx, sy, sz), each in [-127, 127], packed into one int
__host__ __device__ inline int lr_shift_code(int sx, int sy, int sz) {
  return (sx + 128) | ((sy + 128) << 8) | ((sz + 128) << 16);
}
template <bool kSepC6, bool kF32>
__global__ void __launch_bounds__(kLrWarps * 32, 2) k_long_range(
    int n, int row0, const double *__restrict__ xw, CellGrid g, const int *__restrict__ cell,
    const int *__restrict__ cell_start, const int *__restrict__ cell_count, const int *__restrict__ image_of,
    const int *__restrict__ image_start, int reach, int rows_per_fill, LrStencil st, double rc2,
    const double4 *__restrict__ pos4, const double4 *__restrict__ par4, const int *__restrict__ z,
    const double *__restrict__ q, const double *__restrict__ h, const double *__restrict__ c6r,
    const double *__restrict__ aref, const double *__restrict__ cref, int table, LrDev p,
    double *__restrict__ e_lr, double *__restrict__ e_elec, double *__restrict__ e_disp, double *__restrict__ dq,
    double *__restrict__ dh, double *__restrict__ dc6, double *__restrict__ f_lr, double *__restrict__ w_lr) {
  __shared__ int qk[kLrWarps][kLrQueue];       // queued candidate (cell-ordered index)
  __shared__ int qs[kLrWarps][kLrQueue];       // its shift code
  __shared__ int sg_first[kLrWarps][kLrSegs];  // range table: first candidate,
  __shared__ int sg_pre[kLrWarps][kLrSegs + 1];  // concatenated offset,
  __shared__ int sg_code[kLrWarps][kLrSegs];   // shift code
  const int wl = threadIdx.x >> 5;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const int i = row0 + warp;
  const double xi = xw[3 * i], yi = xw[3 * i + 1], zi = xw[3 * i + 2];
  const double qi = q[i], hi = h[i], si = kSepC6 ? c6r[i] : 0.0;
  const int Zi = z[i];
  const double ai0 = (Zi - 1 >= 0 && Zi - 1 < table) ? aref[Zi - 1] : -1.0;
  const double ci0 = (Zi - 1 >= 0 && Zi - 1 < table) ? cref[Zi - 1] : 0.0;
  const LrConst kc = lr_const(p);
  LrConst32 kc32{};
  if (kF32) kc32 = lr_const32(p);
  double acc_ee = 0, acc_ed = 0, acc_dq = 0, acc_dh = 0, acc_dc = 0, fx = 0, fy = 0, fz = 0;
  double wxx = 0, wyy = 0, wzz = 0, wxy = 0, wxz = 0, wyz = 0;
  int count = 0;  // warp-uniform queue length
  // displacement from atom i to candidate k under the shift with this code
  // (the same expression in the scan and in the pair evaluation: same bits)
  auto displacement = [&](const double4 &pk, int code, double &vx, double &vy, double &vz) {
    const int sx = (code & 255) - 128, sy = ((code >> 8) & 255) - 128, sz = ((code >> 16) & 255) - 128;
    vx = pk.x + (sx == 0 ? 0.0 : sx * g.len[0]) - xi;
    vy = pk.y + (sy == 0 ? 0.0 : sy * g.len[1]) - yi;
    vz = pk.z + (sz == 0 ? 0.0 : sz * g.len[2]) - zi;
  };
  auto evaluate = [&](int slot) {
    const int k = qk[wl][slot];
    const double4 pj = ld4(pos4 + k), hj = ld4(par4 + k);
    double vx, vy, vz;
    displacement(pj, qs[wl][slot], vx, vy, vz);
    const double r = sqrt(vx * vx + vy * vy + vz * vz);
    LrPair o;
    if constexpr (kF32)
      o = lr_pair_f32<kSepC6>(kc32, float(r), float(qi), float(pj.w), float(hi), float(hj.x), float(ai0), float(hj.y),
                              float(ci0), float(hj.z), float(si), float(hj.w));
    else
      o = lr_pair_tab<kSepC6>(p, kc, r, qi, pj.w, hi, hj.x, ai0, hj.y, ci0, hj.z, si, hj.w);
    acc_ee += o.e_elec;
    acc_ed += o.e_disp;
    acc_dq += o.dq;
    acc_dh += o.dh;
    if (kSepC6) acc_dc += o.dc;
    // dE/dr / r: divided by r inside the float64 pair term, here in the float32 one
    const double s = kF32 ? o.radial / r : o.radial;
    fx += s * vx;
    fy += s * vy;
    fz += s * vz;
    wxx -= 0.5 * s * vx * vx;
    wyy -= 0.5 * s * vy * vy;
    wzz -= 0.5 * s * vz * vz;
    wxy -= 0.5 * s * vx * vy;
    wxz -= 0.5 * s * vx * vz;
    wyz -= 0.5 * s * vy * vz;
  };
  // test every candidate of the nseg ranges in the table, in order
  auto scan_table = [&](int nseg) {
    const int total = sg_pre[wl][nseg];
    int sg = 0, sg_nx = 0;  // this lane's range cursors (candidate v and v + 32)
    for (int base = 0; base < total; base += 32) {
      const int v = base + lane;
      bool valid = false;
      int k = 0, code = 0;
      if (v < total) {
        while (sg_pre[wl][sg + 1] <= v) ++sg;
        k = sg_first[wl][sg] + (v - sg_pre[wl][sg]);
        code = sg_code[wl][sg];
        if (v + 32 < total) {  // pull the next batch's candidate into L1
          while (sg_pre[wl][sg_nx + 1] <= v + 32) ++sg_nx;
          asm volatile("prefetch.global.L1 [%0];" ::"l"(pos4 + sg_first[wl][sg_nx] + (v + 32 - sg_pre[wl][sg_nx])));
        }
        double vx, vy, vz;
        displacement(ld4(pos4 + k), code, vx, vy, vz);
        const double r2 = vx * vx + vy * vy + vz * vz;
        valid = r2 > 1.0e-24 && r2 < rc2;
      }
      const unsigned mask = __ballot_sync(0xffffffffu, valid);
      if (valid) {
        const int slot = count + __popc(mask & ((1u << lane) - 1u));
        qk[wl][slot] = k;
        qs[wl][slot] = code;
      }
      count += __popc(mask);
      __syncwarp();
      if (count >= 32) {
        evaluate(lane);
        __syncwarp();
        const int rest = count - 32;
        int mk = 0, mc = 0;
        if (lane < rest) {
          mk = qk[wl][32 + lane];
          mc = qs[wl][32 + lane];
        }
        __syncwarp();
        if (lane < rest) {
          qk[wl][lane] = mk;
          qs[wl][lane] = mc;
        }
        count = rest;
        __syncwarp();
      }
    }
  };
  // Every lane brings m ranges (of one stencil row; at most kLrSegs over the
  // warp), the q-th from run(q, first, len, code): write them to the table in
  // lane order and turn their lengths into concatenated offsets.
  auto fill_table = [&](int m, auto run) {
    __syncwarp();  // the previous table has been read
    int off = m;  // prefix of the lanes' range counts
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, off, d);
      if (lane >= d) off += t;
    }
    const int nseg = __shfl_sync(0xffffffffu, off, 31);
    off -= m;
    for (int qq = 0; qq < m; ++qq) {
      int first, len, code;
      run(qq, first, len, code);
      sg_first[wl][off + qq] = first;
      sg_pre[wl][off + qq + 1] = len;  // lengths for now
      sg_code[wl][off + qq] = code;
    }
    __syncwarp();
    // offsets: lane l sums ranges 2l and 2l + 1, then a warp scan
    const int l0 = 2 * lane < nseg ? sg_pre[wl][2 * lane + 1] : 0;
    const int l1 = 2 * lane + 1 < nseg ? sg_pre[wl][2 * lane + 2] : 0;
    int incl = l0 + l1;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += t;
    }
    __syncwarp();
    if (2 * lane < nseg) sg_pre[wl][2 * lane + 1] = incl - l1;
    if (2 * lane + 1 < nseg) sg_pre[wl][2 * lane + 2] = incl;
    if (lane == 0) sg_pre[wl][0] = 0;
    __syncwarp();
    return nseg;
  };
  if (!g.periodic && !g.open_cells) {
    const int im = image_of[i];
    const int nseg = fill_table(lane == 0 ? 1 : 0, [&](int, int &first, int &len, int &code) {
      first = image_start[im];
      len = image_start[im + 1] - first;
      code = lr_shift_code(0, 0, 0);
    });
    scan_table(nseg);
  } else {
    const int nx = g.ncell[0], ny = g.ncell[1], nz = g.ncell[2];
    const int c = cell[i];
    const int cx = c % nx, cy = (c / nx) % ny, cz = c / (nx * ny);
    const int side = 2 * reach + 1;
    // The atom's offset from its cell's lower corner; along each axis, the gap
    // from the atom to the cells o rows away is at least axis_gap (exact for a
    // cell holding its atoms; a clamped open-grid cell's atoms lie farther out),
    // less a margin far above the rounding of positions and cell bounds. Rows
    // and x cells beyond the cutoff by these gaps hold no pair: trimming them
    // drops only candidates that fail the distance test, in the same order.
    constexpr double kGapMargin = 1.0e-7;
    const double clx = g.len[0] / nx, cly = g.len[1] / ny, clz = g.len[2] / nz;
    const double ux = (xi - g.lo[0]) - cx * clx, uy = (yi - g.lo[1]) - cy * cly, uz = (zi - g.lo[2]) - cz * clz;
    auto axis_gap = [](int o, double u, double cl) {
      const double d = o > 0 ? o * cl - u : (o < 0 ? u + (-o - 1) * cl : 0.0);
      return fmax(d - kGapMargin, 0.0);
    };
    for (int t0 = 0; t0 < side * side; t0 += rows_per_fill) {
      // lane j: stencil row t0 + j, (oz, oy) in the serial order (z outer)
      const int t = t0 + lane;
      const int oz = t / side - reach, oy = t % side - reach;
      int m = 0, row = 0, xa = 0, xb = -1, sx_lo = 0, sy = 0, sz = 0;
      if (lane < rows_per_fill && t < side * side) {
        // cells farther than the cutoff from the home cell (nearest points)
        // cannot hold a neighbour: rows with such (oy, oz) are skipped and each
        // row's x run is trimmed to the cells that can (st.rx, tabulated on the
        // host), then to the cells within the cutoff of the atom itself
        const int rx = st.rx[abs(oy)][abs(oz)];
        const double gy = axis_gap(oy, uy, cly), gz = axis_gap(oz, uz, clz);
        const double rem = rc2 - gy * gy - gz * gz;
        if (rx >= 0 && rem > 0.0) {
          // cells cx + xa .. cx + xb (unwrapped): o > 0 while o clx - ux <= w,
          // o < 0 while ux + (-o - 1) clx <= w, and always the atom's own
          // column (gap 0: on a clamped open grid the atom can lie beyond it)
          const double w = sqrt(rem) + kGapMargin;
          const double hi_d = fmin(fmax(floor((w + ux) / clx), 0.0), double(rx));
          const double lo_d = fmin(fmax(floor((w - ux) / clx + 1.0), 0.0), double(rx));
          xb = cx + int(hi_d);
          xa = cx - int(lo_d);
        }
        if (xa > xb) {
          // nothing of this row is within the cutoff
        } else if (g.open_cells) {
          // one open system on a clamped grid: no wrap and no shift (an atom
          // outside the grid is farther from every other cell than its
          // boundary cell is, so the bounds above still hold)
          const int wz = cz + oz, wy = cy + oy;
          if (wz >= 0 && wz < nz && wy >= 0 && wy < ny && max(0, xa) <= min(nx - 1, xb)) {
            row = (wz * ny + wy) * nx;
            m = 1;
          }
        } else {
          // x runs of constant periodic shift are contiguous
          int wz = cz + oz, wy = cy + oy;
          while (wz < 0) { wz += nz; --sz; }
          while (wz >= nz) { wz -= nz; ++sz; }
          while (wy < 0) { wy += ny; --sy; }
          while (wy >= ny) { wy -= ny; ++sy; }
          row = (wz * ny + wy) * nx;
          sx_lo = xa >= 0 ? 0 : -((nx - 1 - xa) / nx);
          const int sx_hi = xb >= 0 ? xb / nx : -1;
          for (int sx = sx_lo; sx <= sx_hi; ++sx)
            if (max(0, xa - sx * nx) <= min(nx - 1, xb - sx * nx)) ++m;
        }
      }
      const int nseg = fill_table(m, [&](int qq, int &first, int &len, int &code) {
        int lo, hi, sx;
        if (g.open_cells) {
          lo = max(0, xa);
          hi = min(nx - 1, xb);
          sx = 0;
        } else {  // the qq-th non-empty x run of the row
          sx = sx_lo;
          for (int seen = -1;; ++sx) {
            lo = max(0, xa - sx * nx);
            hi = min(nx - 1, xb - sx * nx);
            if (lo <= hi && ++seen == qq) break;
          }
        }
        first = cell_start[row + lo];
        len = cell_start[row + hi] + cell_count[row + hi] - first;
        code = lr_shift_code(sx, sy, sz);
      });
      scan_table(nseg);
    }
  }
  if (lane < count) evaluate(lane);
  acc_ee = warp_sum(acc_ee);
  acc_ed = warp_sum(acc_ed);
  acc_dq = warp_sum(acc_dq);
  acc_dh = warp_sum(acc_dh);
  if (kSepC6) acc_dc = warp_sum(acc_dc);
  fx = warp_sum(fx);
  fy = warp_sum(fy);
  fz = warp_sum(fz);
  wxx = warp_sum(wxx);
  wyy = warp_sum(wyy);
  wzz = warp_sum(wzz);
  wxy = warp_sum(wxy);
  wxz = warp_sum(wxz);
  wyz = warp_sum(wyz);
  if (lane == 0) {
    e_elec[i] = 0.5 * acc_ee;
    e_disp[i] = 0.5 * acc_ed;
    e_lr[i] = 0.5 * acc_ee + 0.5 * acc_ed;
    dq[i] = acc_dq;
    dh[i] = acc_dh;
    if (kSepC6) dc6[i] = acc_dc;
    f_lr[3 * i] = fx;
    f_lr[3 * i + 1] = fy;
    f_lr[3 * i + 2] = fz;
    double *w = w_lr + 6 * i;
    w[0] = wxx; w[1] = wyy; w[2] = wzz; w[3] = wxy; w[4] = wxz; w[5] = wyz;
  }
}

void launch_long_range(int n, int n_cells_atoms, const NeighborState &nb, double rc_lr, const int *z,
                       const double *q, const double *h, const double *c6r, const double *alpha_ref,
                       const double *c6_ref, int table_size, LrDev p, double4 *pos4, double4 *par4, double *e_lr,
                       double *e_elec, double *e_disp, double *dq, double *dh, double *dc6, double *f_lr,
                       double *w_lr, cudaStream_t s, bool f32) {
  if (n == 0) return;
  k_lr_gather<<<(n_cells_atoms + 255) / 256, 256, 0, s>>>(n_cells_atoms, nb.grid.periodic || nb.grid.open_cells,
                                                          nb.cell_atoms, nb.xw, q, h,
                                                          c6r, z, alpha_ref, c6_ref, table_size, pos4, par4);
  SO3_LAUNCH("lr_gather");
  const int reach = sr_reach(nb.grid, rc_lr);
  LrStencil st;
  int rows_per_fill = 32;
  {
    const CellGrid &g = nb.grid;
    const double clx = g.len[0] / g.ncell[0], cly = g.len[1] / g.ncell[1], clz = g.len[2] / g.ncell[2];
    const double rcs = rc_lr * rc_lr * (1.0 + 1e-12) + 1e-12;
    for (int a = 0; a <= kLrMaxReach; ++a)
      for (int b = 0; b <= kLrMaxReach; ++b) {
        int rx = reach;
        if ((g.periodic || g.open_cells) && reach <= kLrMaxReach) {
          const double dy = std::max(a - 1, 0) * cly, dz = std::max(b - 1, 0) * clz;
          const double rem = rcs - dy * dy - dz * dz;
          rx = rem <= 0.0 ? -1 : std::min(reach, int(std::floor(std::sqrt(rem) / clx)) + 1);
        }
        st.rx[a][b] = static_cast<signed char>(rx);
      }
    if ((g.periodic || g.open_cells) && reach > kLrMaxReach)
      throw std::runtime_error("SO3LR long range: cell stencil reach above " +
                                                       std::to_string(kLrMaxReach));
    if (g.periodic) {
      // x runs of one stencil row: one per periodic shift of the row's cells
      // (two when the run wraps once); the kernel's range table holds kLrSegs
      int max_runs = 1;
      const int nx = g.ncell[0];
      for (int a = 0; a <= reach; ++a)
        for (int b = 0; b <= reach; ++b) {
          const int rx = st.rx[a][b];
          if (rx < 0) continue;
          for (int cx = 0; cx < nx; ++cx) {
            const int sx_lo = (cx - rx >= 0) ? 0 : -((rx - cx + nx - 1) / nx), sx_hi = (cx + rx) / nx;
            int runs = 0;
            for (int sx = sx_lo; sx <= sx_hi; ++sx)
              if (std::max(0, cx - rx - sx * nx) <= std::min(nx - 1, cx + rx - sx * nx)) ++runs;
            max_runs = std::max(max_runs, runs);
          }
        }
      rows_per_fill = std::min(32, kLrSegs / max_runs);
    }
  }
  const int threads = kLrWarps * 32;
  const int blocks = (n * 32 + threads - 1) / threads;
  auto go = [&](auto sep, auto f) {
    constexpr bool kSep = decltype(sep)::value, kF = decltype(f)::value;
    k_long_range<kSep, kF><<<blocks, threads, 0, s>>>(n, nb.row0, nb.xw, nb.grid, nb.cell, nb.cell_start,
                                                      nb.cell_count, nb.image_of, nb.image_start, reach,
                                                      rows_per_fill, st, rc_lr * rc_lr, pos4, par4, z, q, h, kSep ? c6r : nullptr,
                                                      alpha_ref, c6_ref, table_size, p, e_lr, e_elec, e_disp, dq, dh,
                                                      kSep ? dc6 : nullptr, f_lr, w_lr);
  };
  using T = std::true_type;
  using F = std::false_type;
  if (c6r != nullptr) {
    if (f32) go(T{}, T{});
    else go(T{}, F{});
  } else {
    if (f32) go(F{}, T{});
    else go(F{}, F{});
  }
  SO3_LAUNCH("long_range");
}

// ---------------------------------------------------------------------------
// assembly: forces, per-atom energies, per-atom virial (gathers over the CSR)
// ---------------------------------------------------------------------------
__global__ void k_assemble(int n, int row0, const int *__restrict__ row_start, const int *__restrict__ edge_pair,
                           const double *__restrict__ geo,
                           const double *__restrict__ gv, const double *__restrict__ e_nn,
                           const double *__restrict__ e_lr, const double *__restrict__ f_lr,
                           const double *__restrict__ w_lr, double *__restrict__ force, double *__restrict__ e_atom,
                           double *__restrict__ e_zbl, double *__restrict__ w_atom) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const int a = row0 + r;
  double fx = 0, fy = 0, fz = 0, ez = 0;
  double w[6] = {0, 0, 0, 0, 0, 0};
  for (int e = row_start[r]; e < row_start[r + 1]; ++e) {
    const int code = edge_pair[e];
    const int p = code >= 0 ? code : ~code;
    const double gx = gv[3 * p], gy = gv[3 * p + 1], gz = gv[3 * p + 2];
    const double *gp = geo + (size_t)p * kGeo;
    ez += gp[6];
    if (code >= 0) {
      fx -= gx; fy -= gy; fz -= gz;
    } else {
      fx += gx; fy += gy; fz += gz;
    }
    // per-atom virial: half of the pair's -v (x) dE/dv to each of its two atoms.
    // v and dE/dv are stored in the pair's canonical orientation, so both atoms
    // (on any GPU) add bit-identical halves; the halves of every pair add up to
    // the global virial of pair_so3lr_native_mpi.cpp:944-990
    {
      const double rr = gp[0];
      const double vx = rr * gp[1], vy = rr * gp[2], vz = rr * gp[3];
      w[0] -= 0.5 * (vx * gx);
      w[1] -= 0.5 * (vy * gy);
      w[2] -= 0.5 * (vz * gz);
      w[3] -= 0.25 * (vx * gy + vy * gx);
      w[4] -= 0.25 * (vx * gz + vz * gx);
      w[5] -= 0.25 * (vy * gz + vz * gy);
    }
  }
  force[3 * a] = fx + f_lr[3 * a];
  force[3 * a + 1] = fy + f_lr[3 * a + 1];
  force[3 * a + 2] = fz + f_lr[3 * a + 2];
  e_zbl[a] = ez;
  e_atom[a] = e_nn[a] + ez + e_lr[a];
  for (int k = 0; k < 6; ++k) w_atom[6 * a + k] = w[k] + w_lr[6 * a + k];
}

void launch_assemble(const NeighborState &nb, const double *geo, const double *gv, const double *e_nn,
                     const double *e_lr, const double *f_lr, const double *w_lr, double *force, double *e_atom,
                     double *e_zbl, double *w_atom, cudaStream_t s) {
  const int n = nb.n_own;
  if (n == 0) return;
  k_assemble<<<(n + 127) / 128, 128, 0, s>>>(n, nb.row0, nb.row_start, nb.edge_pair, geo, gv, e_nn,
                                              e_lr, f_lr, w_lr, force, e_atom, e_zbl, w_atom);
  SO3_LAUNCH("assemble");
}


// q = raw + (Q_img - sum_img raw) / N_img (output_heads.cpp:441-451; image_segments.cpp:49-98);
// also the per-image mean of the charge seeds (image_segments.cpp:104-141).
__global__ void k_charge_correct(int n, const double *__restrict__ raw, const double *__restrict__ raw_sum,
                                 const double *__restrict__ qtot, const int *__restrict__ image_of,
                                 const int *__restrict__ image_start, double *__restrict__ q) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int im = image_of[i];
  const double count = double(image_start[im + 1] - image_start[im]);
  q[i] = raw[i] + (qtot[im] - raw_sum[im]) / count;
}
__global__ void k_seed_mean(int nimg, const double *__restrict__ dq_sum, const int *__restrict__ image_start,
                            double *__restrict__ mean) {
  const int im = blockIdx.x * blockDim.x + threadIdx.x;
  if (im >= nimg) return;
  mean[im] = dq_sum[im] / double(image_start[im + 1] - image_start[im]);
}

void launch_charge_correct(int n, const double *raw, const double *raw_sum, const double *qtot,
                           const int *image_of_atom, const int *image_start, double *q, double *dq_mean_out,
                           const double *dq_sum, cudaStream_t s) {
  if (q) {
    k_charge_correct<<<(n + 255) / 256, 256, 0, s>>>(n, raw, raw_sum, qtot, image_of_atom, image_start, q);
    SO3_LAUNCH("charge_correct");
  }
  if (dq_mean_out) {
    // n here is the image count
    k_seed_mean<<<(n + 255) / 256, 256, 0, s>>>(n, dq_sum, image_start, dq_mean_out);
    SO3_LAUNCH("seed_mean");
  }
}

// ---------------------------------------------------------------------------
// velocity Verlet (LAMMPS fix nve, metal units)
// ---------------------------------------------------------------------------
__global__ void k_verlet_first(int n, double *__restrict__ x, double *__restrict__ v, const double *__restrict__ f,
                               const double *__restrict__ inv_mass, double dt, double dtf) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= 3 * n) return;
  const double im = inv_mass[k / 3];
  const double vv = v[k] + dtf * f[k] * im;
  v[k] = vv;
  x[k] += dt * vv;
}
__global__ void k_verlet_second(int n, double *__restrict__ v, const double *__restrict__ f,
                                const double *__restrict__ inv_mass, double dtf) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= 3 * n) return;
  v[k] += dtf * f[k] * inv_mass[k / 3];
}
void launch_verlet_first(int n, double *x, double *v, const double *f, const double *inv_mass, double dt,
                         double ftm2v, cudaStream_t s) {
  k_verlet_first<<<(3 * n + 255) / 256, 256, 0, s>>>(n, x, v, f, inv_mass, dt, 0.5 * dt * ftm2v);
  SO3_LAUNCH("verlet_first");
}
void launch_verlet_second(int n, double *v, const double *f, const double *inv_mass, double dt, double ftm2v,
                          cudaStream_t s) {
  k_verlet_second<<<(3 * n + 255) / 256, 256, 0, s>>>(n, v, f, inv_mass, 0.5 * dt * ftm2v);
  SO3_LAUNCH("verlet_second");
}

}  // namespace so3lr_b200
