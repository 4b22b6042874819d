// Nose-Hoover chain thermostat for the device-resident MD harness (NVT runs of
// the multi-GPU benchmark workload).
//
// The reference leaves integration to LAMMPS (fix nvt). This is the published
// Nose-Hoover chain of Martyna, Tuckerman and Klein (Mol. Phys. 87, 1117
// (1996)) with the Trotter splitting of its thermostat propagator: a half step
// of the chain before and after each velocity-Verlet step. Chain masses
// Q_1 = N_f kT tau^2 and Q_j = kT tau^2 (j > 1), N_f = 3N - 3. The kinetic
// energy entering the chain is an exact fixed-point sum, and every GPU updates
// the chain with the same single-thread kernel, so the velocity scale factor is
// bit-identical on every rank.
#include "kernels.cuh"

namespace so3lr_b200 {
namespace {

// 2K per owned row (eV): m v^2 mvv2e
__global__ void k_two_ke(int n, const double *__restrict__ v, const double *__restrict__ mass, double mvv2e,
                         double *__restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double vx = v[3 * i], vy = v[3 * i + 1], vz = v[3 * i + 2];
  out[i] = mass[i] * (vx * vx + vy * vy + vz * vz) * mvv2e;
}

__device__ inline double chain_force(const NhcState &s, const double *ve, double two_k, int j) {
  if (j == 0) return (two_k - s.ndof * s.kt) / s.q[0];
  return (s.q[j - 1] * ve[j - 1] * ve[j - 1] - s.kt) / s.q[j];
}

// One half step (dt / 2) of the chain for kinetic energy *two_k; writes the
// velocity scale factor to *scale.
__global__ void k_nhc_half(NhcState *__restrict__ st, const double *__restrict__ two_k_in, double dt,
                           double *__restrict__ scale) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  NhcState &s = *st;
  const int m = s.chain;
  double *ve = s.veta;
  double two_k = *two_k_in;
  const double d2 = 0.5 * dt, d4 = 0.25 * dt, d8 = 0.125 * dt;
  // thermostat velocities from the end of the chain down to the particles
  ve[m - 1] += d4 * chain_force(s, ve, two_k, m - 1);
  for (int j = m - 2; j >= 0; --j) {
    const double f = exp(-d8 * ve[j + 1]);
    ve[j] = (ve[j] * f + d4 * chain_force(s, ve, two_k, j)) * f;
  }
  const double sc = exp(-d2 * ve[0]);
  two_k *= sc * sc;
  for (int j = 0; j < m; ++j) s.eta[j] += d2 * ve[j];
  // and back up
  for (int j = 0; j < m - 1; ++j) {
    const double f = exp(-d8 * ve[j + 1]);
    ve[j] = (ve[j] * f + d4 * chain_force(s, ve, two_k, j)) * f;
  }
  ve[m - 1] += d4 * chain_force(s, ve, two_k, m - 1);
  *scale = sc;
}

__global__ void k_scale_v(int n, double *__restrict__ v, const double *__restrict__ scale) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k < 3 * n) v[k] *= *scale;
}

}  // namespace

void launch_two_ke(int n, const double *v, const double *mass, double mvv2e, double *out, cudaStream_t s) {
  if (n == 0) return;
  k_two_ke<<<(n + 255) / 256, 256, 0, s>>>(n, v, mass, mvv2e, out);
  SO3_LAUNCH("two_ke");
}

void launch_nhc_half(NhcState *st, const double *two_k, double dt, double *scale, cudaStream_t s) {
  k_nhc_half<<<1, 32, 0, s>>>(st, two_k, dt, scale);
  SO3_LAUNCH("nhc_half");
}

void launch_scale_v(int n, double *v, const double *scale, cudaStream_t s) {
  if (n == 0) return;
  k_scale_v<<<(3 * n + 255) / 256, 256, 0, s>>>(n, v, scale);
  SO3_LAUNCH("scale_v");
}

}  // namespace so3lr_b200
