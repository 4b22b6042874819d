// Real spherical harmonics l = 1..4 of a unit vector (24 channels, ordered
// m = -l..l within each degree) and the vector-Jacobian product of the same
// polynomials with respect to the unit vector's components.
//
// Same normalisation and channel order as the reference
// (src/kokkos_learned_energy_forces.cpp:14-63); the VJP differentiates each
// polynomial as written (treating x, y, z as independent), and the caller
// projects out the radial part, as learned_energy_forces.cpp:259-305 does.
#pragma once

namespace so3lr_b200 {

struct ShConst {
  double c1, a2, b2, c2, a3, b3, c3, d3, e3, a4, b4, c4, d4, e4, f4, g4;
};

__host__ __device__ inline ShConst sh_constants() {
  constexpr double pi = 3.141592653589793238462643383279502884;
  ShConst k;
  k.c1 = sqrt(3.0 / (4.0 * pi));
  k.a2 = 0.5 * sqrt(15.0 / pi);
  k.b2 = 0.25 * sqrt(5.0 / pi);
  k.c2 = 0.25 * sqrt(15.0 / pi);
  k.a3 = 0.25 * sqrt(35.0 / (2.0 * pi));
  k.b3 = 0.5 * sqrt(105.0 / pi);
  k.c3 = 0.25 * sqrt(21.0 / (2.0 * pi));
  k.d3 = 0.25 * sqrt(7.0 / pi);
  k.e3 = 0.25 * sqrt(105.0 / pi);
  k.a4 = 0.75 * sqrt(35.0 / pi);
  k.b4 = 0.75 * sqrt(35.0 / (2.0 * pi));
  k.c4 = 0.75 * sqrt(5.0 / pi);
  k.d4 = 0.75 * sqrt(5.0 / (2.0 * pi));
  k.e4 = 0.1875 * sqrt(1.0 / pi);
  k.f4 = 0.375 * sqrt(5.0 / pi);
  k.g4 = 0.1875 * sqrt(35.0 / pi);
  return k;
}

__device__ inline void real_sh(double x, double y, double z, double *o) {
  const ShConst k = sh_constants();
  const double xx = x * x, yy = y * y, zz = z * z;
  o[0] = k.c1 * y;
  o[1] = k.c1 * z;
  o[2] = k.c1 * x;
  o[3] = k.a2 * x * y;
  o[4] = k.a2 * y * z;
  o[5] = k.b2 * (3.0 * zz - 1.0);
  o[6] = k.a2 * x * z;
  o[7] = k.c2 * (xx - yy);
  o[8] = k.a3 * y * (3.0 * xx - yy);
  o[9] = k.b3 * x * y * z;
  o[10] = k.c3 * y * (5.0 * zz - 1.0);
  o[11] = k.d3 * (5.0 * zz * z - 3.0 * z);
  o[12] = k.c3 * x * (5.0 * zz - 1.0);
  o[13] = k.e3 * (xx - yy) * z;
  o[14] = k.a3 * x * (xx - 3.0 * yy);
  o[15] = k.a4 * x * y * (xx - yy);
  o[16] = k.b4 * y * (3.0 * xx - yy) * z;
  o[17] = k.c4 * x * y * (7.0 * zz - 1.0);
  o[18] = k.d4 * y * (7.0 * zz * z - 3.0 * z);
  o[19] = k.e4 * (35.0 * zz * zz - 30.0 * zz + 3.0);
  o[20] = k.d4 * x * (7.0 * zz * z - 3.0 * z);
  o[21] = k.f4 * (xx - yy) * (7.0 * zz - 1.0);
  o[22] = k.b4 * x * (xx - 3.0 * yy) * z;
  o[23] = k.g4 * (xx * (xx - 3.0 * yy) - yy * (3.0 * xx - yy));
}

// d/d(x,y,z) of sum_m g[m] * Y_m(x, y, z)
__device__ inline void real_sh_vjp(double x, double y, double z, const double *g, double &gx, double &gy,
                                   double &gz) {
  const ShConst k = sh_constants();
  const double xx = x * x, yy = y * y, zz = z * z;
  double ax = 0.0, ay = 0.0, az = 0.0;
  // l = 1
  ay += g[0] * k.c1;
  az += g[1] * k.c1;
  ax += g[2] * k.c1;
  // l = 2
  ax += g[3] * k.a2 * y;  ay += g[3] * k.a2 * x;
  ay += g[4] * k.a2 * z;  az += g[4] * k.a2 * y;
  az += g[5] * 6.0 * k.b2 * z;
  ax += g[6] * k.a2 * z;  az += g[6] * k.a2 * x;
  ax += g[7] * 2.0 * k.c2 * x;  ay -= g[7] * 2.0 * k.c2 * y;
  // l = 3
  ax += g[8] * 6.0 * k.a3 * x * y;  ay += g[8] * 3.0 * k.a3 * (xx - yy);
  ax += g[9] * k.b3 * y * z;  ay += g[9] * k.b3 * x * z;  az += g[9] * k.b3 * x * y;
  ay += g[10] * k.c3 * (5.0 * zz - 1.0);  az += g[10] * 10.0 * k.c3 * y * z;
  az += g[11] * k.d3 * (15.0 * zz - 3.0);
  ax += g[12] * k.c3 * (5.0 * zz - 1.0);  az += g[12] * 10.0 * k.c3 * x * z;
  ax += g[13] * 2.0 * k.e3 * x * z;  ay -= g[13] * 2.0 * k.e3 * y * z;  az += g[13] * k.e3 * (xx - yy);
  ax += g[14] * 3.0 * k.a3 * (xx - yy);  ay -= g[14] * 6.0 * k.a3 * x * y;
  // l = 4
  ax += g[15] * k.a4 * y * (3.0 * xx - yy);  ay += g[15] * k.a4 * x * (xx - 3.0 * yy);
  ax += g[16] * 6.0 * k.b4 * x * y * z;  ay += g[16] * 3.0 * k.b4 * (xx - yy) * z;
  az += g[16] * k.b4 * y * (3.0 * xx - yy);
  ax += g[17] * k.c4 * y * (7.0 * zz - 1.0);  ay += g[17] * k.c4 * x * (7.0 * zz - 1.0);
  az += g[17] * 14.0 * k.c4 * x * y * z;
  ay += g[18] * k.d4 * (7.0 * zz * z - 3.0 * z);  az += g[18] * k.d4 * y * (21.0 * zz - 3.0);
  az += g[19] * k.e4 * (140.0 * zz * z - 60.0 * z);
  ax += g[20] * k.d4 * (7.0 * zz * z - 3.0 * z);  az += g[20] * k.d4 * x * (21.0 * zz - 3.0);
  ax += g[21] * 2.0 * k.f4 * x * (7.0 * zz - 1.0);  ay -= g[21] * 2.0 * k.f4 * y * (7.0 * zz - 1.0);
  az += g[21] * 14.0 * k.f4 * z * (xx - yy);
  ax += g[22] * 3.0 * k.b4 * (xx - yy) * z;  ay -= g[22] * 6.0 * k.b4 * x * y * z;
  az += g[22] * k.b4 * x * (xx - 3.0 * yy);
  ax += g[23] * 4.0 * k.g4 * x * (xx - 3.0 * yy);  ay += g[23] * 4.0 * k.g4 * y * (yy - 3.0 * xx);
  gx = ax;
  gy = ay;
  gz = az;
}

}  // namespace so3lr_b200
