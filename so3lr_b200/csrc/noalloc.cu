// Long-range (Coulomb + dispersion) evaluation of an open-boundary system that
// allocates no device memory.
//
// Who needs it: host programs that own the whole device-memory budget and hand
// a library only the buffers it must fill, and that therefore cannot let the
// library call cudaMalloc/cudaFree on its own once a run has started -- for
// example an MD engine whose device memory comes from its own pool or arena,
// or a coupling loop that must not touch the driver allocator between steps.
// Such a caller passes its input and output buffers; the scratch this kernel
// needs (the cell-ordered copy of every atom's position, charge, Hirshfeld
// ratio and reference polarisability/C6, and the one-image offsets) lives in the
// fixed-size arrays below instead of in memory the library would allocate.
//
// The arrays are ordinary file-scope device variables: every GPU that loads this
// library holds them (about 1 MiB) until the process exits. Calls that use them
// share them, so two calls that overlap on the GPU (on different streams, or on
// different host threads) race on this scratch and must be serialised by the
// caller. Each call overwrites every scratch element it reads before reading it,
// so no clearing between calls is needed. The scratch addresses are resolved
// once per device and kept for the life of the process, so the entry point must
// not be used after a reset of the device's primary context (cudaDeviceReset).
#include <mutex>

#include "kernels.cuh"
#include "model_host.hpp"

namespace so3lr_b200 {

constexpr int kNoAllocMaxAtoms = 16384;

// scratch: pos4[N] and par4[N] as double4 (8 doubles per atom)
static __device__ __align__(256) double g_lr_partner_scratch[8 * kNoAllocMaxAtoms];
// scratch: image_of[N] (all zero: one image) and image_start[2] = {0, N}
static __device__ __align__(256) int g_lr_image_scratch[kNoAllocMaxAtoms + 2];

namespace {

__global__ void k_single_image(int n, int *__restrict__ image_of, int *__restrict__ image_start) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) image_of[i] = 0;
  if (i == 0) {
    image_start[0] = 0;
    image_start[1] = n;
  }
}

struct Scratch {
  double *partners = nullptr;
  int *images = nullptr;
};

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
Scratch g_scratch[kMaxDevices];

// Device addresses of the scratch arrays for the current device, resolved once
// per device with that device current. In host code the array names are
// host-side stand-ins, never device addresses.
Scratch scratch_for_current_device() {
  int dev = 0;
  SO3_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) throw Error("SO3LR no-alloc long range: device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  Scratch &s = g_scratch[dev];
  if (s.partners == nullptr) {
    void *p = nullptr, *q = nullptr;
    const cudaError_t e1 = cudaGetSymbolAddress(&p, g_lr_partner_scratch);
    if (e1 != cudaSuccess)
      throw Error(std::string("SO3LR no-alloc long range: cudaGetSymbolAddress(partner scratch) failed: ") +
                  cudaGetErrorString(e1));
    const cudaError_t e2 = cudaGetSymbolAddress(&q, g_lr_image_scratch);
    if (e2 != cudaSuccess)
      throw Error(std::string("SO3LR no-alloc long range: cudaGetSymbolAddress(image scratch) failed: ") +
                  cudaGetErrorString(e2));
    s.images = static_cast<int *>(q);
    s.partners = static_cast<double *>(p);
  }
  return s;
}

}  // namespace

int noalloc_max_atoms() { return kNoAllocMaxAtoms; }

// Same kernels and arithmetic as the long-range step of the full evaluation,
// with open boundaries and all scratch in the arrays above.
void long_range_noalloc(int n, const double *x, const double *q, const double *h, const int *z,
                        const double *alpha_ref, const double *c6_ref, int table_size, const LrDev &p, double rc_lr,
                        double *e_lr, double *e_elec, double *e_disp, double *dq, double *dh, double *f,
                        double *w_atom, cudaStream_t s) {
  if (n <= 0) throw Error("SO3LR no-alloc long range: the system has no atoms");
  if (n > kNoAllocMaxAtoms)
    throw Error("SO3LR no-alloc long range: " + std::to_string(n) + " atoms exceed the fixed scratch of " +
                std::to_string(kNoAllocMaxAtoms) + " atoms; use the allocating entry points for larger systems");
  const Scratch sc = scratch_for_current_device();
  k_single_image<<<(n + 255) / 256, 256, 0, s>>>(n, sc.images, sc.images + kNoAllocMaxAtoms);
  SO3_LAUNCH("noalloc_single_image");
  NeighborState nb{};
  nb.grid.periodic = 0;
  nb.xw = const_cast<double *>(x);  // read only
  nb.image_of = sc.images;
  nb.image_start = sc.images + kNoAllocMaxAtoms;
  double4 *pos4 = reinterpret_cast<double4 *>(sc.partners);
  double4 *par4 = pos4 + kNoAllocMaxAtoms;
  nb.row0 = 0;
  nb.n_own = n;
  launch_long_range(n, n, nb, rc_lr, z, q, h, nullptr, alpha_ref, c6_ref, table_size, p, pos4, par4, e_lr, e_elec,
                    e_disp, dq, dh, nullptr, f, w_atom, s);
}

}  // namespace so3lr_b200
