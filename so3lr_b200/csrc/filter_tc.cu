// Mixed-precision pair-filter forward on the fifth-generation tensor cores
// (tcgen05, TF32 kind): the same outputs as k_filter_forward_mixed
// (filter_mixed.cu) -- both filters of every pair in float64, float32 silu' of
// the rbf hidden layer for the reverse, d rbf/dr -- with the GEMMs issued as
// tcgen05.mma from shared-memory descriptors into a TMEM accumulator.
//
// Tile: 128 pairs (one TMEM lane per pair). Per tile and filter
//   D1 = rbf W0^T                      (K = 32)   TMEM columns   0..127
//   u  = silu(D1 + b0)                 (epilogue warps, split into TF32 hi/lo)
//   D2 = u W1^T + w V1^T               (K = 128 + 32) columns 128..255
//   f  = D2 + b1 + c1                  (float64 to global)
// with w = silu(L0 V0^T + c0) computed by the epilogue warps. Every product is
// three TF32 MMAs (A_lo B_hi, A_hi B_lo, A_hi B_hi; see filter_mixed.cu).
//
// Warp roles: warps 0-7 build the A operands (rbf, w, u) in shared memory and
// read the accumulators back (warp w owns TMEM lanes 32 (w % 4) .. + 31, i.e.
// its pairs, and column half w / 4 of every 32-column chunk); warp 8 (one
// elected lane) streams the weight K-chunks into a three-slot ring with bulk
// asynchronous copies (cp.async.bulk, this GPU's own global memory, no
// multicast) and issues the MMAs. The hidden layer is handed to the MMA in
// 32-column chunks through a two-slot ring, so the second GEMM starts while
// the epilogue still works on later chunks. All hand-offs are mbarriers; every
// wait gives up after about two seconds, records where in an error word and
// the CTA stops (no spin without a bound).
//
// Weights come pre-split and pre-swizzled (FilterW32::tc_fwd). Shared-memory
// operands use the 128-byte-swizzled K-major layout: a [128 x 32] float tile is
// 16 KB, row n, column k at byte 1024 (n / 8) + 128 (n % 8) + 16 ((k / 4) xor
// (n % 8)) + 4 (k % 4); the descriptor's stride byte offset is 1024 (one 8-row
// group) and each K step of 8 advances its start address by 32 bytes.
//
// The silu' values go to the buffer of the float64 path in a column-major
// per-tile layout (sp_tc_index) that the tcgen05 reverse reads.
#include "filter_common.cuh"
#include "kernels.cuh"

SO3LR_SHAPE_BEGIN
namespace {

constexpr int kTcRows = 128;
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = (kTcEpiWarps + 1) * 32;
constexpr uint32_t kTile = 128 * 32 * 4;  // one [128 x 32] float tile, 16 KB
constexpr int kBSlots = 3;
constexpr uint32_t kOffA1 = 0;                             // rbf: hi, lo
constexpr uint32_t kOffA3 = kOffA1 + 2 * kTile;            // ev hidden w: hi, lo
constexpr uint32_t kOffA2 = kOffA3 + 2 * kTile;            // hidden u chunks: 2 slots x (hi, lo)
constexpr uint32_t kOffB = kOffA2 + 4 * kTile;             // weight chunks: kBSlots x (hi, lo)
constexpr uint32_t kOffBar = kOffB + kBSlots * 2 * kTile;  // mbarriers
constexpr int kNumBars = 16;
constexpr uint32_t kSmemTc = kOffBar + kNumBars * 8 + 16 + 1024;  // + TMEM address + alignment slack
// mbarrier indices
constexpr int kFullB = 0;      // 3: weight chunk landed (transaction bytes)
constexpr int kEmptyB = 3;     // 3: MMAs reading the weight slot done
constexpr int kFullA = 6;      // 2: hidden chunk written (8 epilogue warps)
constexpr int kEmptyA = 8;     // 2: MMAs reading the hidden slot done
constexpr int kOpnd = 10;      // rbf (first filter) and w written (8 warps)
constexpr int kD1Full = 11;    // D1 complete
constexpr int kD2Full = 12;    // D2 complete
constexpr int kD1Free = 13;    // D1 read by every epilogue warp (8)
constexpr int kD2Free = 14;    // D2 read by every epilogue warp (8)
constexpr int kDrain = 15;     // all MMAs of the CTA complete (teardown)
constexpr long long kWaitCycles = 4000000000LL;  // about 2 s at 1.9 GHz

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Wait for the completion of the phase with the given parity, at most
// kWaitCycles; false (and the error word set to `where`) when it gives up or
// when another thread of the CTA already gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag, int *err,
                                          int where) {
  uint32_t done = 0;
  const long long t0 = clock64();
  while (true) {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      atomicCAS(err, 0, where);
      return false;
    }
  }
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte swizzle, 8-row groups 1024 bytes apart (sm100 descriptor)
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3fff) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}
// kind::tf32, D float32, A and B TF32 K-major, M = 128, N = n
constexpr uint32_t idesc_tf32(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(128 >> 4) << 24);
}
constexpr uint32_t kIdesc = idesc_tf32(128);
constexpr uint32_t kIdesc32 = idesc_tf32(32);

__device__ __forceinline__ void mma_tf32_tc(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// D (+)= A B^T over one 32-wide K-chunk in three TF32 passes; A, B: hi tile then lo tile
__device__ __forceinline__ void mma_chunk(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi,
                                          uint32_t b_lo, bool accumulate, uint32_t idesc = kIdesc) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const uint32_t o = 32u * ks;
    mma_tf32_tc(d_tmem, smem_desc(a_lo + o), smem_desc(b_hi + o), idesc, (accumulate || ks > 0) ? 1u : 0u);
    mma_tf32_tc(d_tmem, smem_desc(a_hi + o), smem_desc(b_lo + o), idesc, 1u);
    mma_tf32_tc(d_tmem, smem_desc(a_hi + o), smem_desc(b_hi + o), idesc, 1u);
  }
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// 16 consecutive float32 columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive float32 columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  float a[16], b[16];
  tmem_ld16(taddr, a);
  tmem_ld16(taddr + 16, b);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = a[i];
    v[16 + i] = b[i];
  }
}

__device__ __forceinline__ float tf32_hi(float x) {
  unsigned r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// 16 values of row `row`, columns 16 hh .. + 15 of a [128 x 32] tile pair (hi, lo)
__device__ __forceinline__ void store_row16(char *hi_tile, char *lo_tile, int row, int hh, const float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int chunk = (4 * hh + q) ^ (row & 7);
    const uint32_t off = (row >> 3) * 1024 + (row & 7) * 128 + chunk * 16;
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h[e] = tf32_hi(v[4 * q + e]);
      l[e] = tf32_hi(v[4 * q + e] - h[e]);
    }
    *reinterpret_cast<float4 *>(hi_tile + off) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4 *>(lo_tile + off) = make_float4(l[0], l[1], l[2], l[3]);
  }
}
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// position of silu'(row `row` of 128-pair tile `tile`, column `col`) in the
// tcgen05 kernels' layout: column-major per tile and filter, so a warp's 32
// consecutive rows of one column are one 128-byte line (the mma.sync kernels
// use their own layout, sp_offset; the two kernel pairs do not mix)
__device__ __forceinline__ size_t sp_tc_index(int tile, int filt, int row, int col) {
  return ((size_t(tile) * 2 + filt) * 128 + col) * 128 + row;
}

}  // namespace

// Forward pipeline. Epilogue warps 0-15: warp w owns TMEM lanes 32 (w % 4)
// .. + 31 (its 32 pairs) and columns 8 (w / 4) .. + 7 of every 32-column
// chunk; warp 16 (one lane) loads weights and issues MMAs. The layer-2
// accumulator D2 has two buffers (TMEM columns 128-255 and 256-383), so the
// MMAs of the next (tile, filter) run while the epilogue writes the outputs of
// the current one; the next operands (rbf, w) are built before that.
namespace {
constexpr int kFwdEpiWarps = 16;
constexpr int kFwdThreads = (kFwdEpiWarps + 1) * 32;
constexpr int kFwdBars = 22;
constexpr uint32_t kSmemFwd = kOffBar + kFwdBars * 8 + 16 + 1024;
constexpr int kFFullB = 0, kFEmptyB = 3, kFFullA = 6, kFEmptyA = 8, kFOpnd = 10, kFD1Full = 11, kFD2Full = 12,
              kFD1Free = 14, kFD2Free = 15, kFDrain = 17, kFQuarter = 18;  // kFQuarter + q: 4 warps of row quarter q
// Output staging in the hidden ring, which is free while the outputs are
// written: row quarter q stages its 32 rows x 32 doubles in the bytes that hold
// its own rows of ring slot 0 (rows 0-15 where its rows of the hi tile are,
// rows 16-31 where those of the lo tile are: 4 KB each), so quarters that run
// ahead into the next step never touch another quarter's staging. The 16-byte
// chunks of a 256-byte staging row are swizzled with the row (conflict-free
// 16-byte writes by rows and 8-byte reads along a row).
__device__ __forceinline__ double *stage_at(unsigned char *sm, int q, int r, int col) {
  const uint32_t off = kOffA2 + (r < 16 ? 0u : kTile) + 4096u * q + uint32_t(r & 15) * 256u +
                       uint32_t(((col >> 1) ^ (r & 15)) * 16 + (col & 1) * 8);
  return reinterpret_cast<double *>(sm + off);
}

// 8 consecutive float32 columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// 8 values of row `row`, columns 8 part .. + 7 of a [128 x 32] tile pair (hi, lo)
__device__ __forceinline__ void store_row8(char *hi_tile, char *lo_tile, int row, int part, const float (&v)[8]) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int chunk = (2 * part + q) ^ (row & 7);
    const uint32_t off = (row >> 3) * 1024 + (row & 7) * 128 + chunk * 16;
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h[e] = tf32_hi(v[4 * q + e]);
      l[e] = tf32_hi(v[4 * q + e] - h[e]);
    }
    *reinterpret_cast<float4 *>(hi_tile + off) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4 *>(lo_tile + off) = make_float4(l[0], l[1], l[2], l[3]);
  }
}
}  // namespace

__global__ void __launch_bounds__(kFwdThreads, 1) k_filter_forward_tc(
    int P, int ntiles, const double *__restrict__ geo, const int *__restrict__ pa, const int *__restrict__ pb,
    const double *__restrict__ ev, const __grid_constant__ TcFwdConsts c, FilterW32 finv, FilterW32 fev,
    float *__restrict__ f_inv, float *__restrict__ f_ev, float *__restrict__ sp, double *__restrict__ drbf,
    int *__restrict__ err) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-byte alignment for the swizzled tiles
  unsigned char *sm = smem_raw + (base - raw);
  const uint32_t bars = base + kOffBar;
  auto bar = [&](int i) { return bars + 8u * i; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kOffBar + kFwdBars * 8);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + kOffBar + kFwdBars * 8 + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(bar(kFFullB + i), 1);
    for (int i = 0; i < 3; ++i) mbar_init(bar(kFEmptyB + i), 1);
    for (int i = 0; i < 2; ++i) mbar_init(bar(kFFullA + i), kFwdEpiWarps);
    for (int i = 0; i < 2; ++i) mbar_init(bar(kFEmptyA + i), 1);
    mbar_init(bar(kFOpnd), kFwdEpiWarps);
    mbar_init(bar(kFD1Full), 1);
    for (int i = 0; i < 2; ++i) mbar_init(bar(kFD2Full + i), 1);
    mbar_init(bar(kFD1Free), kFwdEpiWarps);
    for (int i = 0; i < 2; ++i) mbar_init(bar(kFD2Free + i), kFwdEpiWarps);
    mbar_init(bar(kFDrain), 1);
    for (int i = 0; i < 4; ++i) mbar_init(bar(kFQuarter + i), 4);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kFwdEpiWarps) {  // the MMA warp owns the TMEM: D1 (128 columns), two D2 buffers (128 each)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
  const int total_tf = 2 * my_tiles;  // (tile, filter) steps of this CTA

  if (warp == kFwdEpiWarps) {
    // ------------------------------------------------------------------ MMA warp
    if (lane == 0) {
      const int total = total_tf * 6;  // 6 weight chunks (MMA groups) per (tile, filter)
      int next_load = 0, landed = 0;
      bool ok = true;
      for (int g = 0; g < total && ok; ++g) {
        while (ok && next_load < total && next_load <= g + kBSlots - 1) {  // up to kBSlots chunks in flight
          const int s = next_load % kBSlots, n = next_load / kBSlots;
          ok = mbar_wait(bar(kFEmptyB + s), (n & 1) ^ 1, abort_flag, err, 1);
          if (!ok) break;
          const int tf = next_load / 6, gi = next_load % 6;
          const FilterW32 &W = (tf & 1) ? fev : finv;
          mbar_expect_tx(bar(kFFullB + s), 2 * kTile);
          bulk_load(base + kOffB + s * 2 * kTile, W.tc_fwd + size_t(gi) * (2 * kTile / 4), 2 * kTile,
                    bar(kFFullB + s));
          ++next_load;
        }
        if (!ok) break;
        const int tf = g / 6, gi = g % 6, d2b = tf & 1, d2use = tf >> 1;
        const int s = g % kBSlots;
        const uint32_t b_hi = base + kOffB + s * 2 * kTile, b_lo = b_hi + kTile;
        const uint32_t d2 = tmem + 128 + 128 * d2b;
        if (gi == 0) {
          ok = mbar_wait(bar(kFOpnd), tf & 1, abort_flag, err, 2) &&
               mbar_wait(bar(kFD1Free), (tf & 1) ^ 1, abort_flag, err, 3);
        } else if (gi <= 4) {
          const int ch = gi - 1, slot = ch & 1, use = tf * 2 + (ch >> 1);
          ok = mbar_wait(bar(kFFullA + slot), use & 1, abort_flag, err, 4);
          if (ok && ch == 0) ok = mbar_wait(bar(kFD2Free + d2b), (d2use & 1) ^ 1, abort_flag, err, 5);
        }
        if (ok) ok = mbar_wait(bar(kFFullB + s), (g / kBSlots) & 1, abort_flag, err, 6);
        if (!ok) break;
        landed = g + 1;
        tc_fence_after();
        if (gi == 0) {
          mma_chunk(tmem, base + kOffA1, base + kOffA1 + kTile, b_hi, b_lo, false);
          tc_commit(bar(kFEmptyB + s));
          tc_commit(bar(kFD1Full));
        } else if (gi <= 4) {
          const int ch = gi - 1, slot = ch & 1;
          const uint32_t a_hi = base + kOffA2 + slot * 2 * kTile;
          mma_chunk(d2, a_hi, a_hi + kTile, b_hi, b_lo, ch > 0);
          tc_commit(bar(kFEmptyB + s));
          tc_commit(bar(kFEmptyA + slot));
        } else {
          mma_chunk(d2, base + kOffA3, base + kOffA3 + kTile, b_hi, b_lo, true);
          tc_commit(bar(kFEmptyB + s));
          tc_commit(bar(kFD2Full + d2b));
        }
      }
      // teardown: every MMA issued has completed and, after a wait that gave
      // up, every weight copy still in flight has landed (bounded)
      tc_commit(bar(kFDrain));
      mbar_wait(bar(kFDrain), 0, abort_flag, err, 7);
      for (int i = landed; i < next_load; ++i) {
        const long long t0 = clock64();
        uint32_t d = 0;
        while (!d && clock64() - t0 < kWaitCycles)
          asm volatile(
              "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
              " selp.u32 %0, 1, 0, p;\n}\n"
              : "=r"(d)
              : "r"(bar(kFFullB + i % kBSlots)), "r"(uint32_t((i / kBSlots) & 1))
              : "memory");
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int q = warp & 3, part = warp >> 2;
    const int row = 32 * q + lane;
    const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
    double l0[4] = {0, 0, 0, 0};
    // operands of (tile, filter) step tf: rbf into A1 (first filter of a tile), w into A3
    auto prepare = [&](int tf) {
      const int f = tf & 1;
      const int p = (int(blockIdx.x) + (tf >> 1) * int(gridDim.x)) * kTcRows + row;
      const bool valid = p < P;
      if (f == 0) {
        const double r = valid ? geo[(size_t)p * kGeo] : 1.0;
        const double raw_x = exp(-c.gamma * r);
        double x = raw_x;
        if (x < 1.0e-6) x = 1.0e-6;
        if (x > 1.0 - 1.0e-6) x = 1.0 - 1.0e-6;
        const double lx = log(x), l1x = log(1.0 - x);
        const bool live = raw_x > 1.0e-6 && raw_x < 1.0 - 1.0e-6;
        const double ratio = live ? raw_x / (1.0 - raw_x) : 0.0;
        float v[8];
        double d[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k = 8 * part + i;
          const double b = exp_tang(c.rb[k] + c.rk[k] * lx + c.rkr[k] * l1x);
          v[i] = float(b);
          d[i] = live ? b * (-c.gamma * c.rk[k] + c.gamma * c.rkr[k] * ratio) : 0.0;
        }
        store_row8(reinterpret_cast<char *>(sm + kOffA1), reinterpret_cast<char *>(sm + kOffA1 + kTile), row, part,
                   v);
        if (drbf != nullptr && valid) {
          double2 *dst = reinterpret_cast<double2 *>(drbf + (size_t)p * kR + 8 * part);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_double2(d[2 * i], d[2 * i + 1]);
        }
        l0[0] = l0[1] = l0[2] = l0[3] = 0.0;
        if (ev != nullptr && valid) {
          const int a = pa[p], b = pb[p];
#pragma unroll
          for (int m = 0; m < kEV; ++m) {
            const double diff = ev[(size_t)b * kEV + m] - ev[(size_t)a * kEV + m];
            l0[degree_of_channel(m)] += diff * diff * c.cg[m];
          }
        }
      }
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int j = 8 * part + i;
        const float s = float(l0[0]) * c.v0[f][j * 4] + float(l0[1]) * c.v0[f][j * 4 + 1] +
                        float(l0[2]) * c.v0[f][j * 4 + 2] + float(l0[3]) * c.v0[f][j * 4 + 3] + c.c0[f][j];
        v[i] = s * sigmoid_fast(s);
      }
      store_row8(reinterpret_cast<char *>(sm + kOffA3), reinterpret_cast<char *>(sm + kOffA3 + kTile), row, part, v);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kFOpnd));
    };

    bool ok = true;
    int quarter_phase = 0;  // completed phases of this row quarter's staging barrier
    if (total_tf > 0) prepare(0);
    for (int tf = 0; tf < total_tf && ok; ++tf) {
      const int f = tf & 1, d2b = tf & 1, d2use = tf >> 1;
      const int p = (int(blockIdx.x) + (tf >> 1) * int(gridDim.x)) * kTcRows + row;
      const bool valid = p < P;
      float *out = f ? f_ev : f_inv;
      {  // the next tile's per-pair inputs into L2 ahead of its preparation
        const int pn = p + int(gridDim.x) * kTcRows;
        if (pn < P && part == 0) {
          if (f == 0) {
            prefetch_l2(geo + (size_t)pn * kGeo);
            prefetch_l2(pa + pn);
            prefetch_l2(pb + pn);
          } else if (ev != nullptr) {
            const int a = pa[pn], b = pb[pn];
            prefetch_l2(ev + (size_t)a * kEV);
            prefetch_l2(ev + (size_t)a * kEV + 16);
            prefetch_l2(ev + (size_t)b * kEV);
            prefetch_l2(ev + (size_t)b * kEV + 16);
          }
        }
      }
      // hidden layer: D1 + b0 -> silu, in 32-column chunks through the hidden ring
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kFD1Full), tf & 1, abort_flag, err, 8));
      if (!ok) break;
      tc_fence_after();
      for (int ch = 0; ch < 4 && ok; ++ch) {
        const int slot = ch & 1, use = tf * 2 + (ch >> 1);
        ok = __all_sync(0xffffffffu, mbar_wait(bar(kFEmptyA + slot), (use & 1) ^ 1, abort_flag, err, 9));
        if (!ok) break;
        const int col0 = 32 * ch + 8 * part;
        float v[8], u[8];
        tmem_ld8(lane_base + col0, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float x = v[i] + c.b0[f][col0 + i];
          const float sg = sigmoid_fast(x);
          u[i] = x * sg;
          v[i] = sg * (1.0f + x * (1.0f - sg));  // silu'
        }
        char *a_hi = reinterpret_cast<char *>(sm + kOffA2 + slot * 2 * kTile);
        store_row8(a_hi, a_hi + kTile, row, part, u);
        {  // every row of the tile (finite values past P); a warp writes one line per column
          const int tile = p >> 7;
#pragma unroll
          for (int i = 0; i < 8; ++i) sp[sp_tc_index(tile, f, row, col0 + i)] = v[i];
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kFFullA + slot));
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kFD1Free));
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kFD2Full + d2b), d2use & 1, abort_flag, err, 10));
      if (!ok) break;
      tc_fence_after();
      // the next step's operands first (A1 and A3 are free: every MMA of this
      // step has completed), so its MMAs overlap the output writes below
      if (tf + 1 < total_tf) prepare(tf + 1);
      // output: D2 + b1 + c1 in float32, 32 columns at a time through the
      // quarter's staging block, so that each store writes 128 contiguous bytes
      // of one row (8 rows per warp)
      const int tile_row0 = (p >> 7) * kTcRows + 32 * q;  // first pair of this quarter
#pragma unroll 1
      for (int ch = 0; ch < 4 && ok; ++ch) {
        const int col0 = 32 * ch + 8 * part;
        float v[8];
        tmem_ld8(lane_base + 128 + 128 * d2b + col0, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          *reinterpret_cast<double2 *>(stage_at(sm, q, lane, 8 * part + 2 * i)) =
              make_double2(double(v[2 * i] + c.bc1[f][col0 + 2 * i]), double(v[2 * i + 1] + c.bc1[f][col0 + 2 * i + 1]));
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kFQuarter + q));
        ok = __all_sync(0xffffffffu, mbar_wait(bar(kFQuarter + q), quarter_phase & 1, abort_flag, err, 11));
        ++quarter_phase;
        if (!ok) break;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = 8 * part + k, pr = tile_row0 + r;
          if (pr < P) out[(size_t)pr * kF + 32 * ch + lane] = float(*stage_at(sm, q, r, lane));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kFQuarter + q));
        ok = __all_sync(0xffffffffu, mbar_wait(bar(kFQuarter + q), quarter_phase & 1, abort_flag, err, 12));
        ++quarter_phase;
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kFD2Free + d2b));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kFwdEpiWarps) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// Fills the float64 outputs of launch_filter_forward_mixed with the tcgen05
// kernel; err (device int, zeroed by the caller) receives the code of a wait
// that gave up (0: none).
void launch_filter_forward_tc(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                              const TcFwdConsts &consts, const FilterW32 &finv, const FilterW32 &fev, float *f_inv,
                              float *f_ev, float *sp, double *drbf, int *err, int num_sms, cudaStream_t s) {
  if (P == 0) return;
  const int ntiles = (P + kTcRows - 1) / kTcRows;
  allow_dynamic_smem(reinterpret_cast<const void *>(k_filter_forward_tc), kSmemFwd);
  const int grid = std::min(ntiles, std::max(1, num_sms));
  k_filter_forward_tc<<<grid, kFwdThreads, kSmemFwd, s>>>(P, ntiles, geo, pair_a, pair_b, ev, consts, finv, fev,
                                                          f_inv, f_ev, sp, drbf, err);
  SO3_LAUNCH("filter_forward_tc");
}

// ---------------------------------------------------------------------------
// reverse on tcgen05: per tile of 128 pairs and per filter
//   D_h = gF W1      (K = 128, N = 128)   TMEM columns   0..127
//   D_w = gF V1      (K = 128, N = 32)                 128..159
//   g_pre = D_h * silu'      (epilogue, split)
//   D_r (+)= g_pre W0 (K = 128, N = 32)                160..191, summed over both filters
// then, per pair, the radial gradient sum_k g_rbf[k] d rbf_k/dr + the cutoff
// term, the harmonic gradient and the L0 gradient, as k_filter_reverse_mixed
// finishes a pair (the L0 part g_pe = (gF V1) * silu'(L0 V0^T + c0) in float64).
// Both filters are handled by one CTA, so the radial-basis gradient of the two
// is summed in the TMEM accumulator instead of across a CTA pair.
// Weight chunks (FilterW32::tc_rev): for k-chunk c = 0..3 a 40 KB group
// [W1^T chunk hi | lo (16 KB each)][V1^T chunk hi | lo (4 KB each)], then for
// c = 0..3 an 8 KB group [W0^T chunk hi | lo (4 KB each)].
// ---------------------------------------------------------------------------
namespace {
constexpr uint32_t kTile32 = 32 * 32 * 4;            // one [32 x 32] float tile, 4 KB
constexpr uint32_t kGrpE12 = 2 * kTile + 2 * kTile32;  // 40 KB
constexpr uint32_t kGrpE3 = 2 * kTile32;              // 8 KB
constexpr int kRevEpiWarps = 16;                      // 4 per TMEM lane quarter, 8 columns of each chunk
constexpr int kRevThreads = (kRevEpiWarps + 1) * 32;
constexpr uint32_t kRevOffA = 0;                      // 2 slots x (hi, lo) of [128 x 32]
constexpr uint32_t kRevOffB = kRevOffA + 4 * kTile;   // kBSlots x 40 KB
constexpr uint32_t kRevRed = kRevOffB + kBSlots * kGrpE12;  // 2 x [4 parts][128 rows][5] doubles
constexpr uint32_t kRevRedBytes = 4 * 128 * 5 * 8;
constexpr uint32_t kRevOffBar = kRevRed + 2 * kRevRedBytes;
constexpr int kRevBars = 19;
constexpr uint32_t kSmemTcRev = kRevOffBar + kRevBars * 8 + 16 + 1024;
constexpr int kRFullB = 0, kREmptyB = 3, kRFullA = 6, kREmptyA = 8, kRDhwFull = 10, kRDhwFree = 11, kRDrFull = 12,
              kRDrFree = 13, kRDrain = 14, kRRed = 15;  // kRRed + q: the 4 warps of row quarter q
}  // namespace

__global__ void __launch_bounds__(kRevThreads, 1) k_filter_reverse_tc(
    int P, int ntiles, const double *__restrict__ geo, const int *__restrict__ pa, const int *__restrict__ pb,
    const double *__restrict__ ev, const __grid_constant__ TcRevConsts c, FilterW32 finv32,
    FilterW32 fev32, const float *__restrict__ g_filt_inv, const float *__restrict__ g_filt_ev,
    const float *__restrict__ sp, const double *__restrict__ drbf, const double *__restrict__ gA,
    const double *__restrict__ pair_sc, int need_l0, int accumulate, double *__restrict__ g_r,
    double *__restrict__ g_y, double *__restrict__ gl0, int *__restrict__ err) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char *sm = smem_raw + (base - raw);
  const uint32_t bars = base + kRevOffBar;
  auto bar = [&](int i) { return bars + 8u * i; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kRevOffBar + kRevBars * 8);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + kRevOffBar + kRevBars * 8 + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(bar(kRFullB + i), 1);
    for (int i = 0; i < 3; ++i) mbar_init(bar(kREmptyB + i), 1);
    for (int i = 0; i < 2; ++i) mbar_init(bar(kRFullA + i), kRevEpiWarps);
    for (int i = 0; i < 2; ++i) mbar_init(bar(kREmptyA + i), 1);
    mbar_init(bar(kRDhwFull), 1);
    mbar_init(bar(kRDhwFree), kRevEpiWarps);
    mbar_init(bar(kRDrFull), 1);
    mbar_init(bar(kRDrFree), kRevEpiWarps);
    mbar_init(bar(kRDrain), 1);
    for (int i = 0; i < 4; ++i) mbar_init(bar(kRRed + i), 4);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kRevEpiWarps) {  // D_h, D_w, D_r: 192 of 256 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;

  if (warp == kRevEpiWarps) {
    // ------------------------------------------------------------------ MMA warp
    if (lane == 0) {
      const int total = my_tiles * 16;  // per tile and filter: 4 (gF W1, gF V1) groups, 4 (g_pre W0) groups
      int next_load = 0, landed = 0;
      bool ok = true;
      for (int g = 0; g < total && ok; ++g) {
        while (ok && next_load < total && next_load <= g + kBSlots - 1) {
          const int s = next_load % kBSlots, n = next_load / kBSlots;
          ok = mbar_wait(bar(kREmptyB + s), (n & 1) ^ 1, abort_flag, err, 21);
          if (!ok) break;
          const int tf = next_load / 8, gi = next_load % 8;
          const FilterW32 &W = (tf & 1) ? fev32 : finv32;
          const uint32_t bytes = gi < 4 ? kGrpE12 : kGrpE3;
          const size_t off = gi < 4 ? size_t(gi) * kGrpE12 : 4 * size_t(kGrpE12) + size_t(gi - 4) * kGrpE3;
          mbar_expect_tx(bar(kRFullB + s), bytes);
          bulk_load(base + kRevOffB + s * kGrpE12, reinterpret_cast<const char *>(W.tc_rev) + off, bytes,
                    bar(kRFullB + s));
          ++next_load;
        }
        if (!ok) break;
        const int tf = g / 8, gi = g % 8, it = tf >> 1, f = tf & 1;
        const int s = g % kBSlots;
        const int use = tf * 8 + gi, slot = use & 1;  // A-ring use: gF chunks 0-3, then g_pre chunks 0-3
        const uint32_t b0 = base + kRevOffB + s * kGrpE12;
        ok = mbar_wait(bar(kRFullA + slot), (use >> 1) & 1, abort_flag, err, 22);
        if (ok && gi == 0) ok = mbar_wait(bar(kRDhwFree), (tf & 1) ^ 1, abort_flag, err, 23);
        if (ok && gi == 4 && f == 0) ok = mbar_wait(bar(kRDrFree), (it & 1) ^ 1, abort_flag, err, 24);
        if (ok) ok = mbar_wait(bar(kRFullB + s), (g / kBSlots) & 1, abort_flag, err, 25);
        if (!ok) break;
        landed = g + 1;
        tc_fence_after();
        const uint32_t a_hi = base + kRevOffA + slot * 2 * kTile, a_lo = a_hi + kTile;
        if (gi < 4) {
          mma_chunk(tmem, a_hi, a_lo, b0, b0 + kTile, gi > 0);
          mma_chunk(tmem + 128, a_hi, a_lo, b0 + 2 * kTile, b0 + 2 * kTile + kTile32, gi > 0, kIdesc32);
          tc_commit(bar(kREmptyB + s));
          tc_commit(bar(kREmptyA + slot));
          if (gi == 3) tc_commit(bar(kRDhwFull));
        } else {
          mma_chunk(tmem + 160, a_hi, a_lo, b0, b0 + kTile32, !(f == 0 && gi == 4), kIdesc32);
          tc_commit(bar(kREmptyB + s));
          tc_commit(bar(kREmptyA + slot));
          if (f == 1 && gi == 7) tc_commit(bar(kRDrFull));
        }
      }
      tc_commit(bar(kRDrain));
      mbar_wait(bar(kRDrain), 0, abort_flag, err, 27);
      for (int i = landed; i < next_load; ++i) {
        const long long t0 = clock64();
        uint32_t d = 0;
        while (!d && clock64() - t0 < kWaitCycles)
          asm volatile(
              "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
              " selp.u32 %0, 1, 0, p;\n}\n"
              : "=r"(d)
              : "r"(bar(kRFullB + i % kBSlots)), "r"(uint32_t((i / kBSlots) & 1))
              : "memory");
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue warps
    // warp w: TMEM lanes 32 (w % 4) .. + 31 (its 32 pairs), columns
    // 8 (w / 4) .. + 7 of every 32-column chunk
    const int q = warp & 3, part = warp >> 2;
    const int row = 32 * q + lane;
    const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
    bool ok = true;
    // this thread's inputs of the tile holding pair pp into L2: its 8-column
    // slices of both filter gradients and of silu' (one 64- or 32-byte run per
    // chunk), its radial-basis derivatives, the pair scalars and geometry
    auto prefetch_tile = [&](int pp) {
      // the filter gradients of the 8 rows this warp loads (512 B per row and
      // filter; lane: row 8 warp + lane / 4, line lane % 4)
      const int pg = pp - row + 8 * warp + (lane >> 2);
      if (pg < P)
        for (int f = 0; f < 2; ++f)
          prefetch_l2(reinterpret_cast<const char *>((f ? g_filt_ev : g_filt_inv) + (size_t)pg * kF) + 128 * (lane & 3));
      if (pp >= P) return;
      prefetch_l2(drbf + (size_t)pp * kR + 8 * part);
      if (part == 0) {
        prefetch_l2(pair_sc + (size_t)pp * kPairScalars);
        prefetch_l2(geo + (size_t)pp * kGeo);
        prefetch_l2(pa + pp);
        prefetch_l2(pb + pp);
      }
    };
    if (my_tiles > 0) prefetch_tile(int(blockIdx.x) * kTcRows + row);
    for (int it = 0; it < my_tiles && ok; ++it) {
      const int tile = int(blockIdx.x) + it * int(gridDim.x);
      const int p = tile * kTcRows + row;
      const bool valid = p < P;
      if (it + 1 < my_tiles) prefetch_tile(p + int(gridDim.x) * kTcRows);
      double l0[4] = {0, 0, 0, 0}, gl[4] = {0, 0, 0, 0};
      if (need_l0 && valid) {
        const int a = pa[p], b = pb[p];
#pragma unroll
        for (int m = 0; m < kEV; ++m) {
          const double diff = ev[(size_t)b * kEV + m] - ev[(size_t)a * kEV + m];
          l0[degree_of_channel(m)] += diff * diff * c.cg[m];
        }
      }
      for (int f = 0; f < 2 && ok; ++f) {
        const int tf = it * 2 + f;
        const float *gsrc = f ? g_filt_ev : g_filt_inv;
        // the filter gradient (float32) into the A ring, 32 columns at a time.
        // The loads need not follow the TMEM rows: warp w loads rows 8 w ..
        // 8 w + 7 of the chunk, two whole 128-byte row segments per instruction
        // (16 lanes per row, two columns per lane), and writes them to the
        // swizzled A tile
        for (int ch = 0; ch < 4 && ok; ++ch) {
          const int use = tf * 8 + ch, slot = use & 1;
          const int k = 2 * (lane & 15);  // column within the chunk
          float2 v2[4];                   // loaded before the wait for the ring slot
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = 8 * warp + 2 * i + (lane >> 4);
            const int pr = tile * kTcRows + r;
            v2[i] = make_float2(0.0f, 0.0f);
            if (pr < P) v2[i] = __ldg(reinterpret_cast<const float2 *>(gsrc + (size_t)pr * kF + 32 * ch + k));
          }
          ok = __all_sync(0xffffffffu, mbar_wait(bar(kREmptyA + slot), ((use >> 1) & 1) ^ 1, abort_flag, err, 28));
          if (!ok) break;
          char *a_hi = reinterpret_cast<char *>(sm + kRevOffA + slot * 2 * kTile);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = 8 * warp + 2 * i + (lane >> 4);
            const uint32_t off = (r >> 3) * 1024 + (r & 7) * 128 + (((k >> 2) ^ (r & 7)) * 16) + (k & 3) * 4;
            const float h0 = tf32_hi(v2[i].x), h1 = tf32_hi(v2[i].y);
            *reinterpret_cast<float2 *>(a_hi + off) = make_float2(h0, h1);
            *reinterpret_cast<float2 *>(a_hi + kTile + off) =
                make_float2(tf32_hi(v2[i].x - h0), tf32_hi(v2[i].y - h1));
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kRFullA + slot));
        }
        if (!ok) break;
        ok = __all_sync(0xffffffffu, mbar_wait(bar(kRDhwFull), tf & 1, abort_flag, err, 29));
        if (!ok) break;
        tc_fence_after();
        if (need_l0) {  // this part's 8 units of the L0 gradient (float64, as the float64 path)
          float gw[8];
          tmem_ld8(lane_base + 128 + 8 * part, gw);
          const double *v0 = c.v0[f];
          const double *c0 = c.c0[f];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int j = 8 * part + i;
            const double pe = l0[0] * v0[j * 4] + l0[1] * v0[j * 4 + 1] + l0[2] * v0[j * 4 + 2] +
                              l0[3] * v0[j * 4 + 3] + c0[j];
            const double gpe = double(gw[i]) * silu_prime(pe);
#pragma unroll
            for (int d = 0; d < 4; ++d) gl[d] += gpe * v0[j * 4 + d];
          }
        }
        // hidden pre-activation gradient g_pre = D_h * silu' into the A ring
        for (int ch = 0; ch < 4 && ok; ++ch) {
          const int use = tf * 8 + 4 + ch, slot = use & 1;
          const int col0 = 32 * ch + 8 * part;
          float sv[8];  // silu', loaded before the waits (one line per column and warp)
#pragma unroll
          for (int i = 0; i < 8; ++i) sv[i] = __ldg(sp + sp_tc_index(tile, f, row, col0 + i));
          ok = __all_sync(0xffffffffu, mbar_wait(bar(kREmptyA + slot), ((use >> 1) & 1) ^ 1, abort_flag, err, 30));
          if (!ok) break;
          float v[8];
          tmem_ld8(lane_base + col0, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] *= sv[i];
          char *a_hi = reinterpret_cast<char *>(sm + kRevOffA + slot * 2 * kTile);
          store_row8(a_hi, a_hi + kTile, row, part, v);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kRFullA + slot));
        }
        if (!ok) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kRDhwFree));
      }
      if (!ok) break;
      // finish the pairs: radial, cutoff, harmonic and L0 gradients
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kRDrFull), it & 1, abort_flag, err, 31));
      if (!ok) break;
      tc_fence_after();
      float grb[8];
      tmem_ld8(lane_base + 160 + 8 * part, grb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kRDrFree));
      // partial sums of the four parts of a row meet in shared memory (a
      // buffer per tile parity; an mbarrier of the row quarter's 4 warps)
      double *red = reinterpret_cast<double *>(sm + kRevRed + (it & 1) * kRevRedBytes);
      {
        double gr = 0.0;
        if (valid) {
          const double *dr = drbf + (size_t)p * kR + 8 * part;
#pragma unroll
          for (int i = 0; i < 8; ++i) gr += double(grb[i]) * dr[i];
        }
        double *mine = red + (size_t(part) * 128 + row) * 5;
        mine[0] = gr;
        for (int d = 0; d < 4; ++d) mine[1 + d] = gl[d];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kRRed + q));
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kRRed + q), it & 1, abort_flag, err, 32));
      if (!ok) break;
      if (valid) {
        const double *sc = pair_sc + (size_t)p * kPairScalars;
        const double dphi = geo[(size_t)p * kGeo + 5], phi = geo[(size_t)p * kGeo + 4];
        if (part == 0) {
          double gr = 0.0, gsum[4] = {0, 0, 0, 0};
          for (int k = 0; k < 4; ++k) {  // the parts in a fixed order
            const double *o = red + (size_t(k) * 128 + row) * 5;
            gr += o[0];
            for (int d = 0; d < 4; ++d) gsum[d] += o[1 + d];
          }
          gr += __dmul_rn(sc[0], dphi);  // cutoff gradient (its weight is orientation-independent)
          g_r[p] = accumulate ? g_r[p] + gr : gr;
          if (need_l0)
            for (int d = 0; d < 4; ++d) gl0[(size_t)p * 4 + d] = gsum[d];
        }
        const int a = pa[p], b = pb[p];
        for (int m = 6 * part; m < 6 * part + 6; ++m) {
          const int d = degree_of_channel(m);
          const double y = __dmul_rn(phi, __dadd_rn(__dmul_rn(sc[1 + d], gA[(size_t)a * kEV + m]),
                                                    parity_sign(d) * __dmul_rn(sc[5 + d], gA[(size_t)b * kEV + m])));
          double *dst = g_y + (size_t)p * kEV + m;
          *dst = accumulate ? *dst + y : y;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kRevEpiWarps) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
  }
}

void launch_filter_reverse_tc(int P, const double *geo, const int *pair_a, const int *pair_b, const double *ev,
                              const TcRevConsts &consts, const FilterW32 &finv32, const FilterW32 &fev32,
                              const float *g_filt_inv, const float *g_filt_ev,
                              const float *sp, const double *drbf, const double *gA, const double *pair_sc,
                              bool need_l0, bool accumulate, double *g_r, double *g_y, double *gl0, int *err,
                              int num_sms, cudaStream_t s) {
  if (P == 0) return;
  const int ntiles = (P + kTcRows - 1) / kTcRows;
  allow_dynamic_smem(reinterpret_cast<const void *>(k_filter_reverse_tc), kSmemTcRev);
  const int grid = std::min(ntiles, std::max(1, num_sms));
  k_filter_reverse_tc<<<grid, kRevThreads, kSmemTcRev, s>>>(P, ntiles, geo, pair_a, pair_b, ev, consts,
                                                           finv32, fev32, g_filt_inv, g_filt_ev, sp, drbf, gA,
                                                           pair_sc, need_l0 ? 1 : 0, accumulate ? 1 : 0, g_r, g_y,
                                                           gl0, err);
  SO3_LAUNCH("filter_reverse_tc");
}

SO3LR_SHAPE_END
