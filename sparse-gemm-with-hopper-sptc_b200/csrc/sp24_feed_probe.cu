// sp24_feed_probe.cu — shared-memory feed probe (measurement only, built into
// bin/sp24_feed_probe; not part of the sp24 C ABI).
//
// What it measures: how fast one CTA per SM can keep a TMA-fed shared-memory
// ring full when its consumer holds every slot for a fixed number of cycles,
// the way the GEMM kernels' MMAs hold a stage until they complete.  The ring
// has the GEMM kernels' shape: slots of three SW128 boxes of 64 16-bit
// columns, a producer warp whose lanes issue one box each after waiting for
// the slot and arming its full barrier, and a consumer warp that waits for
// the slot, spins `hold` cycles and releases it.  Each case prints the
// sustained fill rate and, per slot, where the two warps spend their cycles.
//
//   L2 cases:  a 48 MB buffer that stays in L2; CTA i starts at box 7 i.
//   HBM cases: a 4 GB buffer streamed once, each CTA over its own range, with
//              a varying number of CTAs (one per SM).
//
// Every wait is bounded (sp24_ptx.cuh); a timeout sets the error flag that
// the host checks after each launch.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <vector>

#include "sp24_ptx.cuh"

namespace sp24 {
namespace feed {

constexpr int kMaxSlots = 8;
constexpr int kBoxes = 3;           // boxes per slot
constexpr int kThreads = 128;       // warp 0 producer, warp 3 consumer
constexpr int kCols = 1024;         // 16-bit columns per buffer row (2 KB rows)

struct Args {
  int iters, nslots, box_rows, hold, stream, rows;
  int* err;
  unsigned long long* prof;   // [0..2] consumer wait/hold/arrive, [3..5] producer wait/arm/issue
};

__global__ void __launch_bounds__(kThreads, 1)
    feed_kernel(const __grid_constant__ CUtensorMap tm, const Args a) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxSlots];
  __shared__ __align__(8) uint64_t empty_bar[kMaxSlots];
  __shared__ volatile int abort_sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int box_bytes = a.box_rows * 128;
  const int slot_bytes = box_bytes * kBoxes;
  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < a.nslots; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const uint64_t tmo = 2000000000ull;
  const int colblk = kCols / 64;
  const int nblk = (a.rows / a.box_rows) * colblk;
  const long long first = a.stream ? static_cast<long long>(blockIdx.x) * nblk / gridDim.x
                                   : static_cast<long long>(blockIdx.x) * 7;
  if (warp == 0) {
    long long pw = 0, pa = 0, pi = 0;
    int s = 0;
    uint32_t ph = 0;
    for (int it = 0; it < a.iters; ++it) {
      const long long c0 = clock64();
      int ok = 1;
      if (lane == 0) ok = mbar_wait_fast(&empty_bar[s], ph ^ 1u, &abort_sh, tmo) ? 1 : 0;
      if (__shfl_sync(0xffffffffu, ok, 0) == 0) break;
      const long long c1 = clock64();
      if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(slot_bytes));
      __syncwarp();
      const long long c2 = clock64();
      if (lane < kBoxes) {
        const int blk = static_cast<int>((first + static_cast<long long>(it) * kBoxes + lane) % nblk);
        tma_load_2d(smem + s * slot_bytes + lane * box_bytes, &tm, &full_bar[s],
                    (blk % colblk) * 64, (blk / colblk) * a.box_rows);
      }
      __syncwarp();
      const long long c3 = clock64();
      pw += c1 - c0;
      pa += c2 - c1;
      pi += c3 - c2;
      if (++s == a.nslots) s = 0, ph ^= 1u;
    }
    if (lane == 0) {
      atomicAdd(&a.prof[3], static_cast<unsigned long long>(pw));
      atomicAdd(&a.prof[4], static_cast<unsigned long long>(pa));
      atomicAdd(&a.prof[5], static_cast<unsigned long long>(pi));
    }
  } else if (warp == 3 && lane == 0) {
    long long cw = 0, ch = 0, ca = 0;
    int s = 0;
    uint32_t ph = 0;
    for (int it = 0; it < a.iters; ++it) {
      const long long c0 = clock64();
      if (!mbar_wait_fast(&full_bar[s], ph, &abort_sh, tmo)) break;
      const long long c1 = clock64();
      if (a.hold > 0) {
        while (clock64() - c1 < a.hold) {
        }
      }
      const long long c2 = clock64();
      mbar_arrive(&empty_bar[s]);
      const long long c3 = clock64();
      cw += c1 - c0;
      ch += c2 - c1;
      ca += c3 - c2;
      if (++s == a.nslots) s = 0, ph ^= 1u;
    }
    atomicAdd(&a.prof[0], static_cast<unsigned long long>(cw));
    atomicAdd(&a.prof[1], static_cast<unsigned long long>(ch));
    atomicAdd(&a.prof[2], static_cast<unsigned long long>(ca));
  }
  __syncthreads();
  if (threadIdx.x == 0 && abort_sh) atomicExch(a.err, 1);
#endif
}

}  // namespace feed
}  // namespace sp24

using namespace sp24::feed;

int main() {
  int sms = 0, clk_khz = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, 0);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                       &q) != cudaSuccess || fn == nullptr) {
    std::printf("cuTensorMapEncodeTiled unavailable\n");
    return 1;
  }
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  const int l2_rows = 24576;       // 48 MB
  const int hbm_rows = 2097152;    // 4 GB
  uint16_t *l2buf = nullptr, *hbmbuf = nullptr;
  if (cudaMalloc(&l2buf, static_cast<size_t>(l2_rows) * kCols * 2) != cudaSuccess ||
      cudaMalloc(&hbmbuf, static_cast<size_t>(hbm_rows) * kCols * 2) != cudaSuccess) {
    std::printf("allocation failed\n");
    return 1;
  }
  cudaMemset(l2buf, 0x3c, static_cast<size_t>(l2_rows) * kCols * 2);
  cudaMemset(hbmbuf, 0x3c, static_cast<size_t>(hbm_rows) * kCols * 2);
  int* err = nullptr;
  unsigned long long* prof = nullptr;
  cudaMalloc(&err, sizeof(int));
  cudaMalloc(&prof, 6 * sizeof(unsigned long long));
  cudaMemset(err, 0, sizeof(int));
  cudaFuncSetAttribute(feed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024);

  struct Case { const char* what; int hbm, ctas, nslots, box_rows, hold; };
  const Case cases[] = {
      {"L2, 4 x 48 KB, hold 0", 0, sms, 4, 128, 0},
      {"L2, 4 x 48 KB, hold 600", 0, sms, 4, 128, 600},
      {"L2, 4 x 48 KB, hold 1200", 0, sms, 4, 128, 1200},
      {"L2, 3 x 48 KB, hold 600", 0, sms, 3, 128, 600},
      {"L2, 8 x 24 KB, hold 300", 0, sms, 8, 64, 300},
      {"L2, 3 x 63 KB, hold 790", 0, sms, 3, 168, 790},
      {"L2, 2 x 96 KB, hold 1200", 0, sms, 2, 256, 1200},
      {"HBM, 4 x 48 KB, 16 CTAs", 1, 16, 4, 128, 0},
      {"HBM, 4 x 48 KB, 32 CTAs", 1, 32, 4, 128, 0},
      {"HBM, 4 x 48 KB, 64 CTAs", 1, 64, 4, 128, 0},
      {"HBM, 4 x 48 KB, 96 CTAs", 1, 96, 4, 128, 0},
      {"HBM, 4 x 48 KB, 128 CTAs", 1, 128, 4, 128, 0},
      {"HBM, 4 x 48 KB, all SMs", 1, sms, 4, 128, 0},
  };
  std::printf("# %d SMs; per slot: consumer wait/hold/arrive, producer wait/arm/issue (cycles)\n",
              sms);
  for (const Case& c : cases) {
    const int rows = c.hbm ? hbm_rows : l2_rows;
    CUtensorMap tm;
    cuuint64_t dims[2] = {kCols, static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {kCols * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(c.box_rows)};
    cuuint32_t estr[2] = {1, 1};
    if (encode(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, c.hbm ? hbmbuf : l2buf, dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      std::printf("tensor map encode failed\n");
      return 1;
    }
    const int slot_bytes = c.box_rows * 128 * kBoxes;
    Args a{};
    a.iters = static_cast<int>(3000LL * 49152 / slot_bytes);
    if (c.hbm) {   // each CTA streams its own range once: no box is read twice
      const int per_cta = (rows / c.box_rows) * (kCols / 64) / c.ctas;
      a.iters = std::min(2000, per_cta / kBoxes);
    }
    a.nslots = c.nslots;
    a.box_rows = c.box_rows;
    a.hold = c.hold;
    a.stream = c.hbm;
    a.rows = rows;
    a.err = err;
    a.prof = prof;
    const int smem = c.nslots * slot_bytes + 1024;
    float best_ms = 0;
    for (int rep = 0; rep < 2; ++rep) {
      cudaMemset(prof, 0, 6 * sizeof(unsigned long long));
      cudaEvent_t e0, e1;
      cudaEventCreate(&e0);
      cudaEventCreate(&e1);
      cudaEventRecord(e0);
      feed_kernel<<<c.ctas, kThreads, smem>>>(tm, a);
      cudaEventRecord(e1);
      if (cudaGetLastError() != cudaSuccess || cudaEventSynchronize(e1) != cudaSuccess) {
        std::printf("launch failed: %s\n", c.what);
        return 1;
      }
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      if (rep == 0 || ms < best_ms) best_ms = ms;
    }
    int herr = 0;
    unsigned long long hp[6];
    cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost);
    cudaMemcpy(hp, prof, sizeof(hp), cudaMemcpyDeviceToHost);
    if (herr) {
      std::printf("%s: a wait timed out\n", c.what);
      return 2;
    }
    const double bytes = static_cast<double>(c.ctas) * a.iters * slot_bytes;
    const double n = static_cast<double>(c.ctas) * a.iters;
    const double per_sm = bytes / c.ctas / (best_ms * 1e-3);
    std::printf("%-26s %6.2f TB/s  %6.1f GB/s/SM  %5.1f B/clk/SM@%d MHz | %4.0f %5.0f %3.0f | %4.0f %4.0f %4.0f\n",
                c.what, bytes / (best_ms * 1e-3) / 1e12, per_sm / 1e9,
                per_sm / (clk_khz * 1e3), clk_khz / 1000, hp[0] / n, hp[1] / n, hp[2] / n,
                hp[3] / n, hp[4] / n, hp[5] / n);
  }
  return 0;
}
