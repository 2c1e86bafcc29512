// sp24_peak.cu — tensor-core rate probe (measurement only, built into
// lib/libsp24_peak.so; not part of the sp24 C ABI).
//
// Every CTA pair fills one shared-memory stage once (A 128 rows, B 128
// columns per CTA, one metadata atom), then the leader issues the same
// cta_group::2 M=256 x N=256 MMAs against it back to back: no TMA, no ring,
// no epilogue.  The rate it reaches is the ceiling of the tensor pipe for
// the GEMM kernels' own instruction shape, at whatever clock the GPU holds
// while it runs:
//   sparse: tcgen05.mma.sp.cta_group::2, K = 32 (f16/bf16) or 64 (e4m3)
//   dense:  tcgen05.mma.cta_group::2,    K = 16 (f16/bf16) or 32 (e4m3)
// Shared-memory layouts and descriptors are the CTA-pair kernel's
// (PairCfg<DT, 0, 256>): A_c SW128 K-major, B SW128 MN-major, the metadata
// atom lane-major.  Operand values are pseudo-random (so the switching power
// is a real GEMM's), metadata codes are the six valid 2:4 patterns.
#include <cuda_runtime.h>

#include <cstdint>

#include "sp24_gemm2sm_kernel.cuh"

namespace sp24 {
namespace probe {

constexpr int kProbeThreads = 128;

SP24_DEV uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

template <int KIND>
SP24_DEV void tc_mma_dense_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                uint32_t accumulate) {
  if constexpr (KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// DT: 0 f16, 1 bf16, 2 e4m3.  SPARSE: 1 tcgen05.mma.sp, 0 dense tcgen05.mma.
template <int DT, int SPARSE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kProbeThreads, 1)
    mma_rate_kernel(int iters, int* status, unsigned long long timeout_ns) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using C = PairCfg<DT, 0, 256, 1>;
  constexpr int STAGE = C::A_BYTES + C::B_BYTES + kAtomBytes;
  constexpr int MMA_K = SPARSE ? C::MMA_K : C::MMA_K / 2;   // dense K per instruction
  constexpr int B_STEP = MMA_K * C::B_SPAN;                  // bytes of B per instruction
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t rank = cluster_ctarank();
  const int warp = threadIdx.x >> 5;

  // Operands: pseudo-random bf16/f16 in (-1, 1) or e4m3 bytes without NaN;
  // metadata: one of the six valid codes per nibble.
  const uint32_t seed = mix32(blockIdx.x * 7919u + 17u);
  uint32_t* w = reinterpret_cast<uint32_t*>(smem);
  for (int i = threadIdx.x; i < (C::A_BYTES + C::B_BYTES) / 4; i += kProbeThreads) {
    const uint32_t h = mix32(seed ^ static_cast<uint32_t>(i));
    // 16-bit: exponent bits forced to 0b01111xx (|v| < 2); e4m3: bytes with
    // bit 6 clear never reach the NaN encodings.
    w[i] = (C::ESZ == 2) ? ((h & 0x807f807fu) | 0x3f003f00u) : (h & 0xb7b7b7b7u);
  }
  const uint8_t codes[6] = {0x4, 0x8, 0xC, 0x9, 0xD, 0xE};
  uint8_t* e = smem + C::A_BYTES + C::B_BYTES;
  for (int i = threadIdx.x; i < kAtomBytes; i += kProbeThreads) {
    const uint32_t h = mix32(seed ^ (0x9e3779b9u + static_cast<uint32_t>(i)));
    e[i] = static_cast<uint8_t>(codes[h % 6] | (codes[(h >> 8) % 6] << 4));
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&done_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  const uint64_t tmo = timeout_ns;

  if (rank == 0 && threadIdx.x == 0) {
    const uint32_t sbase = smem_u32(smem);
    const uint64_t adesc = make_sdesc(sbase, 16, C::A_SBO, C::A_LAYOUT);
    const uint64_t bdesc = make_sdesc(sbase + C::A_BYTES, C::B_LBO, C::B_SBO, C::B_LAYOUT);
    const uint64_t edesc = make_sdesc(sbase + C::A_BYTES + C::B_BYTES, kAtomBytes, 128, kLayoutNone);
    const uint32_t e_tmem = tmem_base + static_cast<uint32_t>(C::E_COL);
    if constexpr (SPARSE) tc_cp<2>(e_tmem, edesc);
    const uint32_t idesc_sp = C::IDESC;
    const uint32_t idesc_dn = C::IDESC & ~7u;   // sparse flag and selector cleared
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t acc = (it > 0 || j > 0) ? 1u : 0u;
        if constexpr (SPARSE) {
          const uint32_t col = (C::KIND == 0) ? static_cast<uint32_t>(j) : static_cast<uint32_t>(2 * j);
          tc_mma<2, C::KIND>(tmem_base, adesc + j * 2, bdesc + j * (B_STEP >> 4),
                             e_tmem + (col & ~1u), idesc_sp | (col & 1u), acc);
        } else {
          tc_mma_dense_pair<C::KIND>(tmem_base, adesc + j * 2, bdesc + j * (B_STEP >> 4),
                                     idesc_dn, acc);
        }
      }
    }
    tc_commit_to<2>(&done_bar, static_cast<uint16_t>(3u));
  }
  if (threadIdx.x == 0) {
    if (!mbar_wait(&done_bar, 0, &abort_sh, tmo) && status != nullptr) atomicExch(status, 1);
  }
  __syncthreads();
  tc_fence_before();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
  (void)STAGE;
#endif
}

template <int DT, int SPARSE>
int run(int sm_count, int iters, int reps, float* ms_out, double* flops_out, int* status,
        cudaStream_t stream) {
  using C = PairCfg<DT, 0, 256, 1>;
  constexpr int STAGE = C::A_BYTES + C::B_BYTES + kAtomBytes;
  auto kern = mma_rate_kernel<DT, SPARSE>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, STAGE + 1024) !=
      cudaSuccess)
    return 5;
  const int pairs = sm_count / 2;
  const unsigned long long tmo = 2000000000ull;
  kern<<<2 * pairs, kProbeThreads, STAGE + 1024, stream>>>(iters, status, tmo);   // warm-up
  if (cudaGetLastError() != cudaSuccess) return 5;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, stream);
  for (int r = 0; r < reps; ++r) kern<<<2 * pairs, kProbeThreads, STAGE + 1024, stream>>>(iters, status, tmo);
  cudaEventRecord(e1, stream);
  const cudaError_t err = cudaEventSynchronize(e1);
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (err != cudaSuccess || cudaGetLastError() != cudaSuccess) return 5;
  const double k_per = SPARSE ? C::MMA_K : C::MMA_K / 2;
  *ms_out = ms / static_cast<float>(reps);
  *flops_out = 2.0 * 256.0 * 256.0 * k_per * 4.0 * static_cast<double>(iters) * pairs;
  return 0;
}

}  // namespace probe
}  // namespace sp24

extern "C" {

// Times `reps` launches of the probe (after one warm-up) on the current
// device: every SM pair issues `iters` x 4 MMAs.  dtype 0 f16, 1 bf16,
// 2 e4m3; sparse 1 = tcgen05.mma.sp, 0 = dense.  Writes the mean launch time
// and the dense-equivalent FLOPs of one launch.  status_dev (device int,
// may be NULL) is set nonzero if the bounded completion wait gave up.
// Returns 0, or 5 on a CUDA error, 8 on a bad argument.
int sp24_probe_mma_rate(int dtype, int sparse, int iters, int reps, float* ms_out,
                        double* flops_out, int* status_dev, void* stream) {
  if (dtype < 0 || dtype > 2 || iters < 1 || reps < 1 || ms_out == nullptr || flops_out == nullptr)
    return 8;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 5;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  using namespace sp24::probe;
  switch (dtype * 2 + (sparse ? 1 : 0)) {
    case 0: return run<0, 0>(sms, iters, reps, ms_out, flops_out, status_dev, s);
    case 1: return run<0, 1>(sms, iters, reps, ms_out, flops_out, status_dev, s);
    case 2: return run<1, 0>(sms, iters, reps, ms_out, flops_out, status_dev, s);
    case 3: return run<1, 1>(sms, iters, reps, ms_out, flops_out, status_dev, s);
    case 4: return run<2, 0>(sms, iters, reps, ms_out, flops_out, status_dev, s);
    default: return run<2, 1>(sms, iters, reps, ms_out, flops_out, status_dev, s);
  }
}

}  // extern "C"
