// sp24_raw_kernel.cuh — wgmma_sp_raw_kernel<Element, BlockN>: the reference's
// launchable kernel (codes1gn/sparse-gemm-with-hopper-sptc,
// wgmma_sp_raw_common.hpp:955-1030), rebuilt on tcgen05 for sm_100a with the
// same signature, argument meaning and launch geometry:
//
//   wgmma_sp_raw_kernel<Element, BlockN><<<dim3(n / BlockN, m / 64), dim3(128)>>>(
//       a_sparse, b, e_bytes, c, n, k);
//
// (wgmma_sp_raw_common.hpp:1078-1080; docs/hopper-sparse-wgmma-usage-guide.md
// :589-593).  Each CTA computes one 64 x BlockN tile of C (fp32, row stride
// n) from a_sparse (m x k/2 compressed values, row stride k/2), e_bytes (the
// reference's row-major metadata nibbles, m x k/8 bytes) and b (k x n,
// row-major).  Element: half, __nv_bfloat16 or __nv_fp8_e4m3; BlockN: 8, 16,
// 32, 64, 128 or 256; k % 32 == 0 (k % 64 for e4m3), n % BlockN == 0.
//
// Inside a CTA (128 threads; the reference launches with no dynamic shared
// memory, so everything lives in static shared memory, at most 44 KB):
//   * the four warps stage each MMA step (32 dense K; 64 for e4m3) into a
//     double-buffered stage with cp.async copies from this GPU's memory,
//     writing the canonical layouts the tcgen05 shared-memory descriptors
//     name: A_c in 32-byte rows with the 32-byte swizzle, K-major; B MN-major
//     in boxes with the swizzle of their row width;
//   * they also rewrite the step's metadata nibbles, read straight from
//     e_bytes, into its word(s) of a TMEM-image atom in shared memory;
//   * one thread issues tcgen05.cp of the atom into TMEM and the step's
//     tcgen05.mma.sp (accumulator in TMEM) and commits them to the stage's
//     mbarrier, which frees the stage for the load two steps later;
//   * after the last step the warps read the accumulator (tcgen05.ld) and
//     store fp32 C.
// Two forms (SP24_RAW_LAYOUT, default 1):
//   1  M = 64, the reference's tile height: accumulator row r at TMEM lane
//      32 (r / 16) + r % 16, and the metadata of rows r and r + 8 (16-bit
//      kinds) or of row r (e4m3) in the lanes of the same lane quarter;
//   0  the MMA runs with M = 128 on rows 0-63 plus 64 zero rows, with the
//      M = 128 layouts of the library's own kernels.
// Both pass the same checks (tests/raw_kernel_check.cu).
// Every wait is bounded (1 s); a wait that runs out sets
// sp24_raw_kernel_status (a __device__ int of this header) and the CTA
// returns after its MMAs in flight have drained.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../csrc/sp24_ptx.cuh"

#ifndef SP24_RAW_LAYOUT
#define SP24_RAW_LAYOUT 1
#endif

// Set to 1 by a CTA of wgmma_sp_raw_kernel whose bounded wait ran out (the
// reference's kernel has no status argument to carry it).
static __device__ int sp24_raw_kernel_status;

namespace sp24_raw {

template <typename Element>
struct ElementTraits;
template <>
struct ElementTraits<half> {
  static constexpr int ESZ = 2, KIND = 0;
  static constexpr uint32_t FMT = 0;
};
template <>
struct ElementTraits<__nv_bfloat16> {
  static constexpr int ESZ = 2, KIND = 0;
  static constexpr uint32_t FMT = 1;
};
template <>
struct ElementTraits<__nv_fp8_e4m3> {
  static constexpr int ESZ = 1, KIND = 1;
  static constexpr uint32_t FMT = 0;
};

template <typename Element, int BlockN, int LAYOUT>
struct RawCfg {
  using T = ElementTraits<Element>;
  static constexpr int ESZ = T::ESZ;
  static constexpr int KIND = T::KIND;
  static constexpr int MMA_K = ESZ == 1 ? 64 : 32;       // dense K per step (one MMA)
  static constexpr int A_ROW = 32;                        // compressed bytes per row per step
  static constexpr int M_MMA = LAYOUT == 0 ? 128 : 64;
  static constexpr int N_MMA = BlockN < 16 ? 16 : BlockN;
  static constexpr int A_BYTES = M_MMA * A_ROW;
  static constexpr int B_ROW = N_MMA * ESZ;              // bytes of one K row of the tile
  static constexpr int B_SPAN = B_ROW >= 128 ? 128 : B_ROW;
  static constexpr int B_BOXES = B_ROW / B_SPAN;
  static constexpr int B_BOX_BYTES = B_SPAN * MMA_K;
  static constexpr int B_BYTES = B_BOX_BYTES * B_BOXES;
  static constexpr uint32_t B_LAYOUT = B_SPAN == 128  ? sp24::kLayoutSW128
                                       : B_SPAN == 64 ? sp24::kLayoutSW64
                                       : B_SPAN == 32 ? sp24::kLayoutSW32
                                                      : sp24::kLayoutNone;
  static constexpr uint32_t B_SWZ = B_SPAN == 128 ? 7u : B_SPAN == 64 ? 3u : B_SPAN == 32 ? 1u : 0u;
  // MN-major canonical layouts (as the library's kernels): swizzled -> LBO =
  // box stride, SBO = 8-row K group stride; unswizzled -> the reverse.
  static constexpr uint32_t B_LBO = B_LAYOUT == sp24::kLayoutNone ? 8 * B_SPAN : B_BOX_BYTES;
  static constexpr uint32_t B_SBO = B_LAYOUT == sp24::kLayoutNone ? B_BOX_BYTES : 8 * B_SPAN;
  static constexpr int E_BYTES = 2048;                    // one atom (128 lanes x 16 B)
  static constexpr int STAGE_RAW = A_BYTES + B_BYTES + E_BYTES;
  static constexpr int STAGE = (STAGE_RAW + 1023) / 1024 * 1024;
  static constexpr int E_COL = N_MMA;                     // two buffers of 4 columns
  static constexpr int COLS = N_MMA + 8;
  static constexpr uint32_t TMEM_COLS = COLS <= 32 ? 32 : COLS <= 64 ? 64 : COLS <= 128 ? 128
                                        : COLS <= 256 ? 256 : 512;
  static constexpr uint32_t IDESC = sp24::make_idesc_sparse(T::FMT, N_MMA, M_MMA, true);
  static_assert(BlockN == 8 || BlockN == 16 || BlockN == 32 || BlockN == 64 || BlockN == 128 ||
                    BlockN == 256,
                "BlockN is one of the reference's tile widths 8 .. 256");
  static_assert(2 * STAGE <= 46 * 1024, "two stages fit the 48 KB of static shared memory");
  static_assert(A_BYTES % 1024 == 0 || B_SPAN <= 32, "B boxes start on their swizzle period");
};

SP24_DEV void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sp24::smem_u32(dst)), "l"(src)
               : "memory");
}
SP24_DEV void cp_async_8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(sp24::smem_u32(dst)), "l"(src)
               : "memory");
}
SP24_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SP24_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset inside a swizzled region: the 16-byte chunk index (address
// bits 4..) is XORed with address bits 7.. under `mask` (7: 128-byte
// swizzle, 3: 64-byte, 1: 32-byte, 0: none), the pattern the descriptor's
// layout type names.
SP24_DEV uint32_t swz(uint32_t off, uint32_t mask) { return off ^ (((off >> 7) & mask) << 4); }

// Stage MMA step [k0, k0 + MMA_K) of the CTA's tile into stage `st`.
template <typename Element, int BlockN, int LAYOUT>
SP24_DEV void load_step(uint8_t* st, const Element* a_sparse, const Element* b, int n, int k,
                        int row0, int col0, int k0) {
  using C = RawCfg<Element, BlockN, LAYOUT>;
  constexpr int ESZ = C::ESZ;
  // A_c: 64 rows x 32 bytes (two 16-byte chunks), 32-byte swizzle.
  const uint8_t* a = reinterpret_cast<const uint8_t*>(a_sparse);
  for (int i = threadIdx.x; i < 64 * 2; i += 128) {
    const int r = i >> 1, ch = i & 1;
    const uint8_t* src = a + (static_cast<size_t>(row0 + r) * (k / 2) + k0 / 2) * ESZ + 16 * ch;
    cp_async_16(st + swz(static_cast<uint32_t>(r * C::A_ROW + 16 * ch), 1u), src);
  }
  // B: MMA_K rows x BlockN columns, MN-major boxes of B_SPAN-byte rows.
  uint8_t* bs = st + C::A_BYTES;
  const uint8_t* bg = reinterpret_cast<const uint8_t*>(b);
  constexpr int ROWB = BlockN * ESZ;          // loaded bytes per K row (8 B for e4m3 x 8)
  if constexpr (ROWB >= 16) {
    constexpr int CPR = ROWB / 16;            // chunks per row
    for (int i = threadIdx.x; i < C::MMA_K * CPR; i += 128) {
      const int y = i / CPR, ch = i - y * CPR;
      const int xb = 16 * ch;                 // byte column inside the tile row
      const int box = xb / C::B_SPAN, xin = xb - box * C::B_SPAN;
      const uint32_t off = static_cast<uint32_t>(box * C::B_BOX_BYTES) +
                           swz(static_cast<uint32_t>(y * C::B_SPAN + xin), C::B_SWZ);
      cp_async_16(bs + off, bg + (static_cast<size_t>(k0 + y) * n + col0) * ESZ + xb);
    }
  } else {
    for (int y = threadIdx.x; y < C::MMA_K; y += 128)
      cp_async_8(bs + y * C::B_SPAN, bg + (static_cast<size_t>(k0 + y) * n + col0) * ESZ);
  }
}

// Writes the step's metadata (rows row0 .. row0+63, dense K [k0, k0 +
// MMA_K)) into the first column(s) of the stage's TMEM-image atom, read
// straight from the reference's row-major nibbles.
//   16-bit (one column): lane 16 m2 + 8 k1 + m0 [M = 128] or 32 m2 + 8 k1
//     + m0 [M = 64] holds row 16 m2 + m0 in bits 0-15 and row 16 m2 + 8 + m0
//     in bits 16-31, both the 16 dense K [k0 + 16 k1, +16): reference bytes
//     (k0 + 16 k1) / 8 and the next of each row.
//   e4m3 (two columns): the lane of row r ([M = 128] r; [M = 64]
//     32 (r / 16) + r % 16) holds the row's 8 reference bytes of the step.
template <typename Element, int BlockN, int LAYOUT>
SP24_DEV void write_meta(uint8_t* es, const uint8_t* e_bytes, int k, int row0, int k0) {
  using C = RawCfg<Element, BlockN, LAYOUT>;
  const int rb = k / 8;
  uint32_t* img = reinterpret_cast<uint32_t*>(es);
  const int i = threadIdx.x;                      // 128 threads, 128 words either way
  if constexpr (C::ESZ == 2) {
    if (i < 64) {
      const int m0 = i & 7, k1 = (i >> 3) & 1, m2 = i >> 4;
      const uint8_t* s0 =
          e_bytes + static_cast<size_t>(row0 + 16 * m2 + m0) * rb + (k0 + 16 * k1) / 8;
      const uint8_t* s1 = s0 + static_cast<size_t>(8) * rb;
      const uint32_t lo = s0[0] | (s0[1] << 8), hi = s1[0] | (s1[1] << 8);
      const int lane = (LAYOUT == 0 ? 16 * m2 : 32 * m2) + 8 * k1 + m0;
      img[lane * 4] = lo | (hi << 16);
    }
  } else {
    const int r = i & 63, w = i >> 6;
    const uint8_t* s = e_bytes + static_cast<size_t>(row0 + r) * rb + k0 / 8 + 4 * w;
    const uint32_t word = s[0] | (s[1] << 8) | (s[2] << 16) | (static_cast<uint32_t>(s[3]) << 24);
    const int lane = LAYOUT == 0 ? r : 32 * (r >> 4) + (r & 15);
    img[lane * 4 + w] = word;
  }
}

}  // namespace sp24_raw

template <typename Element, int BlockN>
__global__ void __launch_bounds__(128) wgmma_sp_raw_kernel(Element const* __restrict__ a_sparse,
                                                           Element const* __restrict__ b,
                                                           uint8_t const* __restrict__ e_bytes,
                                                           float* __restrict__ c, int n, int k) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  constexpr int LAYOUT = SP24_RAW_LAYOUT;
  using C = sp24_raw::RawCfg<Element, BlockN, LAYOUT>;
  __shared__ __align__(1024) uint8_t smem[2 * C::STAGE];
  __shared__ __align__(8) uint64_t mma_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.y * 64;
  const int col0 = blockIdx.x * BlockN;
  const unsigned long long tmo = 1000000000ull;

  // Both stages start zeroed (padding rows of A, padding columns of B), and
  // metadata lanes that no row of the tile feeds hold the valid code 0x4.
  for (int i = threadIdx.x; i < 2 * C::STAGE / 16; i += 128)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * 512; i += 128)
    reinterpret_cast<uint32_t*>(smem + (i >> 9) * C::STAGE + C::A_BYTES + C::B_BYTES)[i & 511] =
        0x44444444u;
  if (threadIdx.x == 0) {
    abort_sh = 0;
    sp24::mbar_init(&mma_bar[0], 1);
    sp24::mbar_init(&mma_bar[1], 1);
    sp24::fence_barrier_init();
  }
  if (warp == 0) {
    sp24::tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    sp24::tmem_relinquish();
  }
  sp24::tc_fence_before();
  __syncthreads();
  sp24::tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  const int steps = k / C::MMA_K;
  uint32_t phase[2] = {0u, 0u};
  bool ok = true;
  int issued = 0;   // steps whose MMAs were issued (thread 0)
  sp24_raw::load_step<Element, BlockN, LAYOUT>(smem, a_sparse, b, n, k, row0, col0, 0);
  sp24_raw::cp_async_commit();
  for (int s = 0; s < steps; ++s) {
    const int buf = s & 1, nbuf = buf ^ 1;
    if (s + 1 < steps) {
      // Step s - 1's MMA reads stage nbuf: wait for it before reloading it.
      if (s >= 1) {
        if (!sp24::mbar_wait(&mma_bar[nbuf], phase[nbuf], &abort_sh, tmo)) ok = false;
        phase[nbuf] ^= 1u;
      }
      if (ok)
        sp24_raw::load_step<Element, BlockN, LAYOUT>(smem + nbuf * C::STAGE, a_sparse, b, n, k,
                                                     row0, col0, (s + 1) * C::MMA_K);
    }
    sp24_raw::cp_async_commit();
    sp24_raw::cp_async_wait<1>();
    uint8_t* st = smem + buf * C::STAGE;
    sp24_raw::write_meta<Element, BlockN, LAYOUT>(st + C::A_BYTES + C::B_BYTES, e_bytes, k, row0,
                                                  s * C::MMA_K);
    sp24::fence_proxy_async_smem();
    __syncthreads();
    if (!ok || abort_sh) {
      ok = false;
      break;
    }
    if (threadIdx.x == 0) {
      const uint32_t sb = sp24::smem_u32(st);
      const uint64_t adesc = sp24::make_sdesc(sb, 16, 8 * C::A_ROW, sp24::kLayoutSW32);
      const uint64_t bdesc = sp24::make_sdesc(sb + C::A_BYTES, C::B_LBO, C::B_SBO, C::B_LAYOUT);
      const uint64_t edesc =
          sp24::make_sdesc(sb + C::A_BYTES + C::B_BYTES, 2048, 128, sp24::kLayoutNone);
      const uint32_t e_tmem = tmem + static_cast<uint32_t>(C::E_COL + 4 * buf);
      sp24::tc_cp<1>(e_tmem, edesc);
      sp24::tc_mma<1, C::KIND>(tmem, adesc, bdesc, e_tmem, C::IDESC, s > 0 ? 1u : 0u);
      sp24::tc_commit(&mma_bar[buf]);
      issued = s + 1;
    }
  }
  sp24_raw::cp_async_wait<0>();
  // Thread 0's last commit tracks every MMA it issued: wait for it (also on
  // the abort path, so no MMA is in flight when TMEM is released).
  if (threadIdx.x == 0 && issued > 0) {
    const int last = issued - 1;
    volatile int dummy = 0;
    // Completions of stage last & 1 seen so far by the waits above are
    // phase[last & 1]; a wait that already consumed step `last`'s commit
    // cannot have happened (steps are waited two behind), so wait here.
    if (!sp24::mbar_wait(&mma_bar[last & 1], phase[last & 1], &dummy, tmo)) ok = false;
  }
  if (!ok && threadIdx.x == 0) atomicExch(&sp24_raw_kernel_status, 1);
  __syncthreads();
  sp24::tc_fence_after();
  if (ok && !abort_sh) {
    // Warp w reads TMEM lanes 32 w .. 32 w + 31.  M = 128: rows 0-63 live in
    // lanes 0-63 (warps 0 and 1); M = 64: rows 16 w .. 16 w + 15 in lanes
    // 32 w .. 32 w + 15.
    const bool live = LAYOUT == 0 ? warp < 2 : lane < 16;
    const int row = LAYOUT == 0 ? 32 * warp + lane : 16 * warp + lane;
    if (LAYOUT != 0 || warp < 2) {
      constexpr int CH = C::N_MMA < 32 ? C::N_MMA : 32;
      constexpr int NV = BlockN < CH ? BlockN : CH;   // columns stored per chunk
#pragma unroll
      for (int c0 = 0; c0 < BlockN; c0 += CH) {
        uint32_t r[32];
        const uint32_t ta = tmem + (static_cast<uint32_t>(32 * warp) << 16) + static_cast<uint32_t>(c0);
        if constexpr (CH == 32) {
          sp24::tmem_ld_x32(ta, r);
          sp24::tmem_ld_wait(r);
        } else {
          sp24::tmem_ld_x16(ta, *reinterpret_cast<uint32_t(*)[16]>(r));
          sp24::tmem_ld_wait(*reinterpret_cast<uint32_t(*)[16]>(r));
        }
        if (live) {
          float* dst = c + static_cast<size_t>(row0 + row) * n + col0 + c0;
#pragma unroll
          for (int i = 0; i < NV; i += 4)
            *reinterpret_cast<float4*>(dst + i) =
                make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                            __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
        }
      }
    }
  }
  sp24::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sp24::tc_fence_after();
    sp24::tmem_dealloc(tmem, C::TMEM_COLS);
  }
#endif
}
