// sp24_gemm_kernel.cuh — persistent, warp-specialised 2:4 sparse GEMM for
// sm_100a built on tcgen05.mma.sp.
//
//   C[M x N] = alpha * A[M x K] * B[K x N],  A 2:4-sparse along K (compressed
//   values A_c[M x K/2] + 4-bit metadata per group of four), B dense row-major.
//
// Replaces the reference's wgmma_sp_raw_kernel (wgmma_sp_raw_common.hpp:955-1030),
// which computes one 64 x BlockN tile per 128-thread CTA with scalar
// global->shared scatter, one wgmma.mma_async.sp per 32/64-wide K step and a
// wait<0> after every step.  Here:
//   * warp 0      TMA producer: A_c, B and the metadata image go global ->
//                 shared through a STAGES-deep ring (full/empty mbarriers);
//   * warp 1      allocates TMEM and issues, from one lane, tcgen05.cp of the
//                 metadata atom into TMEM followed by the tcgen05.mma.sp's of
//                 the stage (accumulator in TMEM); tcgen05.commit frees ring
//                 slots and publishes finished accumulators;
//   * warps 2..5  epilogue: tcgen05.ld -> registers -> scale -> fp32 and/or
//                 bf16 global stores.  The accumulator is double buffered in
//                 TMEM when 2*BN + 8 columns fit, so the epilogue of tile i
//                 overlaps the main loop of tile i+1.
// CTA tile: 128 rows x BN columns; grid = one CTA per SM walking a grouped
// (GROUP_M) tile order so concurrently running CTAs share A and B tiles in L2.
//
// Shared-memory stage (all regions 1024-byte aligned):
//   A_c  128 rows x 64 B, TMA SWIZZLE_64B, K-major (f16: 32 values = dense K 64;
//        e4m3: 64 values = dense K 128)
//   B    dense-K rows of BN elements, MN-major, TMA boxes of <=128 B with the
//        matching swizzle (SW128 / SW64 / SW32 / none)
//   E    one 2 KB metadata atom (128 lanes x 16 B) per 128 dense K; for f16 one
//        atom serves two stages and only even stages carry it.
#pragma once

#include <cuda_bf16.h>

#include "sp24_ptx.cuh"

namespace sp24 {

constexpr int kBlockM = 128;
constexpr int kThreads = 192;          // 6 warps
constexpr int kAtomBytes = 2048;       // 128 lanes x 16 B metadata atom
constexpr int kSmemBudget = 232448 - 2048;

// Output epilogue shared by every kernel: per row r,
//   v = alpha * acc (+ bias[r]), then the activation (none or SiLU).
// The bias is a per-row vector because A holds the weights (output features
// along M) and B the activations (tokens along N).
enum : int { kActNone = 0, kActSilu = 1 };

SP24_DEV float silu(float v) { return v / (1.0f + __expf(-v)); }

SP24_DEV float epi_value(float acc, float alpha, float bias, bool has_bias, int act) {
  float v = acc * alpha;
  if (has_bias) v += bias;
  return act == kActSilu ? silu(v) : v;
}

// Fused all-gather of C: besides the local output, every finished tile is
// stored into the other ranks' copies of C (peer pointers to the same element
// as c_f32 / c_bf16, same row pitch), over NVLink.  n = 0: local output only.
constexpr int kMaxPeers = 7;
struct PeerOut {
  int n;
  float* f32[kMaxPeers];
  __nv_bfloat16* bf16[kMaxPeers];
};

struct GemmParams {
  int m, n, k;
  int m_blocks, n_tiles, k_stages, num_tiles;
  int group_m;
  const uint8_t* meta_tc;  // tcgen05 metadata image [k_atoms][meta_mblocks][128][16 B]
  int meta_mblocks;        // 128-row blocks in the image (m_blocks rounded up to even)
  float* c_f32;
  __nv_bfloat16* c_bf16;
  long long ldc;
  uint32_t idesc_ab;  // A / B format fields of the instruction descriptor for mixed fp8
                      // (A at bit 7, B at bit 10; e5m2 = 1), 0 otherwise
  float alpha;
  const float* bias;  // optional per-row bias (m floats), added after alpha
  int act;            // kActNone / kActSilu, applied last
  int gate_from_c;    // second pass of a two-pass gated epilogue: multiply by the value
                      // already in C (c_f32 if given, else c_bf16) before storing
  int vec_f32;   // 16-byte vector stores allowed for c_f32
  int vec_bf16;  // 16-byte vector stores allowed for c_bf16
  int* status;   // device word: set to 1 when a bounded wait timed out
  unsigned long long timeout_ns;
  int stall_producer;  // self-test only: producer issues nothing so waits time out
  PeerOut peers;
};

template <int DT, int BN>
struct GemmCfg {
  static constexpr int ESZ = (DT == 2) ? 1 : 2;          // element bytes
  static constexpr int KIND = (DT == 2) ? 1 : 0;         // 0 kind::f16, 1 kind::f8f6f4
  static constexpr int BKD = (DT == 2) ? 128 : 64;       // dense K per stage
  static constexpr int MMA_K = (DT == 2) ? 64 : 32;      // dense K per MMA
  static constexpr int MMAS = BKD / MMA_K;               // MMAs per stage (2)
  static constexpr int STAGES_PER_ATOM = 128 / BKD;      // f16: 2, e4m3: 1
  static constexpr int A_COLS = 64 / ESZ;                // compressed values per stage row
  static constexpr int A_BYTES = kBlockM * 64;
  static constexpr int B_ROW = BN * ESZ;                 // bytes of one K row of the tile
  static constexpr int B_SPAN = B_ROW >= 128 ? 128 : B_ROW;
  static constexpr int B_BOXN = B_SPAN / ESZ;
  static constexpr int B_BOXES = BN / B_BOXN;
  static constexpr int B_BOX_BYTES = B_SPAN * BKD;
  static constexpr int B_BYTES = B_BOX_BYTES * B_BOXES;
  static constexpr uint32_t B_LAYOUT =
      B_SPAN == 128 ? kLayoutSW128 : B_SPAN == 64 ? kLayoutSW64 : B_SPAN == 32 ? kLayoutSW32
                                                                             : kLayoutNone;
  // MN-major canonical layouts: swizzled -> LBO = stride between MN chunks
  // (TMA boxes), SBO = stride between 8-row K groups; no swizzle -> LBO = K
  // group stride, SBO = MN chunk stride.
  static constexpr uint32_t B_LBO = B_LAYOUT == kLayoutNone ? 8 * B_SPAN : B_BOX_BYTES;
  static constexpr uint32_t B_SBO = B_LAYOUT == kLayoutNone ? B_BOX_BYTES : 8 * B_SPAN;
  static constexpr int B_MMA_ADVANCE = MMA_K * B_SPAN;   // bytes per MMA along K
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + kAtomBytes;
  static constexpr int STAGES_RAW = kSmemBudget / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
  static constexpr int ACC = (2 * BN + 8 <= 512) ? 2 : 1;
  static constexpr int E_COL = ACC * BN;
  static constexpr int COLS_NEEDED = E_COL + 8;
  static constexpr uint32_t TMEM_COLS = COLS_NEEDED <= 32    ? 32
                                        : COLS_NEEDED <= 64  ? 64
                                        : COLS_NEEDED <= 128 ? 128
                                        : COLS_NEEDED <= 256 ? 256
                                                             : 512;
  static constexpr uint32_t FMT = (DT == 1) ? 1u : 0u;   // f16 0 / bf16 1 / e4m3 0
  static constexpr uint32_t IDESC = make_idesc_sparse(FMT, BN, kBlockM, true);
  static constexpr int CH = BN < 32 ? BN : 32;           // epilogue column chunk

  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA M=128 needs N % 16 == 0, 16..256");
  static_assert(BN % B_BOXN == 0, "B tile must be whole TMA boxes");
  static_assert(STAGES >= 2, "shared memory too small for two stages");
  static_assert(STAGE_BYTES % 1024 == 0, "stage regions must stay 1024-aligned");
  static_assert(MMAS == 2, "two MMAs per stage (metadata column arithmetic)");
};

SP24_DEV void tile_coords(const GemmParams& P, int t, int& mb, int& nb) {
  const int per_group = P.group_m * P.n_tiles;
  const int g = t / per_group;
  const int first_m = g * P.group_m;
  const int gm = min(P.m_blocks - first_m, P.group_m);
  const int r = t - g * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// Stores N finished values of one row into one copy of C (c32 / c16 with
// P's pitch and vector rules).
template <int N, typename PP>
SP24_DEV void store_values_to(const PP& P, float* c32, __nv_bfloat16* c16, const float (&v)[N],
                              int row, int col) {
  const bool full = (col + N <= P.n);
  if (c32 != nullptr) {
    float* dst = c32 + static_cast<long long>(row) * P.ldc + col;
    if (full && P.vec_f32) {
#pragma unroll
      for (int i = 0; i < N; i += 4)
        *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (col + i < P.n) dst[i] = v[i];
    }
  }
  if (c16 != nullptr) {
    __nv_bfloat16* dst = c16 + static_cast<long long>(row) * P.ldc + col;
    if (full && P.vec_bf16) {
#pragma unroll
      for (int i = 0; i < N; i += 8) {
        uint4 pk;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[i + 0], v[i + 1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        pk.z = *reinterpret_cast<uint32_t*>(&h2);
        pk.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(dst + i) = pk;
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (col + i < P.n) dst[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// Stores N finished values of one row into C and, for a fused all-gather,
// into every peer's copy.  PP: any parameter block with m, n, ldc, c_f32,
// c_bf16, vec_f32, vec_bf16 and peers.
template <int N, typename PP>
SP24_DEV void store_values(const PP& P, const float (&v)[N], int row, int col) {
  if (row >= P.m) return;
  store_values_to<N>(P, P.c_f32, P.c_bf16, v, row, col);
  for (int p = 0; p < P.peers.n; ++p) store_values_to<N>(P, P.peers.f32[p], P.peers.bf16[p], v, row, col);
}

// Value already in C at (row, col) (f32 output if present, else bf16).
template <typename PP>
SP24_DEV float load_c(const PP& P, int row, int col) {
  const long long o = static_cast<long long>(row) * P.ldc + col;
  return P.c_f32 != nullptr ? P.c_f32[o] : __bfloat162float(P.c_bf16[o]);
}

// v[i] *= C[row][col + i] for the N columns of one row segment (the second
// pass of a two-pass gated epilogue).  16-byte loads when the segment is
// whole and C's rows allow them; the same thread stores the segment later.
template <int N, typename PP>
SP24_DEV void gate_mul_row(const PP& P, float* v, int row, int col) {
  const long long o = static_cast<long long>(row) * P.ldc + col;
  const bool full = col + N <= P.n;
  if (full && P.c_f32 != nullptr && P.vec_f32) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 g = *reinterpret_cast<const float4*>(P.c_f32 + o + i);
      v[i] *= g.x, v[i + 1] *= g.y, v[i + 2] *= g.z, v[i + 3] *= g.w;
    }
  } else if (full && P.c_f32 == nullptr && P.vec_bf16 && N % 8 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 8) {
      const uint4 pk = *reinterpret_cast<const uint4*>(P.c_bf16 + o + i);
      const uint32_t w[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[i + 2 * j] *= __uint_as_float(w[j] << 16);
        v[i + 2 * j + 1] *= __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (col + i < P.n) v[i] *= load_c(P, row, col + i);
  }
}

// N accumulator columns of one row -> epilogue -> stores.  PP additionally
// carries alpha, bias, act and gate_from_c.
template <int N, typename PP>
SP24_DEV void store_chunk(const PP& P, uint32_t (&r)[N], int row, int col) {
  if (row >= P.m) return;
  const bool hb = P.bias != nullptr;
  const float b = hb ? P.bias[row] : 0.0f;
  float v[N];
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = epi_value(__uint_as_float(r[i]), P.alpha, b, hb, P.act);
  if (P.gate_from_c) gate_mul_row<N>(P, v, row, col);
  store_values<N>(P, v, row, col);
}

template <int DT, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    sp24_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmParams P) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using C = GemmCfg<DT, BN>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t accf_bar[C::ACC];
  __shared__ __align__(8) uint64_t acce_bar[C::ACC];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < C::ACC; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 4);
    }
    mbar_init(&drain_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  const uint64_t tmo = P.timeout_ns;
  griddep_launch_dependents();

  if (warp == 0) {
    griddep_wait();   // inputs may come from the previous kernel in the stream
    // ------------------------------------------------------------ producer
    if (lane == 0 && !P.stall_producer) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_phase[C::STAGES];
      bool issued[C::STAGES];
#pragma unroll
      for (int i = 0; i < C::STAGES; ++i) issued[i] = false, issued_phase[i] = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < P.num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(P, t, mb, nb);
        for (int ks = 0; ks < P.k_stages; ++ks) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, &abort_sh, tmo)) {
            ok = false;
            break;
          }
          const bool with_e = (ks % C::STAGES_PER_ATOM) == 0;
          uint8_t* st = smem + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[s],
                                C::A_BYTES + C::B_BYTES + (with_e ? kAtomBytes : 0));
          issued[s] = true;
          issued_phase[s] = ph;
          tma_load_2d(st, &tmA, &full_bar[s], ks * C::A_COLS, mb * kBlockM);
#pragma unroll
          for (int bx = 0; bx < C::B_BOXES; ++bx)
            tma_load_2d(st + C::A_BYTES + bx * C::B_BOX_BYTES, &tmB, &full_bar[s],
                        nb * BN + bx * C::B_BOXN, ks * C::BKD);
          if (with_e) {
            const int ka = ks / C::STAGES_PER_ATOM;
            const uint8_t* src =
                P.meta_tc + (static_cast<size_t>(ka) * P.meta_mblocks + mb) * kAtomBytes;
            bulk_load(st + C::A_BYTES + C::B_BYTES, src, kAtomBytes, &full_bar[s]);
          }
          if (++s == C::STAGES) s = 0, ph ^= 1u;
        }
      }
      if (!ok) {
        // Error path: let every copy this thread issued land before the CTA
        // exits (each slot's barrier only advances when its bytes arrive).
        volatile int dummy_abort = 0;
        for (int i = 0; i < C::STAGES; ++i)
          if (issued[i]) mbar_wait(&full_bar[i], issued_phase[i], &dummy_abort, tmo);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Converged warp loop; one elected lane issues each stage's tcgen05 ops.
    {
      const uint32_t a_base = smem_u32(smem);
      const uint64_t adesc0 = make_sdesc(a_base, 16, 512, kLayoutSW64);
      const uint64_t bdesc0 = make_sdesc(a_base + C::A_BYTES, C::B_LBO, C::B_SBO, C::B_LAYOUT);
      const uint64_t edesc0 =
          make_sdesc(a_base + C::A_BYTES + C::B_BYTES, kAtomBytes, 128, kLayoutNone);
      constexpr uint32_t SD = C::STAGE_BYTES >> 4;
      int s = 0;
      uint32_t ph = 0, soff = 0;
      int ab = 0;
      uint32_t aph = 0;
      bool ok = true;
      bool any_issued = false;
      for (int t = blockIdx.x; t < P.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait_warp(&acce_bar[ab], aph ^ 1u, &abort_sh, tmo)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * BN);
        for (int ks = 0; ks < P.k_stages; ++ks) {
          if (!mbar_wait_warp(&full_bar[s], ph, &abort_sh, tmo)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int sub = ks % C::STAGES_PER_ATOM;
          const uint32_t e_tmem =
              tmem_base + static_cast<uint32_t>(C::E_COL + ((ks / C::STAGES_PER_ATOM) & 1) * 4);
          // Metadata column of MMA j inside the atom: kind::f16 uses one
          // 32-bit column per K=32 MMA, kind::f8f6f4 two per K=64 MMA.  The
          // operand address is even; the odd column is picked through the
          // sparsity selector (instruction descriptor bits 0-1).
          const int kleft = P.k - ks * C::BKD;
          const uint32_t acc0 = ks > 0 ? 1u : 0u;
          if (elect_one()) {
            // Metadata atom: 128 rows of 16 B, rows contiguous -> K-major
            // no-swizzle canonical layout, 8-row groups 128 B apart.
            if (sub == 0) tc_cp<1>(e_tmem, edesc0 + soff);
#pragma unroll
            for (int j = 0; j < C::MMAS; ++j) {
              const uint32_t col = (C::KIND == 0) ? static_cast<uint32_t>(sub * C::MMAS + j)
                                                  : static_cast<uint32_t>(2 * j);
              if (j * C::MMA_K < kleft)
                tc_mma<1, C::KIND>(d_tmem, adesc0 + soff + j * 2,
                                   bdesc0 + soff + j * (C::B_MMA_ADVANCE >> 4),
                                   e_tmem + (col & ~1u), C::IDESC | P.idesc_ab | (col & 1u),
                                   j > 0 ? 1u : acc0);
            }
            tc_commit_to<1>(&empty_bar[s], 0);
          }
          __syncwarp();
          any_issued = true;
          soff += SD;
          if (++s == C::STAGES) s = 0, ph ^= 1u, soff = 0;
        }
        if (!ok) break;
        if (elect_one()) tc_commit_to<1>(&accf_bar[ab], 0);
        __syncwarp();
        if (++ab == C::ACC) ab = 0, aph ^= 1u;
      }
      if (!ok && any_issued) {
        // Error path: wait for MMAs in flight before TMEM is released.
        volatile int dummy_abort = 0;
        if (elect_one()) tc_commit_to<1>(&drain_bar, 0);
        __syncwarp();
        if (lane == 0) mbar_wait(&drain_bar, 0, &dummy_abort, tmo);
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int ab = 0;
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < P.num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(P, t, mb, nb);
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&accf_bar[ab], aph, &abort_sh, tmo);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
      const int row = mb * kBlockM + q * 32 + lane;
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(ab * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += C::CH) {
        uint32_t r[C::CH];
        if constexpr (C::CH == 32) {
          tmem_ld_x32(tb + c, r);
        } else {
          tmem_ld_x16(tb + c, r);
        }
        tmem_ld_wait(r);
        if (c + C::CH >= BN) {
          // Last chunk is in registers: hand the accumulator back early.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce_bar[ab]);
        }
        store_chunk<C::CH>(P, r, row, nb * BN + c);
      }
      if (++ab == C::ACC) ab = 0, aph ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (P.peers.n > 0) __threadfence_system();   // peer stores visible before completion
  if (threadIdx.x == 0 && abort_sh != 0 && P.status != nullptr) atomicExch(P.status, 1);
#endif
}

}  // namespace sp24
