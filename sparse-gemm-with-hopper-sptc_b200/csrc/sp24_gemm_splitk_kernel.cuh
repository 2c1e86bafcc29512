// sp24_gemm_splitk_kernel.cuh — the narrow-N 2:4 sparse GEMM (N <= 128):
// large K stages, and split-K across a thread-block cluster reduced through
// distributed shared memory.
//
// With few output columns (an MLP layer applied to a handful of tokens) the
// GEMM is bound by streaming A_c and its metadata from HBM once: per 128-row
// tile the MMAs are tiny and nearly all time goes to moving bytes.  Two things
// decide the rate: the bytes each SM keeps in flight and the number of SMs
// streaming.  This kernel therefore
//   * stages KB "units" per ring slot, a unit being one 128 x 128 B A_c box
//     (SWIZZLE_128B; 128 dense K for 16-bit types, 256 for e4m3), the B rows
//     of the same K range and their metadata atoms, so one slot carries 22-50
//     KB and the ring keeps ~200 KB per SM in flight;
//   * arms every full barrier for its first use at start-up and lets the MMA
//     warp re-arm a slot as soon as it has seen the slot fill, so the
//     producer warp only waits for a free slot and issues its TMA copies, one
//     copy per lane;
//   * splits K over the S CTAs of a cluster (S <= 8) when the 128-row tiles
//     alone cannot occupy the GPU.  Each CTA accumulates its K range in TMEM,
//     parks the fp32 partial tile in its own shared memory, and after a
//     cluster barrier CTA r sums rows [128 r / S, 128 (r+1) / S) of all S
//     partials over DSMEM in rank order (a fixed order: results do not depend
//     on timing) and stores them.  No workspace, no atomics, no second launch.
//
// Gated form (G = 2, the SwiGLU of an MLP): the CTA streams W_gate and W_up
// (same shape, same B) through one ring, accumulates both tiles in TMEM and
// writes act(alpha W_gate B + bias) * (alpha_up W_up B + bias_up) once.  B is
// staged once for both, and the two GEMMs share one launch and one output.
//
// Roles (6 warps, as in sp24_gemm_kernel.cuh): warp 0 TMA producer, warp 1
// TMEM owner and MMA issuer, warps 2..5 epilogue (TMEM lane quarters).
//
// In the default dispatch this kernel takes up to 16 columns, and wider
// narrow tiles only where the CTA-pair kernel's narrow forms do not apply
// (sp24_gemm2sm_kernel.cuh): from 17 columns on, pairs that each stage half
// of B keep more stages in flight than one SM per 128-row tile.
//
// Replaces, for narrow N, the reference's wgmma_sp_raw_kernel<Element,BlockN>
// (wgmma_sp_raw_common.hpp:955-1030), whose BlockN 8..128 variants compute one
// 64 x BlockN tile per CTA with one 32/64-wide K step per iteration.
#pragma once

#include <cuda_bf16.h>

#include "sp24_gemm_kernel.cuh"
#include "sp24_ptx.cuh"

namespace sp24 {

constexpr int kMaxSplits = 8;

struct SplitParams {
  int m, n, k;
  int m_blocks, n_tiles;
  int splits;         // S: CTAs per cluster, each owning a contiguous range of stages
  int stages;         // ceil(K / dense K per stage)
  int katoms;         // metadata atoms along K (ceil(K / 128))
  const uint8_t* meta_tc;
  int meta_mblocks;
  float* c_f32;
  __nv_bfloat16* c_bf16;
  long long ldc;
  uint32_t idesc_ab;  // A / B format fields of the instruction descriptor for mixed fp8
                      // (A at bit 7, B at bit 10; e5m2 = 1), 0 otherwise
  float alpha;
  const float* bias;  // optional per-row bias (m floats)
  int act;            // kActNone / kActSilu
  int gate_from_c;    // second pass of a two-pass gated epilogue: multiply by the value
                      // already in C (c_f32 if given, else c_bf16) before storing
  // Gated form only: the second weight's metadata image, scale and bias.
  const uint8_t* meta_up;
  float alpha_up;
  const float* bias_up;
  int vec_f32;
  int vec_bf16;
  int rotate;          // per-tile rotation of the K order (see the kernel)
  int static_weights;  // A_c / metadata not written by in-flight work: the first
                       // ring of their loads may precede griddepcontrol.wait
  int* status;
  unsigned long long timeout_ns;
  int stall_producer;
  PeerOut peers;
};

// G: weights streamed per CTA (1 plain, 2 gated).
// BN = 8 (16-bit types, N <= 8): 8-column tiles on N = 16 MMAs.  A 16-wide
// box over an 8-column B would be half outside the tensor, and TMA's
// zero-fill of those halves slowed the whole launch (W_up 14336 x 4096, 8
// columns: 16.8 us against 14.8 us at 16 columns).  Instead each unit loads
// one in-bounds 8-column box (16 B rows, no swizzle), and the MMA's second
// 8-column chunk reads a region that the kernel zeroes once, so accumulator
// columns 8..15 stay zero and are never stored.
template <int DT, int BN, int KB, int G = 1>
struct SplitCfg {
  static constexpr int ESZ = (DT == 2) ? 1 : 2;
  static constexpr int MMA_N = BN < 16 ? 16 : BN;         // accumulator columns per weight
  static constexpr int KIND = (DT == 2) ? 1 : 0;
  static constexpr int WEIGHTS = G;
  static constexpr int UK = (DT == 2) ? 256 : 128;        // dense K per unit
  static constexpr int MMA_K = (DT == 2) ? 64 : 32;
  static constexpr int MMAS_U = UK / MMA_K;               // 4
  static constexpr int E_U = UK / 128;                    // metadata atoms per unit
  static constexpr int BKD = KB * UK;                     // dense K per stage
  static constexpr int A_COLS = 128 / ESZ;                // compressed values per A box row
  static constexpr int A_BOX = kBlockM * 128;             // 16 KB
  static constexpr int A_BYTES = G * KB * A_BOX;           // gate units, then up units
  static constexpr int B_ROW = BN * ESZ;
  static constexpr int B_SPAN = B_ROW >= 128 ? 128 : B_ROW;
  static constexpr int B_BOXN = B_SPAN / ESZ;
  static constexpr int B_BOXES = BN / B_BOXN;             // loaded per unit
  static constexpr int B_CHUNKS = MMA_N / B_BOXN;         // read per unit by the MMAs
  static constexpr int B_BOX_BYTES = B_SPAN * UK;
  static constexpr int B_UNIT = B_BOX_BYTES * B_CHUNKS;   // chunks past B_BOXES: zeroes
  static constexpr int B_BYTES = KB * B_UNIT;
  static constexpr int B_LOAD_BYTES = KB * B_BOXES * B_BOX_BYTES;
  static constexpr uint32_t B_LAYOUT =
      B_SPAN == 128 ? kLayoutSW128 : B_SPAN == 64 ? kLayoutSW64 : B_SPAN == 32 ? kLayoutSW32
                                                                             : kLayoutNone;
  static constexpr uint32_t B_LBO = B_LAYOUT == kLayoutNone ? 8 * B_SPAN : B_BOX_BYTES;
  static constexpr uint32_t B_SBO = B_LAYOUT == kLayoutNone ? B_BOX_BYTES : 8 * B_SPAN;
  static constexpr int B_MMA_ADVANCE = MMA_K * B_SPAN;
  static constexpr int E_S = KB * E_U;                    // metadata atoms per stage and weight
  static constexpr int E_BYTES = G * E_S * kAtomBytes;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + E_BYTES;
  static constexpr int STAGES_RAW = (kSmemBudget - 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
  static constexpr int LOADS_A = G * KB;
  static constexpr int LOADS_B = KB * B_BOXES;
  static constexpr int LOADS = LOADS_A + LOADS_B + G * E_S;   // one copy per producer lane
  static constexpr uint32_t LOAD_LANES = LOADS == 32 ? 0xffffffffu : (1u << LOADS) - 1u;
  static constexpr int E_COL = G * MMA_N;                 // accumulators first, then metadata
  static constexpr int COLS_NEEDED = E_COL + 2 * G * E_S * 4;
  static constexpr uint32_t TMEM_COLS = COLS_NEEDED <= 32    ? 32
                                        : COLS_NEEDED <= 64  ? 64
                                        : COLS_NEEDED <= 128 ? 128
                                        : COLS_NEEDED <= 256 ? 256
                                                             : 512;
  static constexpr uint32_t FMT = (DT == 1) ? 1u : 0u;
  static constexpr uint32_t IDESC = make_idesc_sparse(FMT, MMA_N, kBlockM, true);
  static constexpr int CH = MMA_N < 32 ? MMA_N : 32;      // accumulator columns per TMEM load
  static constexpr int CW = CH < BN ? CH : BN;            // ... of which output columns
  static constexpr int RS = BN + 4;                       // partial-tile row stride (floats)

  static_assert((BN % 16 == 0 && BN >= 16 && BN <= 128) || (BN == 8 && ESZ == 2),
                "narrow tiles: N % 16 == 0, 16..128, or 8 for 16-bit types");
  static_assert(BN % B_BOXN == 0, "B tile must be whole TMA boxes");
  static_assert(STAGES >= 2, "shared memory too small for two stages");
  static_assert(STAGE_BYTES % 1024 == 0, "stage regions must stay 1024-aligned");
  static_assert(LOADS <= 32, "one producer lane per copy");
  static_assert(G * kBlockM * RS * 4 <= STAGES * STAGE_BYTES, "partial tiles must fit the ring");
};

// Bytes that land on a slot's full barrier for global stage g: every A and B
// box counts in full (TMA counts zero-filled out-of-range elements too);
// metadata atoms past the image are not loaded.
template <class C>
SP24_DEV uint32_t split_stage_tx(const SplitParams& P, int g) {
  const int a0 = g * C::E_S;
  int atoms = P.katoms - a0;
  atoms = atoms < 0 ? 0 : (atoms > C::E_S ? C::E_S : atoms);
  return static_cast<uint32_t>(C::A_BYTES + C::B_LOAD_BYTES + C::WEIGHTS * atoms * kAtomBytes);
}

// Stores four finished values of one row into one copy of C.
template <typename PP>
SP24_DEV void store_vec4_to(const PP& P, float* c32, __nv_bfloat16* c16, float4 v, int row,
                            int col) {
  const bool full = col + 4 <= P.n;
  if (c32 != nullptr) {
    float* dst = c32 + static_cast<long long>(row) * P.ldc + col;
    if (full && P.vec_f32) {
      *reinterpret_cast<float4*>(dst) = v;
    } else {
      const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (col + i < P.n) dst[i] = e[i];
    }
  }
  if (c16 != nullptr) {
    __nv_bfloat16* dst = c16 + static_cast<long long>(row) * P.ldc + col;
    if (full && P.vec_bf16) {
      __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y);
      __nv_bfloat162 h1 = __floats2bfloat162_rn(v.z, v.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&h0);
      pk.y = *reinterpret_cast<uint32_t*>(&h1);
      *reinterpret_cast<uint2*>(dst) = pk;
    } else {
      const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (col + i < P.n) dst[i] = __float2bfloat16_rn(e[i]);
    }
  }
}

// ... into C and every peer's copy (fused all-gather).
template <typename PP>
SP24_DEV void store_vec4(const PP& P, float4 v, int row, int col) {
  if (row >= P.m) return;
  store_vec4_to(P, P.c_f32, P.c_bf16, v, row, col);
  for (int p = 0; p < P.peers.n; ++p) store_vec4_to(P, P.peers.f32[p], P.peers.bf16[p], v, row, col);
}

// Grid: (m_blocks * n_tiles * S) CTAs in clusters of S along x; CTA rank r of
// cluster t computes tile t over stages [stages*r/S, stages*(r+1)/S).
// Epilogue of one output element from its fp32 sums: the plain form applies
// alpha, bias and the activation; the gated form multiplies the activated
// gate by the up projection.
template <int G>
SP24_DEV float split_out(const SplitParams& P, float g, float u, float bg, float bu) {
  const float a = epi_value(g, P.alpha, bg, P.bias != nullptr, P.act);
  if constexpr (G == 1) {
    (void)u, (void)bu;
    return a;
  } else {
    return a * epi_value(u, P.alpha_up, bu, P.bias_up != nullptr, kActNone);
  }
}

// tmA2: W_up's A_c (gated form; the plain form passes tmA again).
template <int DT, int BN, int KB, int G>
__global__ void __launch_bounds__(kThreads, 1)
    sp24_gemm_splitk_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmA2, const SplitParams P) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using C = SplitCfg<DT, BN, KB, G>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t accf_bar;
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = P.splits;
  const int rank = S > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int tile = static_cast<int>(blockIdx.x) / S;
  const int mb = tile % P.m_blocks;
  const int nb = tile / P.m_blocks;
  const int g0 = static_cast<int>(static_cast<long long>(P.stages) * rank / S);
  const int g1 = static_cast<int>(static_cast<long long>(P.stages) * (rank + 1) / S);
  const int nst = g1 - g0;
  // K order rotated per row block (P.rotate): the tiles of row block mb start
  // at stage mb * nst / m_blocks of their range and wrap around.  B is shared
  // by every row block, and with one order for all, the CTAs that stream at
  // the same time all read the same few rows of B -- the same L2 lines -- at
  // the same moment.  The rotation depends on mb alone, so a column shard of
  // C (N-sharding) sums every element in the same order as the full GEMM.
  const int rot = (P.rotate && nst > 0)
                      ? static_cast<int>(static_cast<long long>(mb) * nst / P.m_blocks)
                      : 0;
  auto stage_of = [&](int i) {   // i-th stage this CTA processes (i < 2 nst)
    const int j = i + rot;
    return g0 + (j >= nst ? j - nst : j);
  };

  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&accf_bar, 1);
    mbar_init(&drain_bar, 1);
    fence_barrier_init();
    // First use of every slot armed here; the MMA warp re-arms each slot for
    // its next stage when it sees the slot fill.
    for (int s = 0; s < C::STAGES && s < nst; ++s)
      mbar_arrive_expect_tx(&full_bar[s], split_stage_tx<C>(P, stage_of(s)));
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (G == 2) tma_prefetch_desc(&tmA2);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  if constexpr (C::B_CHUNKS > C::B_BOXES) {
    // BN = 8: the B chunks that no TMA copy writes hold zeroes for the whole
    // launch, in every unit of every ring slot.
    constexpr int ZV = (C::B_CHUNKS - C::B_BOXES) * C::B_BOX_BYTES / 16;   // stores per unit
    for (int i = threadIdx.x; i < C::STAGES * KB * ZV; i += kThreads) {
      const int slot = i / (KB * ZV);
      const int u = (i / ZV) % KB;
      const int v = i % ZV;
      *reinterpret_cast<uint4*>(smem + slot * C::STAGE_BYTES + C::A_BYTES + u * C::B_UNIT +
                                C::B_BOXES * C::B_BOX_BYTES + v * 16) = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();   // visible to the MMAs (async proxy) after the barrier
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  const uint64_t tmo = P.timeout_ns;
  griddep_launch_dependents();

  if (warp == 0) {
    // Inputs may come from the previous kernel in the stream: wait for it
    // before the first load (with static weights, after the first ring of
    // weight loads; see below).
    if (!P.static_weights) griddep_wait();
    // ------------------------------------------------------------ producer
    // Lane l issues copy l of every stage: A boxes (gate units, then up
    // units), then B boxes, then metadata atoms (gate, then up).
    // Coordinates advance by a constant step per stage.
    if (!P.stall_producer && lane < C::LOADS) {
      const bool is_a = lane < C::LOADS_A;
      const bool is_b = !is_a && lane < C::LOADS_A + C::LOADS_B;
      const int bl = lane - C::LOADS_A;
      const int el = lane - C::LOADS_A - C::LOADS_B;
      const int u = is_a ? lane % KB : (is_b ? bl / C::B_BOXES : 0);
      const bool up = is_a ? (lane >= KB) : (!is_b && el >= C::E_S);
      const CUtensorMap* amap = up ? &tmA2 : &tmA;
      const uint8_t* meta = up ? P.meta_up : P.meta_tc;
      const uint32_t off = is_a   ? static_cast<uint32_t>(lane * C::A_BOX)
                           : is_b ? static_cast<uint32_t>(C::A_BYTES + u * C::B_UNIT +
                                                          (bl % C::B_BOXES) * C::B_BOX_BYTES)
                                  : static_cast<uint32_t>(C::A_BYTES + C::B_BYTES + el * kAtomBytes);
      const int b_x = nb * BN + (bl % C::B_BOXES) * C::B_BOXN;
      const int e_off = up ? el - C::E_S : el;
      // Copy of this lane for global stage gs into ring slot `slot`.
      auto issue = [&](int slot, uint32_t slot_off, int gs) {
        uint8_t* dst = smem + slot_off + off;
        if (is_a) {
          tma_load_2d(dst, amap, &full_bar[slot], (gs * KB + u) * C::A_COLS, mb * kBlockM);
        } else if (is_b) {
          tma_load_2d(dst, &tmB, &full_bar[slot], b_x, (gs * KB + u) * C::UK);
        } else {
          const int atom = gs * C::E_S + e_off;
          if (atom < P.katoms)
            bulk_load(dst, meta + (static_cast<size_t>(atom) * P.meta_mblocks + mb) * kAtomBytes,
                      kAtomBytes, &full_bar[slot]);
        }
      };
      // Static weights: the first ring of A_c and metadata copies (free
      // slots) goes out before the wait for the previous grid; B, which that
      // grid may have produced, follows it.
      const int pre = P.static_weights ? min(C::STAGES, nst) : 0;
      if (P.static_weights) {
        if (!is_b)
          for (int i = 0; i < pre; ++i)
            issue(i, static_cast<uint32_t>(i * C::STAGE_BYTES), stage_of(i));
        griddep_wait();
        if (is_b)
          for (int i = 0; i < pre; ++i)
            issue(i, static_cast<uint32_t>(i * C::STAGE_BYTES), stage_of(i));
      }
      int s = pre % C::STAGES;
      uint32_t ph = pre == C::STAGES ? 1u : 0u;
      uint32_t soff = static_cast<uint32_t>(s * C::STAGE_BYTES);
      uint32_t issued_mask = pre > 0 ? (1u << pre) - 1u : 0u, issued_ph = 0;
      bool ok = true;
      for (int i = pre; i < nst; ++i) {
        int good = 1;
        if (lane == 0) good = mbar_wait_fast(&empty_bar[s], ph ^ 1u, &abort_sh, tmo) ? 1 : 0;
        if (__shfl_sync(C::LOAD_LANES, good, 0) == 0) {
          ok = false;
          break;
        }
        issue(s, soff, stage_of(i));
        if (lane == 0) {
          issued_mask |= 1u << s;
          issued_ph = (issued_ph & ~(1u << s)) | (ph << s);
        }
        soff += C::STAGE_BYTES;
        if (++s == C::STAGES) s = 0, ph ^= 1u, soff = 0;
      }
      if (!ok && lane == 0) {
        // Error path: let every copy issued so far land before the CTA exits.
        volatile int dummy = 0;
        for (int j = 0; j < C::STAGES; ++j)
          if (issued_mask & (1u << j)) mbar_wait(&full_bar[j], (issued_ph >> j) & 1u, &dummy, tmo);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t smem_base = smem_u32(smem);
    const uint64_t adesc0 = make_sdesc(smem_base, 16, 1024, kLayoutSW128);
    const uint64_t bdesc0 = make_sdesc(smem_base + C::A_BYTES, C::B_LBO, C::B_SBO, C::B_LAYOUT);
    const uint64_t edesc0 =
        make_sdesc(smem_base + C::A_BYTES + C::B_BYTES, kAtomBytes, 128, kLayoutNone);
    constexpr uint32_t SD = C::STAGE_BYTES >> 4;
    int s = 0;
    uint32_t ph = 0, soff = 0, ebuf = 0;
    bool ok = true, any = false;
    for (int i = 0; i < nst; ++i) {
      const int g = stage_of(i);
      if (!mbar_wait_warp(&full_bar[s], ph, &abort_sh, tmo)) {
        ok = false;
        break;
      }
      if (lane == 0 && i + C::STAGES < nst)
        mbar_arrive_expect_tx(&full_bar[s], split_stage_tx<C>(P, stage_of(i + C::STAGES)));
      tc_fence_after();
      ebuf ^= static_cast<uint32_t>(G * C::E_S * 4);
      const uint32_t e_tmem = tmem_base + static_cast<uint32_t>(C::E_COL) + ebuf;
      const int kleft = P.k - g * C::BKD;
      if (elect_one()) {
#pragma unroll
        for (int a = 0; a < G * C::E_S; ++a)
          if (g * C::E_S + a % C::E_S < P.katoms)
            tc_cp<1>(e_tmem + 4 * a, edesc0 + soff + a * (kAtomBytes >> 4));
#pragma unroll
        for (int w = 0; w < G; ++w)
#pragma unroll
          for (int u = 0; u < KB; ++u)
#pragma unroll
            for (int j = 0; j < C::MMAS_U; ++j) {
              const int kk = u * C::UK + j * C::MMA_K;   // dense K inside the stage
              if (kk < kleft) {
                const int atom_in = w * C::E_S + kk / 128;
                const uint32_t col = (C::KIND == 0) ? static_cast<uint32_t>((kk % 128) / 32)
                                                    : static_cast<uint32_t>(2 * ((kk % 128) / 64));
                tc_mma<1, C::KIND>(
                    tmem_base + static_cast<uint32_t>(w * C::MMA_N),
                    adesc0 + soff + (w * KB + u) * (C::A_BOX >> 4) + j * 2,
                    bdesc0 + soff + u * (C::B_UNIT >> 4) + j * (C::B_MMA_ADVANCE >> 4),
                    e_tmem + 4 * atom_in + (col & ~1u), C::IDESC | P.idesc_ab | (col & 1u),
                    (i > 0 || kk > 0) ? 1u : 0u);
              }
            }
        tc_commit_to<1>(&empty_bar[s], 0);
      }
      __syncwarp();
      any = true;
      soff += SD;
      if (++s == C::STAGES) s = 0, ph ^= 1u, soff = 0;
    }
    if (ok && elect_one()) tc_commit_to<1>(&accf_bar, 0);
    __syncwarp();
    if (!ok && any) {
      volatile int dummy = 0;
      if (elect_one()) tc_commit_to<1>(&drain_bar, 0);
      __syncwarp();
      if (lane == 0) mbar_wait(&drain_bar, 0, &dummy, tmo);
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    bool ok = true;
    if (lane == 0) ok = mbar_wait_sleepy(&accf_bar, 0, &abort_sh, tmo);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (ok) {
      tc_fence_after();
      const int row_l = q * 32 + lane;
      const int row = mb * kBlockM + row_l;
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      float* red = reinterpret_cast<float*>(smem);   // ring is idle once accf has fired
      const bool live = row < P.m;
      const float bg = (P.bias != nullptr && live) ? P.bias[row] : 0.0f;
      const float bu = (G == 2 && P.bias_up != nullptr && live) ? P.bias_up[row] : 0.0f;
#pragma unroll 1
      for (int c = 0; c < BN; c += C::CH) {
        uint32_t r[G][C::CH];
#pragma unroll
        for (int w = 0; w < G; ++w) {
          if constexpr (C::CH == 32) {
            tmem_ld_x32(tb + static_cast<uint32_t>(w * C::MMA_N + c), r[w]);
          } else {
            tmem_ld_x16(tb + static_cast<uint32_t>(w * C::MMA_N + c), r[w]);
          }
        }
#pragma unroll
        for (int w = 0; w < G; ++w) tmem_ld_wait(r[w]);
        if (S == 1) {
          // Finished values of this lane's row go to the warp's rows of the
          // idle ring; the warp then stores them row by row (below).
          float v[C::CW];
#pragma unroll
          for (int e = 0; e < C::CW; ++e)
            v[e] = split_out<G>(P, __uint_as_float(r[0][e]), __uint_as_float(r[G - 1][e]), bg,
                                bu);
          if (P.gate_from_c && live) gate_mul_row<C::CW>(P, v, row, nb * BN + c);
#pragma unroll
          for (int e = 0; e < C::CW; e += 4)
            *reinterpret_cast<float4*>(red + row_l * C::RS + c + e) =
                make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        } else {
#pragma unroll
          for (int w = 0; w < G; ++w)
#pragma unroll
            for (int v = 0; v < C::CW; v += 4)
              *reinterpret_cast<float4*>(red + (w * kBlockM + row_l) * C::RS + c + v) =
                  make_float4(__uint_as_float(r[w][v]), __uint_as_float(r[w][v + 1]),
                              __uint_as_float(r[w][v + 2]), __uint_as_float(r[w][v + 3]));
        }
      }
      if (S == 1) {
        // Coalesced stores: the warp's 32 rows leave as contiguous row
        // segments (BN / 4 lanes per row, 16 B each), instead of one 16 B
        // piece of 32 different rows per store instruction.
        __syncwarp();
        constexpr int NV = BN / 4;
        for (int idx = lane; idx < 32 * NV; idx += 32) {
          const int rl = q * 32 + idx / NV;
          const int cg = idx - (idx / NV) * NV;
          const float4 o = *reinterpret_cast<const float4*>(red + rl * C::RS + cg * 4);
          store_vec4(P, o, mb * kBlockM + rl, nb * BN + cg * 4);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (S > 1) {
    // Partials of all ranks are complete and visible after this barrier
    // (release/acquire at cluster scope).
    cluster_sync();
    const int r0 = kBlockM * rank / S;
    const int r1 = kBlockM * (rank + 1) / S;
    constexpr int NV = BN / 4;
    const float* red = reinterpret_cast<const float*>(smem);
    for (int idx = threadIdx.x; idx < (r1 - r0) * NV; idx += kThreads) {
      const int rl = r0 + idx / NV;
      const int cg = idx - (idx / NV) * NV;
      const int row = mb * kBlockM + rl;
      float4 acc[G];
#pragma unroll
      for (int w = 0; w < G; ++w) {
        const uint32_t la = smem_u32(red + (w * kBlockM + rl) * C::RS + cg * 4);
        acc[w] = ld_dsmem_f4(mapa_shared(la, 0));
        for (int src = 1; src < S; ++src) {
          const float4 v = ld_dsmem_f4(mapa_shared(la, static_cast<uint32_t>(src)));
          acc[w].x += v.x;
          acc[w].y += v.y;
          acc[w].z += v.z;
          acc[w].w += v.w;
        }
      }
      if (row >= P.m) continue;
      const float bg = P.bias != nullptr ? P.bias[row] : 0.0f;
      const float bu = (G == 2 && P.bias_up != nullptr) ? P.bias_up[row] : 0.0f;
      float4 o = make_float4(split_out<G>(P, acc[0].x, acc[G - 1].x, bg, bu),
                             split_out<G>(P, acc[0].y, acc[G - 1].y, bg, bu),
                             split_out<G>(P, acc[0].z, acc[G - 1].z, bg, bu),
                             split_out<G>(P, acc[0].w, acc[G - 1].w, bg, bu));
      const int col = nb * BN + cg * 4;
      if (P.gate_from_c) {
        if (col + 0 < P.n) o.x *= load_c(P, row, col + 0);
        if (col + 1 < P.n) o.y *= load_c(P, row, col + 1);
        if (col + 2 < P.n) o.z *= load_c(P, row, col + 2);
        if (col + 3 < P.n) o.w *= load_c(P, row, col + 3);
      }
      store_vec4(P, o, row, col);
    }
    // No CTA leaves (and releases its shared memory) while others still read it.
    cluster_sync();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (P.peers.n > 0) __threadfence_system();   // peer stores visible before completion
  if (threadIdx.x == 0 && abort_sh != 0 && P.status != nullptr) atomicExch(P.status, 1);
#endif
}

}  // namespace sp24
