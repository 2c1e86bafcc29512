// sp24_gemm2sm_kernel.cuh — the 2:4 sparse GEMM on CTA pairs: a cluster of
// 2 CTAs computes a 256-row tile with tcgen05.mma.sp.cta_group::2.
//
// Why a pair: one tcgen05.mma.sp.cta_group::2 with M=256, N=BNP reads A_c
// rows 0-127 and B columns [0, BNP/2) from CTA 0's shared memory and A_c
// rows 128-255 and B columns [BNP/2, BNP) from CTA 1's.  Each SM therefore
// stages half of B, which (a) halves B's share of the L2->SM traffic and of
// the shared-memory read bandwidth per MMA and (b) lets the same ring cover
// twice the MMA time.  No TMA multicast is used: each CTA loads its own tiles.
//
// Forms (template parameters of pair_gemm_body):
//   BNP = 256        large problems; the persistent grid walks the tiles.
//   BNP = 32..128    narrow N (an MLP layer over a few tokens): stages of
//                    22-36 KB, 6-8 of them in the ring.
//   G = 2            gated (SwiGLU): W_gate and W_up against the same B
//                    stages into two accumulators.
//   KS = 1           K-split: a cluster of 2 S CTAs per tile, pair p summing
//                    K slice p, partial tiles reduced over distributed shared
//                    memory (narrow N with few row tiles).
//
// Roles per CTA (11 warps):
//   warps 0,10  TMA producers (both CTAs): warp 0 the A_c rows and the
//               metadata atoms of the CTA's own 128 rows, warp 10 its half of
//               the B columns; completion bytes of both CTAs are counted on
//               the pair leader's full barrier, which only the leader arms.
//   warp 1      TMEM owner (alloc/dealloc with cta_group::2 in both CTAs);
//               in the leader one elected lane issues, per stage, tcgen05.cp
//               (metadata of both CTAs into their own TMEM), the pair MMAs and
//               a 2-CTA multicast commit, so both CTAs' ring slots and
//               accumulator barriers advance.
//   warps 2-9   epilogue (both CTAs): two warps per TMEM lane quarter, each
//               pulls BNP/2 accumulator columns of its 32 rows into registers,
//               hands the accumulator back to the leader's MMA warp at once
//               (remote mbarrier arrive), then scales / converts / stores
//               while the next tile's MMAs run.
// Two 256-wide accumulators plus the two metadata buffers would exceed TMEM's
// 512 columns, so the accumulator is single-buffered (in every form); the
// register hand-off keeps the MMA pause to the TMEM read time.
#pragma once

#include <cuda_bf16.h>

#include "sp24_gemm_kernel.cuh"
#include "sp24_gemm_splitk_kernel.cuh"
#include "sp24_ptx.cuh"

namespace sp24 {

constexpr int kPairThreads = 352;   // 11 warps
constexpr int kPairEpiWarps = 8;
constexpr int kPairBWarp = 10;      // second producer warp (B tiles)

struct PairParams {
  int m, n, k;
  int m_blocks;   // 128-row blocks of the metadata image (padded to even)
  int m_pairs;    // 256-row tiles
  int n_tiles;    // 256-column tiles
  int k_stages, num_tiles, group_m;
  int splits;     // K-split form: pairs per cluster (each owns a K slice); 1 otherwise
  float* c_f32;
  __nv_bfloat16* c_bf16;
  long long ldc;
  uint32_t idesc_ab;  // A / B format fields of the instruction descriptor for mixed fp8
                      // (A at bit 7, B at bit 10; e5m2 = 1), 0 otherwise
  float alpha;
  const float* bias;  // optional per-row bias (m floats)
  int act;            // kActNone / kActSilu
  float alpha_up;         // gated form (G = 2): W_up's scale and optional bias
  const float* bias_up;
  int gate_from_c;    // second pass of a two-pass gated epilogue: multiply by the value
                      // already in C (c_f32 if given, else c_bf16) before storing
  int vec_f32;   // 2: 32-byte stores, 1: 16-byte, 0: scalar
  int vec_bf16;
  int c_evict_first;  // 32-byte C stores under an L2 evict-first policy (no peers)
  int static_weights; // A_c / metadata not written by in-flight work: their producer warp
                      // starts before the previous kernel of the stream completes
  int* status;
  unsigned long long timeout_ns;
  int stall_producer;
  PeerOut peers;
};

// FINE selects the stage granularity: 0 = 128 dense K per stage for 16-bit
// types (256 for e4m3), four MMAs per stage; 1 = half of that, two MMAs per
// stage and twice as many stages.  A ring slot is freed only when its MMAs
// complete, so the MMAs queued in the tensor pipe hold part of the ring; finer
// stages leave more of the same shared memory loading.
// BNP is the pair tile width: 256 for large N; 128, 64 or (16-bit types) 32
// for narrow N (an MLP layer applied to a few tokens), where each CTA stages
// only BNP / 2 columns of B, so a stage shrinks to 22-36 KB and the ring
// holds 6-8 of them.
// G = 2 is the gated form (SwiGLU, narrow tiles only): W_gate and W_up stream
// through one ring against the same B stages into two accumulators, and the
// epilogue writes act(alpha W_gate B + b) * (alpha_up W_up B + b_up).
template <int DT, int FINE, int BNP = 256, int G = 1>
struct PairCfg {
  static constexpr int ESZ = (DT == 2) ? 1 : 2;
  static constexpr int KIND = (DT == 2) ? 1 : 0;
  static constexpr int BKD = ((DT == 2) ? 256 : 128) >> FINE;   // dense K per stage
  static constexpr int MMA_K = (DT == 2) ? 64 : 32;             // dense K per MMA
  static constexpr int MMAS = BKD / MMA_K;                      // MMAs per stage
  static constexpr int E_PER = BKD >= 128 ? BKD / 128 : 1;      // atoms loaded with a stage
  static constexpr int SPA = BKD >= 128 ? 1 : 128 / BKD;        // stages sharing one atom
  static constexpr int A_ROW = BKD / 2 * ESZ;                   // bytes of a compressed A row
  static constexpr int A_COLS = A_ROW / ESZ;
  static constexpr int A_ONE = kBlockM * A_ROW;                 // one weight's A_c box
  static constexpr int A_BYTES = G * A_ONE;
  static constexpr uint32_t A_LAYOUT = A_ROW == 128 ? kLayoutSW128 : kLayoutSW64;
  static constexpr uint32_t A_SBO = 8 * A_ROW;                  // 8-row group stride
  static constexpr int BN = BNP;                                // pair tile width
  static constexpr int BN_CTA = BNP / 2;                        // B columns staged per CTA
  static constexpr int B_ROWB = BN_CTA * ESZ;                   // bytes of one K row of it
  static constexpr int B_SPAN = B_ROWB >= 128 ? 128 : B_ROWB;   // swizzle span of a TMA box
  static constexpr int B_BOXN = B_SPAN / ESZ;
  static constexpr int B_BOXES = BN_CTA / B_BOXN;
  static constexpr int B_BOX_BYTES = B_SPAN * BKD;
  static constexpr int B_BYTES = B_BOX_BYTES * B_BOXES;
  static constexpr uint32_t B_LAYOUT =
      B_SPAN == 128 ? kLayoutSW128 : B_SPAN == 64 ? kLayoutSW64 : kLayoutSW32;
  static constexpr uint32_t B_LBO = B_BOX_BYTES;                // MN-major swizzled: chunk stride
  static constexpr uint32_t B_SBO = 8 * B_SPAN;                 // 8-row K group stride
  static constexpr int B_MMA_ADVANCE = MMA_K * B_SPAN;
  static constexpr int CW = BNP / 2;                            // columns per epilogue warp
  static constexpr int RS = BNP + 4;                            // parked partial row stride
  static constexpr int E_BYTES = G * E_PER * kAtomBytes;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + E_BYTES;
  static constexpr int STAGES_RAW = (kSmemBudget - 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
  static constexpr int LOADS = G + B_BOXES + G * E_PER;         // TMA boxes per stage per CTA
  static constexpr int E_COL = 256;                             // two buffers of E_PER*4 columns
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t FMT = (DT == 1) ? 1u : 0u;
  static constexpr uint32_t IDESC = make_idesc_sparse(FMT, BNP, 256, true);
  static_assert(BNP == 32 || BNP == 64 || BNP == 128 || BNP == 256,
                "pair tile width 32, 64, 128 or 256");
  static_assert(B_SPAN >= 32, "B rows of at least 32 bytes per CTA");
  static_assert(STAGE_BYTES % 1024 == 0, "stage regions must stay 1024-aligned");
  static_assert(STAGES >= 3, "pair kernel wants a deep ring");
  static_assert(kBlockM * RS * 4 <= STAGES * STAGE_BYTES, "a parked partial tile fits the ring");
  static_assert(LOADS <= 32, "one lane per TMA box");
  static_assert(G == 1 || (FINE == 0 && BNP >= 64 && G * BNP <= 256),
                "gated form: coarse stages, 64- or 128-wide tiles");
};

SP24_DEV void pair_tile_coords(const PairParams& P, int t, int& mp, int& nb) {
  const int per_group = P.group_m * P.n_tiles;
  const int g = t / per_group;
  const int first = g * P.group_m;
  const int gm = min(P.m_pairs - first, P.group_m);
  const int r = t - g * per_group;
  mp = first + r % gm;
  nb = r / gm;
}

SP24_DEV void st_global_v8_u32(void* p, const uint32_t* v) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

template <int CW>
SP24_DEV void pair_store_row_to(const PairParams& P, float* c32, __nv_bfloat16* c16,
                                uint32_t (&r)[CW], int row, int col0);
template <int CW>
SP24_DEV void pair_epilogue_row(const PairParams& P, uint32_t (&r)[CW], int row, int col0);

// Store CW consecutive accumulator columns of one row (already in registers).
// Warp-collective: every lane of the warp calls it (lane i holding row
// row0 + i); lanes whose row is beyond M compute nothing and store nothing.
template <int CW>
SP24_DEV void pair_store_row(const PairParams& P, uint32_t (&r)[CW], int row, int col0) {
  if (row < P.m) pair_epilogue_row<CW>(P, r, row, col0);
  pair_store_row_to<CW>(P, P.c_f32, P.c_bf16, r, row, col0);
}

// The epilogue of one row, in place on its registers: alpha, bias and the
// activation, then (second pass of a two-pass gated epilogue) the product
// with the value already in C.
template <int CW>
SP24_DEV void pair_epilogue_row(const PairParams& P, uint32_t (&r)[CW], int row, int col0) {
  if (P.bias != nullptr || P.act != kActNone) {
    const bool hb = P.bias != nullptr;
    const float b = hb ? P.bias[row] : 0.0f;
#pragma unroll
    for (int i = 0; i < CW; ++i)
      r[i] = __float_as_uint(epi_value(__uint_as_float(r[i]), P.alpha, b, hb, P.act));
  } else if (P.alpha != 1.0f) {
#pragma unroll
    for (int i = 0; i < CW; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * P.alpha);
  }
  if (P.gate_from_c) gate_mul_row<CW>(P, reinterpret_cast<float*>(r), row, col0);
}

// Fused all-gather, warp-cooperative: after a warp has stored its 32 rows x
// CW columns locally (pair_store_row), it re-reads them from L2 with the
// lanes spread along each row and writes every row segment to the peers as
// contiguous runs (512 B fp32 / 256 B bf16 at CW = 128), i.e. whole 128 B
// lines over NVLink, instead of one scattered 32 B write per lane and row.
template <int CW>
SP24_DEV void pair_push_rows_to_peers(const PairParams& P, int row0, int col0) {
  __syncwarp();  // the warp's local stores are visible to its own loads
  const int lane = threadIdx.x & 31;
  const bool full = col0 + CW <= P.n;
  const bool mine = 4 * lane < CW;   // lanes that cover the segment, 4 columns each
  for (int rr = 0; rr < 32; ++rr) {
    const int row = row0 + rr;
    if (row >= P.m) break;
    const long long o = static_cast<long long>(row) * P.ldc + col0;
    if (P.c_f32 != nullptr) {
      if (full && P.vec_f32) {
        if (mine) {
          const float4 v = *reinterpret_cast<const float4*>(P.c_f32 + o + 4 * lane);
          for (int p = 0; p < P.peers.n; ++p)
            *reinterpret_cast<float4*>(P.peers.f32[p] + o + 4 * lane) = v;
        }
      } else {
        for (int c = lane; c < CW && col0 + c < P.n; c += 32) {
          const float v = P.c_f32[o + c];
          for (int p = 0; p < P.peers.n; ++p) P.peers.f32[p][o + c] = v;
        }
      }
    }
    if (P.c_bf16 != nullptr) {
      if (full && P.vec_bf16) {
        if (mine) {
          const uint2 v = *reinterpret_cast<const uint2*>(P.c_bf16 + o + 4 * lane);
          for (int p = 0; p < P.peers.n; ++p)
            *reinterpret_cast<uint2*>(P.peers.bf16[p] + o + 4 * lane) = v;
        }
      } else {
        for (int c = lane; c < CW && col0 + c < P.n; c += 32) {
          const __nv_bfloat16 v = P.c_bf16[o + c];
          for (int p = 0; p < P.peers.n; ++p) P.peers.bf16[p][o + c] = v;
        }
      }
    }
  }
}

// 4 x 4 transpose of 32-byte units inside each group of four lanes: unit j
// (u[8j .. 8j+7]) of lane 4g+i moves to unit i of lane 4g+j.  Two butterfly
// stages (lane bit 0, then bit 1), 16 shuffles each.  Afterwards unit q of
// lane 4g+p holds what was unit p of lane 4g+q, so when lane 4g+p stores its
// unit q to row (4g+q) at byte offset 32p, the four lanes of a group write
// one 128-byte run of one row.
SP24_DEV void quad_transpose_units(uint32_t (&u)[32]) {
  const int p = threadIdx.x & 3;
#pragma unroll
  for (int m = 1; m <= 2; m <<= 1) {
    const bool hi = (p & m) != 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j & m) continue;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t send = hi ? u[8 * j + e] : u[8 * (j + m) + e];
        const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, m);
        if (hi)
          u[8 * j + e] = recv;
        else
          u[8 * (j + m) + e] = recv;
      }
    }
  }
}

// Warp-collective store of 128-byte row runs: each lane holds 32 words of
// its own row (lane i: row row0 + i, bytes [0, 128) of the run at `base` +
// row * pitch); after the quad transpose every store instruction writes 8
// whole 128-byte runs (rows 4g + q for the 8 groups g) instead of 32
// scattered 32-byte pieces, a quarter of the L2 write requests.
SP24_DEV void store_rows_128b(void* base, long long pitch_bytes, uint32_t (&u)[32], int row0,
                              int m, bool evict_first, uint64_t pol) {
  quad_transpose_units(u);
  const int lane = threadIdx.x & 31;
  const int p = lane & 3, g = lane >> 2;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int row = row0 + 4 * g + q;
    if (row < m) {
      uint8_t* dst = static_cast<uint8_t*>(base) + static_cast<long long>(row) * pitch_bytes + 32 * p;
      if (evict_first)
        st_global_v8_u32_hint(dst, &u[8 * q], pol);
      else
        st_global_v8_u32(dst, &u[8 * q]);
    }
  }
}

// Stores CW finished values of one row (as float bits) into one copy of C.
// Warp-collective (see pair_store_row); r may be reordered on return.
// With 32-byte aligned rows the stores go through the quad transpose:
//   fp32 out:   each 32-column chunk of r is transposed in place and stored
//               as 128-byte runs; a bf16 copy is then converted from the
//               transposed registers, unit by unit, and stored as 64-byte
//               runs (16 bytes per lane);
//   bf16 only:  each 64-column chunk is packed to bf16 pairs in place,
//               transposed and stored as 128-byte runs.
// Narrow or ragged tiles and less aligned outputs store per lane.
template <int CW>
SP24_DEV void pair_store_row_to(const PairParams& P, float* c32, __nv_bfloat16* c16,
                                uint32_t (&r)[CW], int row, int col0) {
  const bool full = col0 + CW <= P.n;   // warp-uniform: one column range per warp
  const bool live = row < P.m;
  const bool ef = P.c_evict_first != 0;
  const uint64_t pol = ef ? l2_evict_first_policy() : 0;
  const int row0 = row - static_cast<int>(threadIdx.x & 31);
  const bool t32 = c32 != nullptr && full && P.vec_f32 == 2 && CW % 32 == 0 &&
                   (c16 == nullptr || P.vec_bf16 >= 1);
  const bool t16 = c32 == nullptr && c16 != nullptr && full && P.vec_bf16 == 2 && CW % 64 == 0;
  if (t32) {
    const int lane = threadIdx.x & 31;
    const int p = lane & 3, g = lane >> 2;
#pragma unroll
    for (int c = 0; c < CW; c += 32) {
      uint32_t(&u)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[c]);
      store_rows_128b(c32 + col0 + c, P.ldc * 4, u, row0, P.m, ef, pol);
      if (c16 != nullptr) {
        // Unit q now holds row 4g+q, columns c + 8p .. c + 8p + 7.
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(u[8 * q + 2 * e]),
                                                     __uint_as_float(u[8 * q + 2 * e + 1]));
            pk[e] = *reinterpret_cast<uint32_t*>(&h);
          }
          const int rr = row0 + 4 * g + q;
          if (rr < P.m) {
            __nv_bfloat16* dst = c16 + static_cast<long long>(rr) * P.ldc + col0 + c + 8 * p;
            if (ef)
              st_global_v4_u32_hint(dst, pk, pol);
            else
              *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
      }
    }
    return;
  }
  if (t16) {
#pragma unroll
    for (int c = 0; c < CW; c += 64) {
      // bf16 pairs packed in place into r[c .. c+31] (each word is written
      // after the two values it replaces have been read).
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[c + 2 * j]),
                                                 __uint_as_float(r[c + 2 * j + 1]));
        r[c + j] = *reinterpret_cast<uint32_t*>(&h);
      }
      store_rows_128b(c16 + col0 + c, P.ldc * 2, *reinterpret_cast<uint32_t(*)[32]>(&r[c]), row0,
                      P.m, ef, pol);
    }
    return;
  }
  if (!live) return;
  if (c16 != nullptr) {
    __nv_bfloat16* dst = c16 + static_cast<long long>(row) * P.ldc + col0;
    if (full && P.vec_bf16 >= 1) {
#pragma unroll
      for (int i = 0; i < CW; i += 16) {
        uint32_t pk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[i + 2 * j]),
                                                   __uint_as_float(r[i + 2 * j + 1]));
          pk[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        if (P.vec_bf16 == 2) {
          if (ef)
            st_global_v8_u32_hint(dst + i, pk, pol);
          else
            st_global_v8_u32(dst + i, pk);
        } else {
          *reinterpret_cast<uint4*>(dst + i) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(dst + i + 8) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < CW; ++i)
        if (col0 + i < P.n) dst[i] = __float2bfloat16_rn(__uint_as_float(r[i]));
    }
  }
  if (c32 != nullptr) {
    float* dst = c32 + static_cast<long long>(row) * P.ldc + col0;
    if (full && P.vec_f32 == 2) {
#pragma unroll
      for (int i = 0; i < CW; i += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[i + j]);
        if (ef)
          st_global_v8_hint(dst + i, v, pol);
        else
          st_global_v8(dst + i, v);
      }
    } else if (full && P.vec_f32 == 1) {
#pragma unroll
      for (int i = 0; i < CW; i += 4)
        *reinterpret_cast<float4*>(dst + i) =
            make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                        __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    } else {
#pragma unroll
      for (int i = 0; i < CW; ++i)
        if (col0 + i < P.n) dst[i] = __uint_as_float(r[i]);
    }
  }
}

// Bytes both CTAs of a pair load for stage ks of a tile (counted on the
// leader's full barrier): every stage carries A_c and B, and the metadata
// atoms come with the first stage of each SPA group.
template <typename C>
SP24_DEV uint32_t pair_stage_tx(int ks) {
  const bool with_e = (C::SPA == 1) || (ks % C::SPA) == 0;
  return 2u * static_cast<uint32_t>(C::STAGE_BYTES - (with_e ? 0 : C::E_BYTES));
}

// The kernel body.  KS = 0: clusters of 2, persistent over the tiles.
// KS = 1 (K-split form, for too few 256-row tiles to occupy the GPU): a
// cluster of 2 S CTAs computes one tile; pair p (CTAs 2p, 2p+1) accumulates
// K slice p in its TMEM, parks its fp32 partial tile in its idle ring, and
// after a cluster barrier each CTA sums its share of rows over all S pairs
// through distributed shared memory (fixed order) and stores them.
template <int DT, int FINE, int BNP, int KS, int G>
SP24_DEV void pair_gemm_body(const CUtensorMap& tmA, const CUtensorMap& tmB,
                             const CUtensorMap& tmE, const CUtensorMap& tmA2,
                             const CUtensorMap& tmE2, const PairParams& P) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using C = PairCfg<DT, FINE, BNP, G>;
  static_assert(!KS || FINE == 0, "K slices start on whole metadata atoms");
  static_assert(!KS || G == 1, "the K-split form is ungated");
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t accf_bar;
  __shared__ __align__(8) uint64_t acce_bar;
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t lead = KS ? (rank & ~1u) : 0u;   // cluster rank of this pair's leader
  const uint32_t prank = rank - lead;             // 0 or 1 inside the pair
  const bool leader = prank == 0;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << lead);
  const int pair = KS ? static_cast<int>(blockIdx.x) / (2 * P.splits)
                      : static_cast<int>(blockIdx.x >> 1);
  const int npairs = KS ? P.num_tiles : static_cast<int>(gridDim.x >> 1);   // KS: one tile
  const int split = KS ? static_cast<int>(rank >> 1) : 0;
  const int kst0 = KS ? P.k_stages * split / P.splits : 0;          // this pair's K slice
  const int kst1 = KS ? P.k_stages * (split + 1) / P.splits : P.k_stages;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&accf_bar, 1);
    mbar_init(&acce_bar, 2 * kPairEpiWarps);
    mbar_init(&drain_bar, 1);
    fence_barrier_init();
    // The leader arms every full barrier for its first use here and the MMA
    // warp re-arms a slot for its next use as soon as it has seen the slot's
    // data arrive: the producers' per-stage work shrinks to one slot wait and
    // one TMA issue.  Coarse stages all carry the same bytes; fine stages
    // carry a metadata atom every SPA-th stage of a tile (pair_stage_tx).
    if (leader)
      for (int s = 0; s < C::STAGES; ++s)
        mbar_arrive_expect_tx(&full_bar[s], pair_stage_tx<C>(s % max(1, kst1 - kst0) + kst0));
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmE);
    if constexpr (G == 2) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmE2);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  const uint64_t tmo = P.timeout_ns;
  griddep_launch_dependents();

  if (warp == 0 || warp == kPairBWarp) {
    // Inputs may come from the previous kernel in the stream.  Under the
    // static-weights hint the A_c / metadata warp starts at once: only B (and,
    // through the mbarrier chain, every C store) waits for that kernel.
    if (warp == kPairBWarp || !P.static_weights) griddep_wait();
    // ------------------------------------------------------------ producers
    // Two warps load each stage: warp 0 the A_c box (lane 0) and the metadata
    // atoms (lanes 1..E_PER), warp 10 the B boxes (one per lane).  Splitting
    // the stage halves the serial chain of shared-memory operations (slot
    // wait, expect_tx, TMA issue) each warp runs per stage; under full
    // tensor-core load every one of those operations queues behind the
    // MMA's operand reads.  Per lane, the box coordinates advance by a
    // constant step per stage.  Completion bytes of both CTAs land on the
    // leader's full barrier, which each leader warp arms with its share.
    if (!P.stall_producer) {
      // Warp 0: lanes 0..G-1 the A_c box of each weight, then the metadata
      // atoms (weight-major); warp 10: the B boxes.
      const bool is_b = warp == kPairBWarp;
      const bool is_a = !is_b && lane < G;
      const int el = lane - G;                                 // metadata lane index
      const int ew = el >= C::E_PER ? 1 : 0;                   // its weight (gated form)
      const uint32_t full0_leader = mapa_shared(smem_u32(&full_bar[0]), lead);
      const CUtensorMap* lane_map = is_b ? &tmB
                                    : is_a ? (lane == 1 ? &tmA2 : &tmA)
                                           : (ew == 1 ? &tmE2 : &tmE);
      const uint32_t lane_off =
          is_b ? static_cast<uint32_t>(C::A_BYTES + lane * C::B_BOX_BYTES)
               : (is_a ? static_cast<uint32_t>(lane * C::A_ONE)
                       : static_cast<uint32_t>(C::A_BYTES + C::B_BYTES + el * kAtomBytes));
      const int lanes_e = is_b ? C::B_BOXES : G + G * C::E_PER;  // stages that carry metadata
      const int lanes_n = is_b ? C::B_BOXES : G;                 // stages that do not
      const int dx = is_a ? C::A_COLS : 0;
      const int dy = is_b ? C::BKD : (is_a ? 0 : C::E_PER * P.m_blocks * 8 / C::SPA);
      int s = 0;
      uint32_t ph = 0;
      uint32_t soff = 0;
      bool ok = true;
      uint32_t armed_mask = 0, armed_ph = 0;
      // 256-wide tiles: every A_c / metadata tile is read again by the pairs
      // of the other column tiles of its raster group, several waves later;
      // an L2 evict-last policy keeps it over B, which is reused within a
      // wave (configurations 2 / 3 / 5: +0.5 / +1.2-2.3 / +0.4%).  Narrow
      // tiles stream their weights once and keep the default policy.
      const bool a_keep = BNP == 256 && !is_b;
      const uint64_t a_pol = a_keep ? l2_evict_last_policy() : 0;
      for (int t = pair; t < P.num_tiles && ok; t += npairs) {
        int mp, nb;
        pair_tile_coords(P, t, mp, nb);
        const int row0 = mp * 256 + static_cast<int>(prank) * 128;
        const int mb = mp * 2 + static_cast<int>(prank);
        int x = is_b ? nb * C::BN + static_cast<int>(prank) * C::BN_CTA + lane * C::B_BOXN : 0;
        int y = is_b ? 0 : (is_a ? row0 : ((el - ew * C::E_PER) * P.m_blocks + mb) * 8);
        x += kst0 * dx;
        y += kst0 * dy;
        for (int ks = kst0; ks < kst1; ++ks) {
          int good = 1;
          if (lane == 0) good = mbar_wait_fast(&empty_bar[s], ph ^ 1u, &abort_sh, tmo) ? 1 : 0;
          if (__shfl_sync(0xffffffffu, good, 0) == 0) {
            ok = false;
            break;
          }
          const bool with_e = (C::SPA == 1) || (ks % C::SPA) == 0;
          if (leader && lane == 0) {
            armed_mask |= 1u << s;
            armed_ph = (armed_ph & ~(1u << s)) | (ph << s);
          }
          if (lane < (with_e ? lanes_e : lanes_n)) {
            const uint32_t bar = full0_leader + static_cast<uint32_t>(s * sizeof(uint64_t));
            if (a_keep)
              tma_load_2d_pair_hint(smem + soff + lane_off, lane_map, bar, x, y, a_pol);
            else
              tma_load_2d_pair(smem + soff + lane_off, lane_map, bar, x, y);
          }
          x += dx;
          y += dy;
          soff += C::STAGE_BYTES;
          if (++s == C::STAGES) s = 0, ph ^= 1u, soff = 0;
        }
      }
      if (!ok && leader && lane == 0) {
        volatile int dummy = 0;
        for (int i = 0; i < C::STAGES; ++i)
          if (armed_mask & (1u << i)) mbar_wait(&full_bar[i], (armed_ph >> i) & 1u, &dummy, tmo);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    // The whole warp runs this loop converged (all operands warp-uniform);
    // one elected lane issues each stage's tcgen05 ops.
    // Descriptors are formed once; per stage only the start-address field
    // moves (stage offset >> 4 added to the 64-bit descriptor), per MMA by a
    // compile-time step.  Metadata: atom a of a stage lives in TMEM columns
    // E_COL + ebuf + a*4 (ebuf alternates between two buffers of E_PER*4
    // columns per atom group); kind::f16 MMAs use one column each (odd
    // columns through the sparsity selector), kind::f8f6f4 MMAs two.
    if (leader) {
      const uint32_t smem_base = smem_u32(smem);
      const uint64_t adesc0 = make_sdesc(smem_base, 16, C::A_SBO, C::A_LAYOUT);
      const uint64_t bdesc0 = make_sdesc(smem_base + C::A_BYTES, C::B_LBO, C::B_SBO, C::B_LAYOUT);
      const uint64_t edesc0 =
          make_sdesc(smem_base + C::A_BYTES + C::B_BYTES, kAtomBytes, 128, kLayoutNone);
      constexpr uint32_t SD = C::STAGE_BYTES >> 4;
      // Per-MMA constants, per position `sub` of the stage inside its atom
      // group: metadata column offset and sparsity selector.
      uint32_t ecol[C::SPA][C::MMAS], isel[C::SPA][C::MMAS];
#pragma unroll
      for (int sb = 0; sb < C::SPA; ++sb)
#pragma unroll
        for (int j = 0; j < C::MMAS; ++j) {
          const int koff = sb * C::BKD + j * C::MMA_K;          // dense K inside the group
          const int kin = (koff % 128) / C::MMA_K;              // MMA index inside its atom
          const uint32_t col = (C::KIND == 0) ? static_cast<uint32_t>(kin)
                                              : static_cast<uint32_t>(2 * kin);
          ecol[sb][j] = 4u * static_cast<uint32_t>(koff / 128) + (col & ~1u);
          isel[sb][j] = C::IDESC | P.idesc_ab | (col & 1u);
        }
      int s = 0;
      uint32_t ph = 0, soff = 0, aph = 0, ebuf = 0;
      bool ok = true, any = false;
      for (int t = pair; t < P.num_tiles && ok; t += npairs) {
        if (!mbar_wait_warp<true>(&acce_bar, aph ^ 1u, &abort_sh, tmo)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int ks = kst0; ks < kst1; ++ks) {
          if (!mbar_wait_warp(&full_bar[s], ph, &abort_sh, tmo)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            // Re-arm the slot for the stage STAGES later in this pair's
            // sequence (it may fall in a later tile, or after the last one,
            // where the arming is never consumed).
            int nks = ks + C::STAGES;
            while (nks >= kst1) nks -= max(1, kst1 - kst0);
            mbar_arrive_expect_tx(&full_bar[s], pair_stage_tx<C>(nks));
          }
          tc_fence_after();
          const int sub = ks % C::SPA;
          if (sub == 0) ebuf ^= static_cast<uint32_t>(G * C::E_PER * 4);
          const uint32_t e_tmem = tmem_base + static_cast<uint32_t>(C::E_COL) + ebuf;
          const int kleft = P.k - ks * C::BKD;
          const uint32_t acc0 = ks > kst0 ? 1u : 0u;
          if (elect_one()) {
            if (sub == 0) {
#pragma unroll
              for (int a = 0; a < G * C::E_PER; ++a)
                tc_cp<2>(e_tmem + 4 * a, edesc0 + soff + a * (kAtomBytes >> 4));
            }
#pragma unroll
            for (int w = 0; w < G; ++w)
#pragma unroll
              for (int j = 0; j < C::MMAS; ++j)
                if (j * C::MMA_K < kleft)
                  tc_mma<2, C::KIND>(
                      tmem_base + static_cast<uint32_t>(w * BNP),
                      adesc0 + soff + w * (C::A_ONE >> 4) + j * 2,
                      bdesc0 + soff + j * (C::B_MMA_ADVANCE >> 4),
                      e_tmem + 4u * static_cast<uint32_t>(w * C::E_PER) +
                          (C::SPA == 1 ? ecol[0][j] : ecol[sub & (C::SPA - 1)][j]),
                      C::SPA == 1 ? isel[0][j] : isel[sub & (C::SPA - 1)][j], j > 0 ? 1u : acc0);
            tc_commit_to<2>(&empty_bar[s], pair_mask);
          }
          __syncwarp();
          any = true;
          soff += SD;
          if (++s == C::STAGES) s = 0, ph ^= 1u, soff = 0;
        }
        if (!ok) break;
        if (elect_one()) tc_commit_to<2>(&accf_bar, pair_mask);
        __syncwarp();
        aph ^= 1u;
      }
      if (!ok && any) {
        volatile int dummy = 0;
        if (elect_one()) tc_commit_to<2>(&drain_bar, static_cast<uint16_t>(1u << lead));
        __syncwarp();
        if (lane == 0) mbar_wait(&drain_bar, 0, &dummy, tmo);
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t acce_leader = mapa_shared(smem_u32(&acce_bar), lead);
    uint32_t aph = 0;
    for (int t = pair; t < P.num_tiles; t += npairs) {
      int mp, nb;
      pair_tile_coords(P, t, mp, nb);
      bool ok = true;
      if (lane == 0) ok = mbar_wait_sleepy(&accf_bar, aph, &abort_sh, tmo);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(half * C::CW);
      uint32_t r[C::CW];
      if constexpr (C::CW == 16) {
        tmem_ld_x16(tb, r);
      } else {
#pragma unroll
        for (int c = 0; c < C::CW; c += 32)
          tmem_ld_x32(tb + static_cast<uint32_t>(c), *reinterpret_cast<uint32_t(*)[32]>(&r[c]));
      }
      tmem_ld_wait(r);
      if constexpr (G == 2) {
        // Gated form: W_up's accumulator sits BNP columns further on.
        uint32_t ru[C::CW];
#pragma unroll
        for (int c = 0; c < C::CW; c += 32)
          tmem_ld_x32(tb + static_cast<uint32_t>(BNP + c), *reinterpret_cast<uint32_t(*)[32]>(&ru[c]));
        tmem_ld_wait(ru);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acce_leader);
        const int row = mp * 256 + static_cast<int>(prank) * 128 + q * 32 + lane;
        if (row < P.m) {
          const bool hg = P.bias != nullptr, hu = P.bias_up != nullptr;
          const float bg = hg ? P.bias[row] : 0.0f, bu = hu ? P.bias_up[row] : 0.0f;
#pragma unroll
          for (int c = 0; c < C::CW; ++c)
            r[c] = __float_as_uint(
                epi_value(__uint_as_float(r[c]), P.alpha, bg, hg, P.act) *
                epi_value(__uint_as_float(ru[c]), P.alpha_up, bu, hu, kActNone));
        }
        pair_store_row_to<C::CW>(P, P.c_f32, P.c_bf16, r, row, nb * C::BN + half * C::CW);
        aph ^= 1u;
        continue;
      }
      tc_fence_before();
      __syncwarp();
      if constexpr (KS) {
        // K slice done: park the raw partial sums in the idle ring.
        float* red = reinterpret_cast<float*>(smem);
        const int rl = q * 32 + lane;
#pragma unroll
        for (int c = 0; c < C::CW; c += 4)
          *reinterpret_cast<float4*>(red + rl * C::RS + half * C::CW + c) =
              make_float4(__uint_as_float(r[c]), __uint_as_float(r[c + 1]),
                          __uint_as_float(r[c + 2]), __uint_as_float(r[c + 3]));
      } else {
        if (lane == 0) mbar_arrive_cluster(acce_leader);
        const int row = mp * 256 + static_cast<int>(prank) * 128 + q * 32 + lane;
        pair_store_row<C::CW>(P, r, row, nb * C::BN + half * C::CW);
        if (P.peers.n > 0)
          pair_push_rows_to_peers<C::CW>(P, row - lane, nb * C::BN + half * C::CW);
      }
      aph ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();   // KS: every pair's partial is parked and visible (release/acquire)
  if constexpr (KS) {
    // CTA (slice p, pair rank pr) finishes rows [128 p / S, 128 (p+1) / S)
    // of its half of the tile: partials of the S pairs summed in slice order.
    int mp, nb;
    pair_tile_coords(P, pair, mp, nb);
    const int S = P.splits;
    const int r0 = kBlockM * split / S;
    const int r1 = kBlockM * (split + 1) / S;
    constexpr int NV = C::BN / 4;
    const float* red = reinterpret_cast<const float*>(smem);
    for (int idx = threadIdx.x; idx < (r1 - r0) * NV; idx += kPairThreads) {
      const int rl = r0 + idx / NV;
      const int cg = idx - (idx / NV) * NV;
      const uint32_t la = smem_u32(red + rl * C::RS + cg * 4);
      float4 acc = ld_dsmem_f4(mapa_shared(la, prank));
      for (int sp = 1; sp < S; ++sp) {
        const float4 v = ld_dsmem_f4(mapa_shared(la, 2u * static_cast<uint32_t>(sp) + prank));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int row = mp * 256 + static_cast<int>(prank) * 128 + rl;
      if (row >= P.m) continue;
      const bool hb = P.bias != nullptr;
      const float b = hb ? P.bias[row] : 0.0f;
      float4 o = make_float4(epi_value(acc.x, P.alpha, b, hb, P.act),
                             epi_value(acc.y, P.alpha, b, hb, P.act),
                             epi_value(acc.z, P.alpha, b, hb, P.act),
                             epi_value(acc.w, P.alpha, b, hb, P.act));
      const int col = nb * C::BN + cg * 4;
      if (P.gate_from_c) {
        if (col + 0 < P.n) o.x *= load_c(P, row, col + 0);
        if (col + 1 < P.n) o.y *= load_c(P, row, col + 1);
        if (col + 2 < P.n) o.z *= load_c(P, row, col + 2);
        if (col + 3 < P.n) o.w *= load_c(P, row, col + 3);
      }
      store_vec4(P, o, row, col);
    }
    // No CTA leaves (releasing its shared memory) while others still read it.
    cluster_sync();
  }
  if (P.peers.n > 0) __threadfence_system();   // peer stores visible before completion
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && abort_sh != 0 && P.status != nullptr) atomicExch(P.status, 1);
#endif
}

// tmA2 / tmE2: W_up's A_c and metadata maps (gated form); the plain form
// passes tmA / tmE again.
template <int DT, int FINE, int BNP, int G>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    sp24_gemm2sm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmE,
                        const __grid_constant__ CUtensorMap tmA2,
                        const __grid_constant__ CUtensorMap tmE2, const PairParams P) {
  pair_gemm_body<DT, FINE, BNP, 0, G>(tmA, tmB, tmE, tmA2, tmE2, P);
}

// K-split form: launched with a run-time cluster of 2 * P.splits CTAs.
template <int DT, int BNP>
__global__ void __launch_bounds__(kPairThreads, 1)
    sp24_gemm2sm_splitk_kernel(const __grid_constant__ CUtensorMap tmA,
                               const __grid_constant__ CUtensorMap tmB,
                               const __grid_constant__ CUtensorMap tmE, const PairParams P) {
  pair_gemm_body<DT, 0, BNP, 1, 1>(tmA, tmB, tmE, tmA, tmE, P);
}

}  // namespace sp24
