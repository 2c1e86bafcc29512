// sp24_prep.cuh — memory-bound companion kernels of the 2:4 GEMM:
//   compress   dense 2:4 A -> A_c + reference-layout metadata
//              (reference: compress_structured_sparse_a,
//               wgmma_sp_raw_common.hpp:140-205)
//   prune      magnitude 2-of-4 pruning (no reference counterpart)
//   repack     reference metadata -> tcgen05 TMEM image
//   amax / quantize   per-tensor fp8 scaling (reference: quantize_fp8_kernel,
//              mma_sp_m16n8k64_fp32fp8.cu:341-347, and the per-tensor
//              448/amax scale of the e4m3 benchmark configuration)
//   unshard    column-block -> row-major permute after a C all-gather
//
// All of them move bytes and never touch tensor cores; they are sized for
// coalesced 16-byte accesses where the layout allows.
#pragma once

#include <cuda_fp8.h>
#include <stdint.h>

namespace sp24 {

// "Nonzero" exactly as the reference tests it: elem_to_float(x) != 0.0f
// (wgmma_sp_raw_common.hpp:156).  For every supported encoding that is
// "any bit other than the sign bit set" (NaN counts as nonzero).
template <int ESZ>
__device__ __forceinline__ bool nz_bits(uint32_t v) {
  if constexpr (ESZ == 2) return (v & 0x7FFFu) != 0;
  else return (v & 0x7Fu) != 0;
}

// Magnitude key for the pruner.  dt: 0 f16, 1 bf16, 2 any fp8 (e4m3, e5m2).
// The fp8 formats are sign-magnitude with the exponent above the mantissa, so
// the seven magnitude bits order exactly like |x| (finite values): the key is
// those bits, which serves both formats.
template <int DT>
__device__ __forceinline__ float mag_bits(uint32_t v) {
  if constexpr (DT == 0) {
    return fabsf(__half2float(__ushort_as_half(static_cast<unsigned short>(v))));
  } else if constexpr (DT == 1) {
    return fabsf(__uint_as_float(v << 16));
  } else {
    return static_cast<float>(v & 0x7Fu);
  }
}

// One thread per chunk of 8 dense elements (two groups -> one metadata byte).
// ESZ = element bytes; elements are moved as raw bits so values stay bit-exact.
template <int ESZ>
__global__ void compress_kernel(const uint8_t* __restrict__ a, int m, int k, long long lda_b,
                                uint8_t* __restrict__ ac, long long ldac_b,
                                uint8_t* __restrict__ meta, unsigned long long* __restrict__ bad) {
  const int chunks = k / 8;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(m) * chunks) return;
  const int row = static_cast<int>(idx / chunks);
  const int ch = static_cast<int>(idx - static_cast<long long>(row) * chunks);
  const uint8_t* src = a + row * lda_b + static_cast<long long>(ch) * 8 * ESZ;
  uint32_t e[8];
  if constexpr (ESZ == 2) {
    const uint4 v = *reinterpret_cast<const uint4*>(src);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) e[2 * i] = w[i] & 0xFFFFu, e[2 * i + 1] = w[i] >> 16;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    const uint32_t w[2] = {v.x, v.y};
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
  }
  uint32_t out[4];
  uint32_t nib[2];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    int i0 = -1, i1 = -1, nz = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (nz_bits<ESZ>(e[4 * g + i])) {
        if (nz == 0) i0 = i;
        else if (nz == 1) i1 = i;
        ++nz;
      }
    }
    if (nz != 2) {
      atomicMin(bad, static_cast<unsigned long long>(row) * (k / 4) + 2 * ch + g);
      i0 = 0, i1 = 1;  // keep going; the call reports the error
    }
    out[2 * g] = e[4 * g + i0];
    out[2 * g + 1] = e[4 * g + i1];
    nib[g] = static_cast<uint32_t>(i0 | (i1 << 2));
  }
  uint8_t* dst = ac + row * ldac_b + static_cast<long long>(ch) * 4 * ESZ;
  if constexpr (ESZ == 2) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(out[0] | (out[1] << 16), out[2] | (out[3] << 16));
  } else {
    *reinterpret_cast<uint32_t*>(dst) = out[0] | (out[1] << 8) | (out[2] << 16) | (out[3] << 24);
  }
  meta[static_cast<long long>(row) * (k / 8) + ch] = static_cast<uint8_t>(nib[0] | (nib[1] << 4));
}

// Magnitude pruning: keep the two largest |x| per group of four; ties keep
// the lower index; the other two become +0.
template <int DT>
__global__ void prune_kernel(const uint8_t* __restrict__ a, int m, int k, long long lda_b,
                             uint8_t* __restrict__ p, long long ldp_b) {
  constexpr int ESZ = DT == 2 ? 1 : 2;
  const int groups = k / 4;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(m) * groups) return;
  const int row = static_cast<int>(idx / groups);
  const int g = static_cast<int>(idx - static_cast<long long>(row) * groups);
  const uint8_t* src = a + row * lda_b + static_cast<long long>(g) * 4 * ESZ;
  uint32_t e[4];
  if constexpr (ESZ == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    e[0] = v.x & 0xFFFFu, e[1] = v.x >> 16, e[2] = v.y & 0xFFFFu, e[3] = v.y >> 16;
  } else {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(src);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = (v >> (8 * i)) & 0xFFu;
  }
  float mg[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) mg[i] = mag_bits<DT>(e[i]);
  int b0 = 0;
#pragma unroll
  for (int i = 1; i < 4; ++i)
    if (mg[i] > mg[b0]) b0 = i;
  int b1 = (b0 == 0) ? 1 : 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (i != b0 && mg[i] > mg[b1]) b1 = i;
  uint8_t* dst = p + row * ldp_b + static_cast<long long>(g) * 4 * ESZ;
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = (i == b0 || i == b1) ? e[i] : 0u;
  if constexpr (ESZ == 2) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(o[0] | (o[1] << 16), o[2] | (o[3] << 16));
  } else {
    *reinterpret_cast<uint32_t*>(dst) = o[0] | (o[1] << 8) | (o[2] << 16) | (o[3] << 24);
  }
}

// Reference metadata (row-major, k/8 bytes per row) -> tcgen05 image.
// Image: [k_atoms][m_blocks][128 lanes][4 x u32]; one atom covers 128 rows x
// 128 dense K; m_blocks = ceil(m/128) rounded up to even so that a CTA pair's
// second 128 rows always have an atom.  Word w of lane L is TMEM column w.
//  16-bit types (kind::f16, one column per K=32 MMA):
//    L = 16*m2 + 8*k1 + m0;  bits [0,16)  = row 16*m2 + m0,     K [32w+16k1, +16)
//                            bits [16,32) = row 16*m2 + 8 + m0, same K range
//  e4m3 (kind::f8f6f4, two columns per K=64 MMA):
//    lane L = row L; the 16 bytes are the row's 16 reference bytes of the atom.
// Groups outside [0,m) x [0,k) get the valid code 0x4 (indices 0,1).
// k16 != nullptr: the source is the reference's m16n8k16 layout instead
// (16-bit types, m % 16 == 0): u32 words [k/16 strips][m/2], word (s, 8b+i)
// holding row 16b+i's four nibbles of strip s in bits 0-15 and row 16b+8+i's
// in bits 16-31 (mma_sp_m16n8k16_fp32fp16.cu:96-110, strips concatenated at
// :277-297).  That pairing of rows r and r+8 per 16-row block is exactly the
// lane pairing of the 16-bit TMEM image, so each image word is one k16 word.
__global__ void repack_meta_kernel(const uint8_t* __restrict__ ref, int m, int k, int is8,
                                   uint32_t* __restrict__ img, int m_blocks, int k_atoms,
                                   const uint32_t* __restrict__ k16 = nullptr) {
  const long long total = static_cast<long long>(k_atoms) * m_blocks * 128 * 4;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int w = static_cast<int>(idx & 3);
  const int L = static_cast<int>((idx >> 2) & 127);
  const long long blk = idx >> 9;
  const int mb = static_cast<int>(blk % m_blocks);
  const int ka = static_cast<int>(blk / m_blocks);
  const int rb = k / 8;  // reference bytes per row
  uint32_t word;
  if (is8) {
    const int row = mb * 128 + L;
    const int byte0 = ka * 16 + 4 * w;  // 4 bytes = 32 dense K
    if (row < m && byte0 < rb) {
      const uint8_t* s = ref + static_cast<long long>(row) * rb + byte0;
      word = s[0] | (s[1] << 8) | (s[2] << 16) | (static_cast<uint32_t>(s[3]) << 24);
    } else {
      word = 0x44444444u;
    }
  } else if (k16 != nullptr) {
    const int m2 = L >> 4, k1 = (L >> 3) & 1, m0 = L & 7;
    const int kr = ka * 128 + 32 * w + 16 * k1;
    const int row = mb * 128 + 16 * m2 + m0;  // its partner row + 8 is valid with it
    word = (row < m && kr < k)
               ? k16[static_cast<long long>(kr / 16) * (m / 2) + (mb * 128 + 16 * m2) / 2 + m0]
               : 0x44444444u;
  } else {
    const int m2 = L >> 4, k1 = (L >> 3) & 1, m0 = L & 7;
    const int kr = ka * 128 + 32 * w + 16 * k1;  // dense K start of the 16-element run
    const int byte0 = kr / 8;
    uint32_t half[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = mb * 128 + 16 * m2 + 8 * h + m0;
      if (row < m && kr < k) {
        const uint8_t* s = ref + static_cast<long long>(row) * rb + byte0;
        half[h] = s[0] | (s[1] << 8);
      } else {
        half[h] = 0x4444u;
      }
    }
    word = half[0] | (half[1] << 16);
  }
  img[idx] = word;
}

__global__ void amax_kernel(const float* __restrict__ x, size_t n, float* __restrict__ amax) {
  float v = 0.f;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    v = fmaxf(v, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    // |x| >= 0, so the IEEE bit pattern orders like an unsigned integer.
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(v));
  }
}

// Per-tensor fp8 quantisation: scale = largest finite value / amax
// (448 for e4m3, 57344 for e5m2), q = fp8_rn_satfinite(x * scale).
template <int E5M2>
__global__ void quantize_fp8_kernel(const float* __restrict__ x, size_t n,
                                    const float* __restrict__ amax, float* __restrict__ scale_out,
                                    uint8_t* __restrict__ q) {
  constexpr float kMax = E5M2 ? 57344.0f : 448.0f;
  constexpr __nv_fp8_interpretation_t kFmt = E5M2 ? __NV_E5M2 : __NV_E4M3;
  const float am = amax[0];
  const float s = am > 0.f ? kMax / am : 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0 && scale_out != nullptr) scale_out[0] = s;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    q[i] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(x[i] * s, __NV_SATFINITE, kFmt));
}

// dst[r][c] = shard(c)[r][c - n0(shard)] where shard r's block starts at
// element offset m * n0(r) in src.
__global__ void unshard_columns_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                       int m, int n, int world, int per, int vec) {
  // Rows are spread over blockIdx.y, columns over x; with vec every 4-column
  // group lies inside one shard (per % 4 == 0, n % 4 == 0) and moves as one
  // 16-byte access.
  const int step = gridDim.x * blockDim.x;
  for (int r = blockIdx.y; r < m; r += gridDim.y) {
    float* drow = dst + static_cast<long long>(r) * n;
    if (vec) {
      for (int c = 4 * (blockIdx.x * blockDim.x + threadIdx.x); c < n; c += 4 * step) {
        const int g = min(c / per, world - 1);
        const int n0 = g * per;
        const int w = min(per, n - n0);
        const float4 v = *reinterpret_cast<const float4*>(
            src + static_cast<long long>(m) * n0 + static_cast<long long>(r) * w + (c - n0));
        *reinterpret_cast<float4*>(drow + c) = v;
      }
    } else {
      for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += step) {
        const int g = min(c / per, world - 1);
        const int n0 = g * per;
        const int w = min(per, n - n0);
        drow[c] = src[static_cast<long long>(m) * n0 + static_cast<long long>(r) * w + (c - n0)];
      }
    }
  }
}

}  // namespace sp24
