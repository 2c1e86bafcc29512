// ref_legacy_mma_sp.cu — TEST INFRASTRUCTURE ONLY.  Compiles the reference's
// four legacy warp-level entry points (mma_sp_m16n8k16_fp32{fp16,bf16}.cu and
// mma_sp_m16n8k32_fp32{fp16,bf16}.cu, included from the reference checkout
// where they lie, each inside its own namespace; nothing is copied) into
// oracle/_ref/libsp24ref_legacy.so, so that tests/golden/make_golden.py can
// record what their own host code produces.
//
// ref_legacy_case replays a main() of those files at a chosen size: the
// mt19937(42) generation in that main's order, its compress_matrix_host, and
// for the m16n8k16 files the main's per-16-column-strip compression with the
// strips' metadata concatenated (:277-297 of the fp16 file).  C is the fp32
// sequential CPU product the mains verify against (their inline loops).  The
// main()s are renamed away.
//
// ref_legacy_launch runs the files' own kernels (warp-level mma.sp, which
// sm_100a still executes) the way their mains launch them: the LOAD_METHOD
// the main picks, grid (N/64, M/64), 256 threads.  Dynamic shared memory is
// 32 KB for all four.  The m16n8k32 fp16 main passes 6272 B (:457-458), less
// than its kernel's own footprint of 6400 B (A 2 KB + B 4 KB + 64 metadata
// words, :317-320), so this launcher does not copy that value.  Every global
// access of these kernels is bounds-checked against M, N and K
// (e.g. mma_sp_m16n8k32_fp32bf16.cu:258-276, 308-316).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <random>
#include <vector>

#define main legacy_main
namespace k16_f16 {
#include "mma_sp_m16n8k16_fp32fp16.cu"
}
namespace k16_bf16 {
#include "mma_sp_m16n8k16_fp32bf16.cu"
}
#undef CHECK_CUDA
#undef LOAD_METHOD_LDMATRIX
#undef LOAD_METHOD_MANUAL
namespace k32_f16 {
#include "mma_sp_m16n8k32_fp32fp16.cu"
}
namespace k32_bf16 {
#include "mma_sp_m16n8k32_fp32bf16.cu"
}
#undef main

namespace {

float to_f(half v) { return __half2float(v); }
float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

// The mains' verification product (e.g. mma_sp_m16n8k16_fp32fp16.cu:337-344,
// mma_sp_m16n8k32_fp32bf16.cu:366-372): per element, fp32 sum over l in order
// of float(A[r][l]) * float(B[l][c]).
template <typename T>
void main_verify_c(const T* a, const T* b, float* c, int m, int n, int k) {
  for (int r = 0; r < m; ++r)
    for (int col = 0; col < n; ++col) {
      float ref = 0.0f;
      for (int l = 0; l < k; ++l)
        ref += to_f(a[static_cast<size_t>(r) * k + l]) * to_f(b[static_cast<size_t>(l) * n + col]);
      c[static_cast<size_t>(r) * n + col] = ref;
    }
}

template <typename T>
T from_f(float v);
template <>
half from_f<half>(float v) { return __float2half(v); }
template <>
__nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

// The m16n8k16 mains (:257-310 of the fp16 file): A through its
// init_structured_sparse_A, then B from U(-1,1), then compression strip by
// strip of 16 columns; metadata words [k/16][m/2], A_c row-major.
template <typename T, typename InitA, typename Compress>
void k16_main(InitA init_a, Compress compress, int m, int n, int k, T* a, T* b, T* ac,
              uint32_t* e) {
  std::vector<T> a_dense(static_cast<size_t>(m) * k), bv(static_cast<size_t>(k) * n);
  std::mt19937 gen(42);
  std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
  init_a(a_dense, m, k, gen);
  for (size_t i = 0; i < bv.size(); ++i) bv[i] = from_f<T>(dist(gen));
  for (int strip = 0; strip < k / 16; ++strip) {
    std::vector<T> sa(static_cast<size_t>(m) * 16);
    for (int r = 0; r < m; ++r)
      for (int c = 0; c < 16; ++c) sa[r * 16 + c] = a_dense[static_cast<size_t>(r) * k + strip * 16 + c];
    std::vector<T> ss;
    std::vector<uint32_t> se;
    compress(sa, ss, se, m, 16);
    for (int r = 0; r < m; ++r)
      for (int c = 0; c < 8; ++c) ac[static_cast<size_t>(r) * (k / 2) + strip * 8 + c] = ss[r * 8 + c];
    for (int i = 0; i < m / 2; ++i) e[static_cast<size_t>(strip) * (m / 2) + i] = se[i];
  }
  std::memcpy(a, a_dense.data(), a_dense.size() * sizeof(T));
  std::memcpy(b, bv.data(), bv.size() * sizeof(T));
}

// The m16n8k32 mains (:414-438 of the fp16 file): A and B filled from
// U(-1,1), then A overwritten by init_structured_sparse_A, then one
// compression; metadata words [m][k/32].
template <typename T, typename InitA, typename Compress>
void k32_main(InitA init_a, Compress compress, int m, int n, int k, T* a, T* b, T* ac,
              uint32_t* e) {
  std::vector<T> a_dense(static_cast<size_t>(m) * k), bv(static_cast<size_t>(k) * n);
  std::mt19937 gen(42);
  std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
  for (size_t i = 0; i < a_dense.size(); ++i) a_dense[i] = from_f<T>(dist(gen));
  for (size_t i = 0; i < bv.size(); ++i) bv[i] = from_f<T>(dist(gen));
  init_a(a_dense, m, k, gen);
  std::vector<T> ss;
  std::vector<uint32_t> se;
  compress(a_dense, ss, se, m, k);
  std::memcpy(a, a_dense.data(), a_dense.size() * sizeof(T));
  std::memcpy(b, bv.data(), bv.size() * sizeof(T));
  std::memcpy(ac, ss.data(), ss.size() * sizeof(T));
  std::memcpy(e, se.data(), se.size() * sizeof(uint32_t));
}

}  // namespace

extern "C" {

// which: 0 m16n8k16 fp16, 1 m16n8k16 bf16, 2 m16n8k32 fp16, 3 m16n8k32 bf16.
// a (m x k), b (k x n), ac (m x k/2) as 16-bit patterns; e: m*k/32 words (the
// same count in both layouts); c (m x n fp32) or NULL to skip the CPU GEMM.
int ref_legacy_case(int which, int m, int n, int k, void* a, void* b, void* ac, uint32_t* e,
                    float* c) {
  if (m % 16 || k % 32 || m <= 0 || n <= 0) return -1;
  switch (which) {
    case 0:
      k16_main<half>(k16_f16::init_structured_sparse_A, k16_f16::compress_matrix_host, m, n, k,
                     static_cast<half*>(a), static_cast<half*>(b), static_cast<half*>(ac), e);
      break;
    case 1:
      k16_main<__nv_bfloat16>(k16_bf16::init_structured_sparse_A, k16_bf16::compress_matrix_host,
                              m, n, k, static_cast<__nv_bfloat16*>(a),
                              static_cast<__nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(ac), e);
      break;
    case 2:
      k32_main<half>(k32_f16::init_structured_sparse_A, k32_f16::compress_matrix_host, m, n, k,
                     static_cast<half*>(a), static_cast<half*>(b), static_cast<half*>(ac), e);
      break;
    case 3:
      k32_main<__nv_bfloat16>(k32_bf16::init_structured_sparse_A, k32_bf16::compress_matrix_host,
                              m, n, k, static_cast<__nv_bfloat16*>(a),
                              static_cast<__nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(ac), e);
      break;
    default:
      return -1;
  }
  if (c != nullptr) {
    if (which == 0 || which == 2)
      main_verify_c(static_cast<const half*>(a), static_cast<const half*>(b), c, m, n, k);
    else
      main_verify_c(static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), c,
                    m, n, k);
  }
  return 0;
}

// Launches the reference kernel of legacy main `which` on `stream` over
// device buffers in that main's formats: a_c M x K/2, b K x N, e as
// ref_legacy_case describes, c M x N fp32 (all row-major, dense pitches).
// Returns the launch's cudaError_t, or -1 for a shape the kernels do not
// tile (M and N multiples of 64, K of 32).
int ref_legacy_launch(int which, const void* a_c, const void* b, float* c, const uint32_t* e,
                      int m, int n, int k, void* stream) {
  if (m <= 0 || n <= 0 || k <= 0 || m % 64 || n % 64 || k % 32) return -1;
  const dim3 grid(n / 64, m / 64), block(256);
  const int smem = 32768;
  // The mains' LOAD_METHOD_MANUAL (k16) and LOAD_METHOD_MANUAL_LANE (k32)
  // are both 2 (their macros are undefined again above).
  constexpr int kManual = 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (which) {
    case 0:
      k16_f16::mma_sp_m16n8k16_fp32fp16_kernel<kManual><<<grid, block, smem, s>>>(
          static_cast<const half*>(a_c), static_cast<const half*>(b), c, e, m, n, k);
      break;
    case 1:
      k16_bf16::mma_sp_m16n8k16_fp32bf16_kernel<kManual>
          <<<grid, block, smem, s>>>(static_cast<const __nv_bfloat16*>(a_c),
                                     static_cast<const __nv_bfloat16*>(b), c, e, m, n, k);
      break;
    case 2:
      k32_f16::mma_sp_m16n8k32_fp32fp16_kernel<kManual>
          <<<grid, block, smem, s>>>(static_cast<const half*>(a_c), static_cast<const half*>(b),
                                     c, e, m, n, k);
      break;
    case 3:
      k32_bf16::mma_sp_m16n8k32_fp32bf16_kernel<kManual>
          <<<grid, block, smem, s>>>(static_cast<const __nv_bfloat16*>(a_c),
                                     static_cast<const __nv_bfloat16*>(b), c, e, m, n, k);
      break;
    default:
      return -1;
  }
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
