// sp24_host_utils.hpp — host-side utilities shared by the two drop-in
// harness headers (wgmma_sp_raw_common.hpp, wgmma_sp_demo_common.hpp).
//
// They restate the reference's host algorithms with the reference's names and
// signatures (codes1gn/sparse-gemm-with-hopper-sptc, wgmma_sp_raw_common.hpp
// :17-291 and the identical copies in wgmma_sp_demo_common.hpp :88-305) so
// that code written against either header keeps compiling and seeded suites
// keep producing the same data: the random-number call order, the value
// snapping, the metadata nibble encoding and the sequential fp32 CPU GEMM
// are all part of the observable contract.
// run_sp24_case is the device half of a suite case: GPU compression (checked
// bit-for-bit against the host compression) and the GEMM through sp24_gemm.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <random>
#include <string>
#include <type_traits>
#include <vector>

#include "sp24.h"

#define CHECK_CUDA(func)                                                                \
  {                                                                                     \
    cudaError_t sp24_err__ = (func);                                                    \
    if (sp24_err__ != cudaSuccess) {                                                    \
      std::cerr << "CUDA Error: " << cudaGetErrorString(sp24_err__) << " at line "      \
                << __LINE__ << std::endl;                                               \
      std::exit(EXIT_FAILURE);                                                          \
    }                                                                                   \
  }

// ------------------------------------------------------------------ element conversions
template <typename T>
inline float elem_to_float(T x);
template <>
inline float elem_to_float<half>(half x) { return __half2float(x); }
template <>
inline float elem_to_float<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
inline float elem_to_float<__nv_fp8_e4m3>(__nv_fp8_e4m3 x) { return static_cast<float>(x); }

template <typename T>
inline T float_to_elem(float x);
template <>
inline half float_to_elem<half>(float x) { return __float2half_rn(x); }
template <>
inline __nv_bfloat16 float_to_elem<__nv_bfloat16>(float x) { return __float2bfloat16(x); }
template <>
inline __nv_fp8_e4m3 float_to_elem<__nv_fp8_e4m3>(float x) { return __nv_fp8_e4m3(x); }

namespace sp24_dropin {
template <typename T>
constexpr sp24_dtype dtype_of() {
  if constexpr (std::is_same_v<T, half>) return SP24_F16;
  else if constexpr (std::is_same_v<T, __nv_bfloat16>) return SP24_BF16;
  else return SP24_E4M3;
}
}  // namespace sp24_dropin

// ------------------------------------------------------------------ generators
// 2:4 A: for each row and aligned group of four, two distinct positions drawn
// uniformly from {0..3} (the second redrawn until it differs), two U(-1,1)
// values with |v| < 0.1 pushed to +-0.5 / +-0.75; all other entries zero.
template <typename Element>
void init_structured_sparse_a(std::vector<Element>& a_dense, int m, int k, std::mt19937& gen) {
  std::uniform_real_distribution<float> uni(-1.0f, 1.0f);
  std::uniform_int_distribution<int> position(0, 3);
  a_dense.assign(static_cast<size_t>(m) * k, float_to_elem<Element>(0.0f));
  for (int r = 0; r < m; ++r) {
    for (int g = 0; g < k / 4; ++g) {
      int p = position(gen);
      int q = position(gen);
      while (q == p) q = position(gen);
      const int lo = std::min(p, q);
      const int hi = std::max(p, q);
      float x = uni(gen);
      float y = uni(gen);
      if (std::fabs(x) < 0.1f) x = (x < 0.0f) ? -0.5f : 0.5f;
      if (std::fabs(y) < 0.1f) y = (y < 0.0f) ? -0.75f : 0.75f;
      Element* grp = a_dense.data() + static_cast<size_t>(r) * k + 4 * g;
      grp[lo] = float_to_elem<Element>(x);
      grp[hi] = float_to_elem<Element>(y);
    }
  }
}

// Known-answer A: positions 0 and 2 of each group, values dyadic in (row, group).
template <typename Element>
void init_pattern_sparse_a(std::vector<Element>& a_dense, int m, int k) {
  a_dense.assign(static_cast<size_t>(m) * k, float_to_elem<Element>(0.0f));
  for (int r = 0; r < m; ++r)
    for (int g = 0; g < k / 4; ++g) {
      Element* grp = a_dense.data() + static_cast<size_t>(r) * k + 4 * g;
      grp[0] = float_to_elem<Element>(1.0f + 0.125f * r + 0.03125f * g);
      grp[2] = float_to_elem<Element>(-0.5f - 0.0625f * r + 0.015625f * g);
    }
}

template <typename Element>
void init_random_b(std::vector<Element>& b, int k, int n, std::mt19937& gen) {
  std::uniform_real_distribution<float> uni(-1.0f, 1.0f);
  b.resize(static_cast<size_t>(k) * n);
  for (size_t i = 0; i < b.size(); ++i) {
    float v = uni(gen);
    if (std::fabs(v) < 0.1f) v = (v < 0.0f) ? -0.25f : 0.25f;
    b[i] = float_to_elem<Element>(v);
  }
}

template <typename Element>
void init_pattern_b(std::vector<Element>& b, int k, int n) {
  b.resize(static_cast<size_t>(k) * n);
  for (int kk = 0; kk < k; ++kk)
    for (int nn = 0; nn < n; ++nn)
      b[static_cast<size_t>(kk) * n + nn] =
          float_to_elem<Element>(0.25f * static_cast<float>(kk % 7 - 3) + 0.5f * (nn + 1));
}

// ------------------------------------------------------------------ compression
// Kept values in index order into a_sparse (m x k/2); 4-bit code i0 | i1 << 2
// per group, even groups in the low nibble of byte row*(k/8) + group/2.
// A group without exactly two nonzeros aborts, as in the reference.
template <typename Element>
void compress_structured_sparse_a(const std::vector<Element>& a_dense,
                                  std::vector<Element>& a_sparse, std::vector<uint8_t>& e_bytes,
                                  int m, int k) {
  a_sparse.assign(static_cast<size_t>(m) * (k / 2), float_to_elem<Element>(0.0f));
  e_bytes.assign(static_cast<size_t>(m) * (k / 8), uint8_t{0});
  for (int r = 0; r < m; ++r)
    for (int g = 0; g < k / 4; ++g) {
      const Element* grp = a_dense.data() + static_cast<size_t>(r) * k + 4 * g;
      int pos[2] = {-1, -1};
      int count = 0;
      for (int i = 0; i < 4; ++i)
        if (elem_to_float(grp[i]) != 0.0f) {
          if (count < 2) pos[count] = i;
          ++count;
        }
      if (count != 2) {
        std::cerr << "Invalid 2:4 structure at row " << r << ", group " << g << std::endl;
        std::exit(EXIT_FAILURE);
      }
      Element* out = a_sparse.data() + static_cast<size_t>(r) * (k / 2) + 2 * g;
      out[0] = grp[pos[0]];
      out[1] = grp[pos[1]];
      const uint8_t code = static_cast<uint8_t>(pos[0] | (pos[1] << 2));
      uint8_t& byte = e_bytes[static_cast<size_t>(r) * (k / 8) + g / 2];
      byte = (g & 1) ? static_cast<uint8_t>(byte | (code << 4)) : code;
    }
}

// ------------------------------------------------------------------ CPU reference
// fp32 accumulation over k in order, on the dense A.
template <typename ElementA, typename ElementB>
void cpu_gemm_ref(const std::vector<ElementA>& a_dense, const std::vector<ElementB>& b,
                  std::vector<float>& c, int m, int n, int k) {
  c.assign(static_cast<size_t>(m) * n, 0.0f);
  for (int r = 0; r < m; ++r)
    for (int col = 0; col < n; ++col) {
      float acc = 0.0f;
      for (int kk = 0; kk < k; ++kk)
        acc += elem_to_float(a_dense[static_cast<size_t>(r) * k + kk]) *
               elem_to_float(b[static_cast<size_t>(kk) * n + col]);
      c[static_cast<size_t>(r) * n + col] = acc;
    }
}

inline int verify_result(const std::string& tag, const std::vector<float>& got,
                         const std::vector<float>& ref, int cols, float atol = 1.0e-2f) {
  int errors = 0;
  for (size_t i = 0; i < got.size(); ++i) {
    const float diff = std::fabs(got[i] - ref[i]);
    if (diff > atol) {
      ++errors;
      if (errors <= 8)
        std::cout << tag << " mismatch at (" << i / cols << "," << i % cols << ") gpu=" << got[i]
                  << " ref=" << ref[i] << " diff=" << diff << std::endl;
    }
  }
  std::cout << tag << " total errors: " << errors << std::endl;
  return errors;
}

// The sm_100 device with the most free memory (-1 if none); made current.
inline int select_best_device() {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  int best = -1;
  size_t best_free = 0;
  for (int d = 0; d < count; ++d) {
    if (sp24_check_device(d) != SP24_OK) continue;
    if (cudaSetDevice(d) != cudaSuccess || cudaFree(nullptr) != cudaSuccess) {
      (void)cudaGetLastError();
      continue;
    }
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
      (void)cudaGetLastError();
      continue;
    }
    if (best < 0 || free_b > best_free) best = d, best_free = free_b;
  }
  if (best < 0) return -1;
  CHECK_CUDA(cudaSetDevice(best));
  CHECK_CUDA(cudaFree(nullptr));
  return best;
}

namespace sp24_dropin {

// Device half of RawWgmmaSparseDemo::run_case / WgmmaSparseDemo::run_case
// (reference wgmma_sp_raw_common.hpp:1047-1094): generate, compress and
// reference-multiply on the host, then compress and multiply on the GPU and
// verify with the reference's abs 1e-2 rule.
template <typename Element>
bool run_sp24_case(const std::string& tag, int m, int n, int k, bool use_pattern,
                   std::mt19937& gen, int block_n) {
    std::vector<Element> a_dense, b;
    if (use_pattern) {
      init_pattern_sparse_a(a_dense, m, k);
      init_pattern_b(b, k, n);
    } else {
      init_structured_sparse_a(a_dense, m, k, gen);
      init_random_b(b, k, n, gen);
    }
    std::vector<Element> a_sparse;
    std::vector<uint8_t> e_bytes;
    compress_structured_sparse_a(a_dense, a_sparse, e_bytes, m, k);
    std::vector<float> c_ref;
    cpu_gemm_ref(a_dense, b, c_ref, m, n, k);

    constexpr sp24_dtype dt = sp24_dropin::dtype_of<Element>();
    Element *d_dense = nullptr, *d_a = nullptr, *d_b = nullptr;
    uint8_t* d_e = nullptr;
    float* d_c = nullptr;
    long long* d_bad = nullptr;
    void* d_ws = nullptr;
    CHECK_CUDA(cudaMalloc(&d_dense, sizeof(Element) * a_dense.size()));
    CHECK_CUDA(cudaMalloc(&d_a, sizeof(Element) * a_sparse.size()));
    CHECK_CUDA(cudaMalloc(&d_b, sizeof(Element) * b.size()));
    CHECK_CUDA(cudaMalloc(&d_e, e_bytes.size()));
    CHECK_CUDA(cudaMalloc(&d_c, sizeof(float) * c_ref.size()));
    CHECK_CUDA(cudaMalloc(&d_bad, sizeof(long long)));
    CHECK_CUDA(cudaMemcpy(d_dense, a_dense.data(), sizeof(Element) * a_dense.size(),
                          cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(d_b, b.data(), sizeof(Element) * b.size(), cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemset(d_c, 0, sizeof(float) * c_ref.size()));

    bool ok = true;
    // Compression on the GPU; must agree bit for bit with the host compression.
    long long bad = -1;
    sp24_status st = sp24_compress(dt, d_dense, m, k, 0, d_a, 0, d_e, d_bad, &bad, nullptr);
    if (st != SP24_OK) {
      std::cout << tag << " sp24_compress: " << sp24_status_string(st) << std::endl;
      ok = false;
    } else {
      std::vector<Element> a_gpu(a_sparse.size());
      std::vector<uint8_t> e_gpu(e_bytes.size());
      CHECK_CUDA(cudaMemcpy(a_gpu.data(), d_a, sizeof(Element) * a_gpu.size(),
                            cudaMemcpyDeviceToHost));
      CHECK_CUDA(cudaMemcpy(e_gpu.data(), d_e, e_gpu.size(), cudaMemcpyDeviceToHost));
      const bool same_a = std::memcmp(a_gpu.data(), a_sparse.data(),
                                      sizeof(Element) * a_gpu.size()) == 0;
      const bool same_e = std::memcmp(e_gpu.data(), e_bytes.data(), e_gpu.size()) == 0;
      if (!same_a || !same_e) {
        std::cout << tag << " GPU compression differs from host compression (values "
                  << (same_a ? "equal" : "differ") << ", metadata "
                  << (same_e ? "equal" : "differ") << ")" << std::endl;
        ok = false;
      }
    }
    if (ok) {
      sp24_gemm_desc d{};
      d.dtype = dt;
      d.m = m;
      d.n = n;
      d.k = k;
      d.a_c = d_a;
      d.meta = d_e;
      d.meta_format = SP24_META_REF;
      d.b = d_b;
      d.c_f32 = d_c;
      d.tile_n = block_n;
      d.alpha = 1.0f;
      const size_t ws = sp24_gemm_workspace_bytes(&d);
      if (ws > 0) CHECK_CUDA(cudaMalloc(&d_ws, ws));
      d.workspace = d_ws;
      d.workspace_bytes = ws;
      st = sp24_gemm(&d, nullptr);
      if (st == SP24_OK) {
        CHECK_CUDA(cudaDeviceSynchronize());
        st = sp24_last_kernel_status(nullptr);
      }
      if (st != SP24_OK) {
        std::cout << tag << " sp24_gemm: " << sp24_status_string(st) << std::endl;
        ok = false;
      }
    }
    std::vector<float> c_gpu(c_ref.size(), 0.0f);
    CHECK_CUDA(cudaMemcpy(c_gpu.data(), d_c, sizeof(float) * c_gpu.size(), cudaMemcpyDeviceToHost));
    const int errors = verify_result(tag, c_gpu, c_ref, n);

    CHECK_CUDA(cudaFree(d_dense));
    CHECK_CUDA(cudaFree(d_a));
    CHECK_CUDA(cudaFree(d_b));
    CHECK_CUDA(cudaFree(d_e));
    CHECK_CUDA(cudaFree(d_c));
    CHECK_CUDA(cudaFree(d_bad));
    if (d_ws) CHECK_CUDA(cudaFree(d_ws));
    return ok && errors == 0;
}

}  // namespace sp24_dropin
