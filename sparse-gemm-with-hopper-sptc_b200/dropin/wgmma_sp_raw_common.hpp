// wgmma_sp_raw_common.hpp — drop-in replacement for the reference harness
// header of the same name (codes1gn/sparse-gemm-with-hopper-sptc,
// wgmma_sp_raw_common.hpp), served by the sm_100a sp24 library.
//
// A translation unit written against the reference header (the per-dtype
// entry points mma_sp_wgmma_cuda_m64n{8..256}k{32,64}_fp32{fp16,bf16,e4m3}.cu)
// compiles unchanged against this one and links with -lsp24.  The names, the
// signatures and the observable behaviour are kept:
//   * host utilities init_* / compress_structured_sparse_a / cpu_gemm_ref /
//     verify_result / select_best_device (reference :27-291), including the
//     exact random-number call order, so seeded suites produce the same data;
//   * RawSparseConfig<T> constants (:297-331);
//   * RawWgmmaSparseDemo<Element,BlockN>::run_case, RawDemoCase and
//     run_raw_demo_suite (:1032-1136): same shape rule, messages, abs 1e-2
//     verification and exit codes.
// What changes is the device side: run_case compresses A on the GPU
// (sp24_compress, checked bit-for-bit against the host compression) and runs
// the GEMM through sp24_gemm (tcgen05.mma.sp) instead of the sm_90a wgmma
// kernel.  The device gate is sm_100 instead of sm_90.
//   * wgmma_sp_raw_kernel<Element, BlockN> (:955-1030) stays launchable with
//     the reference's signature and <<<dim3(n / BlockN, m / 64), 128>>>
//     geometry, for callers that launch it themselves: sp24_raw_kernel.cuh,
//     a tcgen05.mma.sp kernel of that shape (sp24_gemm, with its persistent
//     warp-specialised kernels, is the fast path).
#pragma once

#include "sp24_host_utils.hpp"
#include "sp24_raw_kernel.cuh"

// ------------------------------------------------------------------ configuration
constexpr int kRawBlockM = 64;
constexpr int kRawThreads = 128;
constexpr int kRawFp8MetadataSmemBytes = kRawBlockM * 8;

template <typename Element>
struct RawSparseConfig;

template <>
struct RawSparseConfig<half> {
  static constexpr int kBlockK = 32;
  static constexpr int kSparseK = kBlockK / 2;
  static constexpr int kMetaBytes = kBlockK / 8;
  static constexpr int kASmemElements = kRawBlockM * kSparseK;
  static constexpr int kESmemBytes = kRawBlockM * kMetaBytes;
  static constexpr uint32_t kADescLeading = 64;
  static constexpr uint32_t kADescStride = 8;
};
template <>
struct RawSparseConfig<__nv_bfloat16> {
  static constexpr int kBlockK = 32;
  static constexpr int kSparseK = kBlockK / 2;
  static constexpr int kMetaBytes = kBlockK / 8;
  static constexpr int kASmemElements = kRawBlockM * kSparseK;
  static constexpr int kESmemBytes = kRawBlockM * kMetaBytes;
  static constexpr uint32_t kADescLeading = 64;
  static constexpr uint32_t kADescStride = 8;
};
template <>
struct RawSparseConfig<__nv_fp8_e4m3> {
  static constexpr int kBlockK = 64;
  static constexpr int kSparseK = kBlockK / 2;
  static constexpr int kMetaBytes = kBlockK / 8;
  static constexpr int kASmemElements = kRawBlockM * kSparseK;
  static constexpr int kESmemBytes = kRawFp8MetadataSmemBytes;
  static constexpr uint32_t kADescLeading = 64;
  static constexpr uint32_t kADescStride = 8;
};

// ------------------------------------------------------------------ harness
template <typename Element, int BlockN>
struct RawWgmmaSparseDemo {
  static bool run_case(const std::string& tag, int m, int n, int k, bool use_pattern,
                       std::mt19937& gen) {
    constexpr int kBlockK = RawSparseConfig<Element>::kBlockK;
    if ((m % kRawBlockM) != 0 || (n % BlockN) != 0 || (k % kBlockK) != 0) {
      std::cerr << tag << " requires M%64==0, N%" << BlockN << "==0, K%" << kBlockK << "==0"
                << std::endl;
      return false;
    }
    return sp24_dropin::run_sp24_case<Element>(tag, m, n, k, use_pattern, gen, BlockN);
  }
};

struct RawDemoCase {
  const char* tag;
  int m;
  int n;
  int k;
  bool use_pattern;
};

template <typename Demo, size_t NumCases>
int run_raw_demo_suite(const char* instruction, RawDemoCase const (&cases)[NumCases]) {
  const int device = select_best_device();
  if (device < 0) {
    std::cout << "No sm_100 (B200-class) GPU with available memory was found." << std::endl;
    return 0;
  }
  cudaDeviceProp props{};
  CHECK_CUDA(cudaGetDeviceProperties(&props, device));
  std::cout << "Raw sparse WGMMA demo: " << instruction << " on device " << device << " ("
            << props.name << ") via " << sp24_version() << std::endl;
  std::mt19937 gen(1234);
  bool ok = true;
  for (auto const& c : cases) ok &= Demo::run_case(c.tag, c.m, c.n, c.k, c.use_pattern, gen);
  if (!ok) {
    std::cout << "Verification FAILED" << std::endl;
    return 1;
  }
  std::cout << "Verification PASSED" << std::endl;
  return 0;
}
