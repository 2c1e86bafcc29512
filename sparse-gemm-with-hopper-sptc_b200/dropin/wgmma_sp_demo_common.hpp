// wgmma_sp_demo_common.hpp — drop-in replacement for the reference's CuTe
// harness header of the same name (codes1gn/sparse-gemm-with-hopper-sptc,
// wgmma_sp_demo_common.hpp:408-549), served by the sm_100a sp24 library.
//
// The reference's per-shape wrappers (mma_sp_wgmma_m64n{8,16,32}k32_fp32
// {fp16,bf16}.cu) name their instruction through CuTe's SM90 sparse GMMA atom
// types, e.g.
//   WgmmaSparseDemo<half_t, half_t,
//                   SM90::GMMA::SPARSE::GMMA_64x16x32_F32F16F16_SS<
//                       SM90::GMMA::Major::K, SM90::GMMA::Major::MN>, 16>
// This header provides those names as plain tag types (no CuTe, no CUTLASS:
// the atom only selects element type and tile width and is checked against
// the template arguments), plus WgmmaSparseDemo / DemoCase / run_demo_suite
// with the reference's semantics: same shape rule (M%64, N%BlockN, K%32),
// same mt19937(1234) suite stream, abs 1e-2 verification, exit codes.  The
// GEMM runs through sp24_gemm (tcgen05.mma.sp) on sm_100.
#pragma once

#include "sp24_host_utils.hpp"

namespace sp24_cute {

using half_t = __half;
using bfloat16_t = __nv_bfloat16;
using float_e4m3_t = __nv_fp8_e4m3;

namespace SM90 {
namespace GMMA {
enum class Major { K = 0, MN = 1 };
namespace SPARSE {
// Tag for a sparse GMMA atom: A/B element, N tile, dense K per instruction.
template <class EA, class EB, int N_, int K_>
struct SparseAtomTag {
  using ElementA = EA;
  using ElementB = EB;
  static constexpr int kN = N_;
  static constexpr int kK = K_;
};
#define SP24_SPARSE_ATOMS(N)                                                                    \
  template <Major tA = Major::K, Major tB = Major::K>                                           \
  struct GMMA_64x##N##x32_F32F16F16_SS : SparseAtomTag<half_t, half_t, N, 32> {};               \
  template <Major tA = Major::K, Major tB = Major::K>                                           \
  struct GMMA_64x##N##x32_F32BF16BF16_SS : SparseAtomTag<bfloat16_t, bfloat16_t, N, 32> {};     \
  template <Major tA = Major::K, Major tB = Major::K>                                           \
  struct GMMA_64x##N##x64_F32E4M3E4M3_SS_TN : SparseAtomTag<float_e4m3_t, float_e4m3_t, N, 64> {};
SP24_SPARSE_ATOMS(8)
SP24_SPARSE_ATOMS(16)
SP24_SPARSE_ATOMS(24)
SP24_SPARSE_ATOMS(32)
SP24_SPARSE_ATOMS(40)
SP24_SPARSE_ATOMS(48)
SP24_SPARSE_ATOMS(56)
SP24_SPARSE_ATOMS(64)
SP24_SPARSE_ATOMS(72)
SP24_SPARSE_ATOMS(80)
SP24_SPARSE_ATOMS(88)
SP24_SPARSE_ATOMS(96)
SP24_SPARSE_ATOMS(104)
SP24_SPARSE_ATOMS(112)
SP24_SPARSE_ATOMS(120)
SP24_SPARSE_ATOMS(128)
SP24_SPARSE_ATOMS(136)
SP24_SPARSE_ATOMS(144)
SP24_SPARSE_ATOMS(152)
SP24_SPARSE_ATOMS(160)
SP24_SPARSE_ATOMS(168)
SP24_SPARSE_ATOMS(176)
SP24_SPARSE_ATOMS(184)
SP24_SPARSE_ATOMS(192)
SP24_SPARSE_ATOMS(200)
SP24_SPARSE_ATOMS(208)
SP24_SPARSE_ATOMS(216)
SP24_SPARSE_ATOMS(224)
SP24_SPARSE_ATOMS(232)
SP24_SPARSE_ATOMS(240)
SP24_SPARSE_ATOMS(248)
SP24_SPARSE_ATOMS(256)
#undef SP24_SPARSE_ATOMS
}  // namespace SPARSE
}  // namespace GMMA
}  // namespace SM90

}  // namespace sp24_cute

using namespace sp24_cute;

template <typename ElementA_, typename ElementB_, typename MmaOp_, int BlockN_>
struct WgmmaSparseDemo {
  using ElementA = ElementA_;
  using ElementB = ElementB_;
  using ElementC = float;
  using MmaOp = MmaOp_;
  static constexpr int kBlockM = 64;
  static constexpr int kBlockN = BlockN_;
  static constexpr int kBlockK = MmaOp::kK;
  static constexpr int kSparseK = kBlockK / 2;
  static constexpr int kMetaBytes = kBlockK / 8;
  static_assert(std::is_same_v<ElementA, ElementB>, "A and B share one element type");
  static_assert(std::is_same_v<ElementA, typename MmaOp::ElementA>,
                "element type must match the MMA atom");
  static_assert(MmaOp::kN == BlockN_, "BlockN must match the MMA atom's N");

  static bool run_case(const std::string& tag, int m, int n, int k, bool use_pattern,
                       std::mt19937& gen) {
    if ((m % kBlockM) != 0 || (n % kBlockN) != 0 || (k % kBlockK) != 0) {
      std::cerr << tag << " requires M%64==0, N%" << kBlockN << "==0, K%" << kBlockK << "==0"
                << std::endl;
      return false;
    }
    return sp24_dropin::run_sp24_case<ElementA>(tag, m, n, k, use_pattern, gen, kBlockN);
  }
};

struct DemoCase {
  const char* tag;
  int m;
  int n;
  int k;
  bool use_pattern;
};

template <typename Demo, size_t NumCases>
int run_demo_suite(const char* instruction, DemoCase const (&cases)[NumCases]) {
  const int device = select_best_device();
  if (device < 0) {
    std::cout << "No sm_100 (B200-class) GPU with available memory was found." << std::endl;
    return 0;
  }
  cudaDeviceProp props{};
  CHECK_CUDA(cudaGetDeviceProperties(&props, device));
  std::cout << "Sparse WGMMA demo: " << instruction << " on device " << device << " ("
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
