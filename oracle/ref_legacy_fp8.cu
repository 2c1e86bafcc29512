// ref_legacy_fp8.cu — TEST INFRASTRUCTURE ONLY.  Compiles the reference's
// mixed fp8 entry point, mma_sp_m16n8k64_fp32fp8.cu (included from the
// reference checkout where it lies; nothing is copied), into
// oracle/_ref/libsp24ref_fp8.so, so that tests/golden/make_golden.py can record
// what its own host code produces for every case of its suite.
//
// Only host functions of that file are called, in the order its run_one()
// calls them (:350-593): the A / B generators (:33-124), quantize_fp8
// (:126-130), cpu_gemm_ref_fp8 (:132-150) and compress_matrix_host_fp8_k64
// (:152-193).  Its kernels are compiled but never launched; its main() is
// renamed out of the way.
#define main sp24_reference_legacy_fp8_main
#include "mma_sp_m16n8k64_fp32fp8.cu"
#undef main

#include <cstring>
#include <functional>
#include <string>

namespace {

using Fill = std::function<void(std::vector<float>&)>;

struct LegacyCase {
  std::string tag;
  Fill a, b;
  bool sorted;
};

// run_one's case list, in its order.  Random generators share one
// mt19937(123), as in run_one.
std::vector<LegacyCase> legacy_cases(std::mt19937& gen) {
  std::vector<LegacyCase> cs;
  auto pat = [](int i0, int i1, bool neg) -> Fill {
    return [=](std::vector<float>& A) { init_structured_sparse_A_pattern(A, i0, i1, neg); };
  };
  auto onehot = [](int off, float v) -> Fill {
    return [=](std::vector<float>& B) { init_onehot_B_f32_colmajor(B, off, v); };
  };
  for (int off = 0; off < K; off += 8)
    cs.push_back({"pattern A(0,1) + onehot B (k=" + std::to_string(off) + ".." +
                      std::to_string(off + 7) + ")",
                  pat(0, 1, false), onehot(off, 1.0f), true});
  cs.push_back({"pattern A(2,3) + onehot B (k=0..7)", pat(2, 3, false), onehot(0, 1.0f), true});
  cs.push_back({"pattern A(0,2) + onehot B (k=0..7)", pat(0, 2, false), onehot(0, 1.0f), true});
  cs.push_back({"pattern A(0,3) + onehot B (k=0..7)", pat(0, 3, false), onehot(0, 1.0f), true});
  cs.push_back({"pattern A(1,2) + onehot B (k=0..7)", pat(1, 2, false), onehot(0, 1.0f), true});
  cs.push_back({"pattern A(1,3) + onehot B (k=0..7)", pat(1, 3, false), onehot(0, 1.0f), true});
  cs.push_back({"pattern A(0,1) neg + onehot B (k=0..7)", pat(0, 1, true), onehot(0, 1.0f), true});
  cs.push_back({"pattern A(0,1) + onehot B -1 (k=0..7)", pat(0, 1, false), onehot(0, -1.0f), true});
  cs.push_back({"pattern A(0,1) + twohot B (k=0,1)", pat(0, 1, false),
                [](std::vector<float>& B) { init_twohot_B_f32_colmajor(B, 0, 1, 1.0f); }, true});
  Fill ra = [&gen](std::vector<float>& A) { init_structured_sparse_A_f32(A, gen); };
  cs.push_back({"mma.sp.m16n8k64.fp32.e5m2.e4m3", ra,
                [&gen](std::vector<float>& B) { init_random_B_f32_colmajor(B, gen); }, true});
  cs.push_back({"random A/B (unsorted idx)", ra,
                [&gen](std::vector<float>& B) { init_random_B_f32_colmajor(B, gen); }, false});
  cs.push_back({"random B discrete", ra,
                [&gen](std::vector<float>& B) { init_random_B_f32_colmajor_discrete(B, gen); },
                true});
  cs.push_back({"random B sparse2", ra,
                [&gen](std::vector<float>& B) { init_sparse_B_f32_colmajor(B, gen, 2); }, true});
  cs.push_back({"random B sparse8", ra,
                [&gen](std::vector<float>& B) { init_sparse_B_f32_colmajor(B, gen, 8); }, true});
  cs.push_back({"scalar load path", ra,
                [&gen](std::vector<float>& B) { init_random_B_f32_colmajor(B, gen); }, true});
  return cs;
}

}  // namespace

extern "C" {

int ref_fp8_suite_size() {
  std::mt19937 gen(123);
  return static_cast<int>(legacy_cases(gen).size());
}

// Per case: a_out 16x64 e5m2 bits (the quantised dense A), bt_out 8x64 e4m3
// bits (B column-major, as the reference keeps it), ac_out 16x32 e5m2 bits,
// e_out 16x2 metadata words, c_out 16x8 fp32 (cpu_gemm_ref_fp8).  tags: one
// NUL-padded name of tag_len bytes per case.  Returns the number of cases.
int ref_fp8_suite(uint8_t* a_out, uint8_t* bt_out, uint8_t* ac_out, uint32_t* e_out, float* c_out,
                  char* tags, int tag_len) {
  std::mt19937 gen(123);
  const std::vector<LegacyCase> cs = legacy_cases(gen);
  int i = 0;
  for (const LegacyCase& c : cs) {
    std::vector<float> a_f32, b_f32;
    c.a(a_f32);
    c.b(b_f32);
    std::vector<__nv_fp8_e5m2> a_fp8;
    std::vector<__nv_fp8_e4m3> b_fp8;
    quantize_fp8(a_f32, a_fp8);
    quantize_fp8(b_f32, b_fp8);
    std::vector<float> c_ref;
    cpu_gemm_ref_fp8(a_fp8, b_fp8, c_ref);
    std::vector<__nv_fp8_e5m2> a_sparse;
    std::vector<uint32_t> e;
    compress_matrix_host_fp8_k64(a_f32, a_sparse, e, c.sorted);
    std::memcpy(a_out + static_cast<size_t>(i) * M * K, a_fp8.data(), M * K);
    std::memcpy(bt_out + static_cast<size_t>(i) * N * K, b_fp8.data(), N * K);
    std::memcpy(ac_out + static_cast<size_t>(i) * M * (K / 2), a_sparse.data(), M * (K / 2));
    std::memcpy(e_out + static_cast<size_t>(i) * M * 2, e.data(), M * 2 * sizeof(uint32_t));
    std::memcpy(c_out + static_cast<size_t>(i) * M * N, c_ref.data(), M * N * sizeof(float));
    std::memset(tags + static_cast<size_t>(i) * tag_len, 0, tag_len);
    std::strncpy(tags + static_cast<size_t>(i) * tag_len, c.tag.c_str(), tag_len - 1);
    ++i;
  }
  return i;
}

}  // extern "C"
