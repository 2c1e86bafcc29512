// ref_harness.cu — TEST INFRASTRUCTURE ONLY.  Compiles the reference's own
// host code (wgmma_sp_raw_common.hpp, included from the reference checkout
// where it lies; nothing is copied) into oracle/_ref/libsp24ref.so so that
// tests/golden/make_golden.py can record its outputs and bench.py's
// `--impl reference` arm can time its CPU GEMM + compression path.
//
// Only host functions of the header are called: init_structured_sparse_a /
// init_pattern_sparse_a / init_random_b / init_pattern_b (:63-138),
// compress_structured_sparse_a (:140-205) and cpu_gemm_ref (:207-225).
// The sm_90a kernels in the header are never instantiated (they cannot run on
// sm_100).  Elements cross this ABI as raw bits (uint16 / uint8).
#include <cstring>
#include <random>
#include <thread>
#include <vector>

#include "wgmma_sp_raw_common.hpp"

namespace {

template <typename T>
void to_bits(const std::vector<T>& v, void* out) {
  std::memcpy(out, v.data(), v.size() * sizeof(T));
}
template <typename T>
std::vector<T> from_bits(const void* in, size_t count) {
  std::vector<T> v(count);
  std::memcpy(v.data(), in, count * sizeof(T));
  return v;
}

// One case of RawWgmmaSparseDemo<T,BlockN>::run_case up to (not including)
// the device launch: generation in the reference's order, compression and
// the CPU GEMM (wgmma_sp_raw_common.hpp:1047-1062).
template <typename T>
void run_host_case(std::mt19937& gen, int m, int n, int k, bool use_pattern, void* a_out,
                   void* b_out, void* ac_out, uint8_t* e_out, float* c_out) {
  std::vector<T> a_dense, b;
  if (use_pattern) {
    init_pattern_sparse_a(a_dense, m, k);
    init_pattern_b(b, k, n);
  } else {
    init_structured_sparse_a(a_dense, m, k, gen);
    init_random_b(b, k, n, gen);
  }
  std::vector<T> a_sparse;
  std::vector<uint8_t> e_bytes;
  compress_structured_sparse_a(a_dense, a_sparse, e_bytes, m, k);
  std::vector<float> c_ref;
  cpu_gemm_ref(a_dense, b, c_ref, m, n, k);
  to_bits(a_dense, a_out);
  to_bits(b, b_out);
  to_bits(a_sparse, ac_out);
  std::memcpy(e_out, e_bytes.data(), e_bytes.size());
  std::memcpy(c_out, c_ref.data(), c_ref.size() * sizeof(float));
}

template <typename T>
void gemm_rows(const void* a, const std::vector<T>* bv, float* c, int n, int k, int r0, int r1) {
  // cpu_gemm_ref over a row slice: rows [r0, r1) of A against all of B.
  std::vector<T> a_rows = from_bits<T>(static_cast<const T*>(a) + static_cast<size_t>(r0) * k,
                                       static_cast<size_t>(r1 - r0) * k);
  std::vector<float> c_rows;
  cpu_gemm_ref(a_rows, *bv, c_rows, r1 - r0, n, k);
  std::memcpy(c + static_cast<size_t>(r0) * n, c_rows.data(), c_rows.size() * sizeof(float));
}

template <typename T>
void gemm_threads(const void* a, const void* b, float* c, int m, int n, int k, int threads) {
  const std::vector<T> bv = from_bits<T>(b, static_cast<size_t>(k) * n);
  const int per = (m + threads - 1) / threads;
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    const int r0 = t * per, r1 = std::min(m, r0 + per);
    if (r0 >= r1) break;
    pool.emplace_back(gemm_rows<T>, a, &bv, c, n, k, r0, r1);
  }
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

void* ref_gen_new(unsigned int seed) { return new std::mt19937(seed); }
void ref_gen_free(void* g) { delete static_cast<std::mt19937*>(g); }

// dt: 0 half, 1 __nv_bfloat16, 2 __nv_fp8_e4m3.
void ref_host_case(void* g, int dt, int m, int n, int k, int use_pattern, void* a_out,
                   void* b_out, void* ac_out, uint8_t* e_out, float* c_out) {
  auto& gen = *static_cast<std::mt19937*>(g);
  if (dt == 0)
    run_host_case<half>(gen, m, n, k, use_pattern != 0, a_out, b_out, ac_out, e_out, c_out);
  else if (dt == 1)
    run_host_case<__nv_bfloat16>(gen, m, n, k, use_pattern != 0, a_out, b_out, ac_out, e_out,
                                 c_out);
  else
    run_host_case<__nv_fp8_e4m3>(gen, m, n, k, use_pattern != 0, a_out, b_out, ac_out, e_out,
                                 c_out);
}

// compress_structured_sparse_a on caller data (must be valid 2:4: the
// reference exits the process otherwise).
void ref_compress(int dt, const void* a, int m, int k, void* ac_out, uint8_t* e_out) {
  const size_t cnt = static_cast<size_t>(m) * k;
  std::vector<uint8_t> e;
  if (dt == 2) {
    auto av = from_bits<__nv_fp8_e4m3>(a, cnt);
    std::vector<__nv_fp8_e4m3> ac;
    compress_structured_sparse_a(av, ac, e, m, k);
    to_bits(ac, ac_out);
  } else if (dt == 1) {
    auto av = from_bits<__nv_bfloat16>(a, cnt);
    std::vector<__nv_bfloat16> ac;
    compress_structured_sparse_a(av, ac, e, m, k);
    to_bits(ac, ac_out);
  } else {
    auto av = from_bits<half>(a, cnt);
    std::vector<half> ac;
    compress_structured_sparse_a(av, ac, e, m, k);
    to_bits(ac, ac_out);
  }
  std::memcpy(e_out, e.data(), e.size());
}

// cpu_gemm_ref with rows split across `threads` std::threads (each element's
// arithmetic is the reference's own, unchanged).
void ref_cpu_gemm(int dt, const void* a, const void* b, float* c, int m, int n, int k,
                  int threads) {
  if (threads < 1) threads = 1;
  if (dt == 0) gemm_threads<half>(a, b, c, m, n, k, threads);
  else if (dt == 1) gemm_threads<__nv_bfloat16>(a, b, c, m, n, k, threads);
  else gemm_threads<__nv_fp8_e4m3>(a, b, c, m, n, k, threads);
}

}  // extern "C"
