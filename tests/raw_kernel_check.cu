// raw_kernel_check.cu — test program for the drop-in's launchable
// wgmma_sp_raw_kernel<Element, BlockN> (dropin/sp24_raw_kernel.cuh).
//
// For every (Element, BlockN) of the reference's 18 raw entry points it runs
// the cases those entry points run (mma_sp_wgmma_cuda_m64n{8..256}k{32,64}_
// fp32{fp16,bf16,e4m3}.cu), exactly as the reference's run_case does
// (wgmma_sp_raw_common.hpp:1032-1095): the host generators and compression
// of the drop-in (the reference's mt19937(1234) stream), cpu_gemm_ref,
// cudaMalloc / cudaMemcpy of A_c, B, the metadata bytes and C, then
//
//   wgmma_sp_raw_kernel<Element, BlockN><<<dim3(n / BlockN, m / 64), dim3(128)>>>(
//       d_a, d_b, d_e, d_c, n, k);
//
// and verify_result's abs 1e-2 rule.  Two more cases per entry point cover
// larger grids (several row and column blocks, K beyond one atom).  Prints
// one line per case and "RAW KERNEL CHECK PASSED" / "FAILED"; exit code 0 on
// success.  Built by sparse-gemm-with-hopper-sptc_b200/build.py, run by
// tests/test_dropin_gpu.py.
#include <cstdio>
#include <string>
#include <vector>

#include "wgmma_sp_raw_common.hpp"

template <typename Element, int BlockN>
bool raw_case(const std::string& tag, int m, int n, int k, bool use_pattern, std::mt19937& gen) {
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

  Element *d_a = nullptr, *d_b = nullptr;
  uint8_t* d_e = nullptr;
  float* d_c = nullptr;
  CHECK_CUDA(cudaMalloc(&d_a, sizeof(Element) * a_sparse.size()));
  CHECK_CUDA(cudaMalloc(&d_b, sizeof(Element) * b.size()));
  CHECK_CUDA(cudaMalloc(&d_e, e_bytes.size()));
  CHECK_CUDA(cudaMalloc(&d_c, sizeof(float) * c_ref.size()));
  CHECK_CUDA(cudaMemcpy(d_a, a_sparse.data(), sizeof(Element) * a_sparse.size(),
                        cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(d_b, b.data(), sizeof(Element) * b.size(), cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(d_e, e_bytes.data(), e_bytes.size(), cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemset(d_c, 0, sizeof(float) * c_ref.size()));

  dim3 block(kRawThreads);
  dim3 grid(n / BlockN, m / kRawBlockM);
  wgmma_sp_raw_kernel<Element, BlockN><<<grid, block>>>(d_a, d_b, d_e, d_c, n, k);
  CHECK_CUDA(cudaGetLastError());
  CHECK_CUDA(cudaDeviceSynchronize());

  int timed_out = 0;
  CHECK_CUDA(cudaMemcpyFromSymbol(&timed_out, sp24_raw_kernel_status, sizeof(int)));
  std::vector<float> c_gpu(c_ref.size(), 0.0f);
  CHECK_CUDA(cudaMemcpy(c_gpu.data(), d_c, sizeof(float) * c_gpu.size(), cudaMemcpyDeviceToHost));
  const int errors = verify_result(tag, c_gpu, c_ref, n);
  CHECK_CUDA(cudaFree(d_a));
  CHECK_CUDA(cudaFree(d_b));
  CHECK_CUDA(cudaFree(d_e));
  CHECK_CUDA(cudaFree(d_c));
  if (timed_out) std::cout << tag << ": a bounded wait ran out" << std::endl;
  return errors == 0 && !timed_out;
}

// The entry point's own three cases (pattern, two random), then a wider grid.
template <typename Element, int BlockN>
bool entry(const char* name, int kb, std::mt19937& gen) {
  const std::string p = std::string(name) + "/";
  bool ok = true;
  const int n0 = BlockN;
  ok &= raw_case<Element, BlockN>(p + "pattern", 64, n0, kb, true, gen);
  ok &= raw_case<Element, BlockN>(p + "random_a", 64, n0, 4 * kb, false, gen);
  ok &= raw_case<Element, BlockN>(p + "random_b", 128, n0 * (BlockN <= 64 ? 4 : 2), 8 * kb, false,
                                  gen);
  ok &= raw_case<Element, BlockN>(p + "grid", 320, 3 * BlockN, 40 * kb, false, gen);
  return ok;
}

int main() {
  const int device = select_best_device();
  if (device < 0) {
    std::cout << "No sm_100 GPU found" << std::endl;
    return 2;
  }
  std::mt19937 gen(1234);
  bool ok = true;
  ok &= entry<half, 8>("f16_n8", 32, gen);
  ok &= entry<half, 16>("f16_n16", 32, gen);
  ok &= entry<half, 32>("f16_n32", 32, gen);
  ok &= entry<half, 64>("f16_n64", 32, gen);
  ok &= entry<half, 128>("f16_n128", 32, gen);
  ok &= entry<half, 256>("f16_n256", 32, gen);
  ok &= entry<__nv_bfloat16, 8>("bf16_n8", 32, gen);
  ok &= entry<__nv_bfloat16, 16>("bf16_n16", 32, gen);
  ok &= entry<__nv_bfloat16, 32>("bf16_n32", 32, gen);
  ok &= entry<__nv_bfloat16, 64>("bf16_n64", 32, gen);
  ok &= entry<__nv_bfloat16, 128>("bf16_n128", 32, gen);
  ok &= entry<__nv_bfloat16, 256>("bf16_n256", 32, gen);
  ok &= entry<__nv_fp8_e4m3, 8>("e4m3_n8", 64, gen);
  ok &= entry<__nv_fp8_e4m3, 16>("e4m3_n16", 64, gen);
  ok &= entry<__nv_fp8_e4m3, 32>("e4m3_n32", 64, gen);
  ok &= entry<__nv_fp8_e4m3, 64>("e4m3_n64", 64, gen);
  ok &= entry<__nv_fp8_e4m3, 128>("e4m3_n128", 64, gen);
  ok &= entry<__nv_fp8_e4m3, 256>("e4m3_n256", 64, gen);
  std::cout << (ok ? "RAW KERNEL CHECK PASSED" : "RAW KERNEL CHECK FAILED") << std::endl;
  return ok ? 0 : 1;
}
