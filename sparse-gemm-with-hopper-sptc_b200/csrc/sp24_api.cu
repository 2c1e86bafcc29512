// sp24_api.cu — the C ABI declared in include/sp24.h: argument validation,
// workspace handling, TMA tensor-map construction and kernel dispatch.
//
// Host-side contract mirrored from the reference harness
// (wgmma_sp_raw_common.hpp:1032-1095): the caller owns every device buffer;
// shape problems are reported instead of launched (:1042-1045); CUDA
// failures become SP24_ERR_CUDA instead of exit(EXIT_FAILURE) (:17-25).
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>

#include "../../include/sp24.h"
#include "sp24_gemm2sm_kernel.cuh"
#include "sp24_gemm_kernel.cuh"
#include "sp24_gemm_splitk_kernel.cuh"
#include "sp24_prep.cuh"
#include "../dropin/sp24_raw_kernel.cuh"

namespace {

constexpr int kMaxDevices = 64;
constexpr unsigned long long kDefaultTimeoutNs = 1000000000ull;  // 1 s per bounded wait

// Library-owned per-device status word used when the caller passes none.
__device__ int g_sp24_status_word;

// Fixed scratch of sp24_gemm_noalloc.  In host code this name is only a
// stand-in for the symbol: its device address comes from cudaGetSymbolAddress
// (noalloc_scratch below), looked up once per device with that device current.
static __device__ __align__(256) uint8_t g_sp24_noalloc_scratch[SP24_NOALLOC_SCRATCH_BYTES];

#define SP24_CUDA_TRY(expr)                  \
  do {                                       \
    cudaError_t e__ = (expr);                \
    if (e__ != cudaSuccess) {                \
      (void)cudaGetLastError();              \
      return SP24_ERR_CUDA;                  \
    }                                        \
  } while (0)

inline cudaStream_t as_stream(sp24_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool is_fp8(int dt) { return dt >= SP24_E4M3 && dt <= SP24_E5M2; }
inline int esize(sp24_dtype dt) { return is_fp8(dt) ? 1 : 2; }
inline bool dtype_ok(int dt) { return dt == SP24_F16 || dt == SP24_BF16 || is_fp8(dt); }
// kind::f8f6f4 format fields of the instruction descriptor (e4m3 = 0,
// e5m2 = 1; A at bit 7, B at bit 10).  One set of fp8 kernels serves every
// pairing; 16-bit types carry their format in the kernel's own constant.
inline uint32_t idesc_ab(int dt) {
  const uint32_t a = (dt == SP24_E5M2_E4M3 || dt == SP24_E5M2) ? 1u : 0u;
  const uint32_t b = (dt == SP24_E4M3_E5M2 || dt == SP24_E5M2) ? 1u : 0u;
  return is_fp8(dt) ? (a << 7) | (b << 10) : 0u;
}
inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }
// 128-row blocks of the tcgen05 metadata image, padded to an even count so a
// CTA pair's second half always has an atom to load.
inline int meta_mblocks(int m) { return ((m + 127) / 128 + 1) / 2 * 2; }
inline int meta_katoms(int k) { return (k + 127) / 128; }

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

sp24_status get_encode_fn() {
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    (void)cudaGetLastError();
  });
  return g_encode ? SP24_OK : SP24_ERR_CUDA;
}

PFN_cuMemGetAddressRange_v3020 g_range = nullptr;

// cuMemGetAddressRange (the allocation holding a pointer), resolved at run
// time like the tensor-map encoder.
sp24_status get_range_fn() {
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 3020, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
    (void)cudaGetLastError();
  });
  return g_range ? SP24_OK : SP24_ERR_CUDA;
}

struct DeviceInfo {
  int sm_count = 0;
  int* status_word = nullptr;
  bool ok = false;
};

std::mutex g_dev_mu;
DeviceInfo g_dev[kMaxDevices];

sp24_status device_info(DeviceInfo** out) {
  int dev = 0;
  SP24_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return SP24_ERR_ARG;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& di = g_dev[dev];
  if (!di.ok) {
    cudaDeviceProp prop{};
    SP24_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
    if (prop.major != 10 || prop.minor != 0) return SP24_ERR_ARCH;
    di.sm_count = prop.multiProcessorCount;
    void* p = nullptr;
    SP24_CUDA_TRY(cudaGetSymbolAddress(&p, g_sp24_status_word));
    di.status_word = static_cast<int*>(p);
    di.ok = true;
  }
  *out = &di;
  return SP24_OK;
}

sp24_status encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                      uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle sw) {
  sp24_status st = get_encode_fn();
  if (st != SP24_OK) return st;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SP24_OK : SP24_ERR_ALIGN;
}

CUtensorMapSwizzle swizzle_for_span(int span) {
  switch (span) {
    case 128: return CU_TENSOR_MAP_SWIZZLE_128B;
    case 64: return CU_TENSOR_MAP_SWIZZLE_64B;
    case 32: return CU_TENSOR_MAP_SWIZZLE_32B;
    default: return CU_TENSOR_MAP_SWIZZLE_NONE;
  }
}

// Launch hints of the calling host thread (sp24_set_launch_hints).
thread_local unsigned g_launch_hints = SP24_HINT_NONE;

// Tuning switches from the environment.  None is needed in normal use: they
// force a kernel family or a tile parameter for tests and tuning runs.  They
// are read once, on the first call that needs them, so a launch costs no
// getenv scan; sp24_reload_tuning() reads them again after the caller changed
// the environment.  Every launch works on its own copy, taken under a mutex.
struct Tuning {
  int pdl = 1;                // SP24_PDL=0: no programmatic dependent launch
  int group_m = 0;            // SP24_GROUP_M: CTA-pair tile rasterisation group (0 = default)
  int c_evict = 1;            // SP24_C_EVICT=0: C stores without the evict-first policy
  int splits = 0;             // SP24_SPLITS: split-K slices (0 = chosen per shape)
  int krot = 1;               // SP24_KROT=0: split-K tiles all start at K = 0
  int pair_fine = 0;          // SP24_PAIR_FINE=1: half-size CTA-pair stages
  int kernel_set = 0;         // SP24_KERNEL is set (a forced kernel family wins)
  int kernel = 0;             //   0 other, 1 "1sm", 2 "2sm", 3 "splitk"
  int narrow_pair = -1;       // SP24_NARROW_PAIR=0|1 (-1 unset)
  int pair_splitk = -1;       // SP24_PAIR_SPLITK=0|S (-1 unset)
  int pair_splitk_width = 0;  // SP24_PAIR_SPLITK_WIDTH=64|128 (0 unset)
  int splitk_b8 = 1;          // SP24_SPLITK_B8=0: no 8-column split-K form
  int splitk_kb = 0;          // SP24_SPLITK_KB=1|2 (0 = chosen per tile width)
  int gated = 0;              // SP24_GATED=1|2: gated SwiGLU form forced
  int pair_gated = 1;         // SP24_PAIR_GATED set: gated CTA-pair form off
  int raw_route = 1;          // SP24_RAW_ROUTE=0: tiny reference-layout problems take the
                              //   repack + dispatch path too
};

Tuning read_tuning() {
  Tuning t;
  auto num = [](const char* name, int* out) {
    const char* v = std::getenv(name);
    if (v == nullptr) return false;
    *out = std::atoi(v);
    return true;
  };
  int v = 0;
  if (num("SP24_PDL", &v)) t.pdl = v != 0;
  if (num("SP24_GROUP_M", &v) && v > 0) t.group_m = v;
  if (num("SP24_C_EVICT", &v)) t.c_evict = v != 0;
  if (num("SP24_SPLITS", &v)) t.splits = v;
  if (num("SP24_KROT", &v)) t.krot = v != 0;
  if (num("SP24_PAIR_FINE", &v)) t.pair_fine = v != 0;
  if (const char* k = std::getenv("SP24_KERNEL")) {
    t.kernel_set = 1;
    t.kernel = std::strcmp(k, "1sm") == 0      ? 1
               : std::strcmp(k, "2sm") == 0    ? 2
               : std::strcmp(k, "splitk") == 0 ? 3
                                               : 0;
  }
  if (num("SP24_NARROW_PAIR", &v)) t.narrow_pair = v;
  if (num("SP24_PAIR_SPLITK", &v)) t.pair_splitk = v;
  if (num("SP24_PAIR_SPLITK_WIDTH", &v) && (v == 64 || v == 128)) t.pair_splitk_width = v;
  if (num("SP24_SPLITK_B8", &v)) t.splitk_b8 = v != 0;
  if (num("SP24_SPLITK_KB", &v) && (v == 1 || v == 2)) t.splitk_kb = v;
  if (num("SP24_GATED", &v)) t.gated = v;
  if (std::getenv("SP24_PAIR_GATED") != nullptr) t.pair_gated = 0;
  if (num("SP24_RAW_ROUTE", &v)) t.raw_route = v != 0;
  return t;
}

std::mutex g_tuning_mu;
bool g_tuning_loaded = false;
Tuning g_tuning;

Tuning tuning() {
  std::lock_guard<std::mutex> lk(g_tuning_mu);
  if (!g_tuning_loaded) {
    g_tuning = read_tuning();
    g_tuning_loaded = true;
  }
  return g_tuning;
}

// Sets a kernel's function attributes (dynamic shared memory, and the
// non-portable cluster size when asked) once per device.  `done` is the
// calling launcher's own per-device flag array; the first calls on a device
// from several host threads serialise on the mutex.
std::mutex g_attr_mu;

template <typename Kern>
sp24_status ensure_kernel_attrs(Kern kern, std::atomic<bool> (&done)[kMaxDevices], int smem,
                                bool nonportable_cluster = false) {
  int dev = 0;
  SP24_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return SP24_ERR_ARG;
  if (done[dev].load(std::memory_order_acquire)) return SP24_OK;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (done[dev].load(std::memory_order_relaxed)) return SP24_OK;
  SP24_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  if (nonportable_cluster)
    SP24_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  done[dev].store(true, std::memory_order_release);
  return SP24_OK;
}

// Everything a launch needs after validation / workspace staging.
struct Prepared {
  sp24_dtype dt;
  int m, n, k;
  const void* a_c;
  int64_t lda_c;
  const uint8_t* meta_tc;
  const void* b;
  int64_t ldb;
  float* c_f32;
  void* c_bf16;
  int64_t ldc;
  float alpha;
  uint32_t idesc_ab;
  const float* bias;
  int act;
  const void* a_c_up;  // gated form (split-K kernel only)
  int64_t lda_c_up;
  const uint8_t* meta_up;
  float alpha_up;
  const float* bias_up;
  int gate_from_c;
  int c_reread;         // C is read back by a later launch (two-pass gated): keep it in L2
  sp24::PeerOut peers;
  int static_weights;   // SP24_HINT_STATIC_WEIGHTS in effect (narrow-N kernel)
  int* status;
  unsigned long long timeout_ns;
  int stall_producer;
  Tuning tune;          // the tuning switches in effect for this call
};

// GEMM launches carry programmatic stream serialization: the kernel may be
// scheduled while the previous kernel of the stream finishes, runs its
// prologue (barriers, TMEM allocation, tensor-map prefetch), and its TMA
// producers wait for the previous grid (griddepcontrol.wait) before the
// first load.  SP24_PDL=0 launches without the attribute.
template <typename... KArgs, typename... Args>
sp24_status launch_gemm_kernel(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem,
                               cudaStream_t stream, unsigned cluster, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned na = 0;
  if (cluster > 0) {   // run-time cluster shape; 0 = none (or the kernel's __cluster_dims__)
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  SP24_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
  return SP24_OK;
}

template <int DT, int BN>
sp24_status launch_gemm(const Prepared& p, const DeviceInfo& di, cudaStream_t stream) {
  using C = sp24::GemmCfg<DT, BN>;
  auto kern = sp24::sp24_gemm_kernel<DT, BN>;
  static std::atomic<bool> attr_set[kMaxDevices];
  const sp24_status ast = ensure_kernel_attrs(kern, attr_set, C::SMEM_BYTES);
  if (ast != SP24_OK) return ast;
  const CUtensorMapDataType tdt =
      C::ESZ == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  CUtensorMap ta, tb;
  sp24_status st =
      encode_2d(&ta, tdt, p.a_c, static_cast<uint64_t>(p.k / 2), static_cast<uint64_t>(p.m),
                static_cast<uint64_t>(p.lda_c) * C::ESZ, C::A_COLS, sp24::kBlockM,
                CU_TENSOR_MAP_SWIZZLE_64B);
  if (st != SP24_OK) return st;
  st = encode_2d(&tb, tdt, p.b, static_cast<uint64_t>(p.n), static_cast<uint64_t>(p.k),
                 static_cast<uint64_t>(p.ldb) * C::ESZ, C::B_BOXN, C::BKD,
                 swizzle_for_span(C::B_SPAN));
  if (st != SP24_OK) return st;

  sp24::GemmParams P{};
  P.m = p.m;
  P.n = p.n;
  P.k = p.k;
  P.m_blocks = (p.m + sp24::kBlockM - 1) / sp24::kBlockM;
  P.n_tiles = (p.n + BN - 1) / BN;
  P.k_stages = (p.k + C::BKD - 1) / C::BKD;
  P.num_tiles = P.m_blocks * P.n_tiles;
  P.group_m = 16;
  P.meta_tc = p.meta_tc;
  P.meta_mblocks = meta_mblocks(p.m);
  P.c_f32 = p.c_f32;
  P.c_bf16 = static_cast<__nv_bfloat16*>(p.c_bf16);
  P.ldc = p.ldc;
  P.alpha = p.alpha;
  P.idesc_ab = p.idesc_ab;
  P.bias = p.bias;
  P.act = p.act;
  P.gate_from_c = p.gate_from_c;
  P.peers = p.peers;
  P.vec_f32 = (p.c_f32 != nullptr && aligned16(p.c_f32) && (p.ldc % 4) == 0) ? 1 : 0;
  P.vec_bf16 = (p.c_bf16 != nullptr && aligned16(p.c_bf16) && (p.ldc % 8) == 0) ? 1 : 0;
  P.status = p.status;
  P.timeout_ns = p.timeout_ns;
  P.stall_producer = p.stall_producer;
  const int grid = std::min(P.num_tiles, di.sm_count);
  return launch_gemm_kernel(kern, static_cast<unsigned>(grid), sp24::kThreads, C::SMEM_BYTES, stream,
                            0, p.tune.pdl != 0, ta, tb, P);
}



// Parameter block shared by the CTA-pair kernels; tiles of tile_m x tile_n.
sp24::PairParams pair_params(const Prepared& p, int bkd, int tile_m, int tile_n) {
  sp24::PairParams P{};
  P.m = p.m;
  P.n = p.n;
  P.k = p.k;
  P.m_blocks = meta_mblocks(p.m);
  P.m_pairs = (p.m + tile_m - 1) / tile_m;
  P.n_tiles = (p.n + tile_n - 1) / tile_n;
  P.k_stages = (p.k + bkd - 1) / bkd;
  P.num_tiles = P.m_pairs * P.n_tiles;
  // 12 M tiles per rasterisation group: with A under the evict-last policy a
  // group's A stays in L2 across its waves, and larger groups re-stream B
  // fewer times (same-box A/B against 8: configuration 2 +0.8%, 3 +1.5-2%).
  P.group_m = p.tune.group_m > 0 ? p.tune.group_m : 12;
  P.splits = 1;
  P.c_f32 = p.c_f32;
  P.c_bf16 = static_cast<__nv_bfloat16*>(p.c_bf16);
  P.ldc = p.ldc;
  P.alpha = p.alpha;
  P.idesc_ab = p.idesc_ab;
  P.bias = p.bias;
  P.act = p.act;
  P.alpha_up = p.alpha_up;
  P.bias_up = p.bias_up;
  P.gate_from_c = p.gate_from_c;
  P.peers = p.peers;
  P.vec_f32 = p.c_f32 == nullptr                            ? 0
              : (aligned32(p.c_f32) && (p.ldc % 8) == 0)    ? 2
              : (aligned16(p.c_f32) && (p.ldc % 4) == 0)    ? 1
                                                            : 0;
  P.vec_bf16 = p.c_bf16 == nullptr                          ? 0
               : (aligned32(p.c_bf16) && (p.ldc % 16) == 0) ? 2
               : (aligned16(p.c_bf16) && (p.ldc % 8) == 0)  ? 1
                                                            : 0;
  // C under an L2 evict-first policy, so the output does not push the A and B
  // tiles that other CTAs still read out of L2 (configuration 2, fp32 + bf16
  // out: +1%).  Outputs that are read back keep the default policy: the fused
  // all-gather re-reads its stores, the first gated pass writes the
  // intermediate that the second pass reads, and the second pass reads C
  // itself.  SP24_C_EVICT=0 turns it off.
  P.c_evict_first =
      (p.tune.c_evict && p.peers.n == 0 && !p.gate_from_c && !p.c_reread) ? 1 : 0;
  P.static_weights = p.static_weights;
  P.status = p.status;
  P.timeout_ns = p.timeout_ns;
  P.stall_producer = p.stall_producer;
  return P;
}

// Metadata image viewed as rows of 256 B: one 2 KB atom = an 8-row box.
sp24_status encode_meta_rows(CUtensorMap* te, const Prepared& p, const uint8_t* image = nullptr) {
  const uint64_t lanes = static_cast<uint64_t>(meta_katoms(p.k)) * meta_mblocks(p.m) * 128;
  return encode_2d(te, CU_TENSOR_MAP_DATA_TYPE_UINT8, image != nullptr ? image : p.meta_tc, 256,
                   lanes * 16 / 256, 256, 256, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int DT, int FINE, int BNP = 256, int G = 1>
sp24_status launch_gemm2sm(const Prepared& p, const DeviceInfo& di, cudaStream_t stream) {
  using C = sp24::PairCfg<DT, FINE, BNP, G>;
  auto kern = sp24::sp24_gemm2sm_kernel<DT, FINE, BNP, G>;
  static std::atomic<bool> attr_set[kMaxDevices];
  const sp24_status ast = ensure_kernel_attrs(kern, attr_set, C::SMEM_BYTES);
  if (ast != SP24_OK) return ast;
  const CUtensorMapDataType tdt =
      C::ESZ == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  CUtensorMap ta, tb, te;
  sp24_status st =
      encode_2d(&ta, tdt, p.a_c, static_cast<uint64_t>(p.k / 2), static_cast<uint64_t>(p.m),
                static_cast<uint64_t>(p.lda_c) * C::ESZ, C::A_COLS, sp24::kBlockM,
                C::A_ROW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (st != SP24_OK) return st;
  st = encode_2d(&tb, tdt, p.b, static_cast<uint64_t>(p.n), static_cast<uint64_t>(p.k),
                 static_cast<uint64_t>(p.ldb) * C::ESZ, C::B_BOXN, C::BKD,
                 swizzle_for_span(C::B_SPAN));
  if (st != SP24_OK) return st;
  st = encode_meta_rows(&te, p);
  if (st != SP24_OK) return st;
  CUtensorMap ta2 = ta, te2 = te;
  if constexpr (G == 2) {   // W_up of the gated form
    st = encode_2d(&ta2, tdt, p.a_c_up, static_cast<uint64_t>(p.k / 2), static_cast<uint64_t>(p.m),
                   static_cast<uint64_t>(p.lda_c_up) * C::ESZ, C::A_COLS, sp24::kBlockM,
                   C::A_ROW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != SP24_OK) return st;
    st = encode_meta_rows(&te2, p, p.meta_up);
    if (st != SP24_OK) return st;
  }

  const sp24::PairParams P = pair_params(p, C::BKD, 256, BNP);
  const int pairs = std::max(1, std::min(P.num_tiles, di.sm_count / 2));
  // Cluster shape (2) comes from the kernel's __cluster_dims__.
  return launch_gemm_kernel(kern, static_cast<unsigned>(2 * pairs), sp24::kPairThreads,
                            C::SMEM_BYTES, stream, 0, p.tune.pdl != 0, ta, tb, te, ta2, te2, P);
}

// Largest cluster of split-K CTAs the device keeps resident `tiles` times
// over (cached per device and split factor).
std::mutex g_occ_mu;
// Per device, kernel family (0 split-K, 1 pair K-split) and cluster size.
int g_occ[kMaxDevices][2][sp24::kMaxSplits + 1];

template <typename Kern>
int max_active_clusters(Kern kern, int smem, int csize, int family = 0,
                        unsigned threads = sp24::kThreads) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices ||
      csize > sp24::kMaxSplits) {
    (void)cudaGetLastError();
    return 0;
  }
  std::lock_guard<std::mutex> lk(g_occ_mu);
  int& slot = g_occ[dev][family][csize];
  if (slot == 0) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(csize));
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(csize);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    slot = n > 0 ? n : -1;
  }
  return slot;
}

// K-split factor of the narrow-N kernel.  When the 128-row tiles already
// cover three quarters of the SMs the tiles run unsplit; otherwise K is cut
// into as many slices as there are SMs per tile (at most 8, the portable
// cluster size, and at least two stages per slice), and the factor is
// lowered until all clusters are resident at once.  SP24_SPLITS overrides
// (tests and tuning runs; still clamped to those limits).
template <typename Kern>
int choose_splits(Kern kern, int smem, int tiles, int stages, int sm_count, int forced) {
  int s = forced > 0 ? forced : (tiles * 4 >= sm_count * 3 ? 1 : sm_count / tiles);
  s = std::min(s, sp24::kMaxSplits);
  s = std::min(s, std::max(1, forced > 0 ? stages : stages / 2));
  s = std::max(s, 1);
  if (forced <= 0)
    while (s > 1 && max_active_clusters(kern, smem, s) < tiles) --s;
  return s;
}

// The CTA-pair kernel's K-split form: one 256-row tile per cluster of
// 2 * splits CTAs, pair p summing K slice p (narrow N with few row tiles).
template <int DT, int BNP>
sp24_status launch_gemm2sm_splitk(const Prepared& p, const DeviceInfo& di, cudaStream_t stream,
                                  int splits) {
  using C = sp24::PairCfg<DT, 0, BNP>;
  auto kern = sp24::sp24_gemm2sm_splitk_kernel<DT, BNP>;
  static std::atomic<bool> attr_set[kMaxDevices];
  const sp24_status ast = ensure_kernel_attrs(kern, attr_set, C::SMEM_BYTES, true);
  if (ast != SP24_OK) return ast;
  const CUtensorMapDataType tdt =
      C::ESZ == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  CUtensorMap ta, tb, te;
  sp24_status st =
      encode_2d(&ta, tdt, p.a_c, static_cast<uint64_t>(p.k / 2), static_cast<uint64_t>(p.m),
                static_cast<uint64_t>(p.lda_c) * C::ESZ, C::A_COLS, sp24::kBlockM,
                C::A_ROW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (st != SP24_OK) return st;
  st = encode_2d(&tb, tdt, p.b, static_cast<uint64_t>(p.n), static_cast<uint64_t>(p.k),
                 static_cast<uint64_t>(p.ldb) * C::ESZ, C::B_BOXN, C::BKD,
                 swizzle_for_span(C::B_SPAN));
  if (st != SP24_OK) return st;
  st = encode_meta_rows(&te, p);
  if (st != SP24_OK) return st;
  sp24::PairParams P = pair_params(p, C::BKD, 256, BNP);
  // Every cluster resident at once, at least two stages per slice.
  splits = std::max(1, std::min(splits, P.k_stages / 2));
  while (splits > 1 &&
         max_active_clusters(kern, C::SMEM_BYTES, 2 * splits, 1, sp24::kPairThreads) < P.num_tiles)
    --splits;
  P.splits = splits;
  return launch_gemm_kernel(kern, static_cast<unsigned>(P.num_tiles * 2 * splits),
                            sp24::kPairThreads, C::SMEM_BYTES, stream,
                            static_cast<unsigned>(2 * splits), p.tune.pdl != 0, ta, tb, te, P);
}

template <int DT, int BN, int KB, int G>
sp24_status launch_splitk(const Prepared& p, const DeviceInfo& di, cudaStream_t stream) {
  using C = sp24::SplitCfg<DT, BN, KB, G>;
  auto kern = sp24::sp24_gemm_splitk_kernel<DT, BN, KB, G>;
  static std::atomic<bool> attr_set[kMaxDevices];
  const sp24_status ast = ensure_kernel_attrs(kern, attr_set, C::SMEM_BYTES);
  if (ast != SP24_OK) return ast;
  const CUtensorMapDataType tdt =
      C::ESZ == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  CUtensorMap ta, tb;
  sp24_status st =
      encode_2d(&ta, tdt, p.a_c, static_cast<uint64_t>(p.k / 2), static_cast<uint64_t>(p.m),
                static_cast<uint64_t>(p.lda_c) * C::ESZ, C::A_COLS, sp24::kBlockM,
                CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != SP24_OK) return st;
  st = encode_2d(&tb, tdt, p.b, static_cast<uint64_t>(p.n), static_cast<uint64_t>(p.k),
                 static_cast<uint64_t>(p.ldb) * C::ESZ, C::B_BOXN, C::UK,
                 swizzle_for_span(C::B_SPAN));
  if (st != SP24_OK) return st;
  CUtensorMap ta2 = ta;
  if constexpr (G == 2) {
    st = encode_2d(&ta2, tdt, p.a_c_up, static_cast<uint64_t>(p.k / 2),
                   static_cast<uint64_t>(p.m), static_cast<uint64_t>(p.lda_c_up) * C::ESZ,
                   C::A_COLS, sp24::kBlockM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SP24_OK) return st;
  }

  sp24::SplitParams P{};
  P.m = p.m;
  P.n = p.n;
  P.k = p.k;
  P.m_blocks = (p.m + sp24::kBlockM - 1) / sp24::kBlockM;
  P.n_tiles = (p.n + BN - 1) / BN;
  P.stages = (p.k + C::BKD - 1) / C::BKD;
  P.katoms = meta_katoms(p.k);
  P.meta_tc = p.meta_tc;
  P.meta_mblocks = meta_mblocks(p.m);
  P.c_f32 = p.c_f32;
  P.c_bf16 = static_cast<__nv_bfloat16*>(p.c_bf16);
  P.ldc = p.ldc;
  P.alpha = p.alpha;
  P.idesc_ab = p.idesc_ab;
  P.bias = p.bias;
  P.act = p.act;
  P.gate_from_c = p.gate_from_c;
  P.peers = p.peers;
  P.vec_f32 = (p.c_f32 != nullptr && aligned16(p.c_f32) && (p.ldc % 4) == 0) ? 1 : 0;
  P.vec_bf16 = (p.c_bf16 != nullptr && aligned16(p.c_bf16) && (p.ldc % 8) == 0) ? 1 : 0;
  P.status = p.status;
  P.timeout_ns = p.timeout_ns;
  P.stall_producer = p.stall_producer;
  P.static_weights = p.static_weights;
  P.rotate = p.tune.krot;   // SP24_KROT=0: every tile in K order (tuning runs)
  P.meta_up = p.meta_up;
  P.alpha_up = p.alpha_up;
  P.bias_up = p.bias_up;
  const int tiles = P.m_blocks * P.n_tiles;
  P.splits = choose_splits(kern, C::SMEM_BYTES, tiles, P.stages, di.sm_count, p.tune.splits);

  // Launched with an explicit cluster shape of S CTAs, S = 1 included.
  return launch_gemm_kernel(kern, static_cast<unsigned>(tiles * P.splits), sp24::kThreads,
                            C::SMEM_BYTES, stream, static_cast<unsigned>(P.splits), p.tune.pdl != 0,
                            ta, tb, ta2, P);
}

// Stage granularity of the CTA-pair kernel (PairCfg FINE); SP24_PAIR_FINE=0|1
// overrides for tuning runs.
bool pair_fine_stages(const Tuning& t) { return t.pair_fine != 0; }

// Kernel choice: the CTA-pair kernel for problems with at least one full
// 256 x 256 tile, the single-CTA kernel (narrow N tiles) otherwise.
// SP24_KERNEL=1sm|2sm overrides (benchmarks and tests).
bool use_pair_kernel(int m, int n, int hint, const Tuning& t) {
  if (t.kernel == 1) return false;
  if (t.kernel == 2) return true;
  if (hint != 0 && hint != 256) return false;
  return m >= 256 && n >= 256;
}

// Narrow N (17..128 columns; 33..128 for fp8) with enough 256-row tiles to
// occupy most SMs as CTA pairs: the pair kernel with a 32-, 64- or 128-wide
// tile.  Its
// cta_group::2 MMAs split B over the two SMs, so each stages half of it, and
// the ring holds 6-8 stages; the split-K kernel, one SM per 128-row tile,
// streams a full B per tile and is latency-bound there (W_up, T = 128).
// Returns the tile width or 0.  SP24_NARROW_PAIR=0 turns it off, =1 forces it
// for every eligible shape (tests and tuning runs).
int narrow_pair_width(const sp24_gemm_desc* d, int sm_count, const Tuning& t) {
  const int mode = t.narrow_pair;
  if (mode == 0) return 0;
  if (t.kernel_set && mode != 1) return 0;   // a forced kernel choice wins
  if (d->tile_n != 0 || d->n > 128) return 0;
  // 32-wide tiles stage 16 columns (32 B rows) per CTA: 16-bit types only.
  if (d->n <= 32 && is_fp8(d->dtype)) return 0;
  const int np = d->n <= 32 ? 32 : d->n <= 64 ? 64 : 128;
  if (mode == 1) return np;
  // Up to 16 columns the split-K kernel's 44 KB stages stream A at the HBM
  // rate; the pair tile wins from 17 columns on (W_up, T = 16: 14.7 us
  // against 16.4 us; T = 32: 17.1 us against 16.5 us).
  if (d->n <= 16) return 0;
  const long long pair_tiles =
      static_cast<long long>((d->m + 255) / 256) * ((d->n + np - 1) / np);
  return pair_tiles * 4 >= static_cast<long long>(sm_count / 2) * 3 ? np : 0;
}

// Narrow N (17..128 columns; 33..128 for fp8) with too few 256-row tiles for
// the plain pair kernel: its K-split form, S pairs per tile (*splits), so
// that 2 S CTAs per tile occupy most of the SMs.  Returns the tile width or
// 0.  SP24_PAIR_SPLITK=0 turns it off; =S forces S pairs on every eligible
// shape (tests and tuning runs).
int narrow_pair_splitk_width(const sp24_gemm_desc* d, int sm_count, int* splits,
                             const Tuning& t) {
  const int forced = t.pair_splitk;
  if (forced == 0) return 0;
  if (t.kernel_set && forced < 1) return 0;   // a forced kernel choice wins
  if (d->tile_n != 0 || d->n > 128 || d->n <= (is_fp8(d->dtype) ? 32 : 16)) return 0;
  int np = d->n <= 32 ? 32 : d->n <= 64 ? 64 : 128;
  if (t.pair_splitk_width != 0 && d->n > 32) np = t.pair_splitk_width;   // tuning: 64 or 128
  if (forced >= 1) {
    *splits = std::min(forced, 4);
    return np;
  }
  const long long tiles = static_cast<long long>((d->m + 255) / 256) * ((d->n + np - 1) / np);
  const int s = static_cast<int>(std::min<long long>(4, (sm_count / 2) / std::max(1LL, tiles)));
  if (s < 2) return 0;
  *splits = s;
  return np;
}

// Narrow N with few 256-row tiles and a K too short for the pair K-split
// form to split (fewer than four 128-deep stages, so one pair per tile): the
// plain pair form, which has no reduction phase.  A single 64 x 128 x 32 fp16
// tile takes 4.75 us per launch there, against 6.62 us in the one-pair K-split
// form, 8.49 us on the single-CTA kernel and 10.97 us on the split-K kernel
// (launches back to back from a CUDA graph).  Returns the tile width or 0.
int short_k_pair_width(const sp24_gemm_desc* d, const Tuning& t) {
  if (t.narrow_pair == 0 || t.pair_splitk >= 0 || t.kernel_set) return 0;
  if (d->tile_n != 0 || d->n > 128 || d->n <= (is_fp8(d->dtype) ? 32 : 16)) return 0;
  const int kstep = is_fp8(d->dtype) ? 256 : 128;
  if ((d->k + kstep - 1) / kstep >= 4) return 0;
  return d->n <= 32 ? 32 : d->n <= 64 ? 64 : 128;
}

// Tiles at most 128 wide take the split-K kernel when N itself is narrow or
// the tile count is modest (up to four waves): there its large stages and
// K splitting win.  With thousands of narrow tiles the persistent
// single-CTA kernel, whose grouped tile order shares operands in L2, is
// faster.  SP24_KERNEL=1sm|splitk overrides.
bool use_splitk_kernel(int m, int n, int bn, int sm_count, const Tuning& t) {
  if (t.kernel == 1) return false;
  if (bn > 128) return false;
  if (t.kernel == 3) return true;
  const long long tiles = static_cast<long long>((m + 127) / 128) * ((n + bn - 1) / bn);
  return n <= 128 || tiles <= 4LL * sm_count;
}

// Split-K tile width for a 16-column choice: 8 for 16-bit types with at most
// 8 columns, whose 16-column B boxes would be half outside B (the kernel's
// 8-column form loads in-bounds boxes only).  SP24_SPLITK_B8=0 turns it off.
int splitk_tile_n(const sp24_gemm_desc* d, int bn, const Tuning& t) {
  if (bn != 16 || d->n > 8 || is_fp8(d->dtype)) return bn;
  return t.splitk_b8 ? 8 : bn;
}

// Units per split-K stage: two (32 KB of A_c) for tiles up to 32 wide, one
// above, where B's share of a stage grows.  SP24_SPLITK_KB=1|2 overrides.
int splitk_units(int bn, const Tuning& t) {
  if (t.splitk_kb != 0) return t.splitk_kb;
  return bn <= 32 ? 2 : 1;
}

using LaunchFn = sp24_status (*)(const Prepared&, const DeviceInfo&, cudaStream_t);

using PairSplitFn = sp24_status (*)(const Prepared&, const DeviceInfo&, cudaStream_t, int);

template <int DT>
PairSplitFn pick_pair_splitk(int np) {
  if constexpr (DT != 2) {
    if (np == 32) return launch_gemm2sm_splitk<DT, 32>;
  }
  return np == 64 ? launch_gemm2sm_splitk<DT, 64> : launch_gemm2sm_splitk<DT, 128>;
}

template <int DT>
LaunchFn pick_pair_gated(int np) {
  return np == 64 ? launch_gemm2sm<DT, 0, 64, 2> : launch_gemm2sm<DT, 0, 128, 2>;
}

template <int DT>
LaunchFn pick_narrow_pair(int np) {
  if constexpr (DT != 2) {
    if (np == 32) return launch_gemm2sm<DT, 0, 32>;
  }
  return np == 64 ? launch_gemm2sm<DT, 0, 64> : launch_gemm2sm<DT, 0, 128>;
}

// Pair-kernel variant: the 256 x 256 tile with coarse stages, or its
// fine-staged form (SP24_PAIR_FINE=1).
template <int DT>
LaunchFn pick_pair_dt(const Tuning& t) {
  return pair_fine_stages(t) ? launch_gemm2sm<DT, 1> : launch_gemm2sm<DT, 0>;
}

LaunchFn pick_pair(sp24_dtype dt, const Tuning& t) {
  return dt == SP24_F16 ? pick_pair_dt<0>(t) : dt == SP24_BF16 ? pick_pair_dt<1>(t) : pick_pair_dt<2>(t);
}

template <int DT>
LaunchFn pick_splitk(int bn, int kb) {
  if constexpr (DT != 2) {
    if (bn == 8) return kb == 2 ? launch_splitk<DT, 8, 2, 1> : launch_splitk<DT, 8, 1, 1>;
  }
  switch (bn) {
    case 16: return kb == 2 ? launch_splitk<DT, 16, 2, 1> : launch_splitk<DT, 16, 1, 1>;
    case 32: return kb == 2 ? launch_splitk<DT, 32, 2, 1> : launch_splitk<DT, 32, 1, 1>;
    case 64: return kb == 2 ? launch_splitk<DT, 64, 2, 1> : launch_splitk<DT, 64, 1, 1>;
    default: return kb == 2 ? launch_splitk<DT, 128, 2, 1> : launch_splitk<DT, 128, 1, 1>;
  }
}

// Gated form: two weights per ring slot, so one unit per stage keeps four to
// five slots in flight.
template <int DT>
LaunchFn pick_gated(int bn) {
  if constexpr (DT != 2) {
    if (bn == 8) return launch_splitk<DT, 8, 1, 2>;
  }
  switch (bn) {
    case 16: return launch_splitk<DT, 16, 1, 2>;
    case 32: return launch_splitk<DT, 32, 1, 2>;
    case 64: return launch_splitk<DT, 64, 1, 2>;
    default: return launch_splitk<DT, 128, 1, 2>;
  }
}

template <int DT>
LaunchFn pick_bn(int bn) {
  switch (bn) {
    case 16: return launch_gemm<DT, 16>;
    case 32: return launch_gemm<DT, 32>;
    case 64: return launch_gemm<DT, 64>;
    case 128: return launch_gemm<DT, 128>;
    default: return launch_gemm<DT, 256>;
  }
}

int choose_bn(int m, int n, int hint, int sm_count) {
  if (hint > 0) {
    if (hint <= 16) return 16;
    if (hint <= 32) return 32;
    if (hint <= 64) return 64;
    if (hint <= 128) return 128;
    return 256;
  }
  if (n <= 16) return 16;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  const long long mb = (m + 127) / 128;
  const long long tiles256 = mb * ((n + 255) / 256);
  return tiles256 >= sm_count ? 256 : 128;
}

struct WsPlan {
  size_t meta_off = 0, meta_bytes = 0;
  size_t b_off = 0, b_bytes = 0;
  int64_t b_pitch_elems = 0;
  size_t total = 0;
};

bool b_needs_copy(const sp24_gemm_desc* d) {
  const int es = esize(d->dtype);
  const int64_t ldb = d->ldb ? d->ldb : d->n;
  return !aligned16(d->b) || ((ldb * es) % 16) != 0;
}

WsPlan plan_workspace(const sp24_gemm_desc* d) {
  WsPlan w;
  size_t off = 0;
  if (d->meta_format == SP24_META_REF || d->meta_format == SP24_META_K16) {
    w.meta_off = off;
    w.meta_bytes = sp24_meta_tc_bytes(d->m, d->k);
    off = round_up(off + w.meta_bytes, 256);
  }
  if (b_needs_copy(d)) {
    const int es = esize(d->dtype);
    w.b_pitch_elems = static_cast<int64_t>(round_up(static_cast<size_t>(d->n) * es, 16) / es);
    w.b_off = off;
    w.b_bytes = static_cast<size_t>(w.b_pitch_elems) * es * d->k;
    off = round_up(off + w.b_bytes, 256);
  }
  w.total = off;
  return w;
}

sp24_status validate(const sp24_gemm_desc* d) {
  if (d == nullptr) return SP24_ERR_ARG;
  if (!dtype_ok(d->dtype)) return SP24_ERR_ARG;
  if (d->meta_format != SP24_META_REF && d->meta_format != SP24_META_TC &&
      d->meta_format != SP24_META_K16)
    return SP24_ERR_ARG;
  if (d->meta_format == SP24_META_K16 && (is_fp8(d->dtype) || d->m % 16 != 0))
    return SP24_ERR_SHAPE;
  if (d->m <= 0 || d->n <= 0 || d->k <= 0) return SP24_ERR_SHAPE;
  const int kq = is_fp8(d->dtype) ? 64 : 32;
  if (d->k % kq != 0) return SP24_ERR_SHAPE;
  if (d->a_c == nullptr || d->meta == nullptr || d->b == nullptr) return SP24_ERR_ARG;
  if (d->c_f32 == nullptr && d->c_bf16 == nullptr) return SP24_ERR_ARG;
  const int64_t lda_c = d->lda_c ? d->lda_c : d->k / 2;
  const int64_t ldb = d->ldb ? d->ldb : d->n;
  const int64_t ldc = d->ldc ? d->ldc : d->n;
  if (lda_c < d->k / 2 || ldb < d->n || ldc < d->n) return SP24_ERR_SHAPE;
  if (!aligned16(d->a_c) || ((lda_c * esize(d->dtype)) % 16) != 0) return SP24_ERR_ALIGN;
  if (!aligned16(d->meta)) return SP24_ERR_ALIGN;
  if (d->tile_n < 0 || d->tile_n > 256) return SP24_ERR_ARG;
  return SP24_OK;
}

sp24_status launch_plain(const sp24_gemm_desc* d, const Prepared& p, const DeviceInfo& di,
                         cudaStream_t stream);

// Checks of the epilogue descriptor (after the GEMM descriptor passed validate).
sp24_status validate_epilogue(const sp24_gemm_desc* d, const sp24_epilogue* e) {
  if (e == nullptr) return SP24_OK;
  if (e->act != SP24_ACT_NONE && e->act != SP24_ACT_SILU) return SP24_ERR_ARG;
  if (e->a_c_up == nullptr) return SP24_OK;
  if (e->meta_up == nullptr || d->meta_format != SP24_META_TC) return SP24_ERR_ARG;
  const int64_t lda = e->lda_c_up ? e->lda_c_up : d->k / 2;
  if (lda < d->k / 2) return SP24_ERR_SHAPE;
  if (!aligned16(e->a_c_up) || ((lda * esize(d->dtype)) % 16) != 0 || !aligned16(e->meta_up))
    return SP24_ERR_ALIGN;
  return SP24_OK;
}

// Checks of the fused all-gather destinations.
sp24_status validate_peers(const sp24_gemm_desc* d, const sp24_peer_out* peers) {
  if (peers == nullptr || peers->n_peers == 0) return SP24_OK;
  if (peers->n_peers < 0 || peers->n_peers > SP24_MAX_PEERS) return SP24_ERR_ARG;
  for (int i = 0; i < peers->n_peers; ++i) {
    if (d->c_f32 != nullptr) {
      if (peers->c_f32[i] == nullptr) return SP24_ERR_ARG;
      if ((reinterpret_cast<uintptr_t>(peers->c_f32[i]) & 31u) !=
          (reinterpret_cast<uintptr_t>(d->c_f32) & 31u))
        return SP24_ERR_ALIGN;
    }
    if (d->c_bf16 != nullptr) {
      if (peers->c_bf16[i] == nullptr) return SP24_ERR_ARG;
      if ((reinterpret_cast<uintptr_t>(peers->c_bf16[i]) & 31u) !=
          (reinterpret_cast<uintptr_t>(d->c_bf16) & 31u))
        return SP24_ERR_ALIGN;
    }
  }
  return SP24_OK;
}

// Size limits of the tiny reference-layout route.  Measured on B200, back to
// back from the host, bf16: 64x128x32 6.2 against 9.9 us, 64x256x64 8.2
// against 16.4 us, 128x256x128 9.8 against 16.4 us; 256x256x256 ties (12.3
// us), and from K = 512 on the route loses (256x256x512 18.3 against 12.3).
constexpr int kRawRouteMaxM = 256;
constexpr int kRawRouteMaxN = 256;
constexpr int kRawRouteMaxK = 256;
constexpr long long kRawRouteMaxMNK = 128LL * 256 * 256;

// Tiny problems in the reference's own metadata layout: one launch of the
// launchable M = 64 kernel (dropin/sp24_raw_kernel.cuh), which reads the
// reference's nibbles inside the kernel, instead of a repack launch followed
// by the CTA-pair kernel, whose setup would be most of the time.  The route
// takes exactly what that kernel takes: fp16 / bf16 / e4m3, fp32 output only,
// alpha 1, packed rows (A_c k / 2, B and C n), M % 64 == 0, K % 32 (e4m3:
// % 64), 16-byte aligned operands, no fused epilogue and no peers.  Returns
// the tile width to launch, 0 when the problem does not take the route.
int raw_route_bn(const sp24_gemm_desc* d, const sp24_epilogue* e, const sp24_peer_out* peers,
                 const Tuning& t) {
  if (!t.raw_route || t.kernel_set || e != nullptr || peers != nullptr) return 0;
  if (d->meta_format != SP24_META_REF) return 0;
  if (d->dtype != SP24_F16 && d->dtype != SP24_BF16 && d->dtype != SP24_E4M3) return 0;
  if (d->c_f32 == nullptr || d->c_bf16 != nullptr) return 0;
  if (d->alpha != 0.0f && d->alpha != 1.0f) return 0;
  if (d->m % 64 != 0 || d->m > kRawRouteMaxM || d->n > kRawRouteMaxN || d->k > kRawRouteMaxK ||
      static_cast<long long>(d->m) * d->n * d->k > kRawRouteMaxMNK)
    return 0;
  if (d->k % (d->dtype == SP24_E4M3 ? 64 : 32) != 0) return 0;
  if ((d->lda_c != 0 && d->lda_c != d->k / 2) || (d->ldb != 0 && d->ldb != d->n) ||
      (d->ldc != 0 && d->ldc != d->n))
    return 0;
  if (!aligned16(d->a_c) || !aligned16(d->b) || !aligned16(d->meta) || !aligned16(d->c_f32))
    return 0;
  for (int bn = 256; bn >= 8; bn >>= 1)
    if (d->n % bn == 0 && (d->tile_n == 0 || bn <= d->tile_n)) return bn;
  return 0;
}

template <typename T>
sp24_status launch_raw_t(const sp24_gemm_desc* d, int bn, cudaStream_t stream) {
  const T* a = static_cast<const T*>(d->a_c);
  const T* b = static_cast<const T*>(d->b);
  const dim3 grid(static_cast<unsigned>(d->n / bn), static_cast<unsigned>(d->m / 64));
  switch (bn) {
    case 256: wgmma_sp_raw_kernel<T, 256><<<grid, 128, 0, stream>>>(a, b, d->meta, d->c_f32, d->n, d->k); break;
    case 128: wgmma_sp_raw_kernel<T, 128><<<grid, 128, 0, stream>>>(a, b, d->meta, d->c_f32, d->n, d->k); break;
    case 64: wgmma_sp_raw_kernel<T, 64><<<grid, 128, 0, stream>>>(a, b, d->meta, d->c_f32, d->n, d->k); break;
    case 32: wgmma_sp_raw_kernel<T, 32><<<grid, 128, 0, stream>>>(a, b, d->meta, d->c_f32, d->n, d->k); break;
    case 16: wgmma_sp_raw_kernel<T, 16><<<grid, 128, 0, stream>>>(a, b, d->meta, d->c_f32, d->n, d->k); break;
    default: wgmma_sp_raw_kernel<T, 8><<<grid, 128, 0, stream>>>(a, b, d->meta, d->c_f32, d->n, d->k); break;
  }
  SP24_CUDA_TRY(cudaGetLastError());
  return SP24_OK;
}

sp24_status launch_raw(const sp24_gemm_desc* d, int bn, cudaStream_t stream) {
  if (d->dtype == SP24_F16) return launch_raw_t<half>(d, bn, stream);
  if (d->dtype == SP24_BF16) return launch_raw_t<__nv_bfloat16>(d, bn, stream);
  return launch_raw_t<__nv_fp8_e4m3>(d, bn, stream);
}

sp24_status gemm_impl(const sp24_gemm_desc* d, cudaStream_t stream, unsigned long long timeout_ns,
                      int stall, const sp24_epilogue* e = nullptr,
                      const sp24_peer_out* peers = nullptr) {
  sp24_status st = validate(d);
  if (st != SP24_OK) return st;
  st = validate_epilogue(d, e);
  if (st != SP24_OK) return st;
  st = validate_peers(d, peers);
  if (st != SP24_OK) return st;
  const WsPlan w = plan_workspace(d);
  if (w.total > 0 && (d->workspace == nullptr || d->workspace_bytes < w.total))
    return SP24_ERR_WORKSPACE;
  if (w.total > 0 && !aligned16(d->workspace)) return SP24_ERR_ALIGN;
  DeviceInfo* di = nullptr;
  st = device_info(&di);
  if (st != SP24_OK) return st;
  uint8_t* ws = static_cast<uint8_t*>(d->workspace);

  Prepared p{};
  p.dt = d->dtype;
  p.m = d->m;
  p.n = d->n;
  p.k = d->k;
  p.a_c = d->a_c;
  p.lda_c = d->lda_c ? d->lda_c : d->k / 2;
  p.b = d->b;
  p.ldb = d->ldb ? d->ldb : d->n;
  p.c_f32 = d->c_f32;
  p.c_bf16 = d->c_bf16;
  p.ldc = d->ldc ? d->ldc : d->n;
  p.alpha = d->alpha == 0.0f ? 1.0f : d->alpha;
  p.idesc_ab = idesc_ab(d->dtype);
  if (peers != nullptr) {
    p.peers.n = peers->n_peers;
    for (int i = 0; i < peers->n_peers; ++i) {
      p.peers.f32[i] = d->c_f32 != nullptr ? peers->c_f32[i] : nullptr;
      p.peers.bf16[i] = d->c_bf16 != nullptr ? static_cast<__nv_bfloat16*>(peers->c_bf16[i]) : nullptr;
    }
  }
  if (e != nullptr) {
    p.bias = e->bias;
    p.act = e->act == SP24_ACT_SILU ? sp24::kActSilu : sp24::kActNone;
    p.a_c_up = e->a_c_up;
    p.lda_c_up = e->lda_c_up ? e->lda_c_up : d->k / 2;
    p.meta_up = e->meta_up;
    p.alpha_up = e->alpha_up == 0.0f ? 1.0f : e->alpha_up;
    p.bias_up = e->bias_up;
  }
  p.status = d->status_dev ? d->status_dev : di->status_word;
  p.timeout_ns = timeout_ns;
  p.stall_producer = stall;
  p.static_weights =
      (g_launch_hints & SP24_HINT_STATIC_WEIGHTS) != 0 && d->meta_format == SP24_META_TC ? 1 : 0;
  p.tune = tuning();

  if (const int rbn = raw_route_bn(d, e, peers, p.tune)) return launch_raw(d, rbn, stream);
  if (d->meta_format == SP24_META_REF) {
    st = sp24_repack_meta(d->dtype, d->meta, d->m, d->k, ws + w.meta_off,
                          reinterpret_cast<sp24_stream_t>(stream));
    if (st != SP24_OK) return st;
    p.meta_tc = ws + w.meta_off;
  } else if (d->meta_format == SP24_META_K16) {
    st = sp24_repack_meta_k16(d->dtype, reinterpret_cast<const uint32_t*>(d->meta), d->m, d->k,
                              ws + w.meta_off, reinterpret_cast<sp24_stream_t>(stream));
    if (st != SP24_OK) return st;
    p.meta_tc = ws + w.meta_off;
  } else {
    p.meta_tc = d->meta;
  }
  if (w.b_bytes > 0) {
    const int es = esize(d->dtype);
    uint8_t* bp = ws + w.b_off;
    SP24_CUDA_TRY(cudaMemsetAsync(bp, 0, w.b_bytes, stream));
    SP24_CUDA_TRY(cudaMemcpy2DAsync(bp, static_cast<size_t>(w.b_pitch_elems) * es, d->b,
                                    static_cast<size_t>(p.ldb) * es, static_cast<size_t>(d->n) * es,
                                    static_cast<size_t>(d->k), cudaMemcpyDeviceToDevice, stream));
    p.b = bp;
    p.ldb = w.b_pitch_elems;
  }

  if (p.a_c_up != nullptr) {
    // The gated product, in order of preference (W_gate/W_up 14336 x 4096):
    //  1. 33..128 columns with enough 256-row tiles: one launch of the
    //     CTA-pair kernel's gated form (T = 64: 29.1 us, T = 128: 35.1 us);
    //  2. up to 64 columns, and for wider N while the tile count is modest:
    //     one launch of the split-K kernel's gated form (T = 16: 26.5 us);
    //  3. otherwise two passes, each on the kernel the plain dispatch picks
    //     (65..128 columns with few row tiles: the pair K-split form, which
    //     beat the one split-K launch, 42.7 us against 46.9 us at T = 128).
    // SP24_GATED=1|2 forces 2 or 3; SP24_PAIR_GATED (set) skips 1.
    const int bn = std::min(128, choose_bn(d->m, d->n, d->tile_n, di->sm_count));
    const long long tiles = static_cast<long long>((d->m + 127) / 128) * ((d->n + bn - 1) / bn);
    int pks = 0;
    const Tuning& t = p.tune;
    const bool pairs_narrow = d->n > 64 && d->n <= 128 &&
                              (narrow_pair_width(d, di->sm_count, t) > 0 ||
                               narrow_pair_splitk_width(d, di->sm_count, &pks, t) > 0);
    const int gmode = t.gated;
    const bool one_launch = gmode == 1 || (gmode != 2 && !pairs_narrow &&
                                           (d->n <= 128 || tiles <= 4LL * di->sm_count));
    const int npg = narrow_pair_width(d, di->sm_count, t);
    if (gmode != 1 && gmode != 2 && npg >= 64 && d->n > 32 && t.pair_gated) {
      // 1: W_gate and W_up against the same B stages of a CTA pair.
      LaunchFn pg = d->dtype == SP24_F16    ? pick_pair_gated<0>(npg)
                    : d->dtype == SP24_BF16 ? pick_pair_gated<1>(npg)
                                            : pick_pair_gated<2>(npg);
      return pg(p, *di, stream);
    }
    if (one_launch) {
      // 2: both weights through the split-K kernel's ring.
      const int sbn = splitk_tile_n(d, bn, t);
      LaunchFn gf = d->dtype == SP24_F16    ? pick_gated<0>(sbn)
                    : d->dtype == SP24_BF16 ? pick_gated<1>(sbn)
                                            : pick_gated<2>(sbn);
      return gf(p, *di, stream);
    }
    // 3: two passes with C as the intermediate.  Pass 1 writes
    // act(alpha W_gate B + bias) into C (fp32 when the caller asked for it,
    // else bf16); pass 2 multiplies (alpha_up W_up B + bias_up) by it in its
    // epilogue and writes the result.
    Prepared p1 = p;
    p1.a_c_up = nullptr;
    p1.c_reread = 1;
    if (p1.c_f32 != nullptr) p1.c_bf16 = nullptr;
    st = launch_plain(d, p1, *di, stream);
    if (st != SP24_OK) return st;
    Prepared p2 = p;
    p2.a_c_up = nullptr;
    p2.a_c = p.a_c_up;
    p2.lda_c = p.lda_c_up;
    p2.meta_tc = p.meta_up;
    p2.alpha = p.alpha_up;
    p2.bias = p.bias_up;
    p2.act = sp24::kActNone;
    p2.gate_from_c = 1;
    return launch_plain(d, p2, *di, stream);
  }
  return launch_plain(d, p, *di, stream);
}

// The kernel choice for one plain (or pass-of-two) GEMM.
sp24_status launch_plain(const sp24_gemm_desc* d, const Prepared& p, const DeviceInfo& di_ref,
                         cudaStream_t stream) {
  const DeviceInfo* di = &di_ref;
  const Tuning& t = p.tune;
  if (use_pair_kernel(d->m, d->n, d->tile_n, t)) {
    return pick_pair(d->dtype, t)(p, *di, stream);
  }
  const int bn = choose_bn(d->m, d->n, d->tile_n, di->sm_count);
  int np = narrow_pair_width(d, di->sm_count, t);
  if (np == 0) np = short_k_pair_width(d, t);
  if (np > 0) {
    LaunchFn nf = d->dtype == SP24_F16    ? pick_narrow_pair<0>(np)
                  : d->dtype == SP24_BF16 ? pick_narrow_pair<1>(np)
                                          : pick_narrow_pair<2>(np);
    return nf(p, *di, stream);
  }
  int pks = 0;
  const int npk = narrow_pair_splitk_width(d, di->sm_count, &pks, t);
  if (npk > 0) {
    return d->dtype == SP24_F16    ? pick_pair_splitk<0>(npk)(p, *di, stream, pks)
           : d->dtype == SP24_BF16 ? pick_pair_splitk<1>(npk)(p, *di, stream, pks)
                                   : pick_pair_splitk<2>(npk)(p, *di, stream, pks);
  }
  if (use_splitk_kernel(d->m, d->n, bn, di->sm_count, t)) {
    const int kb = splitk_units(bn, t);
    const int sbn = splitk_tile_n(d, bn, t);
    LaunchFn sf = d->dtype == SP24_F16    ? pick_splitk<0>(sbn, kb)
                  : d->dtype == SP24_BF16 ? pick_splitk<1>(sbn, kb)
                                          : pick_splitk<2>(sbn, kb);
    return sf(p, *di, stream);
  }
  LaunchFn fn = d->dtype == SP24_F16    ? pick_bn<0>(bn)
                : d->dtype == SP24_BF16 ? pick_bn<1>(bn)
                                        : pick_bn<2>(bn);
  return fn(p, *di, stream);
}

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices];

// Device address of the no-alloc scratch for the current device.
sp24_status noalloc_scratch(void** out) {
  int dev = 0;
  SP24_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return SP24_ERR_ARG;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_sp24_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      return SP24_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return SP24_OK;
}

unsigned int grid_for(long long work, int block) {
  long long g = (work + block - 1) / block;
  if (g < 1) g = 1;
  return static_cast<unsigned int>(std::min<long long>(g, 0x7FFFFFFF));
}

}  // namespace

extern "C" {

const char* sp24_version(void) { return "sp24 0.1.0 (sm_100a tcgen05.mma.sp)"; }

const char* sp24_status_string(sp24_status s) {
  switch (s) {
    case SP24_OK: return "ok";
    case SP24_ERR_SHAPE: return "invalid shape";
    case SP24_ERR_ALIGN: return "pointer or stride misaligned for TMA";
    case SP24_ERR_NOT_2OF4: return "A is not 2:4 sparse";
    case SP24_ERR_ARCH: return "device is not sm_100";
    case SP24_ERR_CUDA: return "CUDA runtime error";
    case SP24_ERR_TIMEOUT: return "bounded device wait timed out";
    case SP24_ERR_NCCL: return "NCCL error";
    case SP24_ERR_ARG: return "invalid argument";
    case SP24_ERR_WORKSPACE: return "workspace missing or too small";
    case SP24_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the no-alloc buffer (SP24_NOALLOC_SCRATCH_BYTES)";
  }
  return "unknown status";
}

sp24_status sp24_check_device(int device) {
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SP24_ERR_CUDA;
  }
  return (prop.major == 10 && prop.minor == 0) ? SP24_OK : SP24_ERR_ARCH;
}

size_t sp24_meta_tc_bytes(int m, int k) {
  if (m <= 0 || k <= 0) return 0;
  return static_cast<size_t>(meta_mblocks(m)) * meta_katoms(k) * sp24::kAtomBytes;
}

size_t sp24_gemm_workspace_bytes(const sp24_gemm_desc* d) {
  if (validate(d) != SP24_OK) return 0;
  return plan_workspace(d).total;
}

sp24_status sp24_gemm(const sp24_gemm_desc* d, sp24_stream_t stream) {
  return gemm_impl(d, as_stream(stream), kDefaultTimeoutNs, 0);
}

// sp24_gemm with a fused epilogue (bias, SiLU, or the gated SwiGLU form).
sp24_status sp24_gemm_fused(const sp24_gemm_desc* d, const sp24_epilogue* e,
                            sp24_stream_t stream) {
  return gemm_impl(d, as_stream(stream), kDefaultTimeoutNs, 0, e);
}

sp24_status sp24_gemm_allgather(const sp24_gemm_desc* d, const sp24_peer_out* peers,
                                sp24_stream_t stream) {
  if (peers == nullptr) return SP24_ERR_ARG;
  return gemm_impl(d, as_stream(stream), kDefaultTimeoutNs, 0, nullptr, peers);
}

}  // extern "C"

namespace {

// Peer access between devices of this process, enabled once per ordered
// pair (sp24_gemm_multi's fused all-gather stores into peers' C).
std::mutex g_peer_mu;
bool g_peer_on[kMaxDevices][kMaxDevices];

sp24_status enable_peer(int dev, int peer) {
  std::lock_guard<std::mutex> lk(g_peer_mu);
  if (g_peer_on[dev][peer]) return SP24_OK;
  int can = 0;
  SP24_CUDA_TRY(cudaDeviceCanAccessPeer(&can, dev, peer));
  if (!can) return SP24_ERR_CUDA;
  SP24_CUDA_TRY(cudaSetDevice(dev));
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    return SP24_ERR_CUDA;
  }
  (void)cudaGetLastError();
  g_peer_on[dev][peer] = true;
  return SP24_OK;
}

// Restores the calling thread's current device when it leaves scope.
struct DeviceRestore {
  int dev = -1;
  DeviceRestore() {
    if (cudaGetDevice(&dev) != cudaSuccess) {
      (void)cudaGetLastError();
      dev = -1;
    }
  }
  ~DeviceRestore() {
    if (dev >= 0) (void)cudaSetDevice(dev);
  }
};

// Host-side checks of a multi-GPU descriptor (no CUDA calls).
sp24_status validate_multi(const sp24_multi_desc* md, int allgather_c) {
  if (md == nullptr) return SP24_ERR_ARG;
  const int ng = md->ngpu;
  if (ng < 1 || ng > SP24_MAX_GPUS) return SP24_ERR_ARG;
  if ((md->b_layout != SP24_MULTI_FULL && md->b_layout != SP24_MULTI_SHARD) ||
      (md->c_layout != SP24_MULTI_FULL && md->c_layout != SP24_MULTI_SHARD))
    return SP24_ERR_ARG;
  if (allgather_c && md->c_layout != SP24_MULTI_FULL) return SP24_ERR_ARG;
  const bool want32 = md->c_f32[0] != nullptr, want16 = md->c_bf16[0] != nullptr;
  if (!want32 && !want16) return SP24_ERR_ARG;
  for (int g = 0; g < ng; ++g) {
    if (md->devices[g] < 0 || md->devices[g] >= kMaxDevices) return SP24_ERR_ARG;
    for (int h = 0; h < g; ++h)
      if (md->devices[h] == md->devices[g]) return SP24_ERR_ARG;
    if (md->a_c[g] == nullptr || md->meta[g] == nullptr || md->b[g] == nullptr) return SP24_ERR_ARG;
    if ((md->c_f32[g] != nullptr) != want32 || (md->c_bf16[g] != nullptr) != want16)
      return SP24_ERR_ARG;
  }
  if (md->gemm.m <= 0 || md->gemm.n <= 0 || md->gemm.k <= 0) return SP24_ERR_SHAPE;
  // Whole-matrix layouts address a device's columns through the row stride,
  // which must then span all n columns (a shard's own check sees only its width).
  if (md->b_layout == SP24_MULTI_FULL && md->gemm.ldb != 0 && md->gemm.ldb < md->gemm.n)
    return SP24_ERR_SHAPE;
  if (md->c_layout == SP24_MULTI_FULL && md->gemm.ldc != 0 && md->gemm.ldc < md->gemm.n)
    return SP24_ERR_SHAPE;
  return SP24_OK;
}

// Device g's share of a multi-GPU GEMM as a one-device descriptor; sets
// *empty when the device owns no columns.
sp24_gemm_desc shard_desc(const sp24_multi_desc* md, int g, int* n0_out, bool* empty) {
  const sp24_gemm_desc& G = md->gemm;
  int n0 = 0, n1 = 0;
  sp24_shard_columns(G.n, md->ngpu, g, 256, &n0, &n1);
  *n0_out = n0;
  *empty = n1 <= n0;
  const size_t es = static_cast<size_t>(esize(G.dtype));
  sp24_gemm_desc d = G;
  d.n = std::max(1, n1 - n0);
  d.a_c = md->a_c[g];
  d.meta = md->meta[g];
  if (md->b_layout == SP24_MULTI_FULL) {
    d.b = static_cast<const uint8_t*>(md->b[g]) + static_cast<size_t>(n0) * es;
    d.ldb = G.ldb ? G.ldb : G.n;
  } else {
    d.b = md->b[g];
    d.ldb = n1 - n0;
  }
  if (md->c_layout == SP24_MULTI_FULL) {
    d.c_f32 = md->c_f32[g] != nullptr ? md->c_f32[g] + n0 : nullptr;
    d.c_bf16 = md->c_bf16[g] != nullptr ? static_cast<uint8_t*>(md->c_bf16[g]) + 2 * static_cast<size_t>(n0)
                                        : nullptr;
    d.ldc = G.ldc ? G.ldc : G.n;
  } else {
    d.c_f32 = md->c_f32[g];
    d.c_bf16 = md->c_bf16[g];
    d.ldc = n1 - n0;
  }
  d.workspace = md->workspace[g];
  d.workspace_bytes = md->workspace_bytes;
  d.status_dev = nullptr;
  return d;
}

}  // namespace

extern "C" {

sp24_status sp24_gemm_multi(const sp24_multi_desc* md, int allgather_c) {
  sp24_status st = validate_multi(md, allgather_c);
  if (st != SP24_OK) return st;
  const int ng = md->ngpu;
  sp24_gemm_desc d[SP24_MAX_GPUS];
  int n0[SP24_MAX_GPUS];
  bool empty[SP24_MAX_GPUS];
  for (int g = 0; g < ng; ++g) {
    d[g] = shard_desc(md, g, &n0[g], &empty[g]);
    if (!empty[g]) {
      st = validate(&d[g]);
      if (st != SP24_OK) return st;
    }
  }
  DeviceRestore restore;
  if (allgather_c && ng > 1)
    for (int g = 0; g < ng; ++g)
      for (int h = 0; h < ng; ++h)
        if (h != g) {
          st = enable_peer(md->devices[g], md->devices[h]);
          if (st != SP24_OK) return st;
        }
  for (int g = 0; g < ng; ++g) {
    if (empty[g]) continue;
    SP24_CUDA_TRY(cudaSetDevice(md->devices[g]));
    const cudaStream_t s = as_stream(md->streams[g]);
    if (allgather_c && ng > 1) {
      sp24_peer_out po{};
      for (int h = 0; h < ng; ++h) {
        if (h == g) continue;
        po.c_f32[po.n_peers] = md->c_f32[h] != nullptr ? md->c_f32[h] + n0[g] : nullptr;
        po.c_bf16[po.n_peers] = md->c_bf16[h] != nullptr
                                    ? static_cast<uint8_t*>(md->c_bf16[h]) + 2 * static_cast<size_t>(n0[g])
                                    : nullptr;
        ++po.n_peers;
      }
      st = gemm_impl(&d[g], s, kDefaultTimeoutNs, 0, nullptr, &po);
    } else {
      st = gemm_impl(&d[g], s, kDefaultTimeoutNs, 0);
    }
    if (st != SP24_OK) return st;
  }
  if (allgather_c && ng > 1) {
    // Every stream waits for every device's launch: the gathered C is
    // complete for work enqueued after this call.  Events are per call (no
    // state shared between concurrent callers) and released at once; the
    // waits already enqueued keep what they need.
    cudaEvent_t ev[SP24_MAX_GPUS] = {};
    for (int g = 0; g < ng; ++g) {
      SP24_CUDA_TRY(cudaSetDevice(md->devices[g]));
      SP24_CUDA_TRY(cudaEventCreateWithFlags(&ev[g], cudaEventDisableTiming));
      SP24_CUDA_TRY(cudaEventRecord(ev[g], as_stream(md->streams[g])));
    }
    sp24_status wst = SP24_OK;
    for (int g = 0; g < ng && wst == SP24_OK; ++g) {
      if (cudaSetDevice(md->devices[g]) != cudaSuccess) wst = SP24_ERR_CUDA;
      for (int h = 0; h < ng && wst == SP24_OK; ++h)
        if (h != g && cudaStreamWaitEvent(as_stream(md->streams[g]), ev[h], 0) != cudaSuccess)
          wst = SP24_ERR_CUDA;
    }
    for (int g = 0; g < ng; ++g) {
      (void)cudaSetDevice(md->devices[g]);
      (void)cudaEventDestroy(ev[g]);
    }
    if (wst != SP24_OK) (void)cudaGetLastError();
    return wst;
  }
  return SP24_OK;
}

size_t sp24_gemm_multi_workspace_bytes(const sp24_multi_desc* md) {
  if (validate_multi(md, 0) != SP24_OK) return 0;
  size_t need = 0;
  for (int g = 0; g < md->ngpu; ++g) {
    int n0 = 0;
    bool empty = false;
    const sp24_gemm_desc d = shard_desc(md, g, &n0, &empty);
    if (!empty && validate(&d) == SP24_OK) need = std::max(need, plan_workspace(&d).total);
  }
  return need;
}

sp24_status sp24_replicate(const void* src, int src_device, size_t bytes, int ngpu,
                           const int* devices, void* const* dst, const sp24_stream_t* streams) {
  if (src == nullptr || devices == nullptr || dst == nullptr || ngpu < 1 || ngpu > SP24_MAX_GPUS)
    return SP24_ERR_ARG;
  for (int g = 0; g < ngpu; ++g)
    if (dst[g] == nullptr || devices[g] < 0) return SP24_ERR_ARG;
  DeviceRestore restore;
  for (int g = 0; g < ngpu; ++g) {
    if (dst[g] == src && devices[g] == src_device) continue;
    SP24_CUDA_TRY(cudaSetDevice(devices[g]));
    SP24_CUDA_TRY(cudaMemcpyPeerAsync(dst[g], devices[g], src, src_device, bytes,
                                      as_stream(streams != nullptr ? streams[g] : nullptr)));
  }
  return SP24_OK;
}

sp24_status sp24_ipc_get_handle(const void* dev_ptr, void* handle64, size_t* offset) {
  if (dev_ptr == nullptr || handle64 == nullptr || offset == nullptr) return SP24_ERR_ARG;
  sp24_status st = get_range_fn();
  if (st != SP24_OK) return st;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return SP24_ERR_CUDA;
  cudaIpcMemHandle_t h;
  SP24_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle64, &h, sizeof(h));
  *offset = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return SP24_OK;
}

sp24_status sp24_ipc_open_handle(const void* handle64, void** base) {
  if (handle64 == nullptr || base == nullptr) return SP24_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  SP24_CUDA_TRY(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
  return SP24_OK;
}

sp24_status sp24_ipc_close(void* base) {
  if (base == nullptr) return SP24_ERR_ARG;
  SP24_CUDA_TRY(cudaIpcCloseMemHandle(base));
  return SP24_OK;
}

// Allocation-free sp24_gemm: the scratch sp24_gemm would take from
// d->workspace comes from the fixed device buffer g_sp24_noalloc_scratch.
sp24_status sp24_gemm_noalloc(const sp24_gemm_desc* d, sp24_stream_t stream) {
  sp24_status st = validate(d);
  if (st != SP24_OK) return st;
  if (plan_workspace(d).total > SP24_NOALLOC_SCRATCH_BYTES) return SP24_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st != SP24_OK) return st;
  sp24_gemm_desc local = *d;
  local.workspace = scratch;
  local.workspace_bytes = SP24_NOALLOC_SCRATCH_BYTES;
  return gemm_impl(&local, as_stream(stream), kDefaultTimeoutNs, 0);
}

// Self-test of the bounded-wait path: runs the GEMM with a producer that
// never issues a load, so the MMA and epilogue waits run out after
// `timeout_ns`; the kernel returns and raises the status word.  Synchronises
// `stream` and returns SP24_ERR_TIMEOUT when that happened (the expected
// result), SP24_OK if it did not.
sp24_status sp24_selftest_timeout(const sp24_gemm_desc* d, unsigned long long timeout_ns,
                                  sp24_stream_t stream) {
  if (d == nullptr || d->status_dev == nullptr) return SP24_ERR_ARG;
  cudaStream_t s = as_stream(stream);
  SP24_CUDA_TRY(cudaMemsetAsync(d->status_dev, 0, sizeof(int), s));
  sp24_status st = gemm_impl(d, s, timeout_ns, 1);
  if (st != SP24_OK) return st;
  int h = 0;
  SP24_CUDA_TRY(cudaMemcpyAsync(&h, d->status_dev, sizeof(int), cudaMemcpyDeviceToHost, s));
  SP24_CUDA_TRY(cudaStreamSynchronize(s));
  return h ? SP24_ERR_TIMEOUT : SP24_OK;
}

void sp24_set_launch_hints(unsigned hints) { g_launch_hints = hints; }

void sp24_reload_tuning(void) {
  const Tuning t = read_tuning();
  std::lock_guard<std::mutex> lk(g_tuning_mu);
  g_tuning = t;
  g_tuning_loaded = true;
}

unsigned sp24_get_launch_hints(void) { return g_launch_hints; }

sp24_status sp24_last_kernel_status(sp24_stream_t stream) {
  DeviceInfo* di = nullptr;
  sp24_status st = device_info(&di);
  if (st != SP24_OK) return st;
  cudaStream_t s = as_stream(stream);
  int h = 0, hr = 0;
  SP24_CUDA_TRY(cudaMemcpyAsync(&h, di->status_word, sizeof(int), cudaMemcpyDeviceToHost, s));
  // The tiny reference-layout route's kernel keeps its own flag.
  SP24_CUDA_TRY(cudaMemcpyFromSymbolAsync(&hr, sp24_raw_kernel_status, sizeof(int), 0,
                                          cudaMemcpyDeviceToHost, s));
  SP24_CUDA_TRY(cudaStreamSynchronize(s));
  if (h || hr) {
    const int zero = 0;
    if (h) SP24_CUDA_TRY(cudaMemsetAsync(di->status_word, 0, sizeof(int), s));
    if (hr)
      SP24_CUDA_TRY(cudaMemcpyToSymbolAsync(sp24_raw_kernel_status, &zero, sizeof(int), 0,
                                            cudaMemcpyHostToDevice, s));
    SP24_CUDA_TRY(cudaStreamSynchronize(s));
    return SP24_ERR_TIMEOUT;
  }
  return SP24_OK;
}

sp24_status sp24_compress(sp24_dtype dtype, const void* a_dense, int m, int k, int64_t lda,
                          void* a_c, int64_t ldac, uint8_t* meta_ref, long long* bad_dev,
                          long long* bad_host, sp24_stream_t stream) {
  if (!dtype_ok(dtype) || a_dense == nullptr || a_c == nullptr || meta_ref == nullptr ||
      bad_dev == nullptr)
    return SP24_ERR_ARG;
  if (m <= 0 || k <= 0 || k % 8 != 0) return SP24_ERR_SHAPE;
  if (lda == 0) lda = k;
  if (ldac == 0) ldac = k / 2;
  if (lda < k || ldac < k / 2) return SP24_ERR_SHAPE;
  const int es = esize(dtype);
  const int need = es == 2 ? 16 : 8;
  if ((reinterpret_cast<uintptr_t>(a_dense) % need) != 0 || (lda * es) % need != 0 ||
      (reinterpret_cast<uintptr_t>(a_c) % (need / 2)) != 0 || (ldac * es) % (need / 2) != 0)
    return SP24_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  SP24_CUDA_TRY(cudaMemsetAsync(bad_dev, 0xFF, sizeof(long long), s));
  const int chunks_per_thread = 4;                  // compress_kernel's U
  const long long work = static_cast<long long>(m) * (k / 8);
  // The kernel indexes units with 32-bit arithmetic (work plus one block's span).
  if (work + static_cast<long long>(sp24::kPrepThreads) * chunks_per_thread >= (1LL << 32))
    return SP24_ERR_SHAPE;
  const unsigned int g = grid_for(work, sp24::kPrepThreads * chunks_per_thread);
  auto* bad = reinterpret_cast<unsigned long long*>(bad_dev);
  const auto* a8 = static_cast<const uint8_t*>(a_dense);
  auto* c8 = static_cast<uint8_t*>(a_c);
  if (es == 2)
    sp24::compress_kernel<2><<<g, sp24::kPrepThreads, 0, s>>>(a8, m, k, lda * 2, c8, ldac * 2, meta_ref, bad);
  else
    sp24::compress_kernel<1><<<g, sp24::kPrepThreads, 0, s>>>(a8, m, k, lda, c8, ldac, meta_ref, bad);
  SP24_CUDA_TRY(cudaGetLastError());
  long long h = -1;
  SP24_CUDA_TRY(cudaMemcpyAsync(&h, bad_dev, sizeof(long long), cudaMemcpyDeviceToHost, s));
  SP24_CUDA_TRY(cudaStreamSynchronize(s));
  if (bad_host) *bad_host = h;
  return h < 0 ? SP24_OK : SP24_ERR_NOT_2OF4;
}

sp24_status sp24_prune_2of4(sp24_dtype dtype, const void* a, int m, int k, int64_t lda,
                            void* a_pruned, int64_t ldp, sp24_stream_t stream) {
  if (!dtype_ok(dtype) || a == nullptr || a_pruned == nullptr) return SP24_ERR_ARG;
  if (m <= 0 || k <= 0 || k % 4 != 0) return SP24_ERR_SHAPE;
  if (lda == 0) lda = k;
  if (ldp == 0) ldp = k;
  if (lda < k || ldp < k) return SP24_ERR_SHAPE;
  const int es = esize(dtype);
  const int need = 4 * es;
  if ((reinterpret_cast<uintptr_t>(a) % need) || (reinterpret_cast<uintptr_t>(a_pruned) % need) ||
      (lda * es) % need || (ldp * es) % need)
    return SP24_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  const int groups_per_thread = 8;                  // prune_kernel's U
  const long long work = static_cast<long long>(m) * (k / 4);
  if (work + static_cast<long long>(sp24::kPrepThreads) * groups_per_thread >= (1LL << 32))
    return SP24_ERR_SHAPE;
  const unsigned int g = grid_for(work, sp24::kPrepThreads * groups_per_thread);
  const auto* a8 = static_cast<const uint8_t*>(a);
  auto* p8 = static_cast<uint8_t*>(a_pruned);
  if (dtype == SP24_F16)
    sp24::prune_kernel<0><<<g, sp24::kPrepThreads, 0, s>>>(a8, m, k, lda * 2, p8, ldp * 2);
  else if (dtype == SP24_BF16)
    sp24::prune_kernel<1><<<g, sp24::kPrepThreads, 0, s>>>(a8, m, k, lda * 2, p8, ldp * 2);
  else
    sp24::prune_kernel<2><<<g, sp24::kPrepThreads, 0, s>>>(a8, m, k, lda, p8, ldp);
  SP24_CUDA_TRY(cudaGetLastError());
  return SP24_OK;
}

sp24_status sp24_repack_meta(sp24_dtype dtype, const uint8_t* meta_ref, int m, int k,
                             uint8_t* meta_tc, sp24_stream_t stream) {
  if (!dtype_ok(dtype) || meta_ref == nullptr || meta_tc == nullptr) return SP24_ERR_ARG;
  if (m <= 0 || k <= 0 || k % (is_fp8(dtype) ? 64 : 32) != 0) return SP24_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(meta_tc) & 3u) != 0) return SP24_ERR_ALIGN;
  const int mb = meta_mblocks(m);
  const int ka = meta_katoms(k);
  const long long total = static_cast<long long>(ka) * mb * 128 * 4;
  cudaStream_t s = as_stream(stream);
  sp24::repack_meta_kernel<<<grid_for(total, 256), 256, 0, s>>>(
      meta_ref, m, k, is_fp8(dtype) ? 1 : 0, reinterpret_cast<uint32_t*>(meta_tc), mb, ka);
  SP24_CUDA_TRY(cudaGetLastError());
  return SP24_OK;
}

sp24_status sp24_repack_meta_k16(sp24_dtype dtype, const uint32_t* meta_k16, int m, int k,
                                 uint8_t* meta_tc, sp24_stream_t stream) {
  if (!dtype_ok(dtype) || is_fp8(dtype) || meta_k16 == nullptr || meta_tc == nullptr)
    return SP24_ERR_ARG;
  if (m <= 0 || k <= 0 || k % 32 != 0 || m % 16 != 0) return SP24_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(meta_tc) & 3u) != 0 ||
      (reinterpret_cast<uintptr_t>(meta_k16) & 3u) != 0)
    return SP24_ERR_ALIGN;
  const int mb = meta_mblocks(m);
  const int ka = meta_katoms(k);
  const long long total = static_cast<long long>(ka) * mb * 128 * 4;
  cudaStream_t s = as_stream(stream);
  sp24::repack_meta_kernel<<<grid_for(total, 256), 256, 0, s>>>(
      nullptr, m, k, 0, reinterpret_cast<uint32_t*>(meta_tc), mb, ka, meta_k16);
  SP24_CUDA_TRY(cudaGetLastError());
  return SP24_OK;
}

sp24_status sp24_amax_f32(const float* x, size_t count, float* amax_dev, sp24_stream_t stream) {
  if (x == nullptr || amax_dev == nullptr) return SP24_ERR_ARG;
  cudaStream_t s = as_stream(stream);
  SP24_CUDA_TRY(cudaMemsetAsync(amax_dev, 0, sizeof(float), s));
  if (count == 0) return SP24_OK;
  DeviceInfo* di = nullptr;
  sp24_status st = device_info(&di);
  if (st != SP24_OK) return st;
  const unsigned int g = std::min<unsigned int>(grid_for(static_cast<long long>(count), 256),
                                                static_cast<unsigned int>(di->sm_count) * 8u);
  if (aligned16(x))
    sp24::amax_kernel<1><<<g, 256, 0, s>>>(x, count, amax_dev);
  else
    sp24::amax_kernel<0><<<g, 256, 0, s>>>(x, count, amax_dev);
  SP24_CUDA_TRY(cudaGetLastError());
  return SP24_OK;
}

}  // extern "C"

namespace {
template <int E5M2>
sp24_status quantize_fp8(const float* x, size_t count, const float* amax_dev, float* scale_dev,
                         uint8_t* q, sp24_stream_t stream) {
  if (x == nullptr || amax_dev == nullptr || q == nullptr) return SP24_ERR_ARG;
  if (count == 0) return SP24_OK;
  DeviceInfo* di = nullptr;
  sp24_status st = device_info(&di);
  if (st != SP24_OK) return st;
  cudaStream_t s = as_stream(stream);
  const unsigned int g = std::min<unsigned int>(grid_for(static_cast<long long>(count), 256),
                                                static_cast<unsigned int>(di->sm_count) * 16u);
  if (aligned16(x) && (reinterpret_cast<uintptr_t>(q) & 3u) == 0)
    sp24::quantize_fp8_kernel<E5M2, 1><<<g, 256, 0, s>>>(x, count, amax_dev, scale_dev, q);
  else
    sp24::quantize_fp8_kernel<E5M2, 0><<<g, 256, 0, s>>>(x, count, amax_dev, scale_dev, q);
  SP24_CUDA_TRY(cudaGetLastError());
  return SP24_OK;
}
}  // namespace

extern "C" {

sp24_status sp24_quantize_e4m3(const float* x, size_t count, const float* amax_dev,
                               float* scale_dev, uint8_t* q, sp24_stream_t stream) {
  return quantize_fp8<0>(x, count, amax_dev, scale_dev, q, stream);
}

sp24_status sp24_quantize_e5m2(const float* x, size_t count, const float* amax_dev,
                               float* scale_dev, uint8_t* q, sp24_stream_t stream) {
  return quantize_fp8<1>(x, count, amax_dev, scale_dev, q, stream);
}

void sp24_shard_columns(int n, int world, int rank, int align, int* n0, int* n1) {
  if (world < 1) world = 1;
  if (align < 1) align = 1;
  const int per_raw = (n + world - 1) / world;
  const int per = (per_raw + align - 1) / align * align;
  int a = std::min(rank * per, n);
  int b = (rank == world - 1) ? n : std::min(a + per, n);
  if (n0) *n0 = a;
  if (n1) *n1 = b;
}

sp24_status sp24_unshard_columns_f32(const float* src, float* dst, int m, int n, int world,
                                     int align, sp24_stream_t stream) {
  if (src == nullptr || dst == nullptr || world < 1) return SP24_ERR_ARG;
  if (m <= 0 || n <= 0) return SP24_ERR_SHAPE;
  int n0 = 0, n1 = 0;
  sp24_shard_columns(n, world, 0, align, &n0, &n1);
  const int per = std::max(1, n1 - n0);
  cudaStream_t s = as_stream(stream);
  const int vec = (per % 4 == 0 && n % 4 == 0 && aligned16(src) && aligned16(dst)) ? 1 : 0;
  const int per_row = vec ? (n + 3) / 4 : n;
  const unsigned gx = static_cast<unsigned>(std::min(64, std::max(1, (per_row + 255) / 256)));
  const unsigned gy = static_cast<unsigned>(std::min(m, 65535));
  sp24::unshard_columns_kernel<<<dim3(gx, gy), 256, 0, s>>>(src, dst, m, n, world, per, vec);
  SP24_CUDA_TRY(cudaGetLastError());
  return SP24_OK;
}

}  // extern "C"
