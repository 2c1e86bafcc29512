// sp24_oracle.cpp — TEST INFRASTRUCTURE ONLY.  CPU restatement of the
// reference's host-side algorithms for the 2:4 sparse GEMM path, used as the
// parity checker by tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline leg.  Nothing in the product library links or calls this file.
//
// Parity is pinned: tests/test_oracle.py checks every function below
// bit-for-bit against golden vectors produced by the reference's own code
// (tests/golden/, made by tests/golden/make_golden.py through oracle/_ref).
//
// Restated from codes1gn/sparse-gemm-with-hopper-sptc, wgmma_sp_raw_common.hpp:
//   gen_structured_sparse_a   :63-98   (pair pick with rejection, U(-1,1), snap)
//   gen_pattern_sparse_a      :100-112 (known-answer dyadic A)
//   gen_random_b              :114-127
//   gen_pattern_b             :129-138
//   compress                  :140-205 (nibble = i0 | i1 << 2; the e4m3 table at
//                                        :176-193 yields the same codes)
//   gemm_ref                  :207-225 (fp32, sequential over k, dense A)
//   count_abs_errors          :227-248 (abs tolerance 1e-2)
// plus, with no reference counterpart: magnitude pruning, the tcgen05
// metadata image and the per-tensor e4m3 quantiser.
//
// Element encodings cross this ABI as raw bits: uint16_t for fp16/bf16,
// uint8_t for e4m3 and e5m2.  Conversions use the CUDA headers' host conversions (the
// same ones the reference calls, :48-61), compiled by the host compiler.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

// Element codes (one matrix at a time).  e5m2 appears as A of the reference's
// mixed fp8 entry point (mma_sp_m16n8k64_fp32fp8.cu, A __nv_fp8_e5m2).
enum { DT_F16 = 0, DT_BF16 = 1, DT_E4M3 = 2, DT_E5M2 = 3 };

__nv_fp8_interpretation_t fp8_kind(int dt) { return dt == DT_E5M2 ? __NV_E5M2 : __NV_E4M3; }

float to_f(int dt, uint32_t bits) {
  if (dt == DT_F16) {
    __half_raw r;
    r.x = static_cast<unsigned short>(bits);
    return __half2float(__half(r));
  }
  if (dt == DT_BF16) {
    uint32_t w = bits << 16;
    float f;
    std::memcpy(&f, &w, 4);
    return f;
  }
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(bits), fp8_kind(dt));
  return __half2float(__half(h));
}

uint32_t from_f(int dt, float v) {
  if (dt == DT_F16) {
    __half h = __float2half_rn(v);
    return static_cast<__half_raw>(h).x;
  }
  if (dt == DT_BF16) {
    __nv_bfloat16 b = __float2bfloat16(v);
    return static_cast<__nv_bfloat16_raw>(b).x;
  }
  return __nv_cvt_float_to_fp8(v, __NV_SATFINITE, fp8_kind(dt));
}

int esz(int dt) { return dt >= DT_E4M3 ? 1 : 2; }

uint32_t ld(int dt, const void* p, size_t i) {
  if (esz(dt) == 2) return static_cast<const uint16_t*>(p)[i];
  return static_cast<const uint8_t*>(p)[i];
}
void st(int dt, void* p, size_t i, uint32_t v) {
  if (esz(dt) == 2) static_cast<uint16_t*>(p)[i] = static_cast<uint16_t>(v);
  else static_cast<uint8_t*>(p)[i] = static_cast<uint8_t>(v);
}

bool nonzero(int dt, uint32_t bits) { return to_f(dt, bits) != 0.0f; }

}  // namespace

extern "C" {

// ---------------------------------------------------------------- generator
// Opaque mt19937 shared across the cases of one suite, seeded 1234 by the
// reference suite runner (wgmma_sp_raw_common.hpp:1123).
void* oracle_gen_new(unsigned int seed) { return new std::mt19937(seed); }
void oracle_gen_free(void* g) { delete static_cast<std::mt19937*>(g); }

// Per row, per group of four: draw two distinct positions from {0..3} (redraw
// the second until it differs), order them, draw two U(-1,1) values, push
// |v| < 0.1 away from zero (to +-0.5 for the first, +-0.75 for the second).
void oracle_gen_structured_sparse_a(void* g, int dt, int m, int k, void* a_out) {
  auto& gen = *static_cast<std::mt19937*>(g);
  std::uniform_real_distribution<float> uni(-1.0f, 1.0f);
  std::uniform_int_distribution<int> pos(0, 3);
  const uint32_t zero = from_f(dt, 0.0f);
  for (size_t i = 0; i < static_cast<size_t>(m) * k; ++i) st(dt, a_out, i, zero);
  for (int r = 0; r < m; ++r) {
    for (int grp = 0; grp < k / 4; ++grp) {
      int p = pos(gen);
      int q = pos(gen);
      while (q == p) q = pos(gen);
      const int lo = std::min(p, q), hi = std::max(p, q);
      float x = uni(gen);
      float y = uni(gen);
      if (std::fabs(x) < 0.1f) x = x < 0.0f ? -0.5f : 0.5f;
      if (std::fabs(y) < 0.1f) y = y < 0.0f ? -0.75f : 0.75f;
      const size_t base = static_cast<size_t>(r) * k + grp * 4;
      st(dt, a_out, base + lo, from_f(dt, x));
      st(dt, a_out, base + hi, from_f(dt, y));
    }
  }
}

// Known-answer A: positions 0 and 2 of every group, values dyadic in (row, group).
void oracle_gen_pattern_sparse_a(int dt, int m, int k, void* a_out) {
  const uint32_t zero = from_f(dt, 0.0f);
  for (size_t i = 0; i < static_cast<size_t>(m) * k; ++i) st(dt, a_out, i, zero);
  for (int r = 0; r < m; ++r)
    for (int grp = 0; grp < k / 4; ++grp) {
      const size_t base = static_cast<size_t>(r) * k + grp * 4;
      st(dt, a_out, base + 0, from_f(dt, 1.0f + 0.125f * r + 0.03125f * grp));
      st(dt, a_out, base + 2, from_f(dt, -0.5f - 0.0625f * r + 0.015625f * grp));
    }
}

void oracle_gen_random_b(void* g, int dt, int k, int n, void* b_out) {
  auto& gen = *static_cast<std::mt19937*>(g);
  std::uniform_real_distribution<float> uni(-1.0f, 1.0f);
  for (int kk = 0; kk < k; ++kk)
    for (int nn = 0; nn < n; ++nn) {
      float v = uni(gen);
      if (std::fabs(v) < 0.1f) v = v < 0.0f ? -0.25f : 0.25f;
      st(dt, b_out, static_cast<size_t>(kk) * n + nn, from_f(dt, v));
    }
}

void oracle_gen_pattern_b(int dt, int k, int n, void* b_out) {
  for (int kk = 0; kk < k; ++kk)
    for (int nn = 0; nn < n; ++nn) {
      const float v = static_cast<float>((kk % 7) - 3) * 0.25f + static_cast<float>(nn + 1) * 0.5f;
      st(dt, b_out, static_cast<size_t>(kk) * n + nn, from_f(dt, v));
    }
}

// The legacy warp-level entry points' generation (mma_sp_m16n8k16_fp32fp16.cu /
// mma_sp_m16n8k32_fp32fp16.cu and their bf16 twins), mt19937(42):
//   A: per row, per group of four, two distinct positions (second redrawn until
//      it differs, then ordered) and two U(-1,1) values, 0 replaced by +1 / -1
//      (init_structured_sparse_A, :29-56);
//   order (which = 0, m16n8k16 mains, :265-268): A, then B[i] = U(-1,1);
//   order (which = 1, m16n8k32 mains, :426-437): A[i] = U(-1,1) and
//      B[i] = U(-1,1) for every element, then A overwritten as above.
void oracle_gen_legacy(int which, int dt, int m, int n, int k, void* a_out, void* b_out) {
  std::mt19937 gen(42);
  std::uniform_real_distribution<float> uni(-1.0f, 1.0f);
  auto structured = [&]() {
    std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
    std::uniform_int_distribution<int> pos(0, 3);
    const uint32_t zero = from_f(dt, 0.0f);
    for (size_t i = 0; i < static_cast<size_t>(m) * k; ++i) st(dt, a_out, i, zero);
    for (int r = 0; r < m; ++r)
      for (int grp = 0; grp < k / 4; ++grp) {
        int p = pos(gen);
        int q = pos(gen);
        while (q == p) q = pos(gen);
        const int lo = std::min(p, q), hi = std::max(p, q);
        float x = dist(gen);
        float y = dist(gen);
        if (x == 0.0f) x = 1.0f;
        if (y == 0.0f) y = -1.0f;
        const size_t base = static_cast<size_t>(r) * k + grp * 4;
        st(dt, a_out, base + lo, from_f(dt, x));
        st(dt, a_out, base + hi, from_f(dt, y));
      }
  };
  if (which == 0) {
    structured();
    for (size_t i = 0; i < static_cast<size_t>(k) * n; ++i) st(dt, b_out, i, from_f(dt, uni(gen)));
  } else {
    for (size_t i = 0; i < static_cast<size_t>(m) * k; ++i) st(dt, a_out, i, from_f(dt, uni(gen)));
    for (size_t i = 0; i < static_cast<size_t>(k) * n; ++i) st(dt, b_out, i, from_f(dt, uni(gen)));
    structured();
  }
}

// ---------------------------------------------------------------- compress
// Returns -1 when every group holds exactly two nonzeros, else the first bad
// group as row*(k/4)+group (the reference prints it and exits).
long long oracle_compress(int dt, const void* a, int m, int k, void* a_c, uint8_t* meta) {
  const int groups = k / 4;
  std::memset(meta, 0, static_cast<size_t>(m) * (k / 8));
  for (size_t i = 0; i < static_cast<size_t>(m) * (k / 2); ++i) st(dt, a_c, i, 0);
  for (int r = 0; r < m; ++r)
    for (int grp = 0; grp < groups; ++grp) {
      const size_t base = static_cast<size_t>(r) * k + grp * 4;
      int idx[2] = {-1, -1}, cnt = 0;
      for (int i = 0; i < 4; ++i)
        if (nonzero(dt, ld(dt, a, base + i))) {
          if (cnt < 2) idx[cnt] = i;
          ++cnt;
        }
      if (cnt != 2) return static_cast<long long>(r) * groups + grp;
      const size_t out = static_cast<size_t>(r) * (k / 2) + grp * 2;
      st(dt, a_c, out, ld(dt, a, base + idx[0]));
      st(dt, a_c, out + 1, ld(dt, a, base + idx[1]));
      const uint8_t code = static_cast<uint8_t>(idx[0] | (idx[1] << 2));
      uint8_t& byte = meta[static_cast<size_t>(r) * (k / 8) + grp / 2];
      byte = (grp & 1) ? static_cast<uint8_t>(byte | (code << 4)) : code;
    }
  return -1;
}

// Inverse of compress: rebuild the dense A from A_c + reference metadata.
void oracle_decompress(int dt, const void* a_c, const uint8_t* meta, int m, int k, void* a_out) {
  for (size_t i = 0; i < static_cast<size_t>(m) * k; ++i) st(dt, a_out, i, 0);
  for (int r = 0; r < m; ++r)
    for (int grp = 0; grp < k / 4; ++grp) {
      const uint8_t byte = meta[static_cast<size_t>(r) * (k / 8) + grp / 2];
      const int code = (grp & 1) ? (byte >> 4) : (byte & 15);
      const size_t base = static_cast<size_t>(r) * k + grp * 4;
      const size_t in = static_cast<size_t>(r) * (k / 2) + grp * 2;
      st(dt, a_out, base + (code & 3), ld(dt, a_c, in));
      st(dt, a_out, base + ((code >> 2) & 3), ld(dt, a_c, in + 1));
    }
}

// ---------------------------------------------------------------- GEMM
// c[r][n] = sum over k, in order, of float(a[r][k]) * float(b[k][n]) in fp32.
// The threaded driver splits rows across threads and leaves the arithmetic of
// each element unchanged; B is converted to float once and shared.
static void gemm_rows_f(int dt, const void* a, const float* bf, float* c, int n, int k, int r0,
                        int r1) {
  // dt: A's element code (B arrives already converted to float).
  std::vector<float> arow(k);
  for (int r = r0; r < r1; ++r) {
    for (int kk = 0; kk < k; ++kk) arow[kk] = to_f(dt, ld(dt, a, static_cast<size_t>(r) * k + kk));
    for (int col = 0; col < n; ++col) {
      float acc = 0.0f;
      for (int kk = 0; kk < k; ++kk) acc += arow[kk] * bf[static_cast<size_t>(kk) * n + col];
      c[static_cast<size_t>(r) * n + col] = acc;
    }
  }
}

void oracle_gemm_rows(int dt, const void* a, const void* b, float* c, int m, int n, int k, int r0,
                      int r1) {
  (void)m;
  std::vector<float> bf(static_cast<size_t>(k) * n);
  for (size_t i = 0; i < bf.size(); ++i) bf[i] = to_f(dt, ld(dt, b, i));
  gemm_rows_f(dt, a, bf.data(), c, n, k, r0, r1);
}

// A and B of different element codes (the mixed fp8 pairs); same arithmetic.
void oracle_gemm_mixed(int dta, int dtb, const void* a, const void* b, float* c, int m, int n,
                       int k, int threads) {
  std::vector<float> bf(static_cast<size_t>(k) * n);
  for (size_t i = 0; i < bf.size(); ++i) bf[i] = to_f(dtb, ld(dtb, b, i));
  const int dt = dta;
  if (threads <= 1) {
    gemm_rows_f(dt, a, bf.data(), c, n, k, 0, m);
    return;
  }
  std::vector<std::thread> pool;
  const int per = (m + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const int r0 = t * per, r1 = std::min(m, r0 + per);
    if (r0 >= r1) break;
    pool.emplace_back(gemm_rows_f, dt, a, bf.data(), c, n, k, r0, r1);
  }
  for (auto& th : pool) th.join();
}

void oracle_gemm(int dt, const void* a, const void* b, float* c, int m, int n, int k,
                 int threads) {
  oracle_gemm_mixed(dt, dt, a, b, c, m, n, k, threads);
}

int oracle_count_abs_errors(const float* got, const float* ref, size_t count, float atol) {
  int errors = 0;
  for (size_t i = 0; i < count; ++i)
    if (std::fabs(got[i] - ref[i]) > atol) ++errors;
  return errors;
}

// ---------------------------------------------------------------- extras
// Magnitude 2:4 pruning: keep the two largest |x| per group, ties to the
// lower index, others set to +0.
void oracle_prune_2of4(int dt, const void* a, int m, int k, void* out) {
  for (int r = 0; r < m; ++r)
    for (int grp = 0; grp < k / 4; ++grp) {
      const size_t base = static_cast<size_t>(r) * k + grp * 4;
      float mg[4];
      for (int i = 0; i < 4; ++i) mg[i] = std::fabs(to_f(dt, ld(dt, a, base + i)));
      int b0 = 0;
      for (int i = 1; i < 4; ++i)
        if (mg[i] > mg[b0]) b0 = i;
      int b1 = b0 == 0 ? 1 : 0;
      for (int i = 0; i < 4; ++i)
        if (i != b0 && mg[i] > mg[b1]) b1 = i;
      for (int i = 0; i < 4; ++i) st(dt, out, base + i, (i == b0 || i == b1) ? ld(dt, a, base + i) : 0);
    }
}

// tcgen05 metadata image: [ceil(k/128)][mb][128 lanes][4 x u32], mb = ceil(m/128)
// rounded up to even (a CTA pair always finds an atom for its second half).
//  16-bit types: lane L = 16*m2 + 8*k1 + m0, word w holds in bits [16h, 16h+16)
//    the 16 dense-K run [128*ka + 32*w + 16*k1, +16) of row 16*m2 + 8*h + m0.
//  e4m3: lane L = row L, 16 bytes = the row's reference bytes of the atom.
// Padding (rows >= m or K >= k) holds the valid code 0x4 in every nibble.
void oracle_meta_tc_image(int dt, const uint8_t* meta, int m, int k, uint32_t* img) {
  const int mb_n = ((m + 127) / 128 + 1) / 2 * 2, ka_n = (k + 127) / 128, rb = k / 8;
  for (int ka = 0; ka < ka_n; ++ka)
    for (int mb = 0; mb < mb_n; ++mb)
      for (int L = 0; L < 128; ++L)
        for (int w = 0; w < 4; ++w) {
          uint32_t word = 0;
          if (esz(dt) == 1) {
            const int row = mb * 128 + L, b0 = ka * 16 + 4 * w;
            if (row < m && b0 < rb) {
              const uint8_t* s = meta + static_cast<size_t>(row) * rb + b0;
              word = s[0] | (s[1] << 8) | (s[2] << 16) | (static_cast<uint32_t>(s[3]) << 24);
            } else {
              word = 0x44444444u;
            }
          } else {
            const int m2 = L / 16, k1 = (L / 8) % 2, m0 = L % 8;
            const int kr = ka * 128 + 32 * w + 16 * k1;
            for (int h = 0; h < 2; ++h) {
              const int row = mb * 128 + 16 * m2 + 8 * h + m0;
              uint32_t half = 0x4444u;
              if (row < m && kr < k) {
                const uint8_t* s = meta + static_cast<size_t>(row) * rb + kr / 8;
                half = s[0] | (s[1] << 8);
              }
              word |= half << (16 * h);
            }
          }
          img[((static_cast<size_t>(ka) * mb_n + mb) * 128 + L) * 4 + w] = word;
        }
}

// Reference-layout metadata -> the m16n8k16 layout of the legacy entry points
// (mma_sp_m16n8k16_fp32fp16.cu:96-110, strips concatenated at :277-297): word
// (s, 8b+i) = row 16b+i's 16-bit strip s (bytes 2s, 2s+1 of its metadata row)
// | row 16b+8+i's << 16.  m % 16 == 0, k % 16 == 0.
void oracle_meta_k16_from_ref(const uint8_t* meta, int m, int k, uint32_t* out) {
  const int rb = k / 8;
  for (int strip = 0; strip < k / 16; ++strip)
    for (int blk = 0; blk < m / 16; ++blk)
      for (int i = 0; i < 8; ++i) {
        const uint8_t* lo = meta + static_cast<size_t>(16 * blk + i) * rb + 2 * strip;
        const uint8_t* hi = meta + static_cast<size_t>(16 * blk + 8 + i) * rb + 2 * strip;
        out[static_cast<size_t>(strip) * (m / 2) + 8 * blk + i] =
            (lo[0] | (lo[1] << 8)) | (static_cast<uint32_t>(hi[0] | (hi[1] << 8)) << 16);
      }
}

// Per-tensor fp8 quantisation: scale = largest finite value / amax (448 for
// e4m3, 57344 for e5m2), q = fp8_rn_satfinite(x * scale).
static float quantize_fp8(int dt, float max_finite, const float* x, size_t count, uint8_t* q) {
  float amax = 0.0f;
  for (size_t i = 0; i < count; ++i) amax = std::max(amax, std::fabs(x[i]));
  const float s = amax > 0.0f ? max_finite / amax : 1.0f;
  for (size_t i = 0; i < count; ++i) q[i] = static_cast<uint8_t>(from_f(dt, x[i] * s));
  return s;
}
float oracle_quantize_e4m3(const float* x, size_t count, uint8_t* q) {
  return quantize_fp8(DT_E4M3, 448.0f, x, count, q);
}
float oracle_quantize_e5m2(const float* x, size_t count, uint8_t* q) {
  return quantize_fp8(DT_E5M2, 57344.0f, x, count, q);
}

// Element conversions for the test harness (bits <-> float).
void oracle_to_float(int dt, const void* src, size_t count, float* dst) {
  for (size_t i = 0; i < count; ++i) dst[i] = to_f(dt, ld(dt, src, i));
}
void oracle_from_float(int dt, const float* src, size_t count, void* dst) {
  for (size_t i = 0; i < count; ++i) st(dt, dst, i, from_f(dt, src[i]));
}

}  // extern "C"
