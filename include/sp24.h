/*
 * sp24.h — C ABI of the B200 (sm_100a) 2:4 structured-sparse GEMM library.
 *
 *   C[M x N] (fp32 accumulate) = A[M x K] * B[K x N]
 *
 * A is 2:4-sparse along K and is passed compressed: A_c holds the two kept
 * values of every aligned group of four (M x K/2, row-major) and the metadata
 * holds one 4-bit code per group (i0 | i1 << 2, i0 < i1).  B is dense, K x N,
 * row-major.  Element types: fp16, bf16 and fp8 (A and B share the type, except
 * that the fp8 formats e4m3 and e5m2 may be mixed between A and B).
 *
 * Every entry point is stream-ordered, never exits the process and reports
 * errors through sp24_status.  Pointers are device pointers unless a comment
 * says otherwise.  No torch or C++ types cross this boundary.
 *
 * Reference interfaces each entry point replaces (paths inside
 * codes1gn/sparse-gemm-with-hopper-sptc):
 *   sp24_gemm            wgmma_sp_raw_common.hpp:955-1030 (wgmma_sp_raw_kernel,
 *                        launched at :1078-1080) and the CuTe twin
 *                        wgmma_sp_demo_common.hpp:307-406
 *   sp24_compress        wgmma_sp_raw_common.hpp:140-205
 *                        (compress_structured_sparse_a)
 *   sp24_repack_meta     the per-tile metadata placement of
 *                        wgmma_sp_raw_common.hpp:415-445 (smem_e_index*,
 *                        e_thread_byte_offset*) re-targeted to tcgen05 TMEM
 *   sp24_prune_2of4      (no counterpart: the reference only generates
 *                        already-pruned A, wgmma_sp_raw_common.hpp:63-98)
 */
#ifndef SP24_H_
#define SP24_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* sp24_stream_t; /* == cudaStream_t; NULL = legacy default stream */

typedef enum sp24_status {
  SP24_OK = 0,
  SP24_ERR_SHAPE = 1,      /* M/N/K or leading dimensions invalid (reference: run_case returns
                              false, wgmma_sp_raw_common.hpp:1042-1045) */
  SP24_ERR_ALIGN = 2,      /* pointer or stride breaks a 16-byte TMA rule and no workspace given */
  SP24_ERR_NOT_2OF4 = 3,   /* a group of four does not hold exactly two nonzeros (reference exits,
                              wgmma_sp_raw_common.hpp:163-166) */
  SP24_ERR_ARCH = 4,       /* device is not sm_100 (reference gate: major < 9,
                              wgmma_sp_raw_common.hpp:1115-1118) */
  SP24_ERR_CUDA = 5,       /* a CUDA runtime call failed (reference: CHECK_CUDA exit, :17-25) */
  SP24_ERR_TIMEOUT = 6,    /* a bounded device-side wait gave up; the kernel returned early */
  SP24_ERR_NCCL = 7,       /* collective failure (multi-GPU all-gather) */
  SP24_ERR_ARG = 8,        /* NULL pointer / bad enum */
  SP24_ERR_WORKSPACE = 9,  /* workspace missing or too small */
  SP24_ERR_SCRATCH_LIMIT = 10 /* sp24_gemm_noalloc: the problem needs more scratch than the
                                 library's fixed device buffer (SP24_NOALLOC_SCRATCH_BYTES) */
} sp24_status;

typedef enum sp24_dtype {
  SP24_F16 = 0,   /* reference: half           (RawSparseConfig<half>, :300-309)          */
  SP24_BF16 = 1,  /* reference: __nv_bfloat16  (RawSparseConfig<__nv_bfloat16>, :311-320) */
  SP24_E4M3 = 2,  /* reference: __nv_fp8_e4m3  (RawSparseConfig<__nv_fp8_e4m3>, :322-331) */
  /* Mixed fp8 (kind::f8f6f4 takes independent A and B formats).  The first
     named format is A's, the second B's; for the single-matrix entry points
     (compress, prune, repack) the dtype names A's element type.
     reference: mma.sp ... .f32.e5m2.e4m3.f32, mma_sp_m16n8k64_fp32fp8.cu:197-217
     (A __nv_fp8_e5m2, B __nv_fp8_e4m3). */
  SP24_E5M2_E4M3 = 3,
  SP24_E4M3_E5M2 = 4, /* no reference counterpart */
  SP24_E5M2 = 5       /* A and B e5m2; no reference counterpart */
} sp24_dtype;

typedef enum sp24_meta_format {
  /* The reference layout: M rows x K/8 bytes, row-major; group g of row r is the
     low (g even) or high (g odd) nibble of byte r*(K/8) + g/2
     (wgmma_sp_raw_common.hpp:197-202).  Needs workspace (repacked on the fly). */
  SP24_META_REF = 0,
  /* The tcgen05 image written by sp24_repack_meta (sp24_meta_tc_bytes bytes). */
  SP24_META_TC = 1,
  /* The m16n8k16 layout of the reference's legacy warp-level entry points
     (mma_sp_m16n8k16_fp32{fp16,bf16}.cu:96-110, strips concatenated at :277-297):
     u32 words [K/16][M/2]; word (s, 8b+i) holds row 16b+i's four nibbles of the
     16-wide K strip s in bits 0-15 and row 16b+8+i's in bits 16-31.  fp16/bf16
     only, M % 16 == 0.  Needs workspace (repacked on the fly).
     (The m16n8k32 entry points' metadata, u32 words [M][K/32] with group g of a
     word at bits 4g..4g+3 (mma_sp_m16n8k32_fp32fp16.cu:112-118), is the
     SP24_META_REF byte stream read little-endian: pass it as SP24_META_REF.) */
  SP24_META_K16 = 2
} sp24_meta_format;

/* Output selection bits for sp24_gemm_desc.c_f32 / c_bf16: either may be NULL,
   not both. */
typedef struct sp24_gemm_desc {
  sp24_dtype dtype;
  int m, n, k;                 /* dense problem size                                  */
  const void* a_c;             /* compressed A, m x k/2 elements, row stride lda_c      */
  int64_t lda_c;               /* elements; 0 = k/2                                     */
  const uint8_t* meta;         /* metadata in meta_format                               */
  sp24_meta_format meta_format;
  const void* b;               /* dense B, k x n elements, row stride ldb               */
  int64_t ldb;                 /* elements; 0 = n                                       */
  float* c_f32;                /* optional fp32 output, m x n, row stride ldc           */
  void* c_bf16;                /* optional bf16 output, m x n, row stride ldc           */
  int64_t ldc;                 /* elements; 0 = n                                       */
  float alpha;                 /* C = alpha * (A*B); fp8: 1/(scale_a*scale_b). 0 = 1.0  */
  int tile_n;                  /* 0 = auto; 8..256 selects the reference's BlockN
                                  variant (8 runs on the 16-wide tile)                  */
  void* workspace;             /* device scratch for META_REF repack / B padding        */
  size_t workspace_bytes;
  int* status_dev;             /* optional device int: kernel writes nonzero on a
                                  bounded-wait timeout; NULL = library-owned word        */
} sp24_gemm_desc;

/* Library / device queries ------------------------------------------------ */
const char* sp24_version(void);
const char* sp24_status_string(sp24_status s);
/* SP24_OK if `device` is an sm_100 part the kernels were built for. */
sp24_status sp24_check_device(int device);
/* Bytes of the tcgen05 metadata image for an m x k A (padded to 128 x 128 atoms). */
size_t sp24_meta_tc_bytes(int m, int k);
/* Workspace sp24_gemm needs for this descriptor (0 if none). */
size_t sp24_gemm_workspace_bytes(const sp24_gemm_desc* d);

/* Compression: dense 2:4 A (m x k, row stride lda elements) -> A_c (m x k/2,
   row stride ldac) + reference-layout metadata (m x k/8 bytes).
   bad_dev: device int64 written with the first invalid group as
   row*(k/4)+group, or -1 when every group is valid.  The call synchronises
   `stream` and returns SP24_ERR_NOT_2OF4 when a group is invalid
   (bad_host, if not NULL, receives the same value).
   Reference: compress_structured_sparse_a, wgmma_sp_raw_common.hpp:140-205. */
sp24_status sp24_compress(sp24_dtype dtype, const void* a_dense, int m, int k, int64_t lda,
                          void* a_c, int64_t ldac, uint8_t* meta_ref, long long* bad_dev,
                          long long* bad_host, sp24_stream_t stream);

/* Magnitude 2:4 pruning: keep the two largest |a| of every group of four
   (ties keep the lower index), zero the rest; writes the pruned dense A.
   No reference counterpart (see file header). */
sp24_status sp24_prune_2of4(sp24_dtype dtype, const void* a, int m, int k, int64_t lda,
                            void* a_pruned, int64_t ldp, sp24_stream_t stream);

/* Repack reference-layout metadata into the tcgen05 image consumed by
   sp24_gemm with SP24_META_TC.  Padding groups get the valid code 0x4. */
sp24_status sp24_repack_meta(sp24_dtype dtype, const uint8_t* meta_ref, int m, int k,
                             uint8_t* meta_tc, sp24_stream_t stream);

/* The same image from metadata in the m16n8k16 layout (SP24_META_K16). */
sp24_status sp24_repack_meta_k16(sp24_dtype dtype, const uint32_t* meta_k16, int m, int k,
                                 uint8_t* meta_tc, sp24_stream_t stream);

/* The GEMM.  Reference: wgmma_sp_raw_kernel<Element,BlockN>
   (wgmma_sp_raw_common.hpp:955-1030), grid (N/BlockN, M/64) x 128 threads,
   fp32 C.  Preconditions of the reference (M%64, N%BlockN, K%32 / K%64 for
   e4m3; :1042-1045) are relaxed to: k % 32 == 0 (k % 64 for fp8), m,n >= 1. */
sp24_status sp24_gemm(const sp24_gemm_desc* d, sp24_stream_t stream);

/* Reads and clears the library-owned device status word that kernels raise
   when a bounded wait timed out (used when sp24_gemm_desc.status_dev is NULL).
   Synchronises `stream`.  SP24_ERR_TIMEOUT if a timeout happened.
   (No reference counterpart: the reference never bounds a wait.) */
sp24_status sp24_last_kernel_status(sp24_stream_t stream);

/* Launch hints for later GEMM calls made from the calling host thread (no
   reference counterpart).  GEMM kernels are launched with programmatic
   dependent launch: they may start while the previous kernel of the stream
   finishes and wait for it before their first load.
   SP24_HINT_STATIC_WEIGHTS: the caller guarantees that A_c and the metadata
   image (SP24_META_TC) of later calls are not written by work still in flight
   in the stream -- inference weights.  The narrow-N kernel then issues its
   first ring of A_c and metadata loads before that wait, hiding their HBM
   latency behind the previous kernel; B is still read, and C written, only
   after the wait.  Ignored for SP24_META_REF / SP24_META_K16, whose image the
   library itself writes just before the GEMM.  Default: SP24_HINT_NONE. */
#define SP24_HINT_NONE 0u
#define SP24_HINT_STATIC_WEIGHTS 1u
void sp24_set_launch_hints(unsigned hints);
unsigned sp24_get_launch_hints(void);

/* Re-reads the SP24_* tuning variables of the environment (no reference
   counterpart).  The library reads them once, on the first GEMM call, so
   that a launch scans no environment; they only force a kernel family or a
   tile parameter for tests and tuning runs.  A caller that changes them
   afterwards calls this, with no GEMM call in progress on another thread. */
void sp24_reload_tuning(void);

/* Self-test of the bounded-wait path (no reference counterpart): launches the
   GEMM of `d` with a producer that issues no load, so the consumers' waits run
   out after `timeout_ns`; the kernel frees its TMEM and returns.  Requires
   d->status_dev.  Synchronises; returns SP24_ERR_TIMEOUT (expected) or
   SP24_OK if no wait ran out. */
sp24_status sp24_selftest_timeout(const sp24_gemm_desc* d, unsigned long long timeout_ns,
                                  sp24_stream_t stream);

/* Allocation-free GEMM (no counterpart in the reference).
   Same contract and results as sp24_gemm, for callers that must not allocate
   device memory per call: real-time serving loops that forbid
   cudaMalloc/cudaFree after start-up (an allocation can synchronize the
   device and stall every stream), and plugin hosts that own all device memory
   and hand the library only its inputs and outputs.  Instead of
   d->workspace (ignored here) it stages its scratch (the tcgen05 image of
   reference-layout metadata and, when B's row pitch breaks the 16-byte TMA
   rule, a padded copy of B) in one fixed buffer of SP24_NOALLOC_SCRATCH_BYTES
   bytes that lives in the library's device image: every GPU that loads the
   library holds it until the process exits.
   - Problems whose scratch need (sp24_gemm_workspace_bytes) exceeds the
     buffer are rejected with SP24_ERR_SCRATCH_LIMIT; nothing is launched.
   - The buffer is shared by every call on a device and keeps the previous
     call's contents; calls that can overlap on the GPU (different streams
     without ordering) race on it.  Serialize them, or use sp24_gemm with
     caller-owned workspaces.
   - The first call on a device looks the buffer's device address up (once,
     with that device current); make that first call before any stream
     capture begins.
   It calls no cudaMalloc, cudaFree or other allocating routine. */
#define SP24_NOALLOC_SCRATCH_BYTES (16u << 20)
sp24_status sp24_gemm_noalloc(const sp24_gemm_desc* d, sp24_stream_t stream);

/* Fused epilogues (no counterpart in the reference; they replace a second
   GEMM and an elementwise kernel that callers of the reference run after it).
   With A the weights (output features along M) and B the activations (tokens
   along N), per output row r:
     plain:  C = act(alpha * A B + bias[r])
     gated:  C = act(alpha * A B + bias[r]) * (alpha_up * A_up B + bias_up[r])
   The gated form is the SwiGLU of an MLP (A = W_gate, A_up = W_up, act = SiLU,
   silu(x) = x / (1 + e^-x)): one launch streams both weights against one
   staged B and writes one output.  A_up has A's shape, dtype and row rules;
   its metadata must be a tcgen05 image (SP24_META_TC) and so must d->meta in
   the gated form.  The gated form runs on the narrow-N kernel (tiles up to
   128 columns; any N). */
typedef enum sp24_activation {
  SP24_ACT_NONE = 0,
  SP24_ACT_SILU = 1
} sp24_activation;

typedef struct sp24_epilogue {
  const float* bias;          /* optional, m floats (device) */
  sp24_activation act;
  const void* a_c_up;         /* gated form when not NULL: compressed A_up, m x k/2 */
  int64_t lda_c_up;           /* elements; 0 = k/2 */
  const uint8_t* meta_up;     /* A_up's tcgen05 metadata image */
  float alpha_up;             /* 0 = 1.0 */
  const float* bias_up;       /* optional, m floats */
} sp24_epilogue;

/* sp24_gemm followed by the epilogue `e` (NULL = none), in one launch. */
sp24_status sp24_gemm_fused(const sp24_gemm_desc* d, const sp24_epilogue* e,
                            sp24_stream_t stream);

/* FP8 helpers.
   sp24_amax_f32: amax_dev[0] = max |x| over count floats (device).
   sp24_quantize_e4m3: q[i] = e4m3_rn_satfinite(x[i] * scale[0]) with
   scale[0] = 448 / amax (computed on device from amax_dev).
   sp24_quantize_e5m2: the same with e5m2 and scale[0] = 57344 / amax.
   Reference: quantize_fp8 / quantize_fp8_kernel (RN conversion through the
   __nv_fp8_* constructors), mma_sp_m16n8k64_fp32fp8.cu:126-130, 341-347; the
   per-tensor 448/amax scale is the e4m3 benchmark configuration's. */
sp24_status sp24_amax_f32(const float* x, size_t count, float* amax_dev, sp24_stream_t stream);
sp24_status sp24_quantize_e4m3(const float* x, size_t count, const float* amax_dev,
                               float* scale_dev, uint8_t* q, sp24_stream_t stream);
sp24_status sp24_quantize_e5m2(const float* x, size_t count, const float* amax_dev,
                               float* scale_dev, uint8_t* q, sp24_stream_t stream);

/* Fused all-gather of C over NVLink (no counterpart in the reference; it
   replaces the optional NCCL all-gather of the column shards and the
   column-block permute after it).  Each rank runs the GEMM of its column shard
   of C with d->c_f32 / d->c_bf16 pointing at the shard's first column inside
   the rank's own full M x N_total C (d->ldc = N_total); the kernel stores
   every finished tile there and, with peer stores over NVLink, at the same
   element of every peer's full C (peers->c_f32[i] / c_bf16[i]: the peer's
   buffer, mapped into this process, plus the same element offset).  Kernels
   never wait on peers.  The gathered C is complete once every rank's call has
   completed: order that with a barrier across the ranks after the launch
   (e.g. a one-element NCCL all-reduce on the same streams).
   Peer pointers must share the local pointer's 32-byte alignment. */
#define SP24_MAX_PEERS 7
typedef struct sp24_peer_out {
  int n_peers;                     /* 0 .. SP24_MAX_PEERS */
  float* c_f32[SP24_MAX_PEERS];    /* when d->c_f32 is set */
  void* c_bf16[SP24_MAX_PEERS];    /* when d->c_bf16 is set */
} sp24_peer_out;
sp24_status sp24_gemm_allgather(const sp24_gemm_desc* d, const sp24_peer_out* peers,
                                sp24_stream_t stream);

/* CUDA IPC plumbing for the peer buffers (host calls, no stream work).
   sp24_ipc_get_handle: 64-byte handle of the allocation holding dev_ptr and
   the byte offset of dev_ptr inside it.  sp24_ipc_open_handle: maps a peer's
   handle into this process (peer access enabled) and returns the
   allocation's base; add the offset.  sp24_ipc_close: unmaps it. */
sp24_status sp24_ipc_get_handle(const void* dev_ptr, void* handle64, size_t* offset);
sp24_status sp24_ipc_open_handle(const void* handle64, void** base);
sp24_status sp24_ipc_close(void* base);

/* One N-sharded GEMM over several GPUs of this process, from one host
   thread (no reference counterpart: the reference runs on one GPU; the
   multi-GPU layout is the one its large GEMMs shard along N).  Device g of
   md->devices owns the columns [n0, n1) = sp24_shard_columns(n, ngpu, g,
   256) of C; A_c and the metadata are replicated (md->a_c[g], md->meta[g]:
   the same contents on every device, e.g. through sp24_replicate), B and C
   are local.  Each device's GEMM is enqueued on md->streams[g] (NULL: that
   device's legacy default stream); the call returns once every launch is
   enqueued and restores the caller's current device.
     md->gemm       the whole problem: dtype, m, n (all columns), k, lda_c,
                    meta_format, ldb / ldc (see the layouts), alpha, tile_n.
                    Its pointer, workspace and status fields are ignored.
     b_layout       SP24_MULTI_FULL: md->b[g] is all of B (k x n, row stride
                    ldb >= n, 0 = n); SP24_MULTI_SHARD: md->b[g] is device g's
                    column block alone (k x (n1 - n0), row stride n1 - n0).
     c_layout       the same for md->c_f32[g] / md->c_bf16[g] (row stride
                    ldc >= n, 0 = n, for FULL): a FULL C receives device g's
                    columns, and with allgather_c every device's columns.
     workspace[g]   device g's workspace (META_REF repack, B padding), at
                    least sp24_gemm_multi_workspace_bytes(md) bytes, or NULL
                    when that is 0.
   allgather_c (FULL C only): every device's epilogue also stores its tiles
   into the other devices' C over NVLink (peer access is enabled on first
   use), and each stream is made to wait for every device's launch, so work
   enqueued on md->streams[g] after this call sees the complete C.  The
   kernels never wait on a peer.  All structural checks (ngpu 1 ..
   SP24_MAX_GPUS, distinct devices, layouts, pointers) happen before anything
   is enqueued. */
#define SP24_MAX_GPUS 8
typedef enum sp24_multi_layout { SP24_MULTI_FULL = 0, SP24_MULTI_SHARD = 1 } sp24_multi_layout;
typedef struct sp24_multi_desc {
  sp24_gemm_desc gemm;
  int ngpu;
  int devices[SP24_MAX_GPUS];
  sp24_stream_t streams[SP24_MAX_GPUS];
  const void* a_c[SP24_MAX_GPUS];
  const uint8_t* meta[SP24_MAX_GPUS];
  const void* b[SP24_MAX_GPUS];
  sp24_multi_layout b_layout;
  float* c_f32[SP24_MAX_GPUS];
  void* c_bf16[SP24_MAX_GPUS];
  sp24_multi_layout c_layout;
  void* workspace[SP24_MAX_GPUS];
  size_t workspace_bytes;
} sp24_multi_desc;
sp24_status sp24_gemm_multi(const sp24_multi_desc* md, int allgather_c);
/* Workspace each device needs for sp24_gemm_multi(md, ...): the largest of
   the per-device column-block GEMMs' needs (0 if none, or if md is invalid). */
size_t sp24_gemm_multi_workspace_bytes(const sp24_multi_desc* md);

/* Replication helper for sp24_gemm_multi's A_c / metadata: copies `bytes`
   from src (on device src_device) to dst[g] on each devices[g] (peer copies
   over NVLink, enqueued on streams[g]; a destination equal to src is
   skipped).  No reference counterpart. */
sp24_status sp24_replicate(const void* src, int src_device, size_t bytes, int ngpu,
                           const int* devices, void* const* dst, const sp24_stream_t* streams);

/* Multi-GPU N-sharding helpers (no collective on the GEMM path).
   Columns [n0, n1) of C belong to `rank` of `world`; boundaries are multiples
   of `align` (the tile width) except the last. */
void sp24_shard_columns(int n, int world, int rank, int align, int* n0, int* n1);
/* Column-block -> row-major permute after an all-gather of per-rank C shards:
   src holds world blocks [rank][m][n1-n0] packed back to back (the shard of
   rank r starts at element offset m*n0(r)); dst is m x n row-major. */
sp24_status sp24_unshard_columns_f32(const float* src, float* dst, int m, int n, int world,
                                     int align, sp24_stream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* SP24_H_ */
