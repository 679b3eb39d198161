/* quack_b200 C ABI: block-scale quantizer, block-scaled GEMM with fused epilogue, and the
 * device-side half of the all-gather GEMM, for NVIDIA B200 (sm_100a).
 *
 * Plain C: raw device pointers, sizes, byte strides, enums and a CUDA stream handle.  No
 * torch types.  Every function returns QK_OK (0) or a negative QK_ERR_* code; the message of
 * the last failure on the calling thread is available from qk_last_error().  The library
 * allocates no device memory: outputs, scratch and the 4-int status buffer belong to the
 * caller (host side it keeps a small cache of tensor maps).  Launches are asynchronous on the
 * given stream.
 *
 * Each entry point names the reference interface (file:line in Dao-AILab/quack) it stands
 * in for.  The reference reaches its kernels through TVM-FFI from Python; a maintainer would
 * bind these symbols with ctypes instead.
 */
#ifndef QUACK_B200_H_
#define QUACK_B200_H_

#include <stddef.h>
#include <stdint.h>

#include "../quack_b200/csrc/qk_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Library / build identification. */
int qk_version(void);
const char* qk_last_error(void);

/* Number of bytes of the blocked scale buffer for `rows` rows and `k` logical elements:
 * ceil(rows/128) * ceil(k/(4*vec)) * 512.   quack/blockscaled/quantize.py:637-662 */
size_t qk_scale_blocked_bytes(int format, long long rows, long long k);

/* max|x| over a tensor -> *amax_out (fp32, device), for the NVFP4 per-tensor scale
 * amax / (448*6).  *amax_out must be zero-initialised by the caller (atomic max).
 * Replaces `x.abs().amax()` feeding quack/blockscaled/quantize.py:398-400. */
int qk_amax(const void* x, int x_dtype, long long rows, long long k, long long ldx /*elements*/,
            float* amax_out, void* stream);

/* Block-scale quantizer along the last dim.
 *   MXFP8_E4M3:  codes (rows,k) E4M3 bytes, one E8M0 scale per 32 elements, rceil rule.
 *           quack/blockscaled/quantize.py:47-108, :267-282
 *   NVFP4:  codes (rows,k/2) bytes (even element in the low nibble), one E4M3 scale per 16
 *           elements, divided by *per_tensor_scale when that pointer is non-null.
 *           quack/blockscaled/quantize.py:403-442, :165-215
 * Scale bytes are written directly in the blocked (rm, rk, 32, 4, 4) layout
 * (quack/blockscaled/quantize.py:637-662), pad slots zero-filled; the call stands in for
 * BlockScaledOperand.quantize (quack/blockscaled/operand.py:718-783). */
int qk_quantize_blockscaled(int format, const void* x, int x_dtype, long long rows, long long k,
                            long long ldx /*elements*/, void* codes, long long ld_codes /*bytes*/,
                            void* scale_blocked, const float* per_tensor_scale /*device, may be NULL*/,
                            void* stream);

/* The same with the E8M0 rule of the MX formats chosen by the caller (scaling_mode = QK_SCALING_*), and the
 * other MX element types:
 *   MXFP8_E5M2: E5M2 codes, format maximum 57344 (to_mx(elem_dtype=float8_e5m2), quack/blockscaled/quantize.py:47-114)
 *   MXFP4:      E2M1 codes packed two per byte, floor rule only (to_mxfp4, quack/blockscaled/quantize.py:285-316)
 *   QK_SCALING_FLOOR for MXFP8: scale exponent = exponent(amax) - exponent(format max) (:254-264); block maxima may
 *   saturate.  QK_SCALING_DEFAULT = what the reference's quantizer of that format does by default. */
int qk_quantize_blockscaled_mode(int format, int scaling_mode, const void* x, int x_dtype, long long rows, long long k,
                                 long long ldx /*elements*/, void* codes, long long ld_codes /*bytes*/,
                                 void* scale_blocked, const float* per_tensor_scale /*device, may be NULL*/,
                                 void* stream);

/* Quantisation along dim 0 with a transposed result: x is (rows, cols) row-major and the scale blocks run down its
 * columns (rows % 32 == 0).  codes_t is (cols, rows) row-major [(cols, rows / 2) bytes for the 4-bit formats] and
 * scale_blocked the blocked scales of that (cols, rows) operand: exactly what qk_quantize_blockscaled_mode returns
 * for the transposed matrix, without a transposed high-precision copy in memory.  This is
 * BlockScaledOperand.quantize(x, format, dim=-2) (quack/blockscaled/operand.py:718-783) and, for MXFP8, the
 * arithmetic of to_mx_dim0 (quack/blockscaled/quantize.py:117-162; that function keeps the codes in the input's
 * layout). */
int qk_quantize_blockscaled_dim0(int format, int scaling_mode, const void* x, int x_dtype, long long rows, long long cols,
                                 long long ldx /*elements*/, void* codes_t, long long ld_codes /*bytes*/,
                                 void* scale_blocked, const float* per_tensor_scale /*device, may be NULL*/,
                                 void* stream);

/* (mn, sf_k) row-major scale bytes -> blocked layout (zero padded) and back.
 * quack/blockscaled/quantize.py:637-674 */
int qk_scale_pack_blocked(const void* scale_2d, long long mn, long long sf_k, void* blocked, void* stream);
int qk_scale_unpack_blocked(const void* blocked, long long mn, long long sf_k, void* scale_2d, void* stream);

/* All-gather arrival gate + shard-major schedule (quack/gemm.py:360-375,
 * quack/tile_scheduler.py:123-177, :585-614).  flags == NULL disables it. */
/* (qk_ag_pull_args, the in-kernel transport of the all-gather GEMM, is declared in qk_types.h) */
typedef struct qk_ag_args {
  const int* flags;  /* (num_shards*num_chunks) int32, device; flag >= *epoch (modular) = arrived */
  const int* epoch;  /* (1) int32, device */
  int num_shards;
  int first_shard;
  int num_chunks;
  const qk_ag_pull_args* pull;   /* DEVICE pointer, NULL = shards are delivered by someone else */
} qk_ag_args;

/* D = epilogue(A * B^T): the kernel-level call quack.gemm.gemm (quack/gemm.py:378-443) with
 * SFA/SFB/bs_format_* set, plus the epilogue operands of quack/gemm_default_epi.py:22-67
 * (alpha, bias row vector), quack/epilogue/library.py:527-576 (activation / gated
 * activation with optional pre-activation store) and quack/epilogue/quantize_out.py
 * (re-quantised output with blocked scale factors). */
typedef struct qk_gemm_args {
  int format;                /* format of A: QK_FMT_MXFP8_E4M3, QK_FMT_MXFP8_E5M2, QK_FMT_MXFP4 or QK_FMT_NVFP4 */
  int format_b;              /* format of B; 0 = same as A.  Legal pairs (quack/blockscaled/operand.py:418-483):
                                any two of the MXFP8 formats (kind::mxf8f6f4), MXFP4 x MXFP4 and NVFP4 x NVFP4
                                (kind::mxf4nvf4) */
  int m;                     /* logical extents; k % 32 == 0 */
  int n;
  int k;
  const void* a;             /* (m, k_storage) K-major codes */
  long long lda;             /* row pitch in bytes, multiple of 16 */
  const void* b;             /* (n, k_storage) K-major codes */
  long long ldb;
  const void* sfa;           /* blocked scales of A: atoms of 512 bytes */
  long long sfa_stride_rm;   /* bytes between 128-row atom rows    (multiple of 512) */
  long long sfa_stride_rk;   /* bytes between consecutive K atoms  (multiple of 512) */
  const void* sfb;
  long long sfb_stride_rm;
  long long sfb_stride_rk;
  /* plain output or stored pre-activation; NULL = not stored */
  void* d;
  long long ldd;             /* elements (bytes for quantised codes) */
  int d_dtype;               /* QK_DT_* ; ignored when d receives quantised codes */
  /* activation output; NULL = no activation stage */
  void* post;
  long long ldpost;          /* elements (bytes for quantised codes) */
  int post_dtype;
  int activation;            /* QK_ACT_* */
  int exact_activation;      /* sigmoid / SiLU arithmetic of silu, swiglu and glu.  0: ex2.approx and the approximate
                                division, like the reference's device code (quack/activation.py:54-69); 1: expf and
                                IEEE division, x / (1 + exp(-x)), which reproduces torch's CUDA silu / sigmoid bit for
                                bit (the yardstick of quack/gemm_interface.py:81-102) */
  const void* bias;          /* (n) row vector added after alpha; may be NULL */
  int bias_dtype;
  float alpha;               /* host factor */
  const float* alpha_dev;    /* optional device factor (per-tensor scales), multiplied in */
  const float* alpha_dev2;   /* optional second device factor: alpha = alpha * *alpha_dev * *alpha_dev2 */
  /* residual operand: value = alpha * acc + beta * C + bias (quack/gemm_interface.py:1562-1590 gemm_add,
   * :1934-1960 gemm_add_inplace; C may alias d) */
  const void* c;             /* (m, n) row-major, NULL = none */
  long long ldc;             /* elements */
  int c_dtype;               /* QK_DT_* */
  float beta;                /* host factor (used when c != NULL) */
  const float* beta_dev;     /* optional device factor, multiplied in */
  /* quantised output: applies to `post` when present, else to `d` */
  int out_format;            /* QK_FMT_NONE / QK_FMT_MXFP8_E4M3 / QK_FMT_NVFP4 */
  void* sfd;                 /* blocked output scales, (ceil(m/128), ceil(n_out/(4*vec)), 512 B) */
  long long sfd_stride_rm;   /* bytes */
  float norm_const;          /* 1 / out_per_tensor_scale, host value */
  const float* norm_const_dev; /* optional device value (replaces the host value) */
  qk_ag_args ag;
  int tile_n;                /* 0 = choose; else 64 (one CTA per tile only) / 128 / 192 / 256 */
  int cta_group;             /* 0 = choose; 1 = one CTA per tile, 2 = CTA pair (256-row tiles) */
  int max_ctas;              /* 0 = all SMs; else cap on the persistent grid */
  int scheduler;             /* QK_SCHED_STATIC (0): persistent grid, tile = cluster + i * clusters;
                                QK_SCHED_CLC (1): one cluster per tile, running clusters take over the
                                tiles of clusters not yet started through cluster launch control (the
                                reference's is_dynamic_persistent, quack/gemm_config.py:215-225,
                                quack/tile_scheduler.py); needs max_ctas == 0 and prof == NULL;
                                QK_SCHED_ARRIVAL (2): all-gather mode only (one chunk per shard, <= 32 shards):
                                persistent grid, same tile ownership as the static schedule, but every
                                cluster takes the shards in the order their arrival flags flip instead of
                                strict ring order, so one late sender does not stall the tiles of shards
                                that are already resident (no counterpart in the reference) */
  int split_k;               /* 1 = off; 0 = automatic (splits K over several CTAs per tile when the tiles
                                are fewer than half the SMs and `workspace` is large enough); > 1 = that
                                many splits (error if the workspace is too small).  Partial sums are fp32
                                and summed in split order: the result does not depend on timing.
                                (reference: split_k of quack/gemm.py:378-443, SplitKMode) */
  void* workspace;           /* device scratch for split_k, 16-byte aligned, ZEROED once by the caller; the
                                kernel leaves its counters at zero, except when it gives up a bounded wait
                                (non-zero status): zero the workspace again before the next launch.  One
                                workspace per concurrently running GEMM.  Bytes needed: 256-rounded 16 * tiles * cta_group  +  splits * tiles *
                                cta_group * 128 * tile_n * 4 (tiles of 128 * cta_group rows x tile_n
                                columns).  NULL = never split */
  unsigned long long workspace_bytes;
  int* status;               /* device, 4 ints, zeroed by the caller; non-zero after a bounded
                                wait gave up (QK_STATUS_*) */
  unsigned long long timeout_ns; /* 0 = default (2 s) */
  long long* prof;           /* optional device buffer, 16 int64 per launched CTA: SM-clock cycles each
                                role spent in total and inside its waits (the counterpart of the
                                reference's in-kernel trace ranges, quack/gemm_sm100.py:1326,1466,1805,1973).
                                NULL = off */
  void* stream;              /* cudaStream_t */
} qk_gemm_args;

int qk_gemm_blockscaled(const qk_gemm_args* args);

/* The same GEMM for callers that cannot allocate device memory (a process that fixed its
 * device-memory plan at start-up, a language binding without a CUDA allocator).  No counterpart in
 * the reference.  The status block and the per-CTA cycle counters that qk_gemm_blockscaled takes
 * from its caller live in a static device array of 256 + QK_NOALLOC_MAX_CTAS * 128 bytes per GPU
 * instead; args->status and args->prof must be NULL.  status_out (device, 4 ints) and prof_out
 * (device, 16 * QK_NOALLOC_MAX_CTAS int64) are optional outputs that receive copies on the stream.
 * Launches of more than QK_NOALLOC_MAX_CTAS CTAs are rejected with QK_ERR_TOO_LARGE.  All calls on
 * one GPU share the array: calls that overlap on the GPU race.  The first call on a device resolves
 * the array's device address; make it before any stream capture.  Calls no cudaMalloc / cudaFree. */
#define QK_NOALLOC_MAX_CTAS 256
int qk_gemm_blockscaled_noalloc(const qk_gemm_args* args, int* status_out, long long* prof_out);

/* ---- peer-memory plumbing of the copy-engine all-gather transport ----
 * The reference reaches peer buffers through torch symmetric memory and pushes shards with the copy
 * engines (quack/distributed/all_gather_gemm.py:31-38 transport comparison, :275-815 AllGatherRunner:
 * per-peer buffers, flag writes, cross-rank barrier).  These entry points give a host the same
 * pieces without torch: none of them launches a kernel.
 *
 * qk_ipc_export: `ptr` lies in a cudaMalloc allocation of this process; writes the allocation's
 *   64-byte IPC handle and ptr's byte offset inside it.  Send both to the peer process.
 * qk_ipc_open: maps a peer process's allocation (peer access is enabled as needed); returns its base.
 *   A handle may be opened once per process: cache the result.  qk_ipc_close unmaps it.
 * qk_copy_async: device-to-device cudaMemcpyAsync on `stream`; dst/src may be peer mappings.
 * qk_stream_wait_geq32: `stream` stalls until (int32)(*addr - value) >= 0; no timeout: a value
 *   that never comes stalls the stream, not the GPU (no kernel is waiting).
 * qk_stream_write32: stream-ordered 32-bit store to memory of this device. */
#define QK_IPC_HANDLE_BYTES 64
int qk_ipc_export(const void* ptr, void* handle_out, unsigned long long* offset_out);
int qk_ipc_open(const void* handle, void** base_out);
int qk_ipc_close(void* base);
int qk_copy_async(void* dst, const void* src, unsigned long long bytes, void* stream);
int qk_stream_wait_geq32(void* stream, const void* addr, unsigned int value);
int qk_stream_write32(void* stream, void* addr, unsigned int value);

/* A list of the three operations above, enqueued in order with one call (one all-gather step of the
 * copy-engine transport is ~40 of them; a host that pays per foreign-function call builds the list once
 * and patches the epoch values).  Stops at the first failure. */
#define QK_OP_COPY 0        /* dst, src, bytes */
#define QK_OP_WAIT_GEQ32 1  /* dst = address to watch, value */
#define QK_OP_WRITE32 2     /* dst = address to write, value */
typedef struct qk_stream_op {
  int kind;
  unsigned int value;
  void* stream;
  void* dst;
  const void* src;
  unsigned long long bytes;
} qk_stream_op;
int qk_stream_ops(const qk_stream_op* ops, int count);

/* The library keeps the tensor maps (TMA descriptors) it builds for qk_gemm_blockscaled in a 512-entry cache
 * keyed by address, extents, strides and box shape (the reference's host path reuses a compiled plan per call
 * signature, quack/gemm_tvm_ffi_utils.py:357-425): hits and misses since the library was loaded. */
void qk_tensor_map_cache_stats(long long* hits, long long* misses);

/* Number of kernel launches issued by this library since it was loaded (all entry points). */
long long qk_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* QUACK_B200_H_ */
