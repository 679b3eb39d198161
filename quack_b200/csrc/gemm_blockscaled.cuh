// Persistent, warp-specialised block-scaled GEMM for sm_100a.
//
//   D[M,N] = epilogue( sum_k (A[m,k] * SFA[m,k/vec]) * (B[n,k] * SFB[n,k/vec]) )
//
// Operands are K-major.  Per k-tile (128 bytes of K per row) the producer thread issues TMA
// loads of the A and B tiles into 128-byte-swizzled shared memory and of the scale-factor
// atoms (512-byte blocks covering 128 rows x 4 scale columns) for A and B.  One thread issues
// tcgen05.cp (scale atoms: shared memory -> tensor memory) and four tcgen05.mma.block_scale
// instructions per k-tile; accumulators live in tensor memory.  Four epilogue warps (thread ==
// accumulator row) read the accumulator with tcgen05.ld, apply alpha / bias / activation /
// optional re-quantisation in fp32 and store.
//
// CG == 2 runs one MMA across a pair of CTAs (cta_group::2): each CTA holds 128 rows of A and
// half of the B tile; the leader CTA issues the MMAs; completion is signalled to both CTAs.
// No load uses cluster multicast: each CTA fetches what it needs itself.
//
// Every wait is bounded (a %globaltimer deadline).  When a wait gives up, the CTA records
// where in `status`, raises an abort flag that every role polls, drains and returns; the host
// wrapper turns a non-zero status word into an error.
#pragma once

#include "qk_ptx.cuh"
#include "qk_types.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#ifndef QK_EPI_GROUPS
#define QK_EPI_GROUPS 2
#endif
#ifndef QK_XFER_SLOTS_MAX
#define QK_XFER_SLOTS_MAX 7
#endif
#ifndef QK_XFER_SLOT_BYTES
#define QK_XFER_SLOT_BYTES 4096
#endif
#ifndef QK_XFER_WANT_BYTES
#define QK_XFER_WANT_BYTES 20480
#endif

namespace qk {

struct alignas(64) GemmParams {
  CUtensorMap tm_a, tm_b, tm_sfa, tm_sfb;
  CUtensorMap tm_d, tm_post;  // TMA-store maps of the outputs (valid iff d_tma / post_tma)
  int M, N, K;
  int tiles_m, tiles_n, k_tiles, group_m;
  // plain / pre-activation output (may be null)
  void* d;
  long long ldd;  // elements
  int d_dtype;
  int d_tma, post_tma;
  // activation output (null when there is no activation output)
  void* post;
  long long ldpost;  // elements (packed fp4: bytes)
  int post_dtype;
  int act;
  uint32_t idesc_elem_fmt;   // kind::mxf8f6f4: element-format bits of A and B for the instruction descriptor
  int act_exact;   // 1: sigmoid / SiLU through expf and IEEE division (bit-equal to torch's CUDA kernels)
  const void* bias;
  int bias_dtype;
  float alpha;
  const float* alpha_dev;
  const float* alpha_dev2;
  // residual operand: value = alpha * acc + beta * C + bias
  const void* c;
  long long ldc;   // elements
  int c_dtype;
  int c_vec_ok;    // rows of C start on 16-byte boundaries
  float beta;
  const float* beta_dev;
  // quantised output: scale bytes in the blocked (rm, rk, 32, 4, 4) layout
  // (the output format is a template parameter of the kernel; it applies to `post` when an
  // activation output exists, else to `d`)
  unsigned char* sfd;
  long long sfd_stride_rm;  // bytes
  float norm;
  const float* norm_dev;
  // all-gather arrival gate
  const int* ag_flags;
  const int* ag_epoch;
  int ag_num_shards, ag_first_shard, ag_num_chunks, ag_tiles_m_per_shard;
  // in-kernel transport (device memory; null = the shards are delivered from outside the kernel)
  const qk_ag_pull_args* ag_pull;
  unsigned long long timeout_ns;
  int* status;
  int vec_store_ok;
  // optional per-CTA role counters (16 x int64 per CTA, SM clock cycles); null = off
  long long* prof;
  int prefetch_dist;  // k-tiles the L2 prefetch runs ahead of the loads (0 = off)
  // 1: the grid has one cluster per tile and running clusters take over the tiles of clusters
  // that have not started (cluster launch control); 0: static persistent schedule
  int clc;
  // split-K: every tile is computed by `split_k` work units, each over `kt_per_split` k-tiles; the
  // units leave fp32 partials in `ws_partials` and the last to arrive per 32-row group (counted
  // in `ws_counters`, which it leaves at zero) sums them in split order and runs the epilogue.
  // Partials are stored in 8 KB blocks [split][group][64-column chunk], a block holding the 32
  // rows x 64 columns of one warp as float4 (i, lane) at index i * 32 + lane: writer and reader
  // use the same thread = row mapping, so every warp access is one contiguous 512 bytes (a
  // row-major [M][N] layout put the 32 rows of a warp 16 KB apart, onto the same L2 slices, and
  // made the reduction 10x slower).  split_k == 1: off.
  int split_k, kt_per_split;
  float* ws_partials;
  int* ws_counters;
  int ws_groups;   // 32-row groups in the whole problem: tiles * CTAs per tile * 4
  // Rows of the A box of one load (128 unless the whole problem has fewer rows): zero-filled rows
  // cost as much TMA ingest as real ones (~65 B/clk/SM), and with M <= 64 they were most of a
  // stage.  Rows of the stage beyond the box keep stale bytes; they only feed accumulator rows
  // >= M, which are never stored.
  int a_box_rows;
};

// slots of the per-CTA profile block
enum : int {
  PROF_MMA_TOTAL = 0, PROF_MMA_WAIT_FULL = 1, PROF_MMA_WAIT_ACC = 2, PROF_MMA_TILES = 3,
  PROF_LOAD_TOTAL = 4, PROF_LOAD_WAIT_EMPTY = 5, PROF_LOAD_WAIT_GATE = 6,
  PROF_EPI_TOTAL = 8, PROF_EPI_WAIT_ACC = 9, PROF_EPI_DRAIN = 10, PROF_EPI_TILES = 11,
  PROF_MMA_ISSUE_CP = 7, PROF_MMA_ISSUE_MMA = 14, PROF_MMA_ISSUE_COMMIT = 15,  // issue cycles of the elected MMA lane
  PROF_SPLIT_PUBLISH = 12,  // split-K: fence + arrival counter
  PROF_SPLIT_REDUCE = 13,   // split-K: the last unit's reduction and epilogue
};

// FEW_ROWS: variant for problems of at most 32 rows (single-CTA tiles only).  A stage reserves 32 rows of A
// instead of 128, which more than doubles the pipeline depth in the same shared memory: these problems stream
// the weights through few CTAs and are bound by the bytes each keeps in flight.  The MMA still reads 128 rows
// (whatever follows the 32 in shared memory); they only feed accumulator rows that are never stored.
// PULL: variant with one more warp, the in-kernel transport of the all-gather mode (see `transport_warp`).
template <int KIND, int TILE_N_, int CG_, bool FEW_ROWS_ = false, bool PULL_ = false>
struct GemmCfg {
  static constexpr int TILE_N = TILE_N_;
  static constexpr int CG = CG_;
  static constexpr bool FEW_ROWS = FEW_ROWS_;
  static constexpr bool PULL = PULL_;
  static_assert(!FEW_ROWS || CG_ == 1, "the few-rows variant uses single-CTA tiles");
  static constexpr int TILE_M = 128;                // rows per CTA
  static constexpr int KT_BYTES = 128;              // bytes of K per row per k-tile
  static constexpr int KBLOCKS = 4;                 // MMA instructions per k-tile (32 bytes of K each)
  // scale atoms per k-tile per 128 rows: a k-tile holds 128 (MXFP8) or 256 (fp4) elements, an atom 4 scale
  // columns of 32 (MXFP8, MXFP4) or 16 (NVFP4) elements
  static constexpr int AK = KIND == 0 ? 1 : KIND == 1 ? 4 : 2;
  // B scale atoms cover 128 rows of N; a tile that does not start on an atom boundary starts
  // (n0 % 128) / 32 TMEM columns into its first atom.  NB = most atoms a tile can touch.
  static constexpr int N_GCD = (TILE_N % 128 == 0) ? 128 : (TILE_N % 64 == 0) ? 64 : 32;
  static constexpr int NB = (TILE_N + (128 - N_GCD) + 127) / 128;
  static constexpr int A_ROWS_STORED = FEW_ROWS ? 32 : TILE_M;
  static constexpr int A_BYTES = A_ROWS_STORED * KT_BYTES;
  static constexpr int B_ROWS = TILE_N / CG;
  static constexpr int B_BYTES = B_ROWS * KT_BYTES;
  static constexpr int SFA_BYTES = AK * 512;
  static constexpr int SFB_BYTES = NB * AK * 512;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  static constexpr int SFA_COLS = AK * 4;
  static constexpr int SFB_COLS = NB * AK * 4;
  // Tensor memory (512 columns): two accumulator stages of TILE_N columns.  When the scale
  // factors do not fit next to them (TILE_N = 256) a tile's scale factors are placed in the
  // first columns of the OTHER accumulator stage: that stage holds the previous tile, whose
  // epilogue releases those columns ("head") as soon as it has read its first 64-column chunk.
  static constexpr int ACC_STAGES = 2;
  static constexpr bool OVERLAP_SF = (2 * TILE_N + SFA_COLS + SFB_COLS > 512);
  __host__ __device__ static constexpr int sfa_col0(int acc) { return OVERLAP_SF ? (1 - acc) * TILE_N : 2 * TILE_N; }
  __host__ __device__ static constexpr int sfb_col0(int acc) { return sfa_col0(acc) + SFA_COLS; }
  static constexpr int TMEM_COLS = 512;
  static constexpr int EPI_WARPS = 4;                // warps that drain one accumulator (one per TMEM lane quadrant)
  // Epilogue groups: group g drains the tiles held in accumulator stage g (every other tile), so a
  // tile's drain may take as long as two main loops before it stalls the MMA issuer.
  // Used for the 256-wide pair tiles (the large-problem shape, where a quantising epilogue can outlast a
  // K = 4096 main loop); the other shapes keep one group and their deeper load pipeline.
  static constexpr int EPI_GROUPS = (CG == 2 && TILE_N == 256) ? QK_EPI_GROUPS : 1;
  static constexpr int EPI_WARPS_TOTAL = EPI_WARPS * EPI_GROUPS;
  // 320 threads with two groups: registers are granted per 4 warps, so the compiler's cap is
  // 65536 / 384 = 168 per thread (a 200-register build of this kernel is refused at launch with "too many
  // resources requested"); the two-group variants spill ~120 bytes per thread at that cap.
  static constexpr int XFER_WARP = 2 + EPI_WARPS_TOTAL;   // (PULL only)
  static constexpr int NUM_THREADS = 32 * (2 + EPI_WARPS_TOTAL + (PULL ? 1 : 0));
  // 11 warps are granted registers like 12: bound the kernel as if it had 384 threads, or the compiler
  // may pick a count the launch cannot be given
  static constexpr int LAUNCH_BOUND_THREADS = PULL ? (NUM_THREADS + 127) / 128 * 128 : NUM_THREADS;
  // bias staging: every epilogue warp keeps the 64 bias values of the chunk it is working on (a private
  // copy: no barrier between warps).  Staging the whole tile per warp cost 8 KB with two epilogue groups,
  // which was the difference between 4 and 5 load stages for the 256-wide NVFP4 pair tile.
  static constexpr int BIAS_BYTES = EPI_WARPS_TOTAL * 64 * 4;
  static constexpr int SLAB_BYTES = 4096;                        // 32 rows x 128 bytes
  // staging slabs per epilogue warp: two (one being read by a bulk store while the next is written) with
  // one group; one with two groups (each warp has twice the time per tile, and the 32 KB saved keep the load
  // pipeline as deep as before)
  static constexpr int SLABS_PER_WARP = EPI_GROUPS == 2 ? 1 : 2;
  static constexpr int EPI_BYTES = EPI_WARPS_TOTAL * SLABS_PER_WARP * SLAB_BYTES;
  static constexpr int CTRL_BYTES = 1024;
  // dynamic scheduler ring (offsets inside the control block; the pipeline barriers end below 256)
  static constexpr int SCHED_SLOTS = 8;
  static constexpr int SCHED_FULL_OFF = 256, SCHED_EMPTY_OFF = 320, SCHED_CLC_BAR_OFF = 384, SCHED_TILE_OFF = 448,
                       SCHED_RESP_OFF = 512;
  static_assert(SCHED_RESP_OFF + 16 * SCHED_SLOTS <= CTRL_BYTES, "control block too small");
  // warps that read a tile id per CTA group: MMA + epilogue warps of the leader, and with a CTA
  // pair the producer + epilogue warps of the peer (the leader's producer is the scheduler)
  static constexpr int SCHED_CONSUMERS = CG == 2 ? 2 * (1 + EPI_WARPS_TOTAL) : 1 + EPI_WARPS_TOTAL;
  static constexpr int SMEM_LIMIT = 232448;  // 227 KB opt-in maximum per CTA
  static constexpr int STAGES_MAX = FEW_ROWS ? 12 : 8;
  static constexpr int SMEM_AVAIL = SMEM_LIMIT - 1024 /*align slack*/ - CTRL_BYTES - BIAS_BYTES - EPI_BYTES;
  static constexpr int STAGES_NOX = SMEM_AVAIL / STAGE_BYTES > STAGES_MAX ? STAGES_MAX : SMEM_AVAIL / STAGE_BYTES;
  // Transport ring of the PULL variant: peer memory -> slot -> this GPU's gather buffer.  The ring holds what
  // one SM keeps in flight over NVLink.  Measured (MXFP8 32768 x 28672 x 8192): 5 slots of 4 KB beside 5 pipeline
  // stages move 430 GB/s per GPU at 2 GPUs; 7 slots of 8 KB move 545 GB/s but cost a pipeline stage, and the
  // step was slower (3.42 vs 3.23 ms at 2 GPUs, equal at 8).  The variant gives up a stage only when the
  // remainder of shared memory is smaller than QK_XFER_WANT_BYTES.
  static constexpr int XFER_SLOT_BYTES = QK_XFER_SLOT_BYTES;
  static constexpr int XFER_WANT = QK_XFER_WANT_BYTES;
  static constexpr int STAGES = !PULL ? STAGES_NOX
                                      : (SMEM_AVAIL - STAGES_NOX * STAGE_BYTES >= XFER_WANT ? STAGES_NOX : STAGES_NOX - 1);
  static constexpr int XFER_SLOTS_RAW = (SMEM_AVAIL - STAGES * STAGE_BYTES) / XFER_SLOT_BYTES;
  static constexpr int XFER_SLOTS = !PULL ? 0 : (XFER_SLOTS_RAW > QK_XFER_SLOTS_MAX ? QK_XFER_SLOTS_MAX : XFER_SLOTS_RAW);
  static constexpr int XFER_BYTES = XFER_SLOTS * XFER_SLOT_BYTES;
  // stores that may still be reading their slot while the next loads are issued / loads in flight ahead of them
  static constexpr int XFER_PENDING = XFER_SLOTS >= 6 ? 3 : 2;
  static constexpr int XFER_AHEAD = XFER_SLOTS - XFER_PENDING;
  static_assert(!PULL || (XFER_SLOTS >= 3 && XFER_AHEAD >= 1), "transport ring too small");
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + XFER_BYTES + BIAS_BYTES + CTRL_BYTES;
  // The tensor-memory column offset of the B scale factors, (n0 % 128) / 32, must be even: an odd
  // offset (tile widths that are odd multiples of 32) raises a misaligned-address fault in the MMA.
  static_assert(TILE_N % 64 == 0 && TILE_N >= 64 && TILE_N <= 256, "tile_n: multiple of 64 in [64,256]");
  static_assert((TILE_N / CG) % 8 == 0, "B rows per CTA: whole 8-row swizzle groups");
  static_assert(STAGES >= 3, "need at least 3 pipeline stages");
  static_assert(2 * TILE_N <= 512 && SFA_COLS + SFB_COLS <= 64, "tensor memory budget");
  static_assert(OVERLAP_SF || 2 * TILE_N + SFA_COLS + SFB_COLS <= 512, "tensor memory budget");
  static_assert(B_BYTES % 1024 == 0, "B stage must keep 1024-byte alignment");
};

struct CtaCtl {
  volatile int abort;
};

// Bounded mbarrier wait.  Returns false when the wait was abandoned (this CTA is aborting).
template <bool CLUSTER_SCOPE>
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, CtaCtl* ctl, const GemmParams& p,
                                             int code, int detail) {
  bool done = CLUSTER_SCOPE ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
  if (done) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    done = CLUSTER_SCOPE ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
    if (done) return true;
    if ((++it & 31u) == 0) {
      if (ctl->abort) return false;
      if (globaltimer_ns() - t0 > p.timeout_ns) {
        ctl->abort = 1;
        if (atomicCAS(p.status, 0, code) == 0) {
          p.status[1] = detail;
          p.status[2] = static_cast<int>(blockIdx.x);
          p.status[3] = static_cast<int>(parity);
        }
        return false;
      }
    }
  }
}

struct TileCoord {
  int m_tile;  // cluster tile index along M (128*CG rows each)
  int n_tile;
  int shard;   // all-gather shard the rows belong to (0 when not gated)
};

__device__ __forceinline__ TileCoord decode_tile(const GemmParams& p, int id) {
  TileCoord tc;
  int tiles_m = p.tiles_m, base_m = 0;
  tc.shard = 0;
  if (p.ag_flags != nullptr) {
    // shard-major order starting at the local shard: every tile of a shard before the next
    const int per_shard = p.ag_tiles_m_per_shard * p.tiles_n;
    const int s = id / per_shard;
    id -= s * per_shard;
    int shard = s + p.ag_first_shard;
    if (shard >= p.ag_num_shards) shard -= p.ag_num_shards;
    tc.shard = shard;
    tiles_m = p.ag_tiles_m_per_shard;
    base_m = shard * p.ag_tiles_m_per_shard;
  }
  const int group_sz = p.group_m * p.tiles_n;
  const int g = id / group_sz;
  const int first_m = g * p.group_m;
  const int gm = min(tiles_m - first_m, p.group_m);
  const int r = id - g * group_sz;
  tc.m_tile = base_m + first_m + r % gm;
  tc.n_tile = r / gm;
  return tc;
}

// ------------------------------------------------------------------ epilogue math -------
// The activation is selected ONCE per chunk (a switch around the unrolled loop): a switch per
// element turns into an indirect branch per element and made the epilogue ~5x slower.
// Two arithmetic modes for sigmoid / SiLU:
//   fast  - ex2.approx and the approximate division, like the reference's device code
//           (quack/activation.py:54-69);
//   exact - expf and IEEE division, x / (1 + exp(-x)): the expression of torch's CUDA silu / sigmoid
//           kernels, so a quantising epilogue reproduces torch's fp32 result bit for bit.
template <bool EXACT>
__device__ __forceinline__ float act_sigmoid(float x) {
  if constexpr (EXACT) return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-x)));
  else return __fdividef(1.f, 1.f + __expf(-x));
}
template <bool EXACT>
__device__ __forceinline__ float act_silu(float x) {
  if constexpr (EXACT) return __fdiv_rn(x, __fadd_rn(1.f, expf(-x)));
  else return x * act_sigmoid<false>(x);
}
__device__ __forceinline__ float act_gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}

template <int N>
__device__ __forceinline__ void act_apply_chunk(int act, bool exact, float (&x)[N]) {
#define QK_ACT_LOOP(EXPR)                      \
  _Pragma("unroll") for (int i = 0; i < N; ++i) { \
    const float v = x[i];                      \
    x[i] = (EXPR);                             \
  }
  switch (act) {
    case QK_ACT_RELU: QK_ACT_LOOP(fmaxf(v, 0.f)) break;
    case QK_ACT_RELU_SQ: QK_ACT_LOOP(fmaxf(v, 0.f) * fmaxf(v, 0.f)) break;
    case QK_ACT_SILU:
      if (exact) { QK_ACT_LOOP(act_silu<true>(v)) } else { QK_ACT_LOOP(act_silu<false>(v)) }
      break;
    case QK_ACT_GELU_TANH: QK_ACT_LOOP(act_gelu_tanh(v)) break;
    case QK_ACT_TANH: QK_ACT_LOOP(tanhf(v)) break;
    default: break;
  }
#undef QK_ACT_LOOP
}

// y[i] = f(gate = x[2i], up = x[2i+1])
template <int N>
__device__ __forceinline__ void gated_apply_chunk(int act, bool exact, const float (&x)[2 * N], float (&y)[N]) {
#define QK_GATED_LOOP(EXPR)                      \
  _Pragma("unroll") for (int i = 0; i < N; ++i) { \
    const float g = x[2 * i], u = x[2 * i + 1]; \
    y[i] = (EXPR);                               \
  }
  switch (act) {
    case QK_ACT_SWIGLU:
      if (exact) { QK_GATED_LOOP(__fmul_rn(act_silu<true>(g), u)) } else { QK_GATED_LOOP(act_silu<false>(g) * u) }
      break;
    case QK_ACT_REGLU: QK_GATED_LOOP(fmaxf(g, 0.f) * u) break;
    case QK_ACT_GEGLU: QK_GATED_LOOP(act_gelu_tanh(g) * u) break;
    case QK_ACT_GLU:
      if (exact) { QK_GATED_LOOP(__fmul_rn(act_sigmoid<true>(g), u)) } else { QK_GATED_LOOP(act_sigmoid<false>(g) * u) }
      break;
    default: QK_GATED_LOOP(g * u) break;
  }
#undef QK_GATED_LOOP
}

// x[i] += beta * C[off + i], i < 64; `nvalid` leading elements exist.  16-byte loads when the row
// segment is aligned and complete.
__device__ __forceinline__ void add_residual64(float (&x)[64], const void* c, int dtype, long long off, int nvalid,
                                               bool vec, float beta) {
  if (vec && nvalid == 64) {
    if (dtype == QK_DT_F32) {
      const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(c) + off);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 v = __ldg(src + i);
        x[4 * i] = fmaf(beta, v.x, x[4 * i]);
        x[4 * i + 1] = fmaf(beta, v.y, x[4 * i + 1]);
        x[4 * i + 2] = fmaf(beta, v.z, x[4 * i + 2]);
        x[4 * i + 3] = fmaf(beta, v.w, x[4 * i + 3]);
      }
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(c) + off);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = __ldg(src + i);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float lo, hi;
          if (dtype == QK_DT_BF16) {
            lo = __uint_as_float(u[j] << 16);
            hi = __uint_as_float(u[j] & 0xFFFF0000u);
          } else {
            const __half2 h = *reinterpret_cast<const __half2*>(&u[j]);
            lo = __low2float(h);
            hi = __high2float(h);
          }
          x[8 * i + 2 * j] = fmaf(beta, lo, x[8 * i + 2 * j]);
          x[8 * i + 2 * j + 1] = fmaf(beta, hi, x[8 * i + 2 * j + 1]);
        }
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    if (i < nvalid) {
      float v;
      if (dtype == QK_DT_F32) v = reinterpret_cast<const float*>(c)[off + i];
      else if (dtype == QK_DT_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(c)[off + i]);
      else v = __half2float(reinterpret_cast<const __half*>(c)[off + i]);
      x[i] = fmaf(beta, v, x[i]);
    }
  }
}

__device__ __forceinline__ float load_as_float(const void* p, int dtype, long long i) {
  if (dtype == QK_DT_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == QK_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// Store NV consecutive values of one row (columns [col, col+NV) of an (M, ld) matrix).
template <int NV>
__device__ __forceinline__ void store_row_chunk(void* base, int dtype, long long ld, int row, int col, int n_limit,
                                                const float (&x)[NV], bool vec_ok) {
  const int nvalid = min(NV, n_limit - col);
  if (nvalid <= 0) return;
  if (dtype == QK_DT_F32) {
    float* dst = reinterpret_cast<float*>(base) + static_cast<long long>(row) * ld + col;
    if (vec_ok && nvalid == NV) {
#pragma unroll
      for (int i = 0; i < NV; i += 4)
        *reinterpret_cast<float4*>(dst + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i)
        if (i < nvalid) dst[i] = x[i];
    }
  } else if (dtype == QK_DT_BF16) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(base) + static_cast<long long>(row) * ld + col;
    if (vec_ok && nvalid == NV) {
#pragma unroll
      for (int i = 0; i < NV; i += 8) {
        uint4 v;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(x[i], x[i + 1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(x[i + 2], x[i + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(x[i + 4], x[i + 5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(x[i + 6], x[i + 7]);
        v.x = *reinterpret_cast<uint32_t*>(&h0);
        v.y = *reinterpret_cast<uint32_t*>(&h1);
        v.z = *reinterpret_cast<uint32_t*>(&h2);
        v.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(dst + i) = v;
      }
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i)
        if (i < nvalid) dst[i] = __float2bfloat16_rn(x[i]);
    }
  } else {  // fp16
    __half* dst = reinterpret_cast<__half*>(base) + static_cast<long long>(row) * ld + col;
    if (vec_ok && nvalid == NV) {
#pragma unroll
      for (int i = 0; i < NV; i += 8) {
        uint4 v;
        __half2 h0 = __floats2half2_rn(x[i], x[i + 1]);
        __half2 h1 = __floats2half2_rn(x[i + 2], x[i + 3]);
        __half2 h2 = __floats2half2_rn(x[i + 4], x[i + 5]);
        __half2 h3 = __floats2half2_rn(x[i + 6], x[i + 7]);
        v.x = *reinterpret_cast<uint32_t*>(&h0);
        v.y = *reinterpret_cast<uint32_t*>(&h1);
        v.z = *reinterpret_cast<uint32_t*>(&h2);
        v.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(dst + i) = v;
      }
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i)
        if (i < nvalid) dst[i] = __float2half_rn(x[i]);
    }
  }
}

// ---- shared-memory staged TMA store ----------------------------------------------------
// Each epilogue warp owns two 4 KB slabs (32 rows x up to 128 bytes).  A thread writes the
// 16-byte units of its row with the XOR pattern of the TMA swizzle mode that matches the row
// width (128 / 64 / 32 bytes; 16-byte rows are unswizzled), so the quarter-warp phases of the
// 16-byte shared stores hit distinct banks; one lane then issues the bulk tensor store, which
// clips rows and columns outside the matrix.
struct StoreCtx {
  uint32_t slab0;   // first of this warp's consecutive 4 KB slabs
  uint32_t buf;     // 0 or 1
  uint32_t toggle;  // 1: two slabs used alternately; 0: a single slab
  __device__ __forceinline__ uint32_t cur() const { return slab0 + buf * 4096u; }
};

template <int NU>  // 16-byte units per row of the box: 1, 2, 4 or 8
__device__ __forceinline__ void box_store(const CUtensorMap* tm, StoreCtx& sc, int lane, const uint32_t* w, int c0,
                                          int c1) {
  if (lane == 0) {   // the store that last read this slab is done with it
    if (sc.toggle) tma_store_wait_read<1>();
    else tma_store_wait_read<0>();
  }
  __syncwarp();
  const uint32_t base = sc.cur() + static_cast<uint32_t>(lane) * (NU * 16);
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int pu = NU == 8 ? (u ^ (lane & 7)) : NU == 4 ? (u ^ ((lane >> 1) & 3)) : NU == 2 ? (u ^ ((lane >> 2) & 1)) : u;
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + pu * 16), "r"(w[4 * u]), "r"(w[4 * u + 1]),
                 "r"(w[4 * u + 2]), "r"(w[4 * u + 3])
                 : "memory");
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tm, sc.cur(), c0, c1);
    tma_store_commit();
  }
  sc.buf ^= sc.toggle;
}

__device__ __forceinline__ uint32_t pack2_16(int dtype, float a, float b) {
  if (dtype == QK_DT_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One output matrix of the epilogue.
struct Sink {
  void* base;
  long long ld;
  int dtype;
  const CUtensorMap* tm;
  bool tma;
};

// NV consecutive fp32 values of row `row`, columns [col, col+NV), of a `limit`-wide matrix.
template <int NV>
__device__ __forceinline__ void emit_plain(const Sink& s, StoreCtx& sc, int lane, int row_base, int row, bool row_ok,
                                           int col, int limit, const float (&x)[NV], bool vec_ok) {
  if (s.tma) {
    if (s.dtype == QK_DT_F32) {
#pragma unroll
      for (int b = 0; b < NV / 32; ++b) {
        if (col + b * 32 < limit)
          box_store<8>(s.tm, sc, lane, reinterpret_cast<const uint32_t*>(x) + b * 32, col + b * 32, row_base);
      }
    } else {
      uint32_t w[NV / 2];
#pragma unroll
      for (int i = 0; i < NV / 2; ++i) w[i] = pack2_16(s.dtype, x[2 * i], x[2 * i + 1]);
      box_store<NV / 8>(s.tm, sc, lane, w, col, row_base);
    }
  } else if (row_ok) {
    store_row_chunk<NV>(s.base, s.dtype, s.ld, row, col, limit, x, vec_ok);
  }
}

// ---- output quantiser ------------------------------------------------------------------
// fp32 -> E8M0 byte rounding the exponent up (smallest power of two >= s), zero -> 0,
// clamped to [2^-127, 2^127].
__device__ __forceinline__ uint32_t e8m0_round_up(float s) {
  const uint32_t bits = __float_as_uint(s);
  uint32_t e = (bits >> 23) & 0xFF;
  const uint32_t mant = bits & 0x7FFFFF;
  if (e == 0) {
    // zero -> 2^-127 (byte 0); a subnormal rounds up to the power of two at or above it
    if (mant == 0) return 0;
    const int lz = __clz(mant) - 9;       // leading zeros inside the 23-bit field
    int ex = -127 - lz;                   // floor(log2(s)) = -127 - lz
    if (mant & (mant - 1)) ex += 1;       // not a power of two: round up
    return static_cast<uint32_t>(max(ex, -127) + 127);
  }
  if (mant) e += 1;
  return min(e, 254u);
}
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float e4m3_byte_to_float(uint32_t b) {
  uint32_t h;
  asm("{\n\t.reg .b16 s;\n\tcvt.u16.u32 s, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, s;\n\t}" : "=r"(h) : "r"(b & 0xFF));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFF)));
}

// traits of the output formats: scale vector length, E8M0 (power-of-two) or E4M3 scales, 4-bit or 8-bit codes
__host__ __device__ constexpr int qf_vec(int qf) { return qf == QK_FMT_NVFP4 ? 16 : 32; }
__host__ __device__ constexpr bool qf_e8m0(int qf) { return qf != QK_FMT_NVFP4; }
__host__ __device__ constexpr bool qf_fp4(int qf) { return qf == QK_FMT_NVFP4 || qf == QK_FMT_MXFP4; }

__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Quantise V consecutive fp32 values sharing one scale factor.  Returns the scale byte;
// `q` receives the rescaled values (the saturating conversion happens at the store).  Arithmetic: scale = (amax / dmax) * norm; rcp = norm / scale_q (IEEE divides).
// A NaN among the values makes the block maximum NaN (torch.amax propagates it): the scale byte
// is then the format's NaN (0x7F for E4M3, 0xFF for E8M0), rcp = FLT_MAX like any non-positive
// scale, and the NaN elements themselves stay NaN up to the conversion (E4M3 code 0x7F; E2M1 has
// no NaN and saturates).
template <int QF, int V>
__device__ __forceinline__ uint32_t quantise_vec(float norm, const float* x, float* q) {
  // three-input NaN-propagating maximum: two elements per instruction
  float amax = 0.f;
  static_assert(V % 2 == 0, "pairs");
#pragma unroll
  for (int i = 0; i < V; i += 2) amax = max3_nan(amax, fabsf(x[i]), fabsf(x[i + 1]));
  const bool nan_block = amax != amax;
  constexpr float dmax = qf_fp4(QF) ? 6.f : 448.f;
  const float scale = __fmul_rn(__fdiv_rn(amax, dmax), norm);
  uint32_t byte;
  float scale_q;
  if constexpr (qf_e8m0(QF)) {
    byte = nan_block ? 0xFFu : e8m0_round_up(scale);
    scale_q = byte == 0 ? __uint_as_float(0x00400000u) /* 2^-127 */ : __uint_as_float(byte << 23);
  } else {
    byte = nan_block ? 0x7Fu : (cvt_e4m3x2(fminf(scale, 448.f), 0.f) & 0xFF);
    scale_q = e4m3_byte_to_float(byte);
  }
  // capped at FLT_MAX (quack/blockscaled/quantize_utils.py:9-22): norm / 2^-127 may overflow, and 0 * inf is NaN
  const float rcp = (!nan_block && scale_q > 0.f) ? fminf(__fdiv_rn(norm, scale_q), 3.402823466e+38f) : 3.402823466e+38f;
  // no clamp to +-dmax here: the conversions at the store are cvt.rn.satfinite, which saturate finite and
  // infinite values to the format maximum and keep a NaN a NaN where the format has one
#pragma unroll
  for (int i = 0; i < V; ++i) q[i] = __fmul_rn(x[i], rcp);
  return byte;
}

// Quantise NY consecutive values of one output row (columns [ycol, ycol+NY) of a row that is
// ylimit wide) and store codes + scale bytes.  Scale byte of (row m, scale column k) lives at
// atom (m/128, k/4), byte (m%32)*16 + ((m/32)%4)*4 + k%4 of the blocked layout.  Only
// in-range rows / scale columns are written: the launcher zero-fills buffers that have pad
// slots.
template <int QF, int NY>
__device__ __forceinline__ void quant_store_row(const GemmParams& p, float norm, const Sink& s, StoreCtx& sc, int lane,
                                                int row_base, int row, bool row_ok, int ycol, int ylimit,
                                                float (&y)[NY]) {
  void* out = s.base;
  const long long ldo = s.ld;
  constexpr int VEC = qf_vec(QF);
  constexpr int NSF = NY / VEC;
  constexpr bool FP4 = qf_fp4(QF);
  if (ycol + NY > ylimit) {   // (warp-uniform) only the last chunk of a ragged row
#pragma unroll
    for (int i = 0; i < NY; ++i)
      if (ycol + i >= ylimit) y[i] = 0.f;  // columns past the logical width count as zeros
  }
  float qv[NY];
  uint32_t sfb[NSF];
#pragma unroll
  for (int s = 0; s < NSF; ++s) sfb[s] = quantise_vec<QF, VEC>(norm, y + s * VEC, qv + s * VEC);
  if (s.tma) {
    // codes through the staged bulk store (every lane takes part); scale bytes below
    if constexpr (!FP4) {
      uint32_t w[NY / 4];
#pragma unroll
      for (int i = 0; i < NY / 4; ++i)
        w[i] = cvt_e4m3x2(qv[4 * i], qv[4 * i + 1]) | (cvt_e4m3x2(qv[4 * i + 2], qv[4 * i + 3]) << 16);
      box_store<NY / 16>(s.tm, sc, lane, w, ycol, row_base);
    } else {
      uint32_t w[NY / 8];
#pragma unroll
      for (int i = 0; i < NY / 8; ++i) {
        const float* v = qv + 8 * i;
        w[i] = cvt_e2m1x2(v[0], v[1]) | (cvt_e2m1x2(v[2], v[3]) << 8) | (cvt_e2m1x2(v[4], v[5]) << 16) |
               (cvt_e2m1x2(v[6], v[7]) << 24);
      }
      box_store<NY / 32>(s.tm, sc, lane, w, ycol / 2, row_base);
    }
  }
  if (!row_ok) return;
  const int sf_cols = (ylimit + VEC - 1) / VEC;
  const int k0 = ycol / VEC;
  unsigned char* rowbase =
      p.sfd + static_cast<long long>(row / 128) * p.sfd_stride_rm + (row % 32) * 16 + ((row / 32) % 4) * 4;
  if (NSF == 4 && k0 + 4 <= sf_cols) {
    *reinterpret_cast<uint32_t*>(rowbase + static_cast<long long>(k0 / 4) * 512) =
        sfb[0] | (sfb[1 % NSF] << 8) | (sfb[2 % NSF] << 16) | (sfb[3 % NSF] << 24);
  } else {
#pragma unroll
    for (int s = 0; s < NSF; ++s) {
      const int k = k0 + s;
      if (k < sf_cols) rowbase[static_cast<long long>(k / 4) * 512 + (k % 4)] = static_cast<unsigned char>(sfb[s]);
    }
  }
  if (s.tma) return;
  const int nvalid = min(NY, ylimit - ycol);
  if constexpr (!FP4) {
    unsigned char* dst = reinterpret_cast<unsigned char*>(out) + static_cast<long long>(row) * ldo + ycol;
    if (p.vec_store_ok && nvalid == NY) {
#pragma unroll
      for (int i = 0; i < NY; i += 16) {
        uint4 v;
        v.x = cvt_e4m3x2(qv[i], qv[i + 1]) | (cvt_e4m3x2(qv[i + 2], qv[i + 3]) << 16);
        v.y = cvt_e4m3x2(qv[i + 4], qv[i + 5]) | (cvt_e4m3x2(qv[i + 6], qv[i + 7]) << 16);
        v.z = cvt_e4m3x2(qv[i + 8], qv[i + 9]) | (cvt_e4m3x2(qv[i + 10], qv[i + 11]) << 16);
        v.w = cvt_e4m3x2(qv[i + 12], qv[i + 13]) | (cvt_e4m3x2(qv[i + 14], qv[i + 15]) << 16);
        *reinterpret_cast<uint4*>(dst + i) = v;
      }
    } else {
#pragma unroll
      for (int i = 0; i < NY; ++i)
        if (i < nvalid) dst[i] = static_cast<unsigned char>(cvt_e4m3x2(qv[i], 0.f) & 0xFF);
    }
  } else {
    // two E2M1 codes per byte, even column in the low nibble; ldo counts bytes
    unsigned char* dst = reinterpret_cast<unsigned char*>(out) + static_cast<long long>(row) * ldo + ycol / 2;
    if (p.vec_store_ok && nvalid == NY) {
#pragma unroll
      for (int i = 0; i < NY; i += 32) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float* s = qv + i + j * 8;
          w[j] = cvt_e2m1x2(s[0], s[1]) | (cvt_e2m1x2(s[2], s[3]) << 8) | (cvt_e2m1x2(s[4], s[5]) << 16) |
                 (cvt_e2m1x2(s[6], s[7]) << 24);
        }
        *reinterpret_cast<uint4*>(dst + i / 2) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < NY; i += 2)
        if (i < nvalid) dst[i / 2] = static_cast<unsigned char>(cvt_e2m1x2(qv[i], (i + 1 < nvalid) ? qv[i + 1] : 0.f));
    }
  }
}

// ------------------------------------------------------------------ the kernel ----------
template <int KIND, int TILE_N, int CG, int QF, bool FEW_ROWS = false, bool PULL = false>
__global__ void __launch_bounds__(GemmCfg<KIND, TILE_N, CG, FEW_ROWS, PULL>::LAUNCH_BOUND_THREADS, 1)
gemm_blockscaled_kernel(const __grid_constant__ GemmParams p) {
  using C = GemmCfg<KIND, TILE_N, CG, FEW_ROWS, PULL>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem_gen = smem_raw + (smem_base - smem_u32(smem_raw));

  const uint32_t sA = smem_base;
  const uint32_t sB = sA + C::STAGES * C::A_BYTES;
  const uint32_t sEpi = sB + C::STAGES * C::B_BYTES;  // staging slabs: 1024-byte aligned (swizzled)
  const uint32_t sXfer = sEpi + C::EPI_BYTES;          // (PULL) transport ring
  const uint32_t sSFA = sXfer + C::XFER_BYTES;
  const uint32_t sSFB = sSFA + C::STAGES * C::SFA_BYTES;
  const uint32_t sBias = sSFB + C::STAGES * C::SFB_BYTES;
  const uint32_t sCtrl = sBias + C::BIAS_BYTES;
  float* bias_smem = reinterpret_cast<float*>(smem_gen + (sBias - smem_base));
  uint8_t* ctrl_gen = smem_gen + (sCtrl - smem_base);
  // control block: barriers (8 B each), then the TMEM base pointer and the abort flag
  const uint32_t bar_full = sCtrl;                        // [STAGES]
  const uint32_t bar_empty = bar_full + 8 * C::STAGES;    // [STAGES]
  const uint32_t bar_acc_full = bar_empty + 8 * C::STAGES;  // [ACC_STAGES]
  const uint32_t bar_acc_empty = bar_acc_full + 8 * 2;      // [ACC_STAGES]
  const uint32_t bar_head_free = bar_acc_empty + 8 * 2;     // [ACC_STAGES] first chunk of a stage drained
  uint32_t* tmem_ptr_smem = reinterpret_cast<uint32_t*>(ctrl_gen + 8 * (2 * C::STAGES + 6));
  CtaCtl* ctl = reinterpret_cast<CtaCtl*>(ctrl_gen + 8 * (2 * C::STAGES + 6) + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta_rank = CG == 2 ? cluster_ctarank() : 0u;
  const bool is_leader = cta_rank == 0;
  const int cluster_id = CG == 2 ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int num_clusters = CG == 2 ? static_cast<int>(num_clusters_x()) : static_cast<int>(gridDim.x);
  // work units: (tile, K split); `num_tiles` counts units
  const int split_k = p.split_k;
  const int num_tiles = p.tiles_m * p.tiles_n * split_k;
  static_assert(8 * (2 * C::STAGES + 6) + 16 <= C::SCHED_FULL_OFF, "control block layout");
  const bool clc = p.clc == 1;       // tile ids come from cluster launch control
  const bool arrival = p.clc == 2;   // all-gather: shards are consumed in the order they arrive
  const bool ring = p.clc != 0;      // either way the ids travel through the scheduler ring
  const uint32_t bar_sched_full = sCtrl + C::SCHED_FULL_OFF;    // [SCHED_SLOTS] tile id published
  const uint32_t bar_sched_empty = sCtrl + C::SCHED_EMPTY_OFF;  // [SCHED_SLOTS] every reader has it (leader's copy)
  const uint32_t bar_clc = sCtrl + C::SCHED_CLC_BAR_OFF;        // [SCHED_SLOTS] answer of the hardware landed
  const uint32_t s_tile = sCtrl + C::SCHED_TILE_OFF;            // [SCHED_SLOTS] int
  const uint32_t s_resp = sCtrl + C::SCHED_RESP_OFF;            // [SCHED_SLOTS] 16 bytes
  const volatile int* tile_slots = reinterpret_cast<const volatile int*>(ctrl_gen + C::SCHED_TILE_OFF);
  const uint32_t sched_empty0 = CG == 2 ? mapa(bar_sched_empty, 0) : bar_sched_empty;
  // Reader side of the scheduler ring (whole warp calls): the next tile id, -1 = no more work,
  // -2 = wait abandoned.
  auto next_tile = [&](int& slot, uint32_t& ph) -> int {
    if (!__all_sync(0xffffffffu, wait_bounded<(CG == 2)>(bar_sched_full + 8 * slot, ph, ctl, p, QK_STATUS_SCHED_TIMEOUT, slot)))
      return -2;
    const int t = tile_slots[slot];
    __syncwarp();
    if (lane == 0) {
      if constexpr (CG == 1) mbar_arrive(sched_empty0 + 8 * slot);
      else mbar_arrive_remote(sched_empty0 + 8 * slot);   // the slot's value is in a register: nothing to release
    }
    if (++slot == C::SCHED_SLOTS) { slot = 0; ph ^= 1u; }
    return t;
  };

  if (threadIdx.x == 0) {
    ctl->abort = 0;
    for (int s2 = 0; s2 < C::SCHED_SLOTS; ++s2) {
      mbar_init(bar_sched_full + 8 * s2, 1);
      mbar_init(bar_sched_empty + 8 * s2, C::SCHED_CONSUMERS);
      mbar_init(bar_clc + 8 * s2, 1);
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);   // the leader's arrive.expect_tx (covers the whole CTA group)
      mbar_init(bar_empty + 8 * s, 1);  // one tcgen05.commit
    }
    for (int a = 0; a < C::ACC_STAGES; ++a) {
      mbar_init(bar_acc_full + 8 * a, 1);
      mbar_init(bar_acc_empty + 8 * a, C::EPI_WARPS * CG);
      mbar_init(bar_head_free + 8 * a, C::EPI_WARPS * CG);
    }
    fence_mbar_init();
    prefetch_tmap(&p.tm_a);
    prefetch_tmap(&p.tm_b);
    prefetch_tmap(&p.tm_sfa);
    prefetch_tmap(&p.tm_sfb);
  }
  if (warp == 1) {
    tmem_alloc<CG>(smem_u32(tmem_ptr_smem), C::TMEM_COLS);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) {
    cluster_arrive();
    cluster_wait();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_ptr_smem;
  // Programmatic dependent launch: everything above touched only shared / tensor memory and kernel
  // parameters.  Let the next GEMM of the stream set itself up on SMs this grid leaves free (a
  // few-row problem uses 32-64 of 148), then wait for the previous grid before the first global access.
  griddep_launch_dependents();
  griddep_wait();

  // alpha = host factor x (device factors): the device factors are the per-tensor scales of
  // NVFP4 operands, multiplied together first like the reference's folding
  float alpha = p.alpha;
  if (p.alpha_dev != nullptr) {
    float dev_scale = __ldg(p.alpha_dev);
    if (p.alpha_dev2 != nullptr) dev_scale = __fmul_rn(dev_scale, __ldg(p.alpha_dev2));
    alpha = (p.alpha == 1.0f) ? dev_scale : __fmul_rn(p.alpha, dev_scale);
  }

  if (warp == 0) {
    // ===================================== producer ========================================
    // The whole warp runs the loop (warp-uniform control flow keeps the address arithmetic in
    // uniform registers); one elected lane issues the copies.
    {
      const bool issuer = elect_one();
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t full0 = CG == 2 ? mapa(bar_full, 0) : bar_full;  // leader's barriers
      bool ok = true;
      const bool prof = p.prof != nullptr;
      long long t_start = prof ? clock64() : 0, t_wait = 0, t_gate = 0;
      // L2 prefetch cursor: runs `pf_dist` k-tiles ahead of the demand loads (across tile
      // boundaries, except under the all-gather gate where later rows may not have arrived), so
      // that the loads that fill a pipeline stage find their sectors in L2.
      const int pf_dist = p.prefetch_dist;
      int pf_tile = cluster_id, pf_kt = 0, pf_row0 = 0, pf_n0 = 0;
      auto pf_decode = [&]() {
        if (pf_tile < num_tiles) {
          const TileCoord t2 = decode_tile(p, pf_tile);
          pf_row0 = (t2.m_tile * CG + static_cast<int>(cta_rank)) * C::TILE_M;
          pf_n0 = t2.n_tile * TILE_N;
        }
      };
      auto pf_step = [&]() {
        if (pf_tile >= num_tiles) return;
        if (issuer) {
          const int kb2 = pf_kt * C::KT_BYTES;
          tma_prefetch_2d(&p.tm_a, kb2, pf_row0);
          tma_prefetch_2d(&p.tm_b, kb2, pf_n0 + (CG == 2 ? static_cast<int>(cta_rank) * C::B_ROWS : 0));
          tma_prefetch_3d(&p.tm_sfa, 0, pf_kt * C::AK, pf_row0 / 128);
          tma_prefetch_3d(&p.tm_sfb, 0, pf_kt * C::AK, pf_n0 / 128);
        }
        if (++pf_kt == p.k_tiles) {
          pf_kt = 0;
          pf_tile += num_clusters;
          if (p.ag_flags != nullptr) pf_tile = num_tiles;   // re-armed when the next tile passes its gate
          pf_decode();
        }
      };
      if (pf_dist > 0 && p.ag_flags == nullptr) {
        pf_decode();
        for (int i = 0; i < pf_dist; ++i) pf_step();
      }
      int sslot = 0;          // scheduler ring position (the leader writes it, the peer reads it)
      uint32_t sphase = 0;
      const int issuer_lane = __ffs(__ballot_sync(0xffffffffu, issuer)) - 1;
      // leader: hand a tile id (or -1 = no more work) to every reader of the ring, in both CTAs
      auto publish_tile = [&](int nt) -> bool {
        if (!__all_sync(0xffffffffu, wait_bounded<(CG == 2)>(bar_sched_empty + 8 * sslot, sphase ^ 1u, ctl, p,
                                                             QK_STATUS_SCHED_TIMEOUT, 16 + sslot)))
          return false;
        if (issuer) {
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(s_tile + 4 * sslot), "r"(nt) : "memory");
          if constexpr (CG == 2) {
            st_shared_cluster_u32(mapa(s_tile + 4 * sslot, 1), static_cast<uint32_t>(nt));
            mbar_arrive_cluster(mapa(bar_sched_full + 8 * sslot, 1));
            mbar_arrive_cluster(mapa(bar_sched_full + 8 * sslot, 0));
          } else {
            mbar_arrive(bar_sched_full + 8 * sslot);
          }
        }
        if (++sslot == C::SCHED_SLOTS) { sslot = 0; sphase ^= 1u; }
        return true;
      };
      // ---- arrival-order schedule of the all-gather mode (leader only) ----
      // Tile ownership is the static one (linear id = ring position of the shard x tiles per shard + j,
      // owned by cluster id % clusters), only the order of the shards follows their arrival flags.
      const int ag_per_shard = p.ag_tiles_m_per_shard * p.tiles_n;
      int ag_ring = -1, ag_j = 0, ag_done_n = 0;
      uint32_t ag_done = 0;
      long long t_gate2 = 0;
      auto ag_next = [&]() -> int {   // next linear tile id, -1 = finished, -2 = gave up waiting
        while (true) {
          if (ag_ring >= 0) {
            if (ag_j < ag_per_shard) {
              const int id = ag_ring * ag_per_shard + ag_j;
              ag_j += num_clusters;
              return id;
            }
            ag_done |= 1u << ag_ring;
            ++ag_done_n;
            ag_ring = -1;
          }
          // shards in which this cluster owns no tile need no waiting
          for (int r = 0; r < p.ag_num_shards; ++r) {
            if ((ag_done >> r) & 1u) continue;
            int j0 = (cluster_id - (r * ag_per_shard) % num_clusters) % num_clusters;
            if (j0 < 0) j0 += num_clusters;
            if (j0 >= ag_per_shard) {
              ag_done |= 1u << r;
              ++ag_done_n;
            }
          }
          if (ag_done_n == p.ag_num_shards) return -1;
          const long long tg0 = prof ? clock64() : 0;
          const int epoch = *reinterpret_cast<const volatile int*>(p.ag_epoch);
          const uint64_t t0 = globaltimer_ns();
          uint32_t it = 0;
          int pick = -1;
          // Every lane polls, but the warp acts on lane 0's view only: the outcome of an iteration (a shard,
          // give up, or poll again) is broadcast before anyone leaves the loop, so the lanes never diverge
          // around the shuffle.
          while (true) {
            int mine = -1;   // >= 0: ring position that has arrived; -2: give up; -1: nothing yet
            for (int r = 0; r < p.ag_num_shards; ++r) {   // ring order: the order the senders serve this rank
              if ((ag_done >> r) & 1u) continue;
              int shard = r + p.ag_first_shard;
              if (shard >= p.ag_num_shards) shard -= p.ag_num_shards;
              if ((*(reinterpret_cast<const volatile int*>(p.ag_flags) + shard) - epoch) >= 0) { mine = r; break; }
            }
            if (mine < 0 && (++it & 7u) == 0) {
              if (ctl->abort) {
                mine = -2;
              } else if (globaltimer_ns() - t0 > p.timeout_ns) {
                mine = -2;
                if (lane == 0) {
                  ctl->abort = 1;
                  if (atomicCAS(p.status, 0, QK_STATUS_GATE_TIMEOUT) == 0) {
                    p.status[1] = -1;
                    p.status[2] = static_cast<int>(ag_done);
                    p.status[3] = epoch;
                  }
                }
              }
            }
            pick = __shfl_sync(0xffffffffu, mine, 0);
            if (pick == -2) return -2;
            if (pick >= 0) break;
            __nanosleep(64);
          }
          if (prof) t_gate2 += clock64() - tg0;
          if (C::PULL && p.ag_pull != nullptr) {
            // the rows were written by other CTAs' bulk stores (or by another GPU through the switch) and
            // published through the flag: order this warp's tensor loads (asynchronous proxy) after the flag read
            __threadfence_system();
            fence_proxy_async_all();
          }
          ag_ring = pick;
          // first tile of this cluster in the shard: (pick * per_shard + j) % clusters == cluster_id
          int j0 = (cluster_id - (pick * ag_per_shard) % num_clusters) % num_clusters;
          if (j0 < 0) j0 += num_clusters;
          ag_j = j0;
        }
      };
      for (int tile = cluster_id; ok;) {
        if (arrival) {
          if (is_leader) {
            tile = ag_next();
            if (tile == -2 || !publish_tile(tile)) { ok = false; break; }
          } else {
            tile = next_tile(sslot, sphase);
            if (tile == -2) { ok = false; break; }
            if (C::PULL && p.ag_pull != nullptr) fence_proxy_async_all();   // (the leader read the flag; see there)
          }
          if (tile < 0) break;
        } else if (tile >= num_tiles) {
          break;
        }
        const int ks = split_k > 1 ? tile % split_k : 0;
        const TileCoord tc = decode_tile(p, split_k > 1 ? tile / split_k : tile);
        const int kt0 = ks * p.kt_per_split, kt1 = min(p.k_tiles, kt0 + p.kt_per_split);
        const int row0 = (tc.m_tile * CG + static_cast<int>(cta_rank)) * C::TILE_M;
        const int n0 = tc.n_tile * TILE_N;
        if (clc && is_leader) {
          // ask for the tile after this one now: the answer arrives while this tile loads
          if (!__all_sync(0xffffffffu, wait_bounded<(CG == 2)>(bar_sched_empty + 8 * sslot, sphase ^ 1u, ctl, p,
                                                               QK_STATUS_SCHED_TIMEOUT, 16 + sslot))) {
            ok = false;
            break;
          }
          if (issuer) {
            mbar_arrive_expect_tx(bar_clc + 8 * sslot, 16);
            clc_try_cancel(s_resp + 16 * sslot, bar_clc + 8 * sslot);
          }
        }
        if (p.ag_flags != nullptr && !arrival) {
          const long long tg0 = prof ? clock64() : 0;
          // arrival gate: the rows of this tile belong to chunk `c` of shard `tc.shard`
          const int rows_per_shard = p.ag_tiles_m_per_shard * C::TILE_M * CG;
          const int rows_per_chunk = rows_per_shard / p.ag_num_chunks;
          const int chunk = (row0 - tc.shard * rows_per_shard) / rows_per_chunk;
          const volatile int* flag = p.ag_flags + tc.shard * p.ag_num_chunks + chunk;
          const int epoch = *reinterpret_cast<const volatile int*>(p.ag_epoch);
          const uint64_t t0 = globaltimer_ns();
          uint32_t it = 0;
          while ((*flag - epoch) < 0) {
            if ((++it & 15u) == 0) {
              if (ctl->abort) { ok = false; break; }
              if (globaltimer_ns() - t0 > p.timeout_ns) {
                ctl->abort = 1;
                if (atomicCAS(p.status, 0, QK_STATUS_GATE_TIMEOUT) == 0) {
                  p.status[1] = tc.shard * p.ag_num_chunks + chunk;
                  p.status[2] = *flag;
                  p.status[3] = epoch;
                }
                ok = false;
                break;
              }
              __nanosleep(64);
            }
          }
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          if (prof) t_gate += clock64() - tg0;
          if (C::PULL && p.ag_pull != nullptr) {
            __threadfence_system();
            fence_proxy_async_all();
          }
          if (pf_dist > 0) {   // this tile's rows are resident now: prefetch its first k-tiles
            pf_tile = tile;
            pf_kt = 0;
            pf_decode();
            for (int i = 0; i < pf_dist && pf_tile == tile; ++i) pf_step();
          }
        }
        for (int kt = kt0; kt < kt1; ++kt) {
          const long long tw0 = prof ? clock64() : 0;
          if (!__all_sync(0xffffffffu, wait_bounded<false>(bar_empty + 8 * stage, phase ^ 1u, ctl, p,
                                                           QK_STATUS_PRODUCER_TIMEOUT, kt))) {
            ok = false;
            break;
          }
          if (prof) t_wait += clock64() - tw0;
          if (pf_dist > 0) pf_step();
          const uint32_t fb = full0 + 8 * stage;
          const int kb = kt * C::KT_BYTES;
          if (issuer) {
            if constexpr (CG == 1) {
              mbar_arrive_expect_tx(fb, C::STAGE_BYTES - C::A_BYTES + p.a_box_rows * C::KT_BYTES);
              tma_load_2d(sA + stage * C::A_BYTES, &p.tm_a, fb, kb, row0);
              tma_load_2d(sB + stage * C::B_BYTES, &p.tm_b, fb, kb, n0);
              tma_load_3d(sSFA + stage * C::SFA_BYTES, &p.tm_sfa, fb, 0, kt * C::AK, row0 / 128);
              tma_load_3d(sSFB + stage * C::SFB_BYTES, &p.tm_sfb, fb, 0, kt * C::AK, n0 / 128);
            } else {
              // the leader arms its barrier with the bytes of both CTAs; the peer's copies
              // complete on that same barrier (they may land before it is armed: the
              // transaction count is signed)
              if (is_leader) mbar_arrive_expect_tx(bar_full + 8 * stage, 2 * C::STAGE_BYTES);
              tma_load_2d_pair(sA + stage * C::A_BYTES, &p.tm_a, fb, kb, row0);
              tma_load_2d_pair(sB + stage * C::B_BYTES, &p.tm_b, fb, kb, n0 + static_cast<int>(cta_rank) * C::B_ROWS);
              tma_load_3d_pair(sSFA + stage * C::SFA_BYTES, &p.tm_sfa, fb, 0, kt * C::AK, row0 / 128);
              tma_load_3d_pair(sSFB + stage * C::SFB_BYTES, &p.tm_sfb, fb, 0, kt * C::AK, n0 / 128);
            }
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        // ---- next tile ----
        if (arrival) {
          // chosen at the top of the loop
        } else if (!clc) {
          tile += num_clusters;
        } else if (is_leader) {
          if (!__all_sync(0xffffffffu, wait_bounded<false>(bar_clc + 8 * sslot, sphase, ctl, p, QK_STATUS_SCHED_TIMEOUT,
                                                           32 + sslot))) {
            ok = false;
            break;
          }
          int nt = -1;
          if (issuer) {
            const int x = clc_query_first_ctaid_x(s_resp + 16 * sslot);
            fence_proxy_async_smem();   // the answer buffer is rewritten by the async proxy later
            nt = x >= 0 ? x / CG : -1;
          }
          nt = __shfl_sync(0xffffffffu, nt, issuer_lane);
          // (the slot's readers were awaited when the request was issued: this returns at once)
          if (!publish_tile(nt)) { ok = false; break; }
          tile = nt < 0 ? num_tiles : nt;
        } else {
          const int nt = next_tile(sslot, sphase);
          if (nt == -2) { ok = false; break; }
          tile = nt < 0 ? num_tiles : nt;
        }
      }
      if (prof && issuer) {
        long long* pb = p.prof + static_cast<long long>(blockIdx.x) * 16;
        pb[PROF_LOAD_TOTAL] = clock64() - t_start;
        pb[PROF_LOAD_WAIT_EMPTY] = t_wait;
        pb[PROF_LOAD_WAIT_GATE] = t_gate + t_gate2;
      }
    }
  } else if (warp == 1) {
    // ===================================== MMA issuer ======================================
    // Warp-uniform loop; one elected lane issues the tcgen05 instructions.  Descriptor halves
    // are 32-bit values derived from the stage index, so they live in uniform registers.
    if (is_leader) {
      const bool issuer = elect_one();
      const uint32_t idesc = make_idesc_block_scaled(KIND, C::TILE_M * CG, TILE_N) | p.idesc_elem_fmt;
      const uint32_t a_lo0 = sdesc_lo_sw128(sA), b_lo0 = sdesc_lo_sw128(sB);
      const uint32_t sfa_lo0 = sdesc_lo_sf(sSFA), sfb_lo0 = sdesc_lo_sf(sSFB);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      const bool prof = p.prof != nullptr;
      long long t_start = prof ? clock64() : 0, t_full = 0, t_acc = 0, t_icp = 0, t_imma = 0, t_icommit = 0;
      int sslot = 0;
      uint32_t sphase = 0;
      int tile_first = cluster_id;
      if (arrival) {   // even the first tile is chosen by the scheduler
        const int nt = next_tile(sslot, sphase);
        if (nt == -2) ok = false;
        tile_first = nt < 0 ? num_tiles : nt;
      }
      for (int tile = tile_first; tile < num_tiles && ok; ++local) {
        const int ks = split_k > 1 ? tile % split_k : 0;
        const TileCoord tc = decode_tile(p, split_k > 1 ? tile / split_k : tile);
        const int kt0 = ks * p.kt_per_split, kt1 = min(p.k_tiles, kt0 + p.kt_per_split);
        const int n0 = tc.n_tile * TILE_N;
        const uint32_t col_off = static_cast<uint32_t>((n0 % 128) / 32);
        const int a = local % C::ACC_STAGES;
        const uint32_t acc_phase = static_cast<uint32_t>(local / C::ACC_STAGES) & 1u;
        if (kt0 < kt1) {
          // The operands of the tile's first k-tile, before the accumulator hand-off: a wait leaves the barrier
          // as it is (the loop below finds it complete), and done in this order the ~400 cycles it takes to
          // observe the load barrier overlap the hand-off instead of following it.
          const long long tf0 = prof ? clock64() : 0;
          if (!__all_sync(0xffffffffu,
                          wait_bounded<false>(bar_full + 8 * stage, phase, ctl, p, QK_STATUS_MMA_FULL_TIMEOUT, kt0))) {
            ok = false;
            break;
          }
          if (prof) t_full += clock64() - tf0;
        }
        const long long ta0 = prof ? clock64() : 0;
        if (!__all_sync(0xffffffffu, wait_bounded<(CG == 2)>(bar_acc_empty + 8 * a, acc_phase ^ 1u, ctl, p,
                                                             QK_STATUS_MMA_ACC_TIMEOUT, local))) {
          ok = false;
          break;
        }
        if constexpr (C::OVERLAP_SF) {
          // this tile's scale factors overwrite the head of the other stage: the previous
          // tile's epilogue must have read those columns
          if (local > 0 &&
              !__all_sync(0xffffffffu, wait_bounded<(CG == 2)>(bar_head_free + 8 * (1 - a),
                                                               static_cast<uint32_t>((local - 1) / 2) & 1u, ctl, p,
                                                               QK_STATUS_MMA_ACC_TIMEOUT, -local))) {
            ok = false;
            break;
          }
        }
        if (prof) t_acc += clock64() - ta0;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(a * TILE_N);
        const uint32_t t_sfa = tmem_base + static_cast<uint32_t>(C::sfa_col0(a));
        const uint32_t t_sfb = tmem_base + static_cast<uint32_t>(C::sfb_col0(a));
        for (int kt = kt0; kt < kt1; ++kt) {
          const long long tf0 = prof ? clock64() : 0;
          if (!__all_sync(0xffffffffu,
                          wait_bounded<false>(bar_full + 8 * stage, phase, ctl, p, QK_STATUS_MMA_FULL_TIMEOUT, kt))) {
            ok = false;
            break;
          }
          if (prof) t_full += clock64() - tf0;
          tc_fence_after();
          const uint32_t a_lo = a_lo0 + static_cast<uint32_t>(stage) * (C::A_BYTES >> 4);
          const uint32_t b_lo = b_lo0 + static_cast<uint32_t>(stage) * (C::B_BYTES >> 4);
          const uint32_t sfa_lo = sfa_lo0 + static_cast<uint32_t>(stage) * (C::SFA_BYTES >> 4);
          const uint32_t sfb_lo = sfb_lo0 + static_cast<uint32_t>(stage) * (C::SFB_BYTES >> 4);
          const uint32_t acc_flag = kt != kt0 ? 1u : 0u;
          if (issuer) {
            const long long ti0 = prof ? clock64() : 0;
            // scale-factor atoms: shared memory -> tensor memory
#pragma unroll
            for (int j = 0; j < C::AK; ++j)
              tc_cp_32x128b_warpx4_lh<CG>(t_sfa + j * 4, sfa_lo + j * (512 >> 4), kSdescHiSf);
#pragma unroll
            for (int nb = 0; nb < C::NB; ++nb)
#pragma unroll
              for (int j = 0; j < C::AK; ++j)
                tc_cp_32x128b_warpx4_lh<CG>(t_sfb + j * (C::NB * 4) + nb * 4, sfb_lo + (nb * C::AK + j) * (512 >> 4),
                                            kSdescHiSf);
            const long long ti1 = prof ? clock64() : 0;
#pragma unroll
            for (int kb = 0; kb < C::KBLOCKS; ++kb) {
              uint32_t id, sfa_t, sfb_t;
              if constexpr (KIND == 0) {
                id = idesc_with_sf_id(idesc, kb, kb);
                sfa_t = t_sfa;
                sfb_t = t_sfb + col_off;
              } else if constexpr (KIND == 1) {
                id = idesc;
                sfa_t = t_sfa + kb * 4;
                sfb_t = t_sfb + kb * (C::NB * 4) + col_off;
              } else {
                // MXFP4: an instruction (64 elements) takes 2 of an atom's 4 scale columns
                id = idesc_with_sf_id(idesc, (kb & 1) * 2, (kb & 1) * 2);
                sfa_t = t_sfa + (kb >> 1) * 4;
                sfb_t = t_sfb + (kb >> 1) * (C::NB * 4) + col_off;
              }
              tc_mma_block_scale_lh<KIND, CG>(d_tmem, a_lo + kb * 2, kSdescHiSw128, b_lo + kb * 2, kSdescHiSw128, id, sfa_t,
                                              sfb_t, kb == 0 ? acc_flag : 1u);
            }
            const long long ti2 = prof ? clock64() : 0;
            // release the smem stage once the MMAs that read it have completed
            if constexpr (CG == 1) tc_commit(bar_empty + 8 * stage);
            else tc_commit_pair(bar_empty + 8 * stage, 3);
            if (prof) {
              const long long ti3 = clock64();
              t_icp += ti1 - ti0;
              t_imma += ti2 - ti1;
              t_icommit += ti3 - ti2;
            }
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if (issuer) {
          if constexpr (CG == 1) tc_commit(bar_acc_full + 8 * a);
          else tc_commit_pair(bar_acc_full + 8 * a, 3);
        }
        if (!ring) {
          tile += num_clusters;
        } else {
          const int nt = next_tile(sslot, sphase);
          if (nt == -2) { ok = false; ++local; break; }
          tile = nt < 0 ? num_tiles : nt;
        }
      }
      if (prof && issuer) {
        long long* pb = p.prof + static_cast<long long>(blockIdx.x) * 16;
        pb[PROF_MMA_TOTAL] = clock64() - t_start;
        pb[PROF_MMA_WAIT_FULL] = t_full;
        pb[PROF_MMA_WAIT_ACC] = t_acc;
        pb[PROF_MMA_TILES] = local;
        pb[PROF_MMA_ISSUE_CP] = t_icp;
        pb[PROF_MMA_ISSUE_MMA] = t_imma;
        pb[PROF_MMA_ISSUE_COMMIT] = t_icommit;
      }
    }
  } else if (C::PULL && warp == C::XFER_WARP) {
    // ===================================== transport (all-gather) ===========================
    // One warp per CTA copies this CTA's share of every remote shard: peer memory -> ring slot -> this GPU's
    // gather buffer.  The reads are per-thread 16-byte asynchronous copies (cp.async, the load/store unit):
    // bulk copies from a peer sit in the SM's copy unit for microseconds, and the main loop's tensor loads queue
    // behind them (measured: the GEMM lost about as much time as the transfer took).  The writes are local and
    // fast: one bulk store per slot.  Shards are taken in the order the GEMM consumes them (rank + 1, rank + 2,
    // ...: at every step the ranks read from distinct peers).  The pieces of a shard are dealt round-robin to
    // the CTAs of the grid; the CTA whose part completes a shard publishes its flag and tells the owner that
    // its buffer has been read.  Nothing here waits for the GEMM warps.
    if (p.ag_pull != nullptr) {
      const qk_ag_pull_args* g = p.ag_pull;
      constexpr int S = C::XFER_SLOTS;
      constexpr uint32_t SLOT = C::XFER_SLOT_BYTES;
      constexpr int AHEAD = C::XFER_AHEAD, PENDING = C::XFER_PENDING;
      const int W = p.ag_num_shards, rank = g->rank;
      const int epoch = *reinterpret_cast<const volatile int*>(p.ag_epoch);
      const unsigned long long sb0 = g->shard_bytes[0];
      const unsigned long long sb1 = g->num_payloads > 1 ? g->shard_bytes[1] : 0ull;
      const long long n0p = static_cast<long long>((sb0 + SLOT - 1) / SLOT), n1p = static_cast<long long>((sb1 + SLOT - 1) / SLOT);
      const long long total = n0p + n1p;
      const long long G = gridDim.x, b = blockIdx.x;
      const long long cnt = b < total ? (total - b + G - 1) / G : 0;   // this CTA's pieces per shard
      char* const l0 = static_cast<char*>(g->local_base[0]);
      char* const l1 = g->num_payloads > 1 ? static_cast<char*>(g->local_base[1]) : nullptr;
      uint32_t issued = 0, landed = 0;   // pieces loaded / stored since the kernel started (slot = n % S)
      bool ok = true;
      const uint64_t t_begin = globaltimer_ns();
      uint64_t t_owner = 0;
      if (g->mode == 1) {
        // ---- multicast push: this rank's own shard goes out once, through the switch, to every rank ----
        // Stores are posted: nothing is held while they travel, so a piece is simply read from local memory
        // into registers (16 x 16 bytes per lane: 8 KB per warp pass cover the local read latency; 4 KB moved
        // 290 GB/s per GPU) and stored through the multicast mapping.
        const char* const s0 = l0 + static_cast<unsigned long long>(rank) * sb0;
        const char* const s1 = sb1 ? l1 + static_cast<unsigned long long>(rank) * sb1 : nullptr;
        char* const m0 = static_cast<char*>(g->mc_base[0]) + static_cast<unsigned long long>(rank) * sb0;
        char* const m1 = sb1 ? static_cast<char*>(g->mc_base[1]) + static_cast<unsigned long long>(rank) * sb1 : nullptr;
        // The shard goes out in `chunks` row chunks, each with its own flag: every receiver then holds the first
        // chunk of every shard after 1/chunks of the exchange (a multicast store reaches all receivers at once,
        // so whole shards would all complete together, at the very end).
        constexpr uint32_t MC_LINES = 16, MC_PIECE = MC_LINES * 512;
        const int chunks = g->chunks > 0 ? g->chunks : 1;
        const unsigned long long cb0 = sb0 / chunks, cb1 = sb1 / chunks;   // bytes of one chunk (multiples of 16)
        const long long m0p = static_cast<long long>((cb0 + MC_PIECE - 1) / MC_PIECE);
        const long long mtotal = m0p + static_cast<long long>((cb1 + MC_PIECE - 1) / MC_PIECE);
        for (int c = 0; c < chunks; ++c) {
        for (long long idx = b; idx < mtotal; idx += G) {
          const bool first = idx < m0p;
          const unsigned long long off = static_cast<unsigned long long>(first ? idx : idx - m0p) * MC_PIECE;
          const unsigned long long left = (first ? cb0 : cb1) - off;
          const uint32_t bytes = static_cast<uint32_t>(left < MC_PIECE ? left : MC_PIECE);
          const unsigned long long coff = off + static_cast<unsigned long long>(c) * (first ? cb0 : cb1);
          const char* src = (first ? s0 : s1) + coff + lane * 16;
          char* dst = (first ? m0 : m1) + coff + lane * 16;
          uint4 v[MC_LINES];
#pragma unroll
          for (uint32_t i = 0; i < MC_LINES; ++i)
            if (i * 512 + lane * 16 < bytes) v[i] = ld_nc_v4(src + i * 512);
#pragma unroll
          for (uint32_t i = 0; i < MC_LINES; ++i)
            if (i * 512 + lane * 16 < bytes) multimem_st_v4(dst + i * 512, v[i]);
        }
        __threadfence_system();
        __syncwarp();
        if (lane == 0) {
          const int slot = rank * chunks + c;
          const int old = atomicAdd(g->arrive + slot, 1);
          if (old == static_cast<int>(G) - 1) {
            __threadfence_system();
            *reinterpret_cast<volatile int*>(g->arrive + slot) = 0;
            multimem_st_u32(g->mc_flags + slot, static_cast<uint32_t>(epoch));
            if (g->publish_ns != nullptr && c == chunks - 1) g->publish_ns[2 * rank] = globaltimer_ns() - t_begin;
          }
        }
        __syncwarp();
        }
      } else
      for (int step = 1; step < W && ok; ++step) {
        int s = rank + step;
        if (s >= W) s -= W;
        {   // the owner has staged its shard of this call (lane 0 polls; the warp follows its verdict)
          int verdict = 1;
          if (lane == 0) {
            const volatile int* pf = g->peer_flags[s] + s;
            const uint64_t t0 = globaltimer_ns();
            uint32_t it = 0;
            while ((*pf - epoch) < 0) {
              __nanosleep(200);
              if ((++it & 15u) == 0) {
                if (ctl->abort) { verdict = 0; break; }
                if (globaltimer_ns() - t0 > p.timeout_ns) {
                  ctl->abort = 1;
                  if (atomicCAS(p.status, 0, QK_STATUS_PULL_TIMEOUT) == 0) {
                    p.status[1] = 1000 + s;
                    p.status[2] = *pf;
                    p.status[3] = epoch;
                  }
                  verdict = 0;
                  break;
                }
              }
            }
            t_owner = globaltimer_ns() - t0;
            __threadfence_system();
          }
          ok = __shfl_sync(0xffffffffu, verdict, 0) != 0;
          __syncwarp();
          if (!ok) break;
        }
        const char* const r0 = static_cast<const char*>(g->peer_base[s][0]) + static_cast<unsigned long long>(s) * sb0;
        const char* const r1 = sb1 ? static_cast<const char*>(g->peer_base[s][1]) + static_cast<unsigned long long>(s) * sb1 : nullptr;
        char* const d0 = l0 + static_cast<unsigned long long>(s) * sb0;
        char* const d1 = sb1 ? l1 + static_cast<unsigned long long>(s) * sb1 : nullptr;
        auto piece = [&](long long t, const char*& src, char*& dst, uint32_t& bytes) {
          long long idx = b + t * G;
          if (idx < n0p) {
            const unsigned long long off = static_cast<unsigned long long>(idx) * SLOT;
            bytes = static_cast<uint32_t>(sb0 - off < SLOT ? sb0 - off : SLOT);
            src = r0 + off;
            dst = d0 + off;
          } else {
            const unsigned long long off = static_cast<unsigned long long>(idx - n0p) * SLOT;
            bytes = static_cast<uint32_t>(sb1 - off < SLOT ? sb1 - off : SLOT);
            src = r1 + off;
            dst = d1 + off;
          }
        };
        // Iteration t issues the reads of piece t (one cp.async group per iteration, empty past the last
        // piece, so that "all but the AHEAD newest groups" always means piece t - AHEAD) and stores piece
        // t - AHEAD.  A slot is reloaded once the bulk store that read it, issued PENDING iterations
        // earlier, has finished reading.
        for (long long t = 0; t < cnt + AHEAD; ++t) {
          const char* src;
          char* dst;
          uint32_t bytes;
          if (t < cnt) {
            const uint32_t slot = issued % S;
            if (issued >= static_cast<uint32_t>(S)) {
              if (lane == 0) tma_store_wait_read<PENDING - 1>();
              __syncwarp();
            }
            piece(t, src, dst, bytes);
            const uint32_t sdst = sXfer + slot * SLOT + lane * 16;
#pragma unroll
            for (uint32_t i = 0; i < SLOT / 512; ++i) {
              const uint32_t off = i * 512 + lane * 16;
              if (off < bytes) cp_async_16(sdst + i * 512, src + off);
            }
            ++issued;
          }
          cp_async_commit();
          const long long k = t - AHEAD;
          if (k >= 0) {
            cp_async_wait_group<AHEAD>();
            fence_proxy_async_smem();   // the slot was written through the generic proxy, the store reads it through the async one
            __syncwarp();
            if (lane == 0) {
              piece(k, src, dst, bytes);
              bulk_store(dst, sXfer + (landed % S) * SLOT, bytes);
              tma_store_commit();
            }
            ++landed;
          }
        }
        if (lane == 0) {
          tma_store_wait<0>();          // this CTA's part of the shard is in global memory
          fence_proxy_async_all();
          __threadfence();
          const int old = atomicAdd(g->arrive + s, 1);
          if (old == static_cast<int>(G) - 1) {
            // last CTA: every part is stored (each CTA fenced before it counted itself)
            __threadfence();
            *reinterpret_cast<volatile int*>(g->arrive + s) = 0;
            *reinterpret_cast<volatile int*>(g->flags_rw + s) = epoch;
            if (g->publish_ns != nullptr) {
              g->publish_ns[2 * s] = globaltimer_ns() - t_begin;
              g->publish_ns[2 * s + 1] = t_owner;
            }
            __threadfence_system();
            *reinterpret_cast<volatile int*>(g->peer_drained[s] + rank) = epoch;
          }
        }
        __syncwarp();
      }
      cp_async_wait_group<0>();
      if (lane == 0) tma_store_wait<0>();   // nothing may still use the ring when shared memory is released
    }
  } else {
    // ===================================== epilogue ========================================
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int ew = warp - 2;
    const int grp = ew / C::EPI_WARPS;   // this warp drains accumulator stage `grp` when there are two groups
    float* my_bias = bias_smem + ew * 64;
    float nb0 = 0.f, nb1 = 0.f;   // bias of columns (lane, lane + 32) of the chunk that is staged next
    const uint32_t acc_empty0 = CG == 2 ? mapa(bar_acc_empty, 0) : bar_acc_empty;
    const uint32_t head_free0 = CG == 2 ? mapa(bar_head_free, 0) : bar_head_free;
    const bool gated = p.act >= QK_ACT_GATED_FIRST;
    const bool act_exact = p.act_exact != 0;
    const float norm = p.norm_dev != nullptr ? __ldg(p.norm_dev) : p.norm;
    const float beta = p.beta_dev != nullptr ? __fmul_rn(p.beta, __ldg(p.beta_dev)) : p.beta;
    constexpr bool kQuant = QF != QK_FMT_NONE;
    const bool has_post = p.post != nullptr;
    const bool vec_ok = p.vec_store_ok != 0;
    const Sink sink_d{p.d, p.ldd, p.d_dtype, &p.tm_d, p.d_tma != 0};
    const Sink sink_post{p.post, p.ldpost, p.post_dtype, &p.tm_post, p.post_tma != 0};
    const bool plain_d = p.d != nullptr && (!kQuant || has_post);  // `d` holds unquantised values
    StoreCtx sc;
    static_assert(C::SLAB_BYTES == 4096, "StoreCtx assumes 4 KB slabs");
    sc.slab0 = sEpi + static_cast<uint32_t>(ew) * (C::SLABS_PER_WARP * C::SLAB_BYTES);
    sc.buf = 0;
    sc.toggle = C::SLABS_PER_WARP == 2 ? 1u : 0u;
    int local = 0;
    bool ok = true;
    const bool prof = p.prof != nullptr && q == 0 && grp == 0;   // the warp that owns rows 0..31 of the tile
    long long t_start = prof ? clock64() : 0, t_accw = 0, t_drain = 0, t_publish = 0, t_reduce = 0;
    int sslot = 0;
    uint32_t sphase = 0;
    int tile_first = cluster_id;
    if (arrival) {
      const int nt = next_tile(sslot, sphase);
      if (nt == -2) ok = false;
      tile_first = nt < 0 ? num_tiles : nt;
    }
    for (int tile = tile_first; tile < num_tiles && ok; ++local) {
      const int ks = split_k > 1 ? tile % split_k : 0;
      const int tile_id = split_k > 1 ? tile / split_k : tile;
      const TileCoord tc = decode_tile(p, tile_id);
      const int row0 = (tc.m_tile * CG + static_cast<int>(cta_rank)) * C::TILE_M;
      const int n0 = tc.n_tile * TILE_N;
      const int a = local % C::ACC_STAGES;
      // the id of the tile after this one (fetched early: the accumulator wait below hides it)
      // (under the arrival-order scheduler the next id may depend on a shard that has not landed: there
      // it is fetched after this tile's drain, see the end of the loop body)
      int tile_next = num_tiles;
      if (!ring) {
        tile_next = tile + num_clusters;
      } else if (!arrival) {
        const int nt = next_tile(sslot, sphase);
        if (nt == -2) { ok = false; break; }
        tile_next = nt < 0 ? num_tiles : nt;
      }
      auto fetch_late = [&]() {
        const int nt = next_tile(sslot, sphase);
        if (nt == -2) ok = false;
        tile_next = nt < 0 ? num_tiles : nt;
      };
      if (C::EPI_GROUPS == 2 && (local & 1) != grp) {   // the other group's tile
        if (arrival) fetch_late();
        tile = tile_next;
        continue;
      }
      const uint32_t acc_phase = static_cast<uint32_t>(local / C::ACC_STAGES) & 1u;
      // bias of the tile's first chunk (the accumulator wait below hides the load)
      auto fetch_bias = [&](int c) {
        const int col = n0 + c * 64 + lane;
        nb0 = col < p.N ? load_as_float(p.bias, p.bias_dtype, col) : 0.f;
        nb1 = col + 32 < p.N ? load_as_float(p.bias, p.bias_dtype, col + 32) : 0.f;
      };
      if (p.bias != nullptr) fetch_bias(0);
      const long long te0 = prof ? clock64() : 0;
      if (!wait_bounded<false>(bar_acc_full + 8 * a, acc_phase, ctl, p, QK_STATUS_EPI_TIMEOUT, local)) {
        ok = false;
        break;
      }
      const long long te1 = prof ? clock64() : 0;
      if (prof) t_accw += te1 - te0;
      tc_fence_after();
      const int row_base = row0 + q * 32;
      const int row = row_base + lane;
      const bool row_ok = row < p.M;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(a * TILE_N);
      constexpr int FULL_CHUNKS = TILE_N / 64;
      auto release_acc = [&]() {
        // the whole accumulator is in registers: hand the TMEM stage back to the MMA issuer
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 1) mbar_arrive(acc_empty0 + 8 * a);
          else mbar_arrive_remote(acc_empty0 + 8 * a);
        }
        if (prof) t_drain += clock64() - te1;
      };
      // epilogue of one 64-column chunk whose raw fp32 sums are in x
      auto finish_chunk = [&](int c, float (&x)[64]) {
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] *= alpha;
        const int col = n0 + c * 64;
        if (p.c != nullptr && row_ok && col < p.N)
          add_residual64(x, p.c, p.c_dtype, static_cast<long long>(row) * p.ldc + col, min(64, p.N - col),
                         p.c_vec_ok != 0, beta);
        if (p.bias != nullptr) {
          // the chunk's 64 bias values: from the two registers every lane fetched ahead, through this
          // warp's shared-memory row; then fetch the next chunk's
          __syncwarp();
          my_bias[lane] = nb0;
          my_bias[lane + 32] = nb1;
          __syncwarp();
          if (c + 1 < TILE_N / 64) fetch_bias(c + 1);
#pragma unroll
          for (int i = 0; i < 64; ++i) x[i] += my_bias[i];
        }
        if (col >= p.N) return;  // warp-uniform
        if (plain_d) emit_plain<64>(sink_d, sc, lane, row_base, row, row_ok, col, p.N, x, vec_ok);
        if (!has_post && !kQuant) return;
        if (has_post && gated) {
          float y[32];
          gated_apply_chunk<32>(p.act, act_exact, x, y);
          if constexpr (kQuant) quant_store_row<QF, 32>(p, norm, sink_post, sc, lane, row_base, row, row_ok, col / 2, p.N / 2, y);
          else emit_plain<32>(sink_post, sc, lane, row_base, row, row_ok, col / 2, p.N / 2, y, vec_ok);
        } else {
          if (has_post) act_apply_chunk<64>(p.act, act_exact, x);
          Sink s;  // member-wise select keeps both candidates in registers
          s.base = has_post ? sink_post.base : sink_d.base;
          s.ld = has_post ? sink_post.ld : sink_d.ld;
          s.dtype = has_post ? sink_post.dtype : sink_d.dtype;
          s.tm = has_post ? sink_post.tm : sink_d.tm;
          s.tma = has_post ? sink_post.tma : sink_d.tma;
          if constexpr (kQuant) quant_store_row<QF, 64>(p, norm, s, sc, lane, row_base, row, row_ok, col, p.N, x);
          else emit_plain<64>(s, sc, lane, row_base, row, row_ok, col, p.N, x, vec_ok);
        }
      };
#pragma unroll 1
      for (int c = 0; c < FULL_CHUNKS; ++c) {
        uint32_t r0[32], r1[32];
        tc_ld_32x32b_x32(t_row + c * 64, r0);
        tc_ld_32x32b_x32(t_row + c * 64 + 32, r1);
        tc_wait_ld();
        if (C::OVERLAP_SF && c == 0) {
          // columns [0, 64) of this stage are in registers: the next tile may put its scale
          // factors there
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (CG == 1) mbar_arrive(head_free0 + 8 * a);
            else mbar_arrive_remote(head_free0 + 8 * a);
          }
        }
        if (c == FULL_CHUNKS - 1) release_acc();
        float x[64];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = __uint_as_float(r0[i]);
          x[32 + i] = __uint_as_float(r1[i]);
        }
        if (split_k > 1) {
          // leave this unit's partial sums of the chunk in the workspace (valid rows and columns)
          const int col = n0 + c * 64;
          if (row_ok && col < p.N) {
            // (columns past N hold the zeros of the zero-filled B rows)
            const int group = (tile_id * CG + static_cast<int>(cta_rank)) * 4 + q;
            float4* dst = reinterpret_cast<float4*>(p.ws_partials) +
                          ((static_cast<long long>(ks) * p.ws_groups + group) * FULL_CHUNKS + c) * 512 + lane;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              __stcg(dst + i * 32, make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]));
          }
          continue;
        }
        finish_chunk(c, x);
      }
      if (split_k > 1 && row_base < p.M) {
        // one counter per 32-row group of the tile: the unit that arrives last owns the epilogue
        const long long ts0 = prof ? clock64() : 0;
        __threadfence();
        __syncwarp();
        int* ctr = p.ws_counters + (tile_id * CG + static_cast<int>(cta_rank)) * 4 + q;
        int old = 0;
        if (lane == 0) old = atomicAdd(ctr, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        const long long ts1 = prof ? clock64() : 0;
        if (prof) t_publish += ts1 - ts0;
        if (old == split_k - 1) {
          if (lane == 0) *ctr = 0;   // ready for the next launch
          __threadfence();
#pragma unroll 1
          for (int c = 0; c < FULL_CHUNKS; ++c) {
            const int col = n0 + c * 64;
            float x[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) x[i] = 0.f;
            if (row_ok && col < p.N) {
              const int group = (tile_id * CG + static_cast<int>(cta_rank)) * 4 + q;
              const long long split_stride = static_cast<long long>(p.ws_groups) * FULL_CHUNKS * 512;
              const float4* src = reinterpret_cast<const float4*>(p.ws_partials) +
                                  (static_cast<long long>(group) * FULL_CHUNKS + c) * 512 + lane;
              // Fixed order s2 = 0, 1, ...: the sum does not depend on who is last.  The loads of
              // two splits (32 x 16 bytes per lane) are issued before the first add: the loop is
              // bound by L2 round trips, not by bytes.
              for (int s2 = 0; s2 < split_k; s2 += 2) {
                const bool two = s2 + 1 < split_k;
                const float4* s0p = src + s2 * split_stride;
                const float4* s1p = two ? s0p + split_stride : s0p;
                float4 v[16], w[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = __ldcg(s0p + i * 32);
#pragma unroll
                for (int i = 0; i < 16; ++i) w[i] = __ldcg(s1p + i * 32);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  x[4 * i] += v[i].x; x[4 * i + 1] += v[i].y; x[4 * i + 2] += v[i].z; x[4 * i + 3] += v[i].w;
                }
                if (two) {
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                    x[4 * i] += w[i].x; x[4 * i + 1] += w[i].y; x[4 * i + 2] += w[i].z; x[4 * i + 3] += w[i].w;
                  }
                }
              }
            }
            finish_chunk(c, x);
          }
          if (prof) t_reduce += clock64() - ts1;
        }
      }
      if (arrival) fetch_late();
      tile = tile_next;
    }
    // bulk stores still reading the slabs must finish before shared memory is released
    if (lane == 0) tma_store_wait<0>();
    if (prof && lane == 0) {
      long long* pb = p.prof + static_cast<long long>(blockIdx.x) * 16;
      pb[PROF_EPI_TOTAL] = clock64() - t_start;
      pb[PROF_EPI_WAIT_ACC] = t_accw;
      pb[PROF_EPI_DRAIN] = t_drain;
      pb[PROF_EPI_TILES] = local;
      pb[PROF_SPLIT_PUBLISH] = t_publish;
      pb[PROF_SPLIT_REDUCE] = t_reduce;
    }
  }

  // ===================================== teardown ==========================================
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if constexpr (C::PULL) {
    // multicast push: the grid's last CTA tells every rank that this rank has finished reading the buffers of
    // this parity (their owners may refill them two calls from now)
    // (also after an abandoned wait: the peers' next calls wait for this word on their streams, without a
    // timeout; the error itself travels through the status word)
    if (threadIdx.x == 0 && p.ag_pull != nullptr && p.ag_pull->mode == 1) {
      const qk_ag_pull_args* g = p.ag_pull;
      __threadfence();
      const int old = atomicAdd(g->done, 1);
      if (old == static_cast<int>(gridDim.x) - 1) {
        *reinterpret_cast<volatile int*>(g->done) = 0;
        __threadfence_system();
        multimem_st_u32(g->mc_drained + g->rank, static_cast<uint32_t>(*reinterpret_cast<const volatile int*>(p.ag_epoch)));
      }
    }
  }
  if (ctl->abort) {
    // an abandoned wait may leave TMA copies or MMAs in flight: give them time to land
    // before shared and tensor memory are released
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
  }
  if constexpr (CG == 2) {
    cluster_arrive();
    cluster_wait();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace qk
