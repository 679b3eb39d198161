/* Enumerations shared by the CUDA kernels, the C ABI (include/quack_b200.h) and the Python
 * host code.  Plain C so that the public header can include it. */
#ifndef QK_TYPES_H_
#define QK_TYPES_H_

/* block-scaled formats */
#define QK_FMT_NONE 0
#define QK_FMT_MXFP8_E4M3 1 /* E4M3 codes, one E8M0 scale per 32 elements          */
#define QK_FMT_NVFP4 2      /* E2M1 codes (2 per byte), one E4M3 scale per 16      */
#define QK_FMT_MXFP8_E5M2 3 /* E5M2 codes, one E8M0 scale per 32 elements          */
#define QK_FMT_MXFP4 4      /* E2M1 codes (2 per byte), one E8M0 scale per 32      */

/* E8M0 scale rule of the MX quantizers (quack/blockscaled/quantize.py:254-282) */
#define QK_SCALING_DEFAULT 0 /* the format's default: rceil for MXFP8, floor for MXFP4 */
#define QK_SCALING_FLOOR 1
#define QK_SCALING_RCEIL 2

/* plain element types */
#define QK_DT_BF16 0
#define QK_DT_F16 1
#define QK_DT_F32 2

/* epilogue activations; values >= QK_ACT_GATED_FIRST consume (gate, up) column pairs */
#define QK_ACT_NONE 0
#define QK_ACT_RELU 1
#define QK_ACT_RELU_SQ 2
#define QK_ACT_SILU 3
#define QK_ACT_GELU_TANH 4
#define QK_ACT_TANH 5
#define QK_ACT_GATED_FIRST 16
#define QK_ACT_SWIGLU 16
#define QK_ACT_REGLU 17
#define QK_ACT_GEGLU 18
#define QK_ACT_GLU 19

/* return codes of the C entry points */
#define QK_OK 0
#define QK_ERR_INVALID_ARG (-1)
#define QK_ERR_UNSUPPORTED (-2)
#define QK_ERR_CUDA (-3)
#define QK_ERR_TOO_LARGE (-4)

/* device status word (status[0]) written by a kernel that abandoned a wait */
/* tile schedulers of the GEMM */
#define QK_SCHED_STATIC 0
#define QK_SCHED_CLC 1
#define QK_SCHED_ARRIVAL 2

#define QK_STATUS_OK 0
#define QK_STATUS_PRODUCER_TIMEOUT 1
#define QK_STATUS_MMA_FULL_TIMEOUT 2
#define QK_STATUS_MMA_ACC_TIMEOUT 3
#define QK_STATUS_EPI_TIMEOUT 4
#define QK_STATUS_GATE_TIMEOUT 5
#define QK_STATUS_SCHED_TIMEOUT 6
#define QK_STATUS_PULL_TIMEOUT 7 /* in-kernel all-gather transport: status[1] = 1000 + shard (the peer had not
                                     staged it) or the slot of the copy that did not land */

#define QK_AG_MAX_RANKS 16
#define QK_AG_MAX_PAYLOADS 2

/* In-kernel transport of the all-gather GEMM ("pull"): one extra warp per CTA of the GEMM copies the remote
 * shards from the peers' gather buffers (mapped into this process, e.g. through qk_ipc_open) into this rank's
 * gather buffers with bulk asynchronous copies through shared memory, shard by shard in the order the GEMM
 * consumes them (rank + 1, rank + 2, ...), and publishes flags[shard] = *epoch when the last CTA has stored
 * its part of the shard; the same CTA then writes *epoch into peer_drained[shard][rank] (the owner may refill
 * that buffer).  Before it reads shard s it waits (bounded) until peer_flags[s][s] >= *epoch, i.e. until peer
 * s has staged its own shard of this call.  The struct lives in DEVICE memory (it is constant per buffer
 * parity: build it once).  This replaces the reference's separate all-gather kernels / copy-engine pushes
 * (quack/distributed/all_gather_gemm.py:31-38, :197-238) with peer loads issued by the GEMM kernel itself;
 * it has no counterpart in the reference.  Needs num_chunks == 1, tile_n == 256 and cta_group == 2 (or 0). */
typedef struct qk_ag_pull_args {
  int num_payloads;                               /* 1 or 2 byte ranges per shard (codes; codes + scale bytes) */
  int rank;
  unsigned long long shard_bytes[QK_AG_MAX_PAYLOADS];   /* bytes of ONE shard; multiples of 16 */
  void* local_base[QK_AG_MAX_PAYLOADS];           /* this rank's gather buffer: shard s at + s * shard_bytes; 16-byte aligned */
  const void* peer_base[QK_AG_MAX_RANKS][QK_AG_MAX_PAYLOADS];  /* peer s's gather buffer (same layout); [rank] unused */
  const int* peer_flags[QK_AG_MAX_RANKS];         /* peer s's flag array */
  int* peer_drained[QK_AG_MAX_RANKS];             /* peer s's drained array (num_shards int32) */
  int* arrive;                                    /* num_shards int32 counters, zero between calls */
  int* flags_rw;                                  /* this rank's flag array (the `flags` of qk_ag_args), writable */
  unsigned long long* publish_ns;                 /* optional (NULL = off): num_shards x 2 words; the CTA that publishes
                                                     shard s stores [2s] = nanoseconds since its own start of the
                                                     kernel, [2s+1] = nanoseconds it waited for the owner's flag */
  /* mode 1 ("multicast push"): instead of reading the peers' shards, every rank stores its OWN shard (read from its
   * rows of local_base) through an NVSwitch multicast mapping that covers the gather buffers of all ranks, so each
   * byte leaves the GPU once and the switch replicates it.  When the last CTA has stored its part the rank's flag is
   * written through the multicast mapping of the flag arrays (flags[rank] = *epoch on every rank), and when the
   * last CTA of the grid has finished its tiles, *epoch is written into drained[rank] on every rank (the buffers of
   * this parity may be refilled).  peer_base / peer_flags / peer_drained are not used in this mode. */
  int mode;                                       /* 0 = pull (above), 1 = multicast push */
  int chunks;                                     /* mode 1: row chunks per rank (0 = 1), pushed and flagged one after the
                                                     other: flag index rank * chunks + c.  The GEMM is then given
                                                     num_shards = ranks * chunks, first_shard = rank * chunks */
  void* mc_base[QK_AG_MAX_PAYLOADS];              /* multicast address of the gather buffers (same layout) */
  int* mc_flags;                                  /* multicast address of the flag arrays */
  int* mc_drained;                                /* multicast address of the drained arrays */
  int* done;                                      /* one int32 counter, zero between calls */
} qk_ag_pull_args;


#endif /* QK_TYPES_H_ */
