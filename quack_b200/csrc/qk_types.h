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

#endif /* QK_TYPES_H_ */
