/* irx_ops.h -- the op-program register file and op numbering. Plain C with no includes, so
 * that the host (C), the prebuilt kernels (nvcc) and the per-graph kernels compiled at run time
 * (NVRTC) all read the one definition. */
#ifndef IRX_OPS_H
#define IRX_OPS_H

/* ---- op programs: straight-line f32 code over a small register file ---- */
#define PROG_MAX_INS  24
#define PROG_NSTREAM  4     /* r0..r3: per-element input streams */
#define PROG_NUNI     12    /* r4..r15: values uniform over a launch or a row */
#define PROG_NTMP     8     /* r16..r23: per-element temporaries */
#define PROG_R_UNI    PROG_NSTREAM
#define PROG_R_TMP    (PROG_NSTREAM + PROG_NUNI)
#define PROG_NREG     (PROG_R_TMP + PROG_NTMP)

/* Op numbering shared by host and device; names and arities follow the reference's op
 * table (src/ops.c:27-54). */
typedef enum {
    OP_NONE = 0, OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_MAX, OP_MIN, OP_RELU, OP_COPY,
    OP_NEG, OP_ABS, OP_SQRT, OP_RSQRT, OP_RCP, OP_TANH, OP_SIN, OP_COS, OP_LOG2,
    OP_EXP, OP_EXPF, OP_LOG, OP_SIGMOID, OP_SILU, OP_SOFTPLUS, OP_POW, OP_COUNT
} irx_op_t;

#endif /* IRX_OPS_H */
