/* irx_kparams.h -- kernel parameter blocks, shared by the host launcher (C) and the sm_100a
 * kernels (CUDA). Each kernel takes one of these by value; the launcher fills it from a
 * plan and the caller's device pointers. Plain C layout, no pointers into host memory. */

#ifndef IRX_KPARAMS_H
#define IRX_KPARAMS_H

#include <stdint.h>
#include <cuda.h>            /* CUtensorMap: the TMA descriptor, 64-byte aligned */
#include "irx_int.h"

/* Threads per block of the full reduction (the launcher and the kernels agree on it). */
#define IRX_RED_ALL_THREADS 256

/* Device-side error word, written by a kernel whose bounded wait ran out. */
#define IRX_KERR_TIMEOUT   1u
#define IRX_KERR_TMEM      2u

typedef struct {
    const void *ptr;        /* UNI_ARG: the const buffer */
    uint32_t    bits;       /* UNI_LIT: f32 bits */
    int32_t     off;        /* UNI_ARG: element offset */
    uint8_t     kind, dt;   /* uni_kind_t, dt_t */
    uint8_t     pad[2];
} irx_kuni_t;

typedef struct {
    const void *in[PROG_NSTREAM];
    void       *out[4];
    irx_kuni_t  uni[PROG_NUNI];
    irx_prog_t  prog[4];
    irx_prog_t  uprog;
    int64_t     begin, end;         /* element range of this launch (a shard) */
    uint8_t     in_dt[PROG_NSTREAM], out_dt[4];
    uint8_t     nin, nout, nuni, vec_ok;
} irx_kpw_t;

/* The per-graph pointwise kernel's parameters (jit.c writes the same layout into its source). */
typedef struct {
    const void *in[PROG_NSTREAM];
    void       *out[4];
    const void *uni[PROG_NUNI];     /* UNI_ARG: the const buffer; others unused */
    int64_t     begin, end;
    int32_t     vec_ok, pad;
} irx_kpwj_t;

typedef struct {
    const void *x;
    void       *y;
    float      *partial;            /* REDUCE_ALL: one float per block (scratch) */
    unsigned   *ticket;             /* REDUCE_ALL: arrival counter (scratch), left at 0 */
    irx_kuni_t  uni[PROG_NUNI];
    irx_prog_t  pre, uprog;
    int64_t     rows, cols;         /* this launch's rows (REDUCE_ALL: 1) */
    int64_t     row0;               /* first row (shards) */
    int64_t     begin, end;         /* REDUCE_ALL: element range of this launch */
    uint8_t     op, x_dt, y_dt, has_pre, out_reg, tot_reg, nuni, accumulate;
    uint8_t     vec_ok, pad[7];
} irx_kred_t;

typedef struct {
    const void *x, *w;
    void       *y;
    irx_kuni_t  uni[PROG_NUNI];
    irx_prog_t  stat_pre[ROW_MAX_STAT], epi, uprog;
    int64_t     rows, cols, row0;
    uint8_t     stat_op[ROW_MAX_STAT], stat_reg[ROW_MAX_STAT];
    uint8_t     x_dt, w_dt, y_dt, has_w, nstat, nuni, bulk_ok, kind;
    uint32_t    eps_bits;
    uint32_t    smem_row_bytes;     /* bytes of one staged row buffer */
    unsigned   *err;                /* device error word */
    uint8_t     ecache;             /* softmax: 1 keep exp(x - max) in the staged f32 row, 0 recompute */
    uint8_t     rk;                 /* written-out forms: 1/2/4 = cols / (256 * 8), the row held in
                                     * registers; 0 the loop form */
    uint8_t     pad2[6];
} irx_krow_t;

typedef struct {
    CUtensorMap tma_a, tma_b;       /* tcgen05 path: A [M,K] and B ([K,N] or [N,K]) tiles */
    CUtensorMap tma_c;              /* wide pair path: C [M, n1] (the launch's columns), stored by TMA */
    const void *a, *b;
    void       *c;
    int64_t     m, n, k;
    int64_t     n0, n1;             /* column range of this launch (N-column shards) */
    unsigned   *err;                /* device error word */
    uint8_t     b_kmajor;
    uint8_t     no_loads;           /* failure injection (tests): the producers issue no loads */
    uint8_t     stages;             /* CTA-pair kernel: depth of the shared-memory ring */
    uint8_t     group;              /* CTA-pair kernel: 256-row tile rows walked together (L2 reuse) */
    uint8_t     pad[4];
    uint64_t    wait_ns;            /* limit of each device wait, ns (0: IRX_WAIT_NS) */
} irx_kmm_t;

typedef struct {
    CUtensorMap tma_q, tma_k, tma_v;  /* tcgen05 path: [B*H*S, D] views */
    const void *q, *k, *v;
    void       *o;
    int64_t     b, h, s, d;
    int64_t     sq, sk, dqk, dv;    /* general shape (SIMT path) */
    int64_t     bh0, bh1;           /* batch*head range of this launch */
    float       scale;
    float       divisor;            /* scale_div: the score is dot / divisor, as the graph writes it */
    unsigned   *err;
    unsigned   *sched;              /* persistent form: the next unit to hand out (zeroed per launch) */
    uint8_t     causal, k_t, scale_div, pad[5];
} irx_kat_t;

#endif /* IRX_KPARAMS_H */
