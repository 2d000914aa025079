/* irx_int.h -- internal types of the irptx-b200 core: limits, the parsed KIR graph, the
 * op-program form and the per-family launch plans.
 *
 * The KIR wire format is the reference's (BhuvanB404/IRptx 0.1.0, src/kir.c:553-675,
 * fe/kirdump.py:90-103); the structures that hold it here are this backend's own. Everything
 * is plain data with fixed bounds: a plan holds no pointers, so it can be copied, cached and
 * handed across the C ABI as bytes. */

#ifndef IRX_INT_H
#define IRX_INT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IRX_VERSION "0.1.0-b200"

/* ---- limits (same magnitudes as the reference's IR_MAX_*, src/irptx.h:23-39) ---- */
#define KIR_MAX_TEXT  (1u << 20)   /* KIR bytes */
#define KIR_MAX_NODE  65536u
#define KIR_MAX_FLD   262144u
#define KIR_MAX_ITEM  262144u
#define KIR_MAX_STR   (1u << 20)
#define KIR_MAX_DEP   64u
#define KIR_MAX_ARG   32u
#define KIR_MAX_DIM   8u
#define KIR_MAX_NAME  63u

/* ---- E-codes: the reference's numbering and ranges (src/err.c:22-64) plus this backend's
 * own, each listed in the table in err.c ---- */
enum {
    E000 = 0,
    E001 = 1, E002 = 2, E003 = 3, E004 = 4, E005 = 5, E009 = 9,
    E010 = 10, E011 = 11, E012 = 12, E013 = 13, E014 = 14, E015 = 15, E019 = 19,
    E020 = 20, E021 = 21, E022 = 22, E024 = 24, E025 = 25, E026 = 26, E027 = 27,
    E028 = 28, E029 = 29, E034 = 34,
    E040 = 40,   /* graph matches no op family this backend has a kernel template for */
    E041 = 41,   /* family recognised, but an index does not cover its buffer as the template needs */
    E042 = 42,   /* family recognised, but a shape or dtype is outside what its template takes */
    E043 = 43,   /* op program longer or wider than the template's register file */
    E059 = 59,
    E090 = 90,   /* CUDA driver missing or failed to initialise */
    E091 = 91,   /* kernel module failed to load or a kernel is missing from it */
    E092 = 92,   /* a launch failed or a device wait ran out (kernel error word set) */
    E093 = 93,   /* bad argument at the C ABI: count, null pointer or shard out of range */
    E094 = 94,   /* device or host memory could not be allocated or copied */
    E080 = 80, E081 = 81, E082 = 82, E099 = 99
};

int irx_fail(int code, const char *what);       /* one stderr line, returns 1 */
const char *irx_etext(int code);
const char *irx_last_msg(void);
int irx_last_code(void);
void irx_clear_error(void);
void irx_set_quiet(int quiet);
void irx_defer(int on);
void irx_emit_last(void);
void irx_save_error(int *code, char *msg, size_t cap);
void irx_restore_error(int code, const char *msg);

/* ---- parsed KIR ---- */
typedef enum {
    KV_NONE = 0, KV_BOOL, KV_INT, KV_FLT, KV_STR, KV_LIST, KV_NODE, KV_OP, KV_DT
} kv_tag_t;

typedef struct {
    uint8_t  tag;
    int64_t  i;            /* KV_INT, KV_BOOL */
    uint32_t fbits;        /* KV_FLT: f32 bits (narrowed once, as the reference does) */
    uint32_t ref;          /* STR/OP/DT: string offset; NODE: node id; LIST: first item */
    uint32_t n;            /* LIST: item count */
} kv_t;

typedef struct { uint32_t name; kv_t val; } kf_t;

typedef struct {
    uint32_t kname;        /* string offset of the node kind (Emmy class name) */
    uint32_t fld0, nfld;
} kn_t;

typedef enum { KA_IN = 0, KA_CONST, KA_OUT } ka_kind_t;
typedef enum { DT_NONE = 0, DT_F32, DT_BF16, DT_OTHER } dt_t;

typedef struct {
    uint32_t name;
    uint8_t  kind, dt, rank;
    int32_t  dim[KIR_MAX_DIM];
} ka_t;

typedef struct {
    char     name[KIR_MAX_NAME + 1];
    int32_t  grid[3], block[3], smem;
    ka_t     arg[KIR_MAX_ARG];
    uint32_t narg;
    uint32_t zero[KIR_MAX_ARG], nzero;
    uint32_t root;
    kn_t     node[KIR_MAX_NODE];   uint32_t nnode;
    kf_t     fld[KIR_MAX_FLD];     uint32_t nfld;
    kv_t     item[KIR_MAX_ITEM];   uint32_t nitem;
    char     str[KIR_MAX_STR];     uint32_t nstr;
} kir_t;

int kir_load(kir_t *k, const char *txt, size_t len);
const char *kir_str(const kir_t *k, uint32_t off);
const kn_t *kir_node(const kir_t *k, const kv_t *v);
const kv_t *kir_fld(const kir_t *k, const kn_t *nd, const char *name);
const kv_t *kir_item(const kir_t *k, const kv_t *lst, uint32_t i);
int kir_is(const kir_t *k, const kn_t *nd, const char *kind);
dt_t kir_dtype(const char *s);

#include "irx_ops.h"

typedef struct { uint8_t op, dst, a, b; } irx_ins_t;

typedef struct {
    uint8_t   nins;
    uint8_t   out;          /* register holding the result */
    uint8_t   pad[2];
    irx_ins_t ins[PROG_MAX_INS];
} irx_prog_t;

/* A uniform value: a rank-0 (or constant-index) const buffer read once on the device, a
 * literal, or (row ops) a reduced row statistic. */
typedef enum { UNI_NONE = 0, UNI_LIT, UNI_ARG, UNI_STAT } uni_kind_t;
typedef struct { uint8_t kind; uint8_t pad[3]; uint32_t v; int32_t off; } irx_uni_t;

/* ---- plans ---- */
typedef enum {
    FAM_NONE = 0, FAM_POINTWISE, FAM_REDUCE_ALL, FAM_REDUCE_ROWS, FAM_ROWOP,
    FAM_MATMUL, FAM_ATTENTION, FAM_KIR
} irx_fam_t;

/* Every family that runs op programs has one uniform program (`uprog`). It runs once
 * per launch (pointwise), once at the start and again once the total is known
 * (reductions), or at the start of a row and after each row statistic (row ops). Each
 * run recomputes every row- or launch-uniform value from the inputs it has so far. */
typedef struct {
    int64_t   n;                    /* elements per stream */
    uint8_t   nin, nout;
    uint8_t   in_arg[PROG_NSTREAM], in_dt[PROG_NSTREAM];
    uint8_t   out_arg[4], out_dt[4];
    irx_prog_t prog[4];             /* one element program per output */
    irx_prog_t uprog;
    irx_uni_t uni[PROG_NUNI];
    uint8_t   nuni;
    uint64_t  jit_key;              /* cache key of the per-graph kernel (0: none yet) */
} irx_pw_t;

typedef struct {
    int64_t   rows, cols;           /* REDUCE_ALL: rows = 1, cols = n */
    uint8_t   op;                   /* OP_ADD / OP_MAX / OP_MIN / OP_MUL */
    uint8_t   x_arg, x_dt, y_arg, y_dt;
    uint8_t   accumulate;           /* the KIR adds the total into y atomically: y = y + total */
    uint8_t   has_pre;              /* 0: the folded value is the loaded element itself */
    uint8_t   out_reg;              /* uniform register holding the written value */
    uint8_t   tot_reg;              /* uniform register the total is placed in */
    uint8_t   has_seed, seed_uni;   /* an Init seed's share, folded into the total by uprog's first
                                     * instruction from the literal uniform uni[seed_uni] */
    irx_prog_t pre;                 /* folded value per element, r0 = x */
    irx_prog_t uprog;
    irx_uni_t uni[PROG_NUNI];
    uint8_t   nuni;
} irx_red_t;

#define ROW_MAX_STAT 4
typedef struct {
    int64_t   rows, cols;
    uint8_t   x_arg, x_dt, w_arg, w_dt, y_arg, y_dt;
    uint8_t   has_w, nstat;
    uint8_t   stat_op[ROW_MAX_STAT];
    uint8_t   stat_reg[ROW_MAX_STAT];  /* uniform register each statistic lands in */
    irx_prog_t stat_pre[ROW_MAX_STAT]; /* r0 = x[row, j], r1 = w[j] */
    irx_prog_t epi;                    /* r0 = x[row, j], r1 = w[j] */
    irx_prog_t uprog;
    irx_uni_t uni[PROG_NUNI];
    uint8_t   nuni;
    uint8_t   kind;                    /* ROWK_*: a recognised specialisation, or generic */
    uint32_t  eps_bits;                /* ROWK_RMSNORM: eps */
} irx_row_t;

enum { ROWK_GENERIC = 0, ROWK_RMSNORM, ROWK_SOFTMAX, ROWK_L2NORM };

typedef struct {
    int64_t m, n, k;
    uint8_t a_arg, b_arg, c_arg, dt;   /* dt: DT_BF16 (tcgen05) or DT_F32 (SIMT) */
    uint8_t b_kmajor;                  /* 1: B stored [N, K]; 0: B stored [K, N] */
} irx_mm_t;

typedef struct {
    int64_t b, h, s, d;                /* the square form: s = sq = sk, d = dqk = dv */
    int64_t sq, sk, dqk, dv;           /* queries, keys, q/k width, v/o width */
    uint8_t q_arg, k_arg, v_arg, o_arg, dt, causal;
    uint8_t k_t;                       /* 1: K stored transposed, [.., dqk, sk] */
    uint8_t scale_div;                 /* 1: the graph divides the dot by div_bits (not * scale) */
    uint32_t scale_bits, div_bits;
} irx_at_t;

/* FAM_KIR: a graph no template takes, written out statement by statement as its own kernel
 * (kirgen.c); the source lives in the process's per-graph kernel store under `key`. */
typedef struct {
    uint64_t key;
    int32_t  grid, block;              /* the KIR's launch line, as the reference's runner uses it */
    int64_t  cells;
    uint32_t src_len;
} irx_kirk_t;

typedef struct {
    uint32_t magic;
    uint8_t  fam;
    uint8_t  narg;
    uint8_t  arg_kind[KIR_MAX_ARG], arg_dt[KIR_MAX_ARG];
    uint8_t  arg_zero[KIR_MAX_ARG];   /* 1: the KIR lists the output on a `zero` line */
    int64_t  arg_elems[KIR_MAX_ARG];
    char     kname[KIR_MAX_NAME + 1];
    union { irx_pw_t pw; irx_red_t red; irx_row_t row; irx_mm_t mm; irx_at_t at; irx_kirk_t kk; } u;
} irx_plan_int_t;

int irx_kirgen(const kir_t *k, irx_plan_int_t *p);

/* Shard s of ns of a plan's units (irx_plan_units): the one split of every launcher; narrowed to
 * [a, b) on this thread while irx_unit_window(a, b) is set (b < 0 clears it). */
void irx_unit_range(long long units, unsigned s, unsigned ns, long long *u0, long long *u1);
void irx_unit_window(long long a, long long b);

#define IRX_PLAN_MAGIC 0x49525842u   /* "IRXB" */

int irx_select_kir(const kir_t *k, irx_plan_int_t *p);
int irx_plan_text(const irx_plan_int_t *p, char *buf, size_t cap);
const char *irx_op_name(int op);
int irx_op_lookup(const char *name, int *arity);
int irx_op_arity(int op);

#ifdef __cplusplus
}
#endif

#endif /* IRX_INT_H */
