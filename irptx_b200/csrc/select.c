/* select.c -- the sm_100a op-family selector.
 *
 * It replaces the reference's instruction selection, verifier and emitter
 * (src/isel.c, src/verify.c, src/emit.c): instead of lowering every KIR statement to PTX
 * records, it evaluates the Tile body symbolically into a dataflow graph and recognises,
 * from the graph alone, which hand-written kernel template computes the same outputs:
 *
 *   pointwise   every global Write is an elementwise function of Loads at its own cell
 *   reductions  a strided per-thread Accum, folded across the block by WarpShuffle and
 *               TreeHalve (src/isel.c:1718-1840), then a Write per row or an atomic add
 *   row ops     one or more such row statistics, then a second strided loop writing an
 *               elementwise function of the row, the statistics and a broadcast vector
 *   matmul      a Loop over K with an Accum of A[i,k]*B[k,j] (src/isel.c:1848-1870)
 *   attention   an online softmax over keys: coupled maximum / rescaled-sum Accums
 *               (src/isel.c:1301-1319) around a dot-product Loop
 *
 * The statement semantics it evaluates are the reference's: the thread model of is_tile
 * (src/isel.c:910-945), Load/Write flattening (mm_flat 404), Accum seeding and `base`
 * (1306-1400), StridedLoop bounds (1430-1445), Cond scopes (1513). Names never decide
 * anything: only the structure of the graph does (the property tests/rename.py pins).
 * Every graph that is not recognised is refused with one E-code line, as the reference
 * refuses what it cannot lower. */

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "irx_int.h"

/* ---------------------------------------------------------------------------------------
 * Affine integer forms over index variables: tile axes, loop variables, lane/warp/tid.
 * ------------------------------------------------------------------------------------ */

#define V_TILE0  0
#define V_LOOP0  8
#define V_LANE   48
#define V_WARP   49
#define V_TID    50
#define AFF_MAXV 6

typedef struct {
    uint8_t ok;                 /* 0: not affine (or not an integer) */
    uint8_t nv;
    uint8_t var[AFF_MAXV];
    int64_t coef[AFF_MAXV];
    int64_t cst;
} aff_t;

static aff_t aff_const(int64_t c) { aff_t a; memset(&a, 0, sizeof a); a.ok = 1; a.cst = c; return a; }
static aff_t aff_var(int v) { aff_t a = aff_const(0); a.nv = 1; a.var[0] = (uint8_t)v; a.coef[0] = 1; return a; }
static aff_t aff_bad(void) { aff_t a; memset(&a, 0, sizeof a); return a; }
static int aff_isc(const aff_t *a) { return a->ok && a->nv == 0; }

static int64_t aff_coef(const aff_t *a, int v)
{
    int i;
    for (i = 0; i < a->nv; i++) if (a->var[i] == v) return a->coef[i];
    return 0;
}

static aff_t aff_add(aff_t a, aff_t b, int64_t sb)
{
    int i, j;
    if (!a.ok || !b.ok) return aff_bad();
    a.cst += sb * b.cst;
    for (j = 0; j < b.nv; j++) {
        for (i = 0; i < a.nv; i++)
            if (a.var[i] == b.var[j]) { a.coef[i] += sb * b.coef[j]; break; }
        if (i == a.nv) {
            if (a.nv >= AFF_MAXV) return aff_bad();
            a.var[a.nv] = b.var[j];
            a.coef[a.nv] = sb * b.coef[j];
            a.nv++;
        }
    }
    for (i = 0; i < a.nv;) {            /* drop zero terms */
        if (a.coef[i] == 0) {
            a.var[i] = a.var[a.nv - 1];
            a.coef[i] = a.coef[a.nv - 1];
            a.nv--;
        } else i++;
    }
    return a;
}

static aff_t aff_scale(aff_t a, int64_t c)
{
    int i;
    if (!a.ok) return a;
    if (c == 0) return aff_const(0);
    a.cst *= c;
    for (i = 0; i < a.nv; i++) a.coef[i] *= c;
    return a;
}

static int aff_eq(const aff_t *a, const aff_t *b)
{
    aff_t d = aff_add(*a, *b, -1);
    return d.ok && d.nv == 0 && d.cst == 0;
}

/* ---------------------------------------------------------------------------------------
 * The symbolic state.
 * ------------------------------------------------------------------------------------ */

enum { FV_CONST = 1, FV_LOAD, FV_OP, FV_PREV, FV_FINAL, FV_OPAQUE };

#define MAX_FV    4096
#define MAX_IDX   1024
#define MAX_ACC   32
#define MAX_LOOP  32
#define MAX_WR    64
#define MAX_SW    32
#define MAX_BIND  2048
#define MAX_PRED  8

typedef struct { aff_t d[KIR_MAX_DIM]; uint8_t rank; } idx_t;

typedef struct {
    uint8_t  kind, op, arg, lane;
    uint16_t a, b;              /* operands (FV_OP) */
    uint16_t idx;               /* FV_LOAD: index table entry */
    uint16_t acc;               /* FV_PREV / FV_FINAL */
    uint32_t bits;              /* FV_CONST */
} fv_t;

typedef struct {
    uint32_t name;
    uint8_t  op;
    int      loop;              /* owning loop id, -1 when not seeded by a loop */
    int      nupd;              /* Accum statements seen */
    uint16_t upd_val, upd_base; /* base 0 = the accumulator itself */
    int      upd_loop;          /* innermost loop of the Accum statement */
    int      shuf_len;          /* WarpShuffle length applied after the loop, 0 none */
    int      tree_len;          /* TreeHalve length, 0 none */
    int      tree_ok;           /* tree folds by `warp` over a buffer fed by lane 0 */
    int      closed;            /* its loop has ended */
    uint16_t final_val;         /* value the accumulator holds after its loop */
    uint8_t  has_seed;          /* an Init started every thread's partial at seed_bits, not the identity */
    uint32_t seed_bits;
} acc_t;

typedef struct {
    int      kind;              /* 1 Loop, 2 StridedLoop */
    int      parent;
    int64_t  ext, step;
    aff_t    start, end;        /* end.ok == 0: none */
    uint32_t name;
} loop_t;

enum { PR_EQ = 1, PR_LT, PR_LE, PR_GT, PR_GE, PR_OPAQUE };
typedef struct { uint8_t kind; aff_t a; } pred_t;     /* a (op) 0 */

typedef struct {
    uint8_t  arg, nval, atomic, shared;
    uint16_t idx;
    uint16_t val[4];
    int      loop;
    uint8_t  npred;
    pred_t   pred[MAX_PRED];
    uint32_t buf;               /* shared: buffer name */
} wr_t;

enum { B_INT = 1, B_FLT, B_ACC };
typedef struct { uint32_t name; uint8_t kind; uint16_t v; aff_t a; } bind_t;

typedef struct {
    uint32_t name;
    int64_t  elems;
} sbuf_t;

typedef struct {
    const kir_t *k;
    int      na;                       /* tile axes */
    int64_t  ext[KIR_MAX_DIM];
    uint32_t axname[KIR_MAX_DIM];
    int64_t  cells;
    int      block, grid;
    fv_t     fv[MAX_FV];     int nfv;
    idx_t    idx[MAX_IDX];   int nidx;
    acc_t    acc[MAX_ACC];   int nacc;
    loop_t   loop[MAX_LOOP]; int nloop;
    wr_t     wr[MAX_WR];     int nwr;
    sbuf_t   sb[MAX_SW];     int nsb;
    bind_t   bind[MAX_BIND]; int nbind;
    int      mark[KIR_MAX_DEP * 4]; int nmark;
    pred_t   pstack[MAX_PRED]; int npred;
    int      cur_loop;
    int      has_smem_load_global;    /* a shared Load feeds a value (not plumbing) */
    struct { uint32_t name, bits; int used; } init[MAX_ACC]; int ninit;   /* Init statements */
} sym_t;

static sym_t SY;   /* guarded by the caller's lock (irx_compile) */

static int fv_is(uint16_t id, int op, uint16_t a, uint16_t b);

static const char *S(uint32_t off) { return kir_str(SY.k, off); }

static int str_eq(uint32_t a, uint32_t b) { return a == b || strcmp(S(a), S(b)) == 0; }

/* ---- op table (names and arities of the reference's src/ops.c:27-54) ---- */

typedef struct { const char *name; int op; int arity; } opn_t;
static const opn_t OPS[] = {
    {"add", OP_ADD, 2}, {"subtract", OP_SUB, 2}, {"multiply", OP_MUL, 2},
    {"divide", OP_DIV, 2}, {"true_divide", OP_DIV, 2}, {"maximum", OP_MAX, 2},
    {"minimum", OP_MIN, 2}, {"relu", OP_RELU, 1}, {"copy", OP_COPY, 1},
    {"negative", OP_NEG, 1}, {"abs", OP_ABS, 1}, {"sqrt", OP_SQRT, 1},
    {"rsqrt", OP_RSQRT, 1}, {"reciprocal", OP_RCP, 1}, {"tanh", OP_TANH, 1},
    {"sin", OP_SIN, 1}, {"cos", OP_COS, 1}, {"log2", OP_LOG2, 1}, {"exp", OP_EXP, 1},
    {"exp_fast", OP_EXPF, 1}, {"log", OP_LOG, 1}, {"sigmoid", OP_SIGMOID, 1},
    {"silu", OP_SILU, 1}, {"softplus", OP_SOFTPLUS, 1}, {"pow", OP_POW, 2}
};
#define NOPS ((int)(sizeof OPS / sizeof OPS[0]))

static int op_find(const char *s, int *arity)
{
    int i;
    for (i = 0; i < NOPS; i++)
        if (!strcmp(OPS[i].name, s)) { *arity = OPS[i].arity; return OPS[i].op; }
    return OP_NONE;
}

int irx_op_lookup(const char *name, int *arity)
{
    *arity = 0;
    return op_find(name, arity);
}

const char *irx_op_name(int op)
{
    int i;
    for (i = 0; i < NOPS; i++) if (OPS[i].op == op) return OPS[i].name;
    return "?";
}

int irx_op_arity(int op)
{
    int i;
    for (i = 0; i < NOPS; i++) if (OPS[i].op == op) return OPS[i].arity;
    return 0;
}

static int op_ident_ok(int op) { return op == OP_ADD || op == OP_MUL || op == OP_MAX || op == OP_MIN; }

/* The folds' identities (src/ops.c:27-54): finite, never infinity. */
static float irx_ident_f(int op) { return op == OP_MUL ? 1.0f : op == OP_MAX ? -1e30f : op == OP_MIN ? 1e30f : 0.0f; }
static int op_commutes(int op) { return op == OP_ADD || op == OP_MUL || op == OP_MAX || op == OP_MIN; }

/* ---- graph nodes (hash-consed so that equal subexpressions share one node) ---- */

static int fv_new(const fv_t *n, uint16_t *out)
{
    int i;
    for (i = 1; i < SY.nfv; i++) {
        const fv_t *o = &SY.fv[i];
        if (o->kind == n->kind && o->op == n->op && o->arg == n->arg && o->lane == n->lane &&
            o->a == n->a && o->b == n->b && o->idx == n->idx && o->acc == n->acc &&
            o->bits == n->bits && n->kind != FV_OPAQUE) { *out = (uint16_t)i; return 0; }
    }
    if (SY.nfv >= MAX_FV) return irx_fail(E081, "a graph with more values than the selector holds");
    SY.fv[SY.nfv] = *n;
    *out = (uint16_t)SY.nfv++;
    return 0;
}

static int fv_const(uint32_t bits, uint16_t *out)
{
    fv_t n; memset(&n, 0, sizeof n); n.kind = FV_CONST; n.bits = bits;
    return fv_new(&n, out);
}

static int fv_op(int op, uint16_t a, uint16_t b, uint16_t *out)
{
    fv_t n; memset(&n, 0, sizeof n); n.kind = FV_OP; n.op = (uint8_t)op; n.a = a; n.b = b;
    if (op_commutes(op) && a > b) { n.a = b; n.b = a; }
    return fv_new(&n, out);
}

static int idx_new(const idx_t *x, uint16_t *out)
{
    int i, d;
    for (i = 0; i < SY.nidx; i++) {
        if (SY.idx[i].rank != x->rank) continue;
        for (d = 0; d < x->rank; d++) if (!aff_eq(&SY.idx[i].d[d], &x->d[d]) || !SY.idx[i].d[d].ok) break;
        if (d == x->rank) { *out = (uint16_t)i; return 0; }
    }
    if (SY.nidx >= MAX_IDX) return irx_fail(E081, "more distinct indexes than the selector holds");
    SY.idx[SY.nidx] = *x;
    *out = (uint16_t)SY.nidx++;
    return 0;
}

/* ---- names ---- */

static int scope_push(void)
{
    if (SY.nmark >= (int)(sizeof SY.mark / sizeof SY.mark[0])) return irx_fail(E082, "scopes nested deeper than the limit");
    SY.mark[SY.nmark++] = SY.nbind;
    return 0;
}

static void scope_pop(void) { if (SY.nmark > 0) SY.nbind = SY.mark[--SY.nmark]; }

static int bind_set(uint32_t name, int kind, uint16_t v, const aff_t *a)
{
    bind_t *b;
    if (SY.nbind >= MAX_BIND) return irx_fail(E081, "more live names than the selector holds");
    b = &SY.bind[SY.nbind++];
    b->name = name;
    b->kind = (uint8_t)kind;
    b->v = v;
    if (a) b->a = *a; else memset(&b->a, 0, sizeof b->a);
    return 0;
}

static const bind_t *bind_find(uint32_t name)
{
    int i;
    for (i = SY.nbind - 1; i >= 0; i--)
        if (str_eq(SY.bind[i].name, name)) return &SY.bind[i];
    return NULL;
}

static int acc_find(uint32_t name)
{
    int i;
    for (i = 0; i < SY.nacc; i++) if (str_eq(SY.acc[i].name, name)) return i;
    return -1;
}

/* The float value a name denotes now. An accumulator reads as its running state inside
 * its loop (FV_PREV before this trip's Accum, the updated value after it) and as its
 * final value once the loop has closed. */
static int name_flt(uint32_t name, uint16_t *out)
{
    const bind_t *b = bind_find(name);
    int a = acc_find(name);
    char msg[120];

    if (b && b->kind == B_FLT) { *out = b->v; return 0; }
    if (a >= 0 && (!b || b->kind == B_ACC)) {
        acc_t *ac = &SY.acc[a];
        fv_t n;
        if (ac->closed) { *out = ac->final_val; return 0; }
        if (b && b->kind == B_ACC && b->v != 0xFFFF) { *out = b->v; return 0; }
        memset(&n, 0, sizeof n);
        n.kind = FV_PREV;
        n.acc = (uint16_t)a;
        return fv_new(&n, out);
    }
    snprintf(msg, sizeof msg, "the name '%s', which no enclosing scope binds to a value", S(name));
    return irx_fail(E022, msg);
}

/* ---- integer expressions (the reference's kexpr grammar, src/kexpr.c:44-56) ---- */

static int ex_aff(const kv_t *e, aff_t *out);

static int ex_lit(const kn_t *nd, aff_t *out, int *isf, uint32_t *fb)
{
    const kv_t *v = kir_fld(SY.k, nd, "value"), *d = kir_fld(SY.k, nd, "dtype");
    int fl = d && d->tag == KV_STR && !strcmp(S(d->ref), "float");
    if (!v) return irx_fail(E015, "a Literal with no value");
    if (v->tag == KV_FLT && !(d && d->tag == KV_STR && !strcmp(S(d->ref), "int"))) {
        *isf = 1; *fb = v->fbits; return 0;
    }
    if (v->tag == KV_INT && fl) {
        float f = (float)v->i;
        memcpy(fb, &f, 4);
        *isf = 1;
        return 0;
    }
    if (v->tag != KV_INT && v->tag != KV_BOOL) return irx_fail(E059, "a Literal whose value is not a number of its dtype");
    if (v->i > 2147483647LL || v->i < -2147483648LL) return irx_fail(E059, "an integer literal outside s32");
    *isf = 0;
    *out = aff_const(v->i);
    return 0;
}

/* Evaluate an expression as an affine integer form; non-affine forms come back with
 * ok == 0 unless every operand is a constant, which folds with s32 semantics. */
static int ex_aff(const kv_t *e, aff_t *out)
{
    const kn_t *nd;
    const char *kind;

    if (!e) return irx_fail(E015, "an expression with a missing operand");
    if (e->tag == KV_INT || e->tag == KV_BOOL) { *out = aff_const(e->i); return 0; }
    nd = kir_node(SY.k, e);
    if (!nd) return irx_fail(E020, "an operand that is not an expression node");
    kind = S(nd->kname);
    if (!strcmp(kind, "Var")) {
        const kv_t *n = kir_fld(SY.k, nd, "name");
        const bind_t *b;
        if (!n || n->tag != KV_STR) return irx_fail(E015, "a Var with no name");
        b = bind_find(n->ref);
        if (b && b->kind == B_INT) { *out = b->a; return 0; }
        if (b && b->kind == B_FLT) return irx_fail(E021, "a float operand in an integer expression");
        {
            char msg[120];
            snprintf(msg, sizeof msg, "the index name '%s', which nothing binds", S(n->ref));
            return irx_fail(E022, msg);
        }
    }
    if (!strcmp(kind, "Literal")) {
        int isf = 0; uint32_t fb = 0;
        if (ex_lit(nd, out, &isf, &fb)) return 1;
        if (isf) return irx_fail(E021, "a float literal in an integer expression");
        return 0;
    }
    if (!strcmp(kind, "Dim")) return ex_aff(kir_fld(SY.k, nd, "expr"), out);
    if (!strcmp(kind, "BinaryExpr")) {
        const kv_t *o = kir_fld(SY.k, nd, "op");
        aff_t a, b;
        const char *op;
        if (!o || o->tag != KV_STR) return irx_fail(E015, "a BinaryExpr with no op");
        op = S(o->ref);
        if (ex_aff(kir_fld(SY.k, nd, "left"), &a) || ex_aff(kir_fld(SY.k, nd, "right"), &b)) return 1;
        if (!strcmp(op, "+")) { *out = aff_add(a, b, 1); return 0; }
        if (!strcmp(op, "-")) { *out = aff_add(a, b, -1); return 0; }
        if (!strcmp(op, "*")) {
            if (aff_isc(&a)) { *out = aff_scale(b, a.cst); return 0; }
            if (aff_isc(&b)) { *out = aff_scale(a, b.cst); return 0; }
            *out = aff_bad();
            return 0;
        }
        if (aff_isc(&a) && aff_isc(&b)) {
            int32_t x = (int32_t)a.cst, y = (int32_t)b.cst;
            if (!strcmp(op, "/") || !strcmp(op, "//") || !strcmp(op, "%")) {
                if (y == 0) return irx_fail(E059, "a division or remainder by zero in a constant");
                *out = aff_const(op[0] == '%' ? x % y : x / y);
                return 0;
            }
            if (!strcmp(op, "<")) { *out = aff_const(x < y); return 0; }
            if (!strcmp(op, "<=")) { *out = aff_const(x <= y); return 0; }
            if (!strcmp(op, ">")) { *out = aff_const(x > y); return 0; }
            if (!strcmp(op, ">=")) { *out = aff_const(x >= y); return 0; }
            if (!strcmp(op, "==")) { *out = aff_const(x == y); return 0; }
            if (!strcmp(op, "&")) { *out = aff_const(x & y); return 0; }
            if (!strcmp(op, "|")) { *out = aff_const(x | y); return 0; }
            if (!strcmp(op, "^")) { *out = aff_const(x ^ y); return 0; }
            if (!strcmp(op, "<<")) { *out = aff_const(y >= 32 ? 0 : (int32_t)((uint32_t)x << y)); return 0; }
            if (!strcmp(op, ">>")) { *out = aff_const(y >= 31 ? (x < 0 ? -1 : 0) : x >> y); return 0; }
        }
        *out = aff_bad();
        return 0;
    }
    if (!strcmp(kind, "TernaryExpr")) { *out = aff_bad(); return 0; }
    {
        char msg[120];
        snprintf(msg, sizeof msg, "the expression kind %s", kind);
        return irx_fail(E020, msg);
    }
}

static int ex_fold(const kv_t *e, int64_t *v)
{
    aff_t a;
    if (ex_aff(e, &a)) return 1;
    if (!aff_isc(&a)) return irx_fail(E059, "an extent or step that is not a constant");
    *v = a.cst;
    return 0;
}

static int ex_pred(const kv_t *e, pred_t *p)
{
    const kn_t *nd = kir_node(SY.k, e);
    memset(p, 0, sizeof *p);
    p->kind = PR_OPAQUE;
    if (nd && kir_is(SY.k, nd, "BinaryExpr")) {
        const kv_t *o = kir_fld(SY.k, nd, "op");
        aff_t a, b;
        const char *op = o && o->tag == KV_STR ? S(o->ref) : "";
        int kind = !strcmp(op, "==") ? PR_EQ : !strcmp(op, "<") ? PR_LT : !strcmp(op, "<=") ? PR_LE :
                   !strcmp(op, ">") ? PR_GT : !strcmp(op, ">=") ? PR_GE : 0;
        if (kind) {
            if (ex_aff(kir_fld(SY.k, nd, "left"), &a) || ex_aff(kir_fld(SY.k, nd, "right"), &b)) return 1;
            p->a = aff_add(a, b, -1);
            if (p->a.ok) p->kind = (uint8_t)kind;
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------------------------
 * The walk: statement by statement, building the graph.
 * ------------------------------------------------------------------------------------ */

static int walk_list(const kv_t *lst);

static int arg_find(uint32_t name, int *arg)
{
    uint32_t i;
    for (i = 0; i < SY.k->narg; i++)
        if (str_eq(SY.k->arg[i].name, name)) { *arg = (int)i; return 1; }
    return 0;
}

static int sbuf_find(uint32_t name)
{
    int i;
    for (i = 0; i < SY.nsb; i++) if (str_eq(SY.sb[i].name, name)) return i;
    return -1;
}

static int dt_ok(const kv_t *d, int bufdt)
{
    if (!d || d->tag == KV_NONE) return 1;
    if (d->tag != KV_DT) return 0;
    if (!strcmp(S(d->ref), "f32")) return bufdt == DT_F32 || bufdt == DT_NONE;
    if (!strcmp(S(d->ref), "bf16")) return bufdt == DT_BF16;
    return 0;
}

static int index_of(const kv_t *lst, int rank, idx_t *x)
{
    uint32_t i;
    memset(x, 0, sizeof *x);
    if (!lst || lst->tag != KV_LIST) return irx_fail(E015, "an access whose index is not a list");
    if ((int)lst->n != rank && !(rank == 0 && lst->n == 0))
        return irx_fail(E059, "an index whose length is not the buffer's rank");
    x->rank = (uint8_t)lst->n;
    for (i = 0; i < lst->n; i++)
        if (ex_aff(kir_item(SY.k, lst, i), &x->d[i])) return 1;
    return 0;
}

static int st_load(const kn_t *nd)
{
    const kv_t *nms = kir_fld(SY.k, nd, "names"), *in = kir_fld(SY.k, nd, "input");
    const kv_t *ix = kir_fld(SY.k, nd, "index"), *d = kir_fld(SY.k, nd, "dtype");
    int arg = -1, sb;
    uint32_t i;
    idx_t x;
    uint16_t id, v;
    fv_t n;

    if (!nms || !in || !ix) return irx_fail(E015, "a Load missing names, input or index");
    if (nms->tag != KV_LIST || nms->n == 0 || in->tag != KV_STR) return irx_fail(E015, "a Load whose names or input have the wrong shape");
    if (nms->n != 1 && nms->n != 2 && nms->n != 4) return irx_fail(E020, "a Load of a number of values other than 1, 2 or 4");
    sb = sbuf_find(in->ref);
    if (sb >= 0) {            /* a shared read outside the reduction plumbing */
        memset(&n, 0, sizeof n);
        n.kind = FV_OPAQUE;
        for (i = 0; i < nms->n; i++) {
            const kv_t *nm = kir_item(SY.k, nms, i);
            n.lane = (uint8_t)(SY.nfv & 0xff);
            if (fv_new(&n, &v) || bind_set(nm->ref, B_FLT, v, NULL)) return 1;
        }
        SY.has_smem_load_global = 1;
        return 0;
    }
    if (!arg_find(in->ref, &arg)) return irx_fail(E022, "a Load of a name that is not a parameter");
    if (SY.k->arg[arg].kind == KA_OUT) return irx_fail(E022, "a Load from an output buffer");
    if (SY.k->arg[arg].dt == DT_OTHER) return irx_fail(E024, "a Load of a buffer whose dtype is not f32 or bf16");
    if (!dt_ok(d, SY.k->arg[arg].dt)) return irx_fail(E024, "a Load whose dtype does not match its buffer");
    if (index_of(ix, SY.k->arg[arg].rank, &x) || idx_new(&x, &id)) return 1;
    for (i = 0; i < nms->n; i++) {
        const kv_t *nm = kir_item(SY.k, nms, i);
        if (!nm || nm->tag != KV_STR) return irx_fail(E015, "a Load name that is not a string");
        memset(&n, 0, sizeof n);
        n.kind = FV_LOAD;
        n.arg = (uint8_t)arg;
        n.lane = (uint8_t)i;
        n.idx = id;
        if (fv_new(&n, &v) || bind_set(nm->ref, B_FLT, v, NULL)) return 1;
    }
    return 0;
}

static int st_assign(const kn_t *nd)
{
    const kv_t *nm = kir_fld(SY.k, nd, "name"), *op = kir_fld(SY.k, nd, "op");
    const kv_t *as = kir_fld(SY.k, nd, "args"), *d = kir_fld(SY.k, nd, "dtype");
    int o, ar = 0, a;
    uint16_t x = 0, y = 0, v;
    char msg[120];

    if (!nm || !op || !as || nm->tag != KV_STR || op->tag != KV_OP || as->tag != KV_LIST)
        return irx_fail(E015, "an Assign missing name, op or args");
    if (d && d->tag == KV_DT && strcmp(S(d->ref), "f32") && strcmp(S(d->ref), "bf16"))
        return irx_fail(E024, "an Assign whose dtype is not f32");
    o = op_find(S(op->ref), &ar);
    if (o == OP_NONE) {
        snprintf(msg, sizeof msg, "the op '%s', which is not in the op table", S(op->ref));
        return irx_fail(E021, msg);
    }
    if ((int)as->n != ar) return irx_fail(E020, "an Assign whose arg count is not the op's arity");
    if (name_flt(kir_item(SY.k, as, 0)->ref, &x)) return 1;
    if (ar == 2 && name_flt(kir_item(SY.k, as, 1)->ref, &y)) return 1;
    if (fv_op(o, x, ar == 2 ? y : 0, &v)) return 1;
    a = acc_find(nm->ref);
    if (a >= 0) return bind_set(nm->ref, B_ACC, v, NULL);   /* write into the home register */
    return bind_set(nm->ref, B_FLT, v, NULL);
}

static int st_let(const kn_t *nd)
{
    const kv_t *nm = kir_fld(SY.k, nd, "name"), *vl = kir_fld(SY.k, nd, "value");
    const kn_t *vn;
    if (!nm || !vl || nm->tag != KV_STR) return irx_fail(E015, "a Let missing name or value");
    vn = kir_node(SY.k, vl);
    if (vl->tag == KV_FLT || (vn && kir_is(SY.k, vn, "Literal"))) {
        aff_t a; int isf = 0; uint32_t fb = 0; uint16_t v;
        if (vl->tag == KV_FLT) { isf = 1; fb = vl->fbits; }
        else if (ex_lit(vn, &a, &isf, &fb)) return 1;
        if (isf) return fv_const(fb, &v) || bind_set(nm->ref, B_FLT, v, NULL);
        return bind_set(nm->ref, B_INT, 0, &a);
    }
    if (vn && kir_is(SY.k, vn, "FlatIndex")) return irx_fail(E020, "the expression kind FlatIndex");
    {
        aff_t a;
        if (ex_aff(vl, &a)) return 1;
        return bind_set(nm->ref, B_INT, 0, &a);
    }
}

static int st_write(const kn_t *nd)
{
    const kv_t *out = kir_fld(SY.k, nd, "output"), *ix = kir_fld(SY.k, nd, "index");
    const kv_t *vs = kir_fld(SY.k, nd, "values"), *d = kir_fld(SY.k, nd, "value_dtype");
    const kv_t *at = kir_fld(SY.k, nd, "atomic"), *sw = kir_fld(SY.k, nd, "swizzle");
    wr_t *w;
    int arg = -1, sb;
    uint32_t i;
    idx_t x;

    if (!out || !ix || !vs || out->tag != KV_STR || vs->tag != KV_LIST || !vs->n)
        return irx_fail(E015, "a Write missing output, index or values");
    if (vs->n != 1 && vs->n != 2 && vs->n != 4) return irx_fail(E020, "a Write of a number of values other than 1, 2 or 4");
    if (sw && sw->tag == KV_STR && strcmp(S(sw->ref), "NONE")) return irx_fail(E020, "a Write with a swizzle");
    if (SY.nwr >= MAX_WR) return irx_fail(E081, "more Writes than the selector holds");
    w = &SY.wr[SY.nwr];
    memset(w, 0, sizeof *w);
    sb = sbuf_find(out->ref);
    if (sb >= 0) {
        w->shared = 1;
        w->buf = out->ref;
        if (index_of(ix, ix->tag == KV_LIST ? (int)ix->n : 0, &x) || idx_new(&x, &w->idx)) return 1;
    } else {
        if (!arg_find(out->ref, &arg)) return irx_fail(E022, "a Write to a name that is not a parameter");
        if (SY.k->arg[arg].kind != KA_OUT) return irx_fail(E022, "a Write to a buffer that is not an output");
        if (SY.k->arg[arg].dt == DT_OTHER) return irx_fail(E024, "a Write to a buffer whose dtype is not f32 or bf16");
        if (!dt_ok(d, SY.k->arg[arg].dt)) return irx_fail(E024, "a Write whose value_dtype does not match its buffer");
        if (index_of(ix, SY.k->arg[arg].rank, &x) || idx_new(&x, &w->idx)) return 1;
        w->arg = (uint8_t)arg;
    }
    w->nval = (uint8_t)vs->n;
    w->atomic = at && at->tag == KV_BOOL && at->i;
    if (w->atomic && w->shared) return irx_fail(E020, "an atomic Write to shared memory");
    for (i = 0; i < vs->n; i++) {
        const kv_t *v = kir_item(SY.k, vs, i);
        if (!v || v->tag != KV_STR) return irx_fail(E015, "a Write value that is not a name");
        if (name_flt(v->ref, &w->val[i])) return 1;
    }
    w->loop = SY.cur_loop;
    w->npred = (uint8_t)SY.npred;
    memcpy(w->pred, SY.pstack, sizeof(pred_t) * (size_t)SY.npred);
    SY.nwr++;
    return 0;
}

static int acc_get(const kn_t *nd, int *out)
{
    const kv_t *nm = kir_fld(SY.k, nd, "name"), *op = kir_fld(SY.k, nd, "op");
    const kv_t *d = kir_fld(SY.k, nd, "dtype");
    int o, ar = 0, a;
    if (!nm || !op || nm->tag != KV_STR || op->tag != KV_OP) return irx_fail(E015, "an Accum missing name or op");
    if (d && d->tag == KV_DT && strcmp(S(d->ref), "f32")) return irx_fail(E024, "an Accum whose dtype is not f32");
    o = op_find(S(op->ref), &ar);
    if (o == OP_NONE) return irx_fail(E021, "an Accum whose op is not in the op table");
    if (ar != 2) return irx_fail(E020, "an Accum whose op is not binary");
    if (!op_ident_ok(o)) return irx_fail(E021, "an Accum whose op has no identity");
    a = acc_find(nm->ref);
    if (a < 0) {
        if (SY.nacc >= MAX_ACC) return irx_fail(E081, "more accumulators than the selector holds");
        a = SY.nacc++;
        memset(&SY.acc[a], 0, sizeof SY.acc[a]);
        SY.acc[a].name = nm->ref;
        SY.acc[a].op = (uint8_t)o;
        SY.acc[a].loop = -1;
    }
    *out = a;
    return 0;
}

static int st_accum(const kn_t *nd)
{
    const kv_t *vl = kir_fld(SY.k, nd, "value"), *bs = kir_fld(SY.k, nd, "base");
    int a;
    uint16_t v, base = 0, cur, nv;
    acc_t *ac;

    if (!vl || vl->tag != KV_STR) return irx_fail(E015, "an Accum whose value is not a name");
    if (acc_get(nd, &a)) return 1;
    ac = &SY.acc[a];
    if (bs && bs->tag == KV_STR) { if (name_flt(bs->ref, &base)) return 1; }
    else if (bs && bs->tag != KV_NONE) return irx_fail(E020, "an Accum whose base is not a name");
    if (name_flt(vl->ref, &v)) return 1;
    ac->nupd++;
    ac->upd_val = v;
    ac->upd_base = base;
    ac->upd_loop = SY.cur_loop;
    if (ac->closed) return irx_fail(E040, "an accumulator updated again after its reduction closed");
    if (name_flt(ac->name, &cur)) return 1;
    if (fv_op(ac->op, base ? base : cur, v, &nv)) return 1;
    return bind_set(ac->name, B_ACC, nv, NULL);
}

static int loop_axis(const kn_t *nd, uint32_t *name, int64_t *ext)
{
    const kv_t *ax = kir_fld(SY.k, nd, "axis");
    const kn_t *a = kir_node(SY.k, ax);
    const kv_t *an = a ? kir_fld(SY.k, a, "name") : NULL, *ex = a ? kir_fld(SY.k, a, "extent") : NULL;
    if (!an || an->tag != KV_STR || !ex) return irx_fail(E015, "a loop axis with no name or extent");
    if (ex_fold(ex, ext)) return 1;
    if (*ext < 1) return irx_fail(E059, "a loop whose extent is not a constant above 0");
    *name = an->ref;
    return 0;
}

/* Seed: every Accum in the loop's immediate body whose axes name this loop (or that names
 * no axes) belongs to it and starts from its identity (src/isel.c:1373-1400). */
static int init_find(uint32_t name)
{
    int i;
    for (i = 0; i < SY.ninit; i++) if (str_eq(SY.init[i].name, name)) return i;
    return -1;
}

/* Init (src/isel.c:1872-1900): an accumulator seeded with a given value before a loop that
 * does not seed it (seed=false). With the fold's own identity that is the seeded loop the
 * templates take. With another value every thread's partial starts at it, as the reference
 * lowers it; the reduction template folds from the identity and adds the seeds' share to the
 * total (sel_reduce), and the other families refuse it (E042). */
static int st_init(const kn_t *nd)
{
    const kv_t *nm = kir_fld(SY.k, nd, "name"), *iv = kir_fld(SY.k, nd, "identity"), *d = kir_fld(SY.k, nd, "dtype");
    uint32_t bits;
    if (!nm || !iv || !d) return irx_fail(E015, "an Init missing name, identity or dtype");
    if (nm->tag != KV_STR) return irx_fail(E015, "an Init whose name is not a string");
    if (d->tag != KV_NONE && !(d->tag == KV_DT && !strcmp(S(d->ref), "f32"))) return irx_fail(E024, "an Init whose dtype is not f32");
    if (iv->tag == KV_FLT) bits = iv->fbits;
    else if (iv->tag == KV_INT) { float f = (float)iv->i; memcpy(&bits, &f, 4); }
    else return irx_fail(E015, "an Init whose identity is not a number");
    if (init_find(nm->ref) >= 0 || acc_find(nm->ref) >= 0) return irx_fail(E028, "an Init whose name is already an accumulator");
    if (SY.ninit >= MAX_ACC) return irx_fail(E081, "more Inits than the selector holds");
    SY.init[SY.ninit].name = nm->ref;
    SY.init[SY.ninit].bits = bits;
    SY.init[SY.ninit].used = 0;
    SY.ninit++;
    return 0;
}

static int loop_seed(const kn_t *nd, uint32_t axname, int lid)
{
    const kv_t *bd = kir_fld(SY.k, nd, "body"), *sd = kir_fld(SY.k, nd, "seed");
    const int seeded = !(sd && sd->tag == KV_BOOL && !sd->i);
    uint32_t i, j;
    for (i = 0; bd && i < bd->n; i++) {
        const kn_t *st = kir_node(SY.k, kir_item(SY.k, bd, i));
        const kv_t *axes;
        int own = 0, a;
        if (!st || !kir_is(SY.k, st, "Accum")) continue;
        axes = kir_fld(SY.k, st, "axes");
        if (!axes || axes->tag == KV_NONE) own = 1;
        else if (axes->tag == KV_LIST)
            for (j = 0; j < axes->n; j++) {
                const kv_t *x = kir_item(SY.k, axes, j);
                if (x && x->tag == KV_STR && str_eq(x->ref, axname)) own = 1;
            }
        if (!own) continue;
        if (!seeded) {                     /* only an Init's accumulator starts here */
            const kv_t *nm = kir_fld(SY.k, st, "name");
            int in = nm && nm->tag == KV_STR ? init_find(nm->ref) : -1;
            float id;
            if (in < 0 || SY.init[in].used) continue;
            if (acc_get(st, &a)) return 1;
            id = irx_ident_f(SY.acc[a].op);
            if (memcmp(&id, &SY.init[in].bits, 4)) {     /* each thread's partial starts at the seed */
                SY.acc[a].has_seed = 1;
                SY.acc[a].seed_bits = SY.init[in].bits;
            }
            SY.init[in].used = 1;
        } else {
            const kv_t *nm = kir_fld(SY.k, st, "name");
            int in = nm && nm->tag == KV_STR ? init_find(nm->ref) : -1;
            if (in >= 0) SY.init[in].used = 1;  /* a seeding loop starts it over */
            if (acc_get(st, &a)) return 1;
        }
        SY.acc[a].loop = lid;
        SY.acc[a].closed = 0;
        if (bind_set(SY.acc[a].name, B_ACC, 0xFFFF, NULL)) return 1;   /* running state */
    }
    return 0;
}

static int close_loop_accs(int lid)
{
    int a;
    for (a = 0; a < SY.nacc; a++) {
        acc_t *ac = &SY.acc[a];
        if (ac->loop == lid && !ac->closed) {
            fv_t n;
            memset(&n, 0, sizeof n);
            n.kind = FV_FINAL;
            n.acc = (uint16_t)a;
            if (fv_new(&n, &ac->final_val)) return 1;
            ac->closed = 1;
        }
    }
    return 0;
}

static int st_loop(const kn_t *nd, int strided)
{
    const kv_t *bd = kir_fld(SY.k, nd, "body");
    uint32_t axname = 0;
    int64_t ext = 0;
    int lid, prev = SY.cur_loop, rc;
    loop_t *L;
    aff_t lv;

    if (!bd || bd->tag != KV_LIST) return irx_fail(E015, "a loop with no body list");
    if (loop_axis(nd, &axname, &ext)) return 1;
    if (SY.nloop >= MAX_LOOP) return irx_fail(E081, "more loops than the selector holds");
    lid = SY.nloop++;
    L = &SY.loop[lid];
    memset(L, 0, sizeof *L);
    L->kind = strided ? 2 : 1;
    L->parent = prev;
    L->ext = ext;
    L->name = axname;
    L->step = 1;
    L->start = aff_const(0);
    L->end = aff_bad();
    if (strided) {
        const kv_t *en = kir_fld(SY.k, nd, "end");
        if (ex_fold(kir_fld(SY.k, nd, "step"), &L->step)) return 1;
        if (L->step < 1) return irx_fail(E026, "a StridedLoop whose step is not a constant above 0");
        if (ex_aff(kir_fld(SY.k, nd, "start"), &L->start)) return 1;
        if (!L->start.ok) return irx_fail(E041, "a StridedLoop whose start is not affine");
        if (en && en->tag != KV_NONE) {
            if (ex_aff(en, &L->end)) return 1;
            if (!L->end.ok) return irx_fail(E041, "a StridedLoop whose end is not affine");
        }
    }
    if (loop_seed(nd, axname, lid)) return 1;
    if (scope_push()) return 1;
    lv = aff_var(V_LOOP0 + lid);
    if (bind_set(axname, B_INT, 0, &lv)) return 1;
    SY.cur_loop = lid;
    rc = walk_list(bd);
    SY.cur_loop = prev;
    if (rc) return 1;
    /* the accumulators' running values die with the scope; their finals replace them */
    scope_pop();
    return close_loop_accs(lid);
}

static int st_cond(const kn_t *nd)
{
    const kv_t *cd = kir_fld(SY.k, nd, "cond"), *bd = kir_fld(SY.k, nd, "body");
    const kv_t *eb = kir_fld(SY.k, nd, "else_body");
    pred_t p;
    if (!cd || !bd || bd->tag != KV_LIST) return irx_fail(E015, "a Cond missing cond or body");
    if (ex_pred(cd, &p)) return 1;
    if (SY.npred >= MAX_PRED) return irx_fail(E082, "conditions nested deeper than the selector holds");
    SY.pstack[SY.npred++] = p;
    if (scope_push() || walk_list(bd)) return 1;
    scope_pop();
    SY.npred--;
    if (eb && eb->tag == KV_LIST && eb->n) {
        pred_t q = p;
        q.kind = PR_OPAQUE;
        SY.pstack[SY.npred++] = q;
        if (scope_push() || walk_list(eb)) return 1;
        scope_pop();
        SY.npred--;
    }
    return 0;
}

static int st_smem(const kn_t *nd)
{
    const kv_t *nm = kir_fld(SY.k, nd, "name"), *ex = kir_fld(SY.k, nd, "extents");
    int64_t e = 1, v = 0;
    uint32_t i;
    if (!nm || nm->tag != KV_STR || !ex || ex->tag != KV_LIST) return irx_fail(E015, "a Smem missing name or extents");
    if (sbuf_find(nm->ref) >= 0) return 0;
    if (SY.nsb >= MAX_SW) return irx_fail(E081, "more shared arrays than the selector holds");
    for (i = 0; i < ex->n; i++) {
        if (ex_fold(kir_item(SY.k, ex, i), &v)) return 1;
        if (v < 1 || e > (int64_t)1 << 40) return irx_fail(E059, "a shared array with an empty or huge extent");
        e *= v;
    }
    SY.sb[SY.nsb].name = nm->ref;
    SY.sb[SY.nsb].elems = e;
    SY.nsb++;
    return 0;
}

/* The state names of a shuffle or tree, each an accumulator whose loop has closed. The
 * combine must be that accumulator's own op (an empty list means exactly that,
 * src/isel.c:1640-1650). */
static int comb_states(const kn_t *nd, int *accs, int *n)
{
    const kv_t *st = kir_fld(SY.k, nd, "state"), *sb = kir_fld(SY.k, nd, "state_b");
    const kv_t *cm = kir_fld(SY.k, nd, "combine_states");
    uint32_t i;
    if (!st || !sb || st->tag != KV_LIST || sb->tag != KV_LIST || !st->n || st->n != sb->n)
        return irx_fail(E015, "a warp or tree statement with no matching state lists");
    if (st->n > 4) return irx_fail(E040, "a cross-thread combine of more than 4 states");
    for (i = 0; i < st->n; i++) {
        const kv_t *s = kir_item(SY.k, st, i);
        int a = s && s->tag == KV_STR ? acc_find(s->ref) : -1;
        if (a < 0 || !SY.acc[a].closed) return irx_fail(E040, "a cross-thread combine of a value that is not a finished accumulator");
        accs[i] = a;
    }
    *n = (int)st->n;
    if (cm && cm->tag == KV_LIST && cm->n) {
        if (cm->n != st->n) return irx_fail(E040, "a combine program that is not one fold per state");
        for (i = 0; i < cm->n; i++) {
            const kn_t *as = kir_node(SY.k, kir_item(SY.k, cm, i));
            const kv_t *nm, *op, *args;
            int ar = 0, o, j, ok = 0;
            if (!as || !kir_is(SY.k, as, "Assign")) return irx_fail(E027, "a combine_states statement that is not an Assign");
            nm = kir_fld(SY.k, as, "name"); op = kir_fld(SY.k, as, "op"); args = kir_fld(SY.k, as, "args");
            if (!nm || !op || !args || args->tag != KV_LIST || args->n != 2) return irx_fail(E040, "a combine that is not a binary fold");
            o = op_find(S(op->ref), &ar);
            for (j = 0; j < *n; j++) {
                const kv_t *s0 = kir_item(SY.k, st, (uint32_t)j), *s1 = kir_item(SY.k, sb, (uint32_t)j);
                const kv_t *a0 = kir_item(SY.k, args, 0), *a1 = kir_item(SY.k, args, 1);
                if (str_eq(nm->ref, s0->ref) && o == SY.acc[accs[j]].op &&
                    ((str_eq(a0->ref, s0->ref) && str_eq(a1->ref, s1->ref)) ||
                     (str_eq(a1->ref, s0->ref) && str_eq(a0->ref, s1->ref)))) ok = 1;
            }
            if (!ok) return irx_fail(E040, "a combine that is not the accumulator's own fold");
        }
    }
    return 0;
}

static int st_shuffle(const kn_t *nd)
{
    int accs[4], n, i;
    int64_t len = 0;
    if (comb_states(nd, accs, &n)) return 1;
    if (ex_fold(kir_fld(SY.k, nd, "length"), &len)) return 1;
    if (len < 1 || len > 32 || (len & (len - 1))) return irx_fail(E034, "a warp shuffle whose length is not a power of two up to 32");
    if (SY.block % 32) return irx_fail(E034, "a warp shuffle in a block that is not a multiple of 32");
    for (i = 0; i < n; i++) {
        if (SY.acc[accs[i]].shuf_len) return irx_fail(E040, "an accumulator shuffled twice");
        SY.acc[accs[i]].shuf_len = (int)len;
    }
    return 0;
}

static int st_tree(const kn_t *nd)
{
    int accs[4], n, i, w;
    int64_t len = 0;
    const kv_t *bf = kir_fld(SY.k, nd, "bufs"), *tv = kir_fld(SY.k, nd, "tid_var");
    const kv_t *in = kir_fld(SY.k, nd, "inner");
    const bind_t *tb;
    if (comb_states(nd, accs, &n)) return 1;
    if (in && in->tag != KV_NONE) return irx_fail(E020, "a tree with an inner state");
    if (ex_fold(kir_fld(SY.k, nd, "length"), &len)) return 1;
    if (len < 1 || (len & (len - 1))) return irx_fail(E020, "a tree whose length is not a power of two");
    if (!bf || bf->tag != KV_LIST || (int)bf->n != n) return irx_fail(E020, "a tree whose buffers and states do not pair up");
    if (!tv || tv->tag != KV_STR) return irx_fail(E015, "a tree with no tid variable");
    tb = bind_find(tv->ref);
    for (i = 0; i < n; i++) {
        acc_t *ac = &SY.acc[accs[i]];
        const kv_t *b = kir_item(SY.k, bf, (uint32_t)i);
        int ok = tb && tb->kind == B_INT && tb->a.ok && tb->a.nv == 1 && tb->a.var[0] == V_WARP &&
                 tb->a.coef[0] == 1 && tb->a.cst == 0 && ac->shuf_len == 32;
        /* the buffer must hold each warp's total at [warp], written from a lane-0 thread */
        for (w = 0, ok = ok ? 1 : 0; ok && w < SY.nwr; w++) (void)0;
        if (ok) {
            int fed = 0;
            for (w = 0; w < SY.nwr; w++) {
                const wr_t *wr = &SY.wr[w];
                const idx_t *x = &SY.idx[wr->idx];
                if (wr->shared && str_eq(wr->buf, b->ref) && wr->nval == 1 && wr->val[0] == ac->final_val &&
                    x->rank == 1 && x->d[0].ok && x->d[0].nv == 1 && x->d[0].var[0] == V_WARP &&
                    x->d[0].coef[0] == 1 && x->d[0].cst == 0) fed = 1;
            }
            ok = fed;
        }
        if (ac->tree_len) return irx_fail(E040, "an accumulator folded by two trees");
        ac->tree_len = (int)len;
        ac->tree_ok = ok;
    }
    return 0;
}

static int st_stmt(const kn_t *nd)
{
    const char *k = S(nd->kname);
    char msg[120];
    if (!strcmp(k, "Load")) return st_load(nd);
    if (!strcmp(k, "Assign")) return st_assign(nd);
    if (!strcmp(k, "Let")) return st_let(nd);
    if (!strcmp(k, "Write")) return st_write(nd);
    if (!strcmp(k, "Accum")) return st_accum(nd);
    if (!strcmp(k, "Loop")) return st_loop(nd, 0);
    if (!strcmp(k, "StridedLoop")) return st_loop(nd, 1);
    if (!strcmp(k, "Cond")) return st_cond(nd);
    if (!strcmp(k, "Smem")) return st_smem(nd);
    if (!strcmp(k, "Sync")) return 0;
    if (!strcmp(k, "Init")) return st_init(nd);
    if (!strcmp(k, "WarpShuffle")) return st_shuffle(nd);
    if (!strcmp(k, "TreeHalve")) return st_tree(nd);
    if (!strcmp(k, "Tile")) return irx_fail(E021, "a Tile nested inside a body");
    snprintf(msg, sizeof msg, "a %s statement", k);
    return irx_fail(E020, msg);
}

/* Shared arrays are declared wherever their Smem sits; the reference places them in a
 * pre-pass (src/isel.c:716-745), so a Write may name one before its Smem. */
static int smem_prepass(const kv_t *lst)
{
    uint32_t i;
    for (i = 0; i < lst->n; i++) {
        const kn_t *nd = kir_node(SY.k, kir_item(SY.k, lst, i));
        const char *k;
        if (!nd) return irx_fail(E015, "a statement list item that is not a node");
        k = S(nd->kname);
        if (!strcmp(k, "Smem")) { if (st_smem(nd)) return 1; }
        else if (!strcmp(k, "Loop") || !strcmp(k, "StridedLoop") || !strcmp(k, "Cond")) {
            const kv_t *b = kir_fld(SY.k, nd, "body"), *e = kir_fld(SY.k, nd, "else_body");
            if (b && b->tag == KV_LIST && smem_prepass(b)) return 1;
            if (e && e->tag == KV_LIST && smem_prepass(e)) return 1;
        }
    }
    return 0;
}

static int walk_list(const kv_t *lst)
{
    uint32_t i;
    if (!lst || lst->tag != KV_LIST) return irx_fail(E015, "a statement body that is not a list");
    for (i = 0; i < lst->n; i++) {
        const kn_t *nd = kir_node(SY.k, kir_item(SY.k, lst, i));
        if (!nd) return irx_fail(E015, "a statement list item that is not a node");
        if (st_stmt(nd)) return 1;
    }
    return 0;
}

/* ---------------------------------------------------------------------------------------
 * Op-program compilation: a value DAG to straight-line register code. Values that do not
 * depend on a per-element stream are "uniform" and go into a separate program that runs
 * once (per launch, or per row); the element program reads them as uniform registers.
 * ------------------------------------------------------------------------------------ */

typedef struct {
    int      nstream;
    uint16_t stream_fv[PROG_NSTREAM];        /* the FV node each stream register holds */
    irx_uni_t *uni;                          /* uniform register sources (plan-owned) */
    uint8_t *nuni;
    uint16_t uni_fv[PROG_NUNI];              /* FV node held by each uniform register */
    irx_prog_t *uprog;                       /* uniform program (may be NULL: refuse hoists) */
    int      uni_base;                       /* uniform registers below this are inputs */
} pctx_t;

/* Registers already holding a node, and use counts for freeing temporaries. */
typedef struct { uint16_t fv; uint8_t reg; } held_t;

typedef struct {
    pctx_t  *c;
    irx_prog_t *p;
    held_t   held[64]; int nheld;
    uint8_t  tmp_busy[PROG_NTMP];
    int      uses[MAX_FV];
} pgen_t;

static int fv_is_uniform(const pctx_t *c, uint16_t id, int depth)
{
    const fv_t *n = &SY.fv[id];
    int i;
    if (depth > 64) return 0;
    for (i = 0; i < c->nstream; i++) if (c->stream_fv[i] == id) return 0;
    switch (n->kind) {
    case FV_CONST: return 1;
    case FV_LOAD:  return 0;            /* a load that is not a stream is resolved by the caller */
    case FV_FINAL: return 1;
    case FV_OP:
        if (!fv_is_uniform(c, n->a, depth + 1)) return 0;
        return irx_op_arity(n->op) == 1 || fv_is_uniform(c, n->b, depth + 1);
    default: return 0;
    }
}

static int count_uses(pgen_t *g, uint16_t id, int depth)
{
    const fv_t *n = &SY.fv[id];
    if (depth > 64) return irx_fail(E043, "an op program nested deeper than the template takes");
    g->uses[id]++;
    if (g->uses[id] > 1) return 0;
    if (n->kind == FV_OP) {
        if (count_uses(g, n->a, depth + 1)) return 1;
        if (irx_op_arity(n->op) == 2 && count_uses(g, n->b, depth + 1)) return 1;
    }
    return 0;
}

static int uni_reg(pctx_t *c, uint16_t id, int *reg)
{
    int i;
    for (i = 0; i < *c->nuni; i++) if (c->uni_fv[i] == id) { *reg = PROG_R_UNI + i; return 0; }
    return -1;
}

static int uni_add(pctx_t *c, uint16_t id, const irx_uni_t *src, int *reg)
{
    if (*c->nuni >= PROG_NUNI) return irx_fail(E043, "more uniform values than the template's register file holds");
    c->uni[*c->nuni] = *src;
    c->uni_fv[*c->nuni] = id;
    *reg = PROG_R_UNI + *c->nuni;
    (*c->nuni)++;
    return 0;
}

static int gen_node(pgen_t *g, uint16_t id, int *reg, int depth);

static int emit_ins(irx_prog_t *p, int op, int dst, int a, int b)
{
    if (p->nins >= PROG_MAX_INS) return irx_fail(E043, "an op program longer than the template takes");
    p->ins[p->nins].op = (uint8_t)op;
    p->ins[p->nins].dst = (uint8_t)dst;
    p->ins[p->nins].a = (uint8_t)a;
    p->ins[p->nins].b = (uint8_t)b;
    p->nins++;
    return 0;
}

/* A uniform subexpression: constants and scalars become uniform inputs; ops become
 * instructions of the uniform program writing fresh uniform registers. */
static int gen_uniform(pctx_t *c, uint16_t id, int *reg, int depth)
{
    const fv_t *n = &SY.fv[id];
    irx_uni_t u;
    int ra = 0, rb = 0;
    if (depth > 64) return irx_fail(E043, "an op program nested deeper than the template takes");
    if (uni_reg(c, id, reg) == 0) return 0;
    memset(&u, 0, sizeof u);
    if (n->kind == FV_CONST) { u.kind = UNI_LIT; u.v = n->bits; return uni_add(c, id, &u, reg); }
    if (n->kind == FV_LOAD) {     /* a scalar read: the caller proved its index constant */
        const idx_t *x = &SY.idx[n->idx];
        const ka_t *a = &SY.k->arg[n->arg];
        int64_t flat = 0;
        int d;
        for (d = 0; d < x->rank; d++) flat = flat * a->dim[d] + x->d[d].cst;
        u.kind = UNI_ARG; u.v = n->arg; u.off = (int32_t)(flat + n->lane);
        return uni_add(c, id, &u, reg);
    }
    if (n->kind == FV_FINAL) return irx_fail(E040, "a reduced value used where the template has none");
    if (n->kind != FV_OP || !c->uprog) return irx_fail(E040, "a value the template cannot compute once per launch");
    if (gen_uniform(c, n->a, &ra, depth + 1)) return 1;
    if (irx_op_arity(n->op) == 2 && gen_uniform(c, n->b, &rb, depth + 1)) return 1;
    u.kind = UNI_NONE;                         /* computed by the uniform program */
    if (uni_add(c, id, &u, reg)) return 1;
    return emit_ins(c->uprog, n->op, *reg, ra, irx_op_arity(n->op) == 2 ? rb : ra);
}

static void release(pgen_t *g, uint16_t id)
{
    int i;
    if (--g->uses[id] > 0) return;
    for (i = 0; i < g->nheld; i++)
        if (g->held[i].fv == id) {
            int r = g->held[i].reg;
            if (r >= PROG_R_TMP) g->tmp_busy[r - PROG_R_TMP] = 0;
            g->held[i] = g->held[--g->nheld];
            return;
        }
}

static int gen_node(pgen_t *g, uint16_t id, int *reg, int depth)
{
    const fv_t *n = &SY.fv[id];
    int i, ra = 0, rb = 0, t;
    for (i = 0; i < g->c->nstream; i++) if (g->c->stream_fv[i] == id) { *reg = i; return 0; }
    for (i = 0; i < g->nheld; i++) if (g->held[i].fv == id) { *reg = g->held[i].reg; return 0; }
    if (fv_is_uniform(g->c, id, 0) || n->kind == FV_LOAD) return gen_uniform(g->c, id, reg, depth);
    if (n->kind != FV_OP) return irx_fail(E040, "a value the elementwise template cannot compute");
    if (gen_node(g, n->a, &ra, depth + 1)) return 1;
    if (irx_op_arity(n->op) == 2) { if (gen_node(g, n->b, &rb, depth + 1)) return 1; }
    else rb = ra;
    release(g, n->a);
    if (irx_op_arity(n->op) == 2) release(g, n->b);
    for (t = 0; t < PROG_NTMP && g->tmp_busy[t]; t++) ;
    if (t == PROG_NTMP) return irx_fail(E043, "an op program with more live values than the template's temporaries");
    g->tmp_busy[t] = 1;
    *reg = PROG_R_TMP + t;
    if (g->nheld >= 64) return irx_fail(E043, "an op program with too many shared values");
    g->held[g->nheld].fv = id;
    g->held[g->nheld].reg = (uint8_t)*reg;
    g->nheld++;
    return emit_ins(g->p, n->op, *reg, ra, rb);
}

static pgen_t PG;

static int prog_build(pctx_t *c, uint16_t root, irx_prog_t *p)
{
    int reg = 0;
    memset(&PG, 0, sizeof PG);
    memset(p, 0, sizeof *p);
    PG.c = c;
    PG.p = p;
    if (count_uses(&PG, root, 0)) return 1;
    PG.uses[root]++;                       /* the result stays live */
    if (gen_node(&PG, root, &reg, 0)) return 1;
    p->out = (uint8_t)reg;
    return 0;
}

/* ---------------------------------------------------------------------------------------
 * Index helpers.
 * ------------------------------------------------------------------------------------ */

/* Row-major flat offset of an index into a buffer of the given dims. */
static aff_t idx_flat(const idx_t *x, const ka_t *a)
{
    aff_t f = aff_const(0);
    int d;
    if (x->rank == 0) return f;
    for (d = 0; d < x->rank; d++) {
        if (!x->d[d].ok) return aff_bad();
        f = aff_add(aff_scale(f, a->dim[d]), x->d[d], 1);
    }
    return f;
}

static int64_t arg_elems(const ka_t *a)
{
    int64_t n = 1;
    int d;
    for (d = 0; d < a->rank; d++) n *= a->dim[d];
    return n;
}

/* The flat cell index of the Tile's row-major decode: sum axis_i * prod(ext_j, j > i). */
static aff_t tile_flat(int first, int last)
{
    aff_t f = aff_const(0);
    int i;
    for (i = first; i < last; i++) f = aff_add(aff_scale(f, SY.ext[i]), aff_var(V_TILE0 + i), 1);
    return f;
}

/* A StridedLoop that splits [0, ext) over the threads of the axes [first, na): its start
 * is the flat index of exactly those axes and its step their cell count. */
static int lane_split(const loop_t *L, int first)
{
    aff_t want = tile_flat(first, SY.na);
    int64_t t = 1;
    int i;
    for (i = first; i < SY.na; i++) t *= SY.ext[i];
    return L->kind == 2 && aff_eq(&L->start, &want) && L->step == t && !L->end.ok;
}

/* ---------------------------------------------------------------------------------------
 * Family recognisers.
 * ------------------------------------------------------------------------------------ */

static int global_writes(int *ids, int max)
{
    int i, n = 0;
    for (i = 0; i < SY.nwr; i++)
        if (!SY.wr[i].shared) { if (n < max) ids[n] = i; n++; }
    return n;
}

/* Pointwise: no loops, no accumulators; every global Write is an elementwise function of
 * Loads at its own cell (or scalars), and the Writes together cover each output once. */
static int sel_pointwise(irx_plan_int_t *p)
{
    irx_pw_t *pw = &p->u.pw;
    int wids[8], nw, i, j, s, vec;
    aff_t want;
    pctx_t c;

    if (SY.nloop || SY.nacc || SY.nsb) return -1;
    nw = global_writes(wids, 8);
    if (nw < 1 || nw > 4) return -1;
    memset(pw, 0, sizeof *pw);
    vec = SY.wr[wids[0]].nval;
    want = aff_scale(tile_flat(0, SY.na), vec);
    for (i = 0; i < nw; i++) {
        const wr_t *w = &SY.wr[wids[i]];
        const ka_t *a = &SY.k->arg[w->arg];
        aff_t f = idx_flat(&SY.idx[w->idx], a);
        if (w->atomic || w->npred || w->nval != vec || !aff_eq(&f, &want) || arg_elems(a) != SY.cells * vec) return -1;
        for (j = 0; j < i; j++) if (SY.wr[wids[j]].arg == w->arg) return -1;
    }
    pw->n = SY.cells * vec;
    /* every load is either at the write's cell (a stream) or at a constant index (a scalar) */
    for (i = 1; i < SY.nfv; i++) {
        const fv_t *n = &SY.fv[i];
        const ka_t *a;
        aff_t f;
        if (n->kind == FV_OPAQUE || n->kind == FV_PREV || n->kind == FV_FINAL) return -1;
        if (n->kind != FV_LOAD) continue;
        a = &SY.k->arg[n->arg];
        f = idx_flat(&SY.idx[n->idx], a);
        if (aff_isc(&f)) continue;
        if (!aff_eq(&f, &want) || arg_elems(a) != pw->n) return -1;
        for (s = 0; s < pw->nin; s++) if (pw->in_arg[s] == n->arg) break;
        if (s == pw->nin) {
            if (pw->nin >= PROG_NSTREAM) return irx_fail(E043, "a pointwise graph with more than 4 input streams");
            pw->in_arg[pw->nin] = n->arg;
            pw->in_dt[pw->nin] = a->dt;
            pw->nin++;
        }
    }
    memset(&c, 0, sizeof c);
    c.uni = pw->uni;
    c.nuni = &pw->nuni;
    c.uprog = &pw->uprog;
    c.nstream = pw->nin;
    for (j = 0; j < vec; j++) {
        for (s = 0; s < pw->nin; s++) {
            c.stream_fv[s] = 0xFFFF;
            for (i = 1; i < SY.nfv; i++) {
                const fv_t *n = &SY.fv[i];
                if (n->kind == FV_LOAD && n->arg == pw->in_arg[s] && n->lane == j &&
                    !aff_isc(&SY.idx[n->idx].d[0])) c.stream_fv[s] = (uint16_t)i;
            }
        }
        for (i = 0; i < nw; i++) {
            irx_prog_t prog;
            if (prog_build(&c, SY.wr[wids[i]].val[j], &prog)) return 1;
            if (j == 0) {
                pw->prog[i] = prog;
                pw->out_arg[i] = SY.wr[wids[i]].arg;
                pw->out_dt[i] = SY.k->arg[SY.wr[wids[i]].arg].dt;
            } else if (memcmp(&prog, &pw->prog[i], sizeof prog)) {
                return irx_fail(E040, "a vectorised pointwise graph whose lanes compute different things");
            }
        }
    }
    pw->nout = (uint8_t)nw;
    p->fam = FAM_POINTWISE;
    return 0;
}

/* The per-block combine of an accumulator: none when the row's threads are one thread, a
 * full-warp butterfly when they are one warp, the butterfly plus a tree over the warps by
 * `warp` when they are the whole block. */
static int combine_ok(const acc_t *ac, int64_t lanes)
{
    if (lanes == 1) return ac->shuf_len == 0 && ac->tree_len == 0;
    if (lanes == 32) return ac->shuf_len == 32 && ac->tree_len == 0;
    if (lanes == SY.block && lanes % 32 == 0 && lanes > 32)
        return ac->shuf_len == 32 && ac->tree_len == lanes / 32 && ac->tree_ok;
    return 0;
}

/* Predicates of a Write: each must be `var == constant` on a thread-position variable.
 * *pinned gets one bit per tile axis (bits 0..7) and V_LANE/V_WARP/V_TID (bits 8..10)
 * that the predicates fix. Returns 0 when some predicate is of another form. */
static int preds_pin(const wr_t *w, int first_lane, unsigned *pinned)
{
    int i;
    *pinned = 0;
    for (i = 0; i < w->npred; i++) {
        const pred_t *p = &w->pred[i];
        int v;
        int64_t val;
        if (p->kind != PR_EQ || p->a.nv != 1 || p->a.coef[0] != 1) return 0;
        v = p->a.var[0];
        val = -p->a.cst;
        if (v >= V_TILE0 + first_lane && v < V_TILE0 + SY.na) {
            if (val < 0 || val >= SY.ext[v - V_TILE0]) return 0;
            *pinned |= 1u << (v - V_TILE0);
        } else if (v == V_LANE || v == V_WARP || v == V_TID) {
            if (val < 0 || (v == V_LANE && val > 31) || (v != V_LANE && val * (v == V_WARP ? 32 : 1) >= SY.block)) return 0;
            *pinned |= 1u << (8 + v - V_LANE);
        } else return 0;
    }
    return 1;
}

/* Find the one non-scalar global Load a value depends on: the reduced stream. */
static int find_stream(uint16_t id, uint16_t *ld, int depth)
{
    const fv_t *n = &SY.fv[id];
    if (depth > 64) return -1;
    if (n->kind == FV_LOAD) {
        aff_t f = idx_flat(&SY.idx[n->idx], &SY.k->arg[n->arg]);
        if (aff_isc(&f)) return 0;
        if (*ld && *ld != id) return -1;
        *ld = id;
        return 0;
    }
    if (n->kind == FV_OP) {
        if (find_stream(n->a, ld, depth + 1)) return -1;
        if (irx_op_arity(n->op) == 2 && find_stream(n->b, ld, depth + 1)) return -1;
        return 0;
    }
    if (n->kind == FV_CONST || n->kind == FV_FINAL) return 0;
    return -1;
}

/* An Init seed other than the fold's identity (src/isel.c:1872-1900): in the reference each of
 * the `lanes` threads that fold into one result starts its partial at the seed, so the result is
 * the fold of the data and `lanes` copies of the seed. The template folds the data from the
 * identity; the uniform program's first instruction then folds in the seeds' share (lanes * s
 * for a sum, s for a maximum or minimum, s^lanes for a product, formed in double and rounded
 * once), kept in its own literal register so that every shard but the first of a sharded full
 * reduction can set it to the identity and the shards' combine counts it once. */
static int seed_total(pctx_t *c, irx_red_t *r, const acc_t *ac, int64_t lanes)
{
    irx_uni_t u;
    int reg = 0, i;
    float s, t;
    memcpy(&s, &ac->seed_bits, 4);
    switch (ac->op) {
    case OP_ADD: t = (float)((double)s * (double)lanes); break;
    case OP_MUL: t = (float)pow((double)s, (double)lanes); break;
    case OP_MAX: case OP_MIN: t = s; break;
    default: return irx_fail(E042, "an Init seed on a fold the reduction template does not take");
    }
    memset(&u, 0, sizeof u);
    u.kind = UNI_LIT;
    memcpy(&u.v, &t, 4);
    if (uni_add(c, 0xFFFE, &u, &reg)) return 1;
    if (r->uprog.nins >= PROG_MAX_INS) return irx_fail(E043, "an op program longer than the template takes");
    for (i = r->uprog.nins; i > 0; i--) r->uprog.ins[i] = r->uprog.ins[i - 1];
    r->uprog.ins[0].op = ac->op;
    r->uprog.ins[0].dst = r->tot_reg;
    r->uprog.ins[0].a = r->tot_reg;
    r->uprog.ins[0].b = (uint8_t)reg;
    r->uprog.nins++;
    r->seed_uni = (uint8_t)(reg - PROG_R_UNI);
    r->has_seed = 1;
    return 0;
}

static int any_seeded(void)
{
    int a;
    for (a = 0; a < SY.nacc; a++) if (SY.acc[a].has_seed) return 1;
    return 0;
}

static int sel_reduce(irx_plan_int_t *p)
{
    irx_red_t *r = &p->u.red;
    int wids[8], nw, lane0, reg = 0;
    const acc_t *ac;
    const loop_t *L;
    const wr_t *w;
    uint16_t xl = 0;
    const fv_t *xn;
    const ka_t *X, *Y;
    aff_t lf, rowf, want, wf;
    int64_t lanes = 1, rows;
    unsigned pinned;
    pctx_t c;
    irx_uni_t u;
    int i;

    if (SY.nacc != 1 || SY.nloop != 1) return -1;
    nw = global_writes(wids, 8);
    if (nw != 1) return -1;
    ac = &SY.acc[0];
    L = &SY.loop[0];
    w = &SY.wr[wids[0]];
    if (ac->loop != 0 || ac->nupd != 1 || ac->upd_base || ac->upd_loop != 0 || w->loop != -1 || w->nval != 1) return -1;
    if (find_stream(ac->upd_val, &xl, 0) || !xl) return -1;
    xn = &SY.fv[xl];
    X = &SY.k->arg[xn->arg];
    Y = &SY.k->arg[w->arg];
    for (lane0 = SY.na; lane0 >= 0; lane0--) if (lane_split(L, lane0)) break;
    if (lane0 < 0) return irx_fail(E041, "a reduction loop whose start and step do not split the axis over threads");
    for (i = lane0; i < SY.na; i++) lanes *= SY.ext[i];
    lf = idx_flat(&SY.idx[xn->idx], X);
    wf = idx_flat(&SY.idx[w->idx], Y);
    rowf = tile_flat(0, lane0);
    rows = SY.cells / lanes;
    memset(r, 0, sizeof *r);
    r->op = ac->op;
    r->x_arg = xn->arg; r->x_dt = X->dt;
    r->y_arg = w->arg;  r->y_dt = Y->dt;
    if (!preds_pin(w, lane0, &pinned)) return irx_fail(E041, "a reduction result written under a condition the template cannot place");
    if (w->atomic) {
        /* full reduction: every thread of the grid splits the array; each block's total is
         * added into the (zeroed) output by exactly one of its threads */
        int64_t t = 1;
        int bl = SY.na;
        unsigned blockaxes = 0;
        if (lane0 != 0) return irx_fail(E041, "an atomic reduction whose loop does not span the whole grid");
        want = aff_var(V_LOOP0 + 0);
        if (!aff_eq(&lf, &want) || arg_elems(X) != L->ext) return irx_fail(E041, "a full reduction that does not read its whole input once");
        if (ac->op != OP_ADD) return irx_fail(E040, "a cross-block atomic add of a reduction that is not a sum");
        while (bl > 0 && t < SY.block) { t *= SY.ext[--bl]; blockaxes |= 1u << bl; }
        if (t != SY.block) return irx_fail(E041, "a full reduction whose blocks are not whole tile axes");
        if (!combine_ok(ac, SY.block)) return irx_fail(E041, "a block combine that does not fold every thread of the block");
        if ((pinned & blockaxes) != blockaxes && !(pinned & (1u << 10)) && (pinned & 0x300u) != 0x300u)
            return irx_fail(E041, "a block total added by more than one thread of its block");
        if (arg_elems(Y) != 1 || !aff_isc(&wf) || wf.cst != 0) return irx_fail(E041, "a full reduction written to other than a single element");
        r->rows = 1;
        r->cols = L->ext;
        r->accumulate = 1;
        p->fam = FAM_REDUCE_ALL;
    } else {
        want = aff_add(aff_scale(rowf, L->ext), aff_var(V_LOOP0 + 0), 1);
        if (!aff_eq(&lf, &want) || arg_elems(X) != rows * L->ext)
            return irx_fail(E041, "a row reduction whose load is not x[row, loop]");
        if (!aff_eq(&wf, &rowf) || arg_elems(Y) != rows)
            return irx_fail(E041, "a row reduction whose write is not y[row]");
        if (lanes > 1 && lanes != SY.block && lanes != 32) return irx_fail(E041, "a row split over a thread count the combine does not cover");
        if (!combine_ok(ac, lanes)) return irx_fail(E041, "a block combine that does not fold every thread of the row");
        r->rows = rows;
        r->cols = L->ext;
        p->fam = rows == 1 ? FAM_REDUCE_ALL : FAM_REDUCE_ROWS;
    }
    memset(&c, 0, sizeof c);
    c.uni = r->uni;
    c.nuni = &r->nuni;
    c.uprog = &r->uprog;
    memset(&u, 0, sizeof u);
    u.kind = UNI_STAT;
    if (uni_add(&c, ac->final_val, &u, &reg)) return 1;
    r->tot_reg = (uint8_t)reg;
    if (ac->has_seed && seed_total(&c, r, ac, lanes)) return 1;
    c.nstream = 1;
    c.stream_fv[0] = xl;
    r->has_pre = ac->upd_val != xl;
    if (r->has_pre && prog_build(&c, ac->upd_val, &r->pre)) return 1;
    c.nstream = 0;
    if (gen_uniform(&c, w->val[0], &reg, 0)) return 1;
    r->out_reg = (uint8_t)reg;
    if (r->accumulate && r->out_reg != r->tot_reg) {
        /* sum over blocks of post(block total) equals post(total) only for a linear post:
         * accept a divide or a multiply of the total by a launch-uniform value (a mean) */
        const irx_ins_t *q = &r->uprog.ins[r->uprog.nins - 1];
        if (q->dst != r->out_reg || (q->op != OP_DIV && q->op != OP_MUL) || (q->a != r->tot_reg && q->b != r->tot_reg) ||
            (q->op == OP_DIV && q->a != r->tot_reg))
            return irx_fail(E040, "a non-linear function of a block total added across blocks");
    }
    return 0;
}

/* Loads of a loop's own row element x[row, j] and broadcast vector w[j] become the two
 * stream registers of that loop's program. */
static void row_streams(pctx_t *c, const irx_row_t *r, int lid)
{
    int i;
    c->nstream = 2;
    c->stream_fv[0] = c->stream_fv[1] = 0xFFFF;
    for (i = 1; i < SY.nfv; i++) {
        const fv_t *n = &SY.fv[i];
        aff_t f;
        if (n->kind != FV_LOAD) continue;
        f = idx_flat(&SY.idx[n->idx], &SY.k->arg[n->arg]);
        if (aff_coef(&f, V_LOOP0 + lid) != 1) continue;
        if (n->arg == r->x_arg) c->stream_fv[0] = (uint16_t)i;
        else if (r->has_w && n->arg == r->w_arg) c->stream_fv[1] = (uint16_t)i;
    }
}

/* ---- recognising the three BASELINE row ops in a row graph ---- */

static int fv_const_is(uint16_t id, float *v)
{
    if (SY.fv[id].kind != FV_CONST) return 0;
    memcpy(v, &SY.fv[id].bits, 4);
    return 1;
}

static int fv_op1(uint16_t id, int op, uint16_t *a)
{
    if (SY.fv[id].kind != FV_OP || SY.fv[id].op != op) return 0;
    *a = SY.fv[id].a;
    return 1;
}

static int fv_op2(uint16_t id, int op, uint16_t *a, uint16_t *b)
{
    if (SY.fv[id].kind != FV_OP || SY.fv[id].op != op) return 0;
    *a = SY.fv[id].a;
    *b = SY.fv[id].b;
    return 1;
}

/* mean(x^2) + eps: (F / cols) + eps or (F * (1/cols)) + eps; the eps bits land in *eps. */
static int match_ms_eps(uint16_t id, uint16_t F, int64_t cols, uint32_t *eps)
{
    uint16_t a, b, m = 0, e = 0, f, c;
    float v, ev;
    if (!fv_op2(id, OP_ADD, &a, &b)) return 0;
    if (fv_const_is(b, &ev)) { m = a; e = b; }
    else if (fv_const_is(a, &ev)) { m = b; e = a; }
    else return 0;
    (void)e;
    if (fv_op2(m, OP_DIV, &f, &c)) { if (f != F || !fv_const_is(c, &v) || v != (float)cols) return 0; }
    else if (fv_op2(m, OP_MUL, &f, &c)) {
        if (f != F) { uint16_t t = f; f = c; c = t; }
        if (f != F || !fv_const_is(c, &v) || v != 1.0f / (float)cols) return 0;
    } else return 0;
    memcpy(eps, &ev, 4);
    return 1;
}

/* x / S * w, (x * w) / S, x * R * w with S = sqrt(q) or R = rsqrt(q); *q gets q. */
static int match_scaled(uint16_t val, uint16_t xe, uint16_t we, int want_w, uint16_t *q)
{
    uint16_t a, b, c, d;
    if (!want_w) {
        if (fv_op2(val, OP_DIV, &a, &b) && a == xe && fv_op1(b, OP_SQRT, q)) return 1;
        if (fv_op2(val, OP_MUL, &a, &b)) {
            if (a == xe && fv_op1(b, OP_RSQRT, q)) return 1;
            if (b == xe && fv_op1(a, OP_RSQRT, q)) return 1;
        }
        return 0;
    }
    if (fv_op2(val, OP_MUL, &a, &b)) {                 /* (x / S) * w, (x * R) * w */
        uint16_t inner = a == we ? b : b == we ? a : 0;
        if (inner && (a == we || b == we)) {
            if (fv_op2(inner, OP_DIV, &c, &d) && c == xe && fv_op1(d, OP_SQRT, q)) return 1;
            if (fv_op2(inner, OP_MUL, &c, &d) && (c == xe || d == xe) && fv_op1(c == xe ? d : c, OP_RSQRT, q)) return 1;
        }
    }
    if (fv_op2(val, OP_DIV, &a, &b) && fv_op2(a, OP_MUL, &c, &d) && ((c == xe && d == we) || (c == we && d == xe)) &&
        fv_op1(b, OP_SQRT, q)) return 1;                 /* (x * w) / S */
    return 0;
}

/* Which written-out kernel (if any) computes this row graph exactly. `xs[k]` is the row
 * element node of statistic k's loop, `xe`/`we` the epilogue's x and w nodes. */
static int row_kind(const irx_row_t *r, const int *acc, const uint16_t *xs, uint16_t xe, uint16_t we, uint16_t val,
                    uint32_t *eps)
{
    uint16_t q = 0, a, b, c, d;
    if (r->nstat == 1 && r->stat_op[0] == OP_ADD && fv_is(SY.acc[acc[0]].upd_val, OP_MUL, xs[0], xs[0])) {
        uint16_t F = SY.acc[acc[0]].final_val;
        if (r->has_w && match_scaled(val, xe, we, 1, &q) && match_ms_eps(q, F, r->cols, eps)) return ROWK_RMSNORM;
        if (!r->has_w && match_scaled(val, xe, we, 0, &q) && q == F) return ROWK_L2NORM;
        return ROWK_GENERIC;
    }
    if (r->nstat == 2 && !r->has_w && r->stat_op[0] == OP_MAX && r->stat_op[1] == OP_ADD &&
        SY.acc[acc[0]].upd_val == xs[0]) {
        uint16_t M = SY.acc[acc[0]].final_val, L = SY.acc[acc[1]].final_val;
        if (!(fv_op1(SY.acc[acc[1]].upd_val, OP_EXP, &a) && fv_op2(a, OP_SUB, &b, &c) && b == xs[1] && c == M)) return ROWK_GENERIC;
        if (fv_op2(val, OP_DIV, &a, &d) && d == L && fv_op1(a, OP_EXP, &b) && fv_op2(b, OP_SUB, &c, &q) && c == xe && q == M)
            return ROWK_SOFTMAX;
    }
    return ROWK_GENERIC;
}

/* Row ops: statistics loops, then one loop writing y[row, j] = f(x[row, j], w[j], stats). */
static int sel_rowop(irx_plan_int_t *p)
{
    irx_row_t *r = &p->u.row;
    int wids[8], nw, lane0 = -1, i, s, el, st, reg = 0;
    const wr_t *w;
    const loop_t *E;
    int64_t lanes = 1, rows, cols;
    aff_t rowf, want, wf;
    pctx_t c;
    irx_uni_t u;
    int sacc[ROW_MAX_STAT];
    uint16_t sxs[ROW_MAX_STAT];

    nw = global_writes(wids, 8);
    if (nw != 1 || SY.nloop < 2 || SY.nacc < 1 || SY.nacc > ROW_MAX_STAT) return -1;
    w = &SY.wr[wids[0]];
    el = w->loop;
    if (el < 0 || el != SY.nloop - 1 || w->atomic || w->nval != 1 || w->npred) return -1;
    E = &SY.loop[el];
    for (i = SY.na; i >= 0; i--) if (lane_split(E, i)) { lane0 = i; break; }
    if (lane0 < 0) return -1;
    for (i = lane0; i < SY.na; i++) lanes *= SY.ext[i];
    cols = E->ext;
    rows = SY.cells / lanes;
    rowf = tile_flat(0, lane0);
    memset(r, 0, sizeof *r);
    r->rows = rows;
    r->cols = cols;
    r->y_arg = w->arg;
    r->y_dt = SY.k->arg[w->arg].dt;
    wf = idx_flat(&SY.idx[w->idx], &SY.k->arg[w->arg]);
    want = aff_add(aff_scale(rowf, cols), aff_var(V_LOOP0 + el), 1);
    if (!aff_eq(&wf, &want) || arg_elems(&SY.k->arg[w->arg]) != rows * cols) return -1;
    if (lanes > 1 && lanes != SY.block && lanes != 32) return -1;
    for (i = 0; i < SY.nloop; i++)
        if (SY.loop[i].parent != -1 || !lane_split(&SY.loop[i], lane0) || SY.loop[i].ext != cols) return -1;
    if (SY.nacc != SY.nloop - 1) return -1;
    /* the streams: x[row, j] of a loop, and optionally w[j] */
    for (i = 1; i < SY.nfv; i++) {
        const fv_t *n = &SY.fv[i];
        aff_t f;
        if (n->kind == FV_OPAQUE) return -1;
        if (n->kind != FV_LOAD) continue;
        f = idx_flat(&SY.idx[n->idx], &SY.k->arg[n->arg]);
        if (aff_isc(&f)) continue;
        for (s = 0; s < SY.nloop; s++) {
            aff_t wx = aff_add(aff_scale(rowf, cols), aff_var(V_LOOP0 + s), 1);
            aff_t wv = aff_var(V_LOOP0 + s);
            if (aff_eq(&f, &wx) && arg_elems(&SY.k->arg[n->arg]) == rows * cols) {
                if (r->x_dt && r->x_arg != n->arg) return -1;
                r->x_arg = n->arg; r->x_dt = SY.k->arg[n->arg].dt;
                break;
            }
            if (aff_eq(&f, &wv) && arg_elems(&SY.k->arg[n->arg]) == cols) {
                if (r->has_w && r->w_arg != n->arg) return -1;
                r->w_arg = n->arg; r->w_dt = SY.k->arg[n->arg].dt; r->has_w = 1;
                break;
            }
        }
        if (s == SY.nloop) return -1;
    }
    if (!r->x_dt) return -1;
    memset(&c, 0, sizeof c);
    c.uni = r->uni;
    c.nuni = &r->nuni;
    c.uprog = &r->uprog;
    /* statistics, in loop order; each lands in a uniform register */
    for (st = 0; st < SY.nloop; st++) {
        int a;
        const acc_t *ac;
        if (st == el) continue;
        for (a = 0; a < SY.nacc && SY.acc[a].loop != st; a++) ;
        if (a == SY.nacc) return -1;
        ac = &SY.acc[a];
        if (ac->nupd != 1 || ac->upd_base || ac->upd_loop != st) return -1;
        if (!combine_ok(ac, lanes)) return irx_fail(E041, "a row statistic whose block combine does not fold every thread of the row");
        row_streams(&c, r, st);
        sacc[r->nstat] = a;
        sxs[r->nstat] = c.stream_fv[0];
        if (ac->upd_val == c.stream_fv[0]) { memset(&r->stat_pre[r->nstat], 0, sizeof(irx_prog_t)); r->stat_pre[r->nstat].out = 0; }
        else if (prog_build(&c, ac->upd_val, &r->stat_pre[r->nstat])) return 1;
        r->stat_op[r->nstat] = ac->op;
        memset(&u, 0, sizeof u);
        u.kind = UNI_STAT; u.v = r->nstat;
        if (uni_add(&c, ac->final_val, &u, &reg)) return 1;
        r->stat_reg[r->nstat] = (uint8_t)reg;
        r->nstat++;
    }
    row_streams(&c, r, el);
    if (prog_build(&c, w->val[0], &r->epi)) return 1;
    r->kind = (uint8_t)row_kind(r, sacc, sxs, c.stream_fv[0], c.stream_fv[1], w->val[0], &r->eps_bits);
    p->fam = FAM_ROWOP;
    return 0;
}

/* ---- matmul ---- */

static int is_load_of(uint16_t id, int *arg, aff_t *flat)
{
    const fv_t *n = &SY.fv[id];
    if (n->kind != FV_LOAD || n->lane) return 0;
    *arg = n->arg;
    *flat = idx_flat(&SY.idx[n->idx], &SY.k->arg[n->arg]);
    return flat->ok;
}

static int sel_matmul(irx_plan_int_t *p)
{
    irx_mm_t *m = &p->u.mm;
    int wids[4], nw, aa, ab, ta, tb;
    const acc_t *ac;
    const wr_t *w;
    const fv_t *pr;
    aff_t fa, fb, fc, want;
    int64_t M, N, K;
    const ka_t *A, *B, *C;

    if (SY.nloop != 1 || SY.nacc != 1 || SY.na != 2 || SY.nsb) return -1;
    nw = global_writes(wids, 4);
    if (nw != 1) return -1;
    ac = &SY.acc[0];
    w = &SY.wr[wids[0]];
    if (SY.loop[0].kind != 1 || ac->op != OP_ADD || ac->nupd != 1 || ac->upd_base || ac->loop != 0) return -1;
    if (w->nval != 1 || w->val[0] != ac->final_val || w->atomic || w->npred || w->loop != -1) return -1;
    pr = &SY.fv[ac->upd_val];
    if (pr->kind != FV_OP || pr->op != OP_MUL) return -1;
    if (!is_load_of(pr->a, &ta, &fa) || !is_load_of(pr->b, &tb, &fb)) return -1;
    M = SY.ext[0]; N = SY.ext[1]; K = SY.loop[0].ext;
    /* which operand is A: the one indexed by the row axis and k */
    want = aff_add(aff_scale(aff_var(V_TILE0 + 0), K), aff_var(V_LOOP0), 1);
    if (aff_eq(&fb, &want)) { int t = ta; aff_t f = fa; ta = tb; fa = fb; tb = t; fb = f; }
    if (!aff_eq(&fa, &want)) return -1;
    A = &SY.k->arg[ta]; B = &SY.k->arg[tb]; C = &SY.k->arg[w->arg];
    aa = ta; ab = tb;
    memset(m, 0, sizeof *m);
    {
        aff_t bn = aff_add(aff_scale(aff_var(V_LOOP0), N), aff_var(V_TILE0 + 1), 1);   /* B[k, j] */
        aff_t bk = aff_add(aff_scale(aff_var(V_TILE0 + 1), K), aff_var(V_LOOP0), 1);   /* B[j, k] */
        if (aff_eq(&fb, &bn)) m->b_kmajor = 0;
        else if (aff_eq(&fb, &bk)) m->b_kmajor = 1;
        else return irx_fail(E041, "a matmul whose B operand is indexed neither [k, j] nor [j, k]");
    }
    fc = idx_flat(&SY.idx[w->idx], C);
    want = aff_add(aff_scale(aff_var(V_TILE0 + 0), N), aff_var(V_TILE0 + 1), 1);
    if (!aff_eq(&fc, &want)) return irx_fail(E041, "a matmul whose output is not written C[i, j]");
    if (arg_elems(A) != M * K || arg_elems(B) != K * N || arg_elems(C) != M * N) return irx_fail(E041, "a matmul whose buffers do not match its loop extents");
    if (A->dt != B->dt || A->dt != C->dt) return irx_fail(E042, "a matmul with mixed operand dtypes");
    m->m = M; m->n = N; m->k = K;
    m->a_arg = (uint8_t)aa; m->b_arg = (uint8_t)ab; m->c_arg = w->arg;
    m->dt = A->dt;
    p->fam = FAM_MATMUL;
    return 0;
}

/* ---- attention ---- */

static int fv_is(uint16_t id, int op, uint16_t a, uint16_t b)
{
    const fv_t *n = &SY.fv[id];
    if (n->kind != FV_OP || n->op != op) return 0;
    if (n->a == a && n->b == b) return 1;
    return op_commutes(op) && n->a == b && n->b == a;
}

static int fv_prev(uint16_t id, int acc)
{
    return SY.fv[id].kind == FV_PREV && SY.fv[id].acc == acc;
}

static int sel_attention(irx_plan_int_t *p)
{
    irx_at_t *t = &p->u.at;
    int wids[4], nw, jl = -1, el = -1, am = -1, al = -1, ao = -1, ad = -1, i;
    const wr_t *w;
    uint16_t sc, scl = 0, mn, alpha, pj, vload = 0;
    float scale = 0.f;
    int64_t B, H, Sq, Dv, Dqk, Skv;
    int lead, kt = 0;
    uint32_t divc = 0;
    int isdiv = 0;
    const fv_t *o;
    int qa, ka_, va;
    aff_t fq, fk, fv, fo, want;

    if (SY.na < 2 || SY.na > 4 || SY.nloop != 2 || SY.nacc != 4 || SY.nsb) return -1;
    nw = global_writes(wids, 4);
    if (nw != 1) return -1;
    w = &SY.wr[wids[0]];
    if (w->nval != 1 || w->atomic || w->npred || w->loop != -1) return -1;
    for (i = 0; i < 2; i++) {
        if (SY.loop[i].parent == -1) jl = i;
        else el = i;
    }
    if (jl < 0 || el < 0 || SY.loop[el].parent != jl || SY.loop[el].kind != 1) return -1;
    for (i = 0; i < 4; i++) {
        const acc_t *ac = &SY.acc[i];
        if (ac->loop == el && ac->op == OP_ADD && !ac->upd_base) ad = i;
        else if (ac->loop == jl && ac->op == OP_MAX && !ac->upd_base) am = i;
        else if (ac->loop == jl && ac->op == OP_ADD && ac->upd_base) {
            /* the output accumulator folds p * V[j, d]; the running sum folds p alone */
            const fv_t *u = &SY.fv[ac->upd_val];
            if (u->kind == FV_OP && u->op == OP_MUL &&
                (SY.fv[u->a].kind == FV_LOAD || SY.fv[u->b].kind == FV_LOAD)) ao = i;
            else al = i;
        }
    }
    if (ad < 0 || am < 0 || al < 0 || ao < 0) return -1;
    /* the score: dot * scale (or dot / c) */
    {
        const fv_t *d = &SY.fv[SY.acc[ad].upd_val];
        if (d->kind != FV_OP || d->op != OP_MUL) return -1;
        if (!is_load_of(d->a, &qa, &fq) || !is_load_of(d->b, &ka_, &fk)) return -1;
    }
    sc = SY.acc[am].upd_val;
    o = &SY.fv[sc];
    if (o->kind != FV_OP) return -1;
    if (o->op == OP_MUL && SY.fv[o->a].kind == FV_FINAL && SY.fv[o->a].acc == ad && SY.fv[o->b].kind == FV_CONST) scl = o->b;
    else if (o->op == OP_MUL && SY.fv[o->b].kind == FV_FINAL && SY.fv[o->b].acc == ad && SY.fv[o->a].kind == FV_CONST) scl = o->a;
    else if (o->op == OP_DIV && SY.fv[o->a].kind == FV_FINAL && SY.fv[o->a].acc == ad && SY.fv[o->b].kind == FV_CONST) {
        float c;
        memcpy(&c, &SY.fv[o->b].bits, 4);
        scale = 1.0f / c;
        scl = 0xFFFF;
        divc = SY.fv[o->b].bits;
    } else return -1;
    if (scl != 0xFFFF) memcpy(&scale, &SY.fv[scl].bits, 4);
    /* running max, rescale and probability */
    {
        uint16_t prevm = 0, prevl = 0, prevo = 0;
        const fv_t *lb, *ob, *ov;
        for (i = 1; i < SY.nfv; i++) {
            if (fv_prev((uint16_t)i, am)) prevm = (uint16_t)i;
            if (fv_prev((uint16_t)i, al)) prevl = (uint16_t)i;
            if (fv_prev((uint16_t)i, ao)) prevo = (uint16_t)i;
        }
        if (!prevm || !prevl || !prevo) return -1;
        mn = 0;
        for (i = 1; i < SY.nfv; i++) if (fv_is((uint16_t)i, OP_MAX, prevm, sc)) mn = (uint16_t)i;
        if (!mn) return -1;
        pj = SY.acc[al].upd_val;                      /* exp(sc - mn) */
        if (SY.fv[pj].kind != FV_OP || SY.fv[pj].op != OP_EXP) return -1;
        if (!fv_is(SY.fv[pj].a, OP_SUB, sc, mn) || SY.fv[SY.fv[pj].a].a != sc) return -1;
        lb = &SY.fv[SY.acc[al].upd_base];             /* l * alpha */
        if (lb->kind != FV_OP || lb->op != OP_MUL) return -1;
        alpha = lb->a == prevl ? lb->b : lb->b == prevl ? lb->a : 0;
        if (!alpha || SY.fv[alpha].kind != FV_OP || SY.fv[alpha].op != OP_EXP) return -1;
        {
            const fv_t *dm = &SY.fv[SY.fv[alpha].a];
            if (dm->kind != FV_OP || dm->op != OP_SUB || dm->a != prevm || dm->b != mn) return -1;
        }
        ob = &SY.fv[SY.acc[ao].upd_base];             /* o * alpha */
        if (!fv_is(SY.acc[ao].upd_base, OP_MUL, prevo, alpha)) return -1;
        (void)ob;
        ov = &SY.fv[SY.acc[ao].upd_val];              /* p * V */
        if (ov->kind != FV_OP || ov->op != OP_MUL) return -1;
        vload = ov->a == pj ? ov->b : ov->b == pj ? ov->a : 0;
        if (!vload || !is_load_of(vload, &va, &fv)) return -1;
    }
    /* output: o / l */
    if (!fv_is(w->val[0], OP_DIV, SY.acc[ao].final_val, SY.acc[al].final_val) ||
        SY.fv[w->val[0]].a != SY.acc[ao].final_val) return -1;
    /* Tile axes: leading batch axes (none, b, or b and h), then the query q and the output
     * column d. The key loop has Sk keys, the dot loop Dqk terms; V and O are Dv wide. */
    lead = SY.na - 2;
    B = lead >= 1 ? SY.ext[0] : 1;
    H = lead >= 2 ? SY.ext[1] : 1;
    Sq = SY.ext[lead]; Dv = SY.ext[lead + 1];
    Skv = SY.loop[jl].ext;
    Dqk = SY.loop[el].ext;
    {
        aff_t bh = aff_const(0), qrow, krow;
        for (i = 0; i < lead; i++) bh = aff_add(aff_scale(bh, SY.ext[i]), aff_var(V_TILE0 + i), 1);
        qrow = aff_add(aff_scale(bh, Sq), aff_var(V_TILE0 + lead), 1);
        krow = aff_add(aff_scale(bh, Skv), aff_var(V_LOOP0 + jl), 1);
        want = aff_add(aff_scale(qrow, Dqk), aff_var(V_LOOP0 + el), 1);
        if (!aff_eq(&fq, &want)) {          /* the dot may list K first */
            int tq = qa; aff_t f = fq; qa = ka_; fq = fk; ka_ = tq; fk = f;
        }
        if (!aff_eq(&fq, &want)) return irx_fail(E041, "an attention whose Q is not read Q[.., q, e]");
        want = aff_add(aff_scale(krow, Dqk), aff_var(V_LOOP0 + el), 1);
        if (!aff_eq(&fk, &want)) {          /* K stored transposed: Kt[.., e, j] */
            want = aff_add(aff_scale(aff_add(aff_scale(bh, Dqk), aff_var(V_LOOP0 + el), 1), Skv),
                           aff_var(V_LOOP0 + jl), 1);
            if (!aff_eq(&fk, &want)) return irx_fail(E041, "an attention whose K is read neither K[.., j, e] nor Kt[.., e, j]");
            kt = 1;
        }
        want = aff_add(aff_scale(krow, Dv), aff_var(V_TILE0 + lead + 1), 1);
        if (!aff_eq(&fv, &want)) return irx_fail(E041, "an attention whose V is not read V[.., j, d]");
        fo = idx_flat(&SY.idx[w->idx], &SY.k->arg[w->arg]);
        want = aff_add(aff_scale(qrow, Dv), aff_var(V_TILE0 + lead + 1), 1);
        if (!aff_eq(&fo, &want)) return irx_fail(E041, "an attention whose output is not written O[.., q, d]");
    }
    memset(t, 0, sizeof *t);
    /* key range: all keys, or a causal prefix 0 .. q */
    {
        const loop_t *J = &SY.loop[jl];
        if (J->kind == 2) {
            aff_t qe = aff_add(aff_var(V_TILE0 + lead), aff_const(1), 1);
            if (J->step != 1 || !aff_isc(&J->start) || J->start.cst != 0) return -1;
            if (!J->end.ok) t->causal = 0;
            else if (aff_eq(&J->end, &qe)) t->causal = 1;
            else return irx_fail(E042, "an attention whose key range is neither all keys nor a causal prefix");
        }
    }
    {
        const ka_t *Q = &SY.k->arg[qa], *K = &SY.k->arg[ka_], *V = &SY.k->arg[va], *O = &SY.k->arg[w->arg];
        if (arg_elems(Q) != B * H * Sq * Dqk || arg_elems(K) != B * H * Skv * Dqk ||
            arg_elems(V) != B * H * Skv * Dv || arg_elems(O) != B * H * Sq * Dv)
            return irx_fail(E041, "an attention whose buffers do not match its extents");
        if (Dqk > 128 || Dv > 128) return irx_fail(E042, "an attention with a head size over 128");
        if (Q->dt != K->dt || Q->dt != V->dt || Q->dt != O->dt) return irx_fail(E042, "an attention with mixed dtypes");
        t->dt = Q->dt;
    }
    t->b = B; t->h = H; t->s = Sq; t->d = Dv;
    t->sq = Sq; t->sk = Skv; t->dqk = Dqk; t->dv = Dv; t->k_t = (uint8_t)kt;
    t->q_arg = (uint8_t)qa; t->k_arg = (uint8_t)ka_; t->v_arg = (uint8_t)va; t->o_arg = w->arg;
    memcpy(&t->scale_bits, &scale, 4);
    isdiv = scl == 0xFFFF;
    t->scale_div = (uint8_t)isdiv;
    t->div_bits = divc;
    p->fam = FAM_ATTENTION;
    return 0;
}

/* ---------------------------------------------------------------------------------------
 * Entry.
 * ------------------------------------------------------------------------------------ */

static int tile_setup(const kir_t *k, const kn_t *tile)
{
    const kv_t *ax = kir_fld(k, tile, "axes"), *aux = kir_fld(k, tile, "aux_threads");
    uint32_t i;
    int64_t tot;
    if (!ax || ax->tag != KV_LIST) return irx_fail(E015, "a Tile with no axes list");
    if (ax->n > KIR_MAX_DIM) return irx_fail(E081, "a Tile with more axes than the limit");
    if (aux && aux->tag == KV_INT && aux->i != 0) return irx_fail(E059, "a Tile with aux_threads");
    if (k->grid[1] != 1 || k->grid[2] != 1 || k->block[1] != 1 || k->block[2] != 1)
        return irx_fail(E025, "a launch with y or z beyond 1");
    SY.cells = 1;
    SY.na = (int)ax->n;
    for (i = 0; i < ax->n; i++) {
        const kn_t *a = kir_node(k, kir_item(k, ax, i));
        const kv_t *nm = a ? kir_fld(k, a, "name") : NULL, *ex = a ? kir_fld(k, a, "extent") : NULL;
        if (!nm || !ex || nm->tag != KV_STR) return irx_fail(E015, "an Axis with no name or extent");
        if (ex_fold(ex, &SY.ext[i])) return 1;
        if (SY.ext[i] < 1) return irx_fail(E059, "a Tile axis whose extent is below 1");
        SY.cells *= SY.ext[i];
        if (SY.cells > 2147483647LL) return irx_fail(E059, "a Tile with more than 2^31 cells");
        SY.axname[i] = nm->ref;
    }
    SY.block = k->block[0];
    SY.grid = k->grid[0];
    tot = (int64_t)SY.grid * SY.block;
    if (tot > 2147483647LL) return irx_fail(E059, "a launch with more threads than s32 holds");
    if (SY.cells > tot) return irx_fail(E059, "a Tile with more cells than the launch has threads");
    {   /* lane, warp and tid are the reference's builtin thread names (src/isel.c:877-890);
         * names compare by text, so any spelling of them in the string pool binds */
        aff_t l = aff_var(V_LANE), w = aff_var(V_WARP), t = aff_var(V_TID);
        uint32_t off;
        for (off = 1; off < k->nstr; off += (uint32_t)strlen(k->str + off) + 1u) {
            const char *s = k->str + off;
            if (!strcmp(s, "lane")) { if (bind_set(off, B_INT, 0, &l)) return 1; }
            else if (!strcmp(s, "warp")) { if (bind_set(off, B_INT, 0, &w)) return 1; }
            else if (!strcmp(s, "tid")) { if (bind_set(off, B_INT, 0, &t)) return 1; }
        }
        for (i = 0; i < ax->n; i++) {
            aff_t av = aff_var(V_TILE0 + (int)i);
            if (bind_set(SY.axname[i], B_INT, 0, &av)) return 1;
        }
    }
    return 0;
}

static int select_templates(const kir_t *k, irx_plan_int_t *p);

/* The op-family templates first; a graph they refuse at selection (a statement kind, a graph
 * shape or an index they do not take: E020, E040-E043) is written out as the generic per-graph
 * kernel (kirgen.c) instead, as the reference lowers any such graph to PTX. When that fails too,
 * the templates' refusal stands. Refusals are printed only once the outcome is known. */
int irx_select_kir(const kir_t *k, irx_plan_int_t *p)
{
    int rc, code;
    char msg[400];
    irx_defer(1);
    rc = select_templates(k, p);
    if (rc) {
        code = irx_last_code();
        if (code == E020 || code == E040 || code == E041 || code == E042 || code == E043) {
            irx_save_error(&code, msg, sizeof msg);
            if (!irx_kirgen(k, p)) {
                irx_defer(0);
                irx_clear_error();
                return 0;
            }
            irx_restore_error(code, msg);
            memset(p, 0, sizeof *p);
        }
        irx_defer(0);
        irx_emit_last();
        return 1;
    }
    irx_defer(0);
    return 0;
}

static int select_templates(const kir_t *k, irx_plan_int_t *p)
{
    const kn_t *tile;
    const kv_t *body;
    uint32_t i, j;
    int rc;

    memset(&SY, 0, sizeof SY);
    memset(p, 0, sizeof *p);
    SY.k = k;
    SY.nfv = 1;                       /* node 0 is "none" */
    SY.cur_loop = -1;
    if (k->root == 0 || k->root > k->nnode || !kir_is(k, &k->node[k->root], "Tile"))
        return irx_fail(E021, "a body that is not exactly one Tile");
    tile = &k->node[k->root];
    body = kir_fld(k, tile, "body");
    if (!body || body->tag != KV_LIST) return irx_fail(E015, "a Tile with no body list");
    for (i = 0; i < k->narg; i++)
        if (k->arg[i].dt == DT_OTHER) return irx_fail(E024, "a buffer whose dtype is not f32 or bf16");
    if (tile_setup(k, tile)) return 1;
    if (smem_prepass(body)) return 1;
    if (walk_list(body)) return 1;

    p->magic = IRX_PLAN_MAGIC;
    p->narg = (uint8_t)k->narg;
    snprintf(p->kname, sizeof p->kname, "%s", k->name);
    for (i = 0; i < k->narg; i++) {
        p->arg_kind[i] = k->arg[i].kind;
        p->arg_dt[i] = k->arg[i].dt;
        p->arg_elems[i] = arg_elems(&k->arg[i]);
        for (j = 0; j < k->nzero; j++)
            if (!strcmp(kir_str(k, k->zero[j]), kir_str(k, k->arg[i].name))) p->arg_zero[i] = 1;
    }
    if (SY.has_smem_load_global) return irx_fail(E040, "a graph that stages values through shared memory outside a reduction");
    rc = sel_pointwise(p);
    if (rc < 0) rc = sel_reduce(p);
    if (rc < 0 && any_seeded())
        return irx_fail(E042, "an Init seed other than its fold's identity outside a plain reduction");
    if (rc < 0) rc = sel_rowop(p);
    if (rc < 0) rc = sel_matmul(p);
    if (rc < 0) rc = sel_attention(p);
    if (rc < 0) return irx_fail(E040, "a graph that matches no op family with an sm_100a kernel template");
    return rc;
}
