/* kirgen.c -- the generic per-graph kernel: a KIR graph that no sm_100a template takes, written
 * out statement by statement as CUDA source and compiled by NVRTC for sm_100a.
 *
 * The op-family templates cover the graphs the benchmarks name; a graph outside them (cp.async
 * tiles of a tiled matmul, an unusual mix of folds and writes) is still a graph the reference
 * lowers to PTX (src/isel.c), so it is lowered here too instead of being refused. The source
 * follows the lockstep SIMT semantics of the reference's lowering, statement by statement:
 *
 *   * the Tile's cells are the threads gid = ctaid * block + tid, decoded row-major into the
 *     Tile's axes (src/isel.c:910-945); `lane`, `warp` and `tid` are bound as well. Cells past
 *     the Tile's size keep running with a false activity predicate, so barriers and shuffles
 *     stay uniform; every memory access and accumulator update is guarded by the predicate;
 *   * Load / Write flatten their index row-major over the buffer's dims; a read outside the
 *     buffer gives NaN and a write outside it is dropped (no fault); bf16 buffers are widened
 *     on load and rounded to nearest even on store; an atomic Write adds with red.global.add;
 *   * Assign applies the op table's function (irx_apply, kernels/ops.cuh: the same arithmetic
 *     as every other kernel here, .rn throughout, no contraction);
 *   * Accum folds with its op (from `base` when given); accumulators are graph-wide, start at
 *     the fold's identity, are reseeded by a Loop or StridedLoop that owns them (seed=true,
 *     src/isel.c:1373-1400) and set by Init (src/isel.c:1872-1900);
 *   * Loop runs its extent; StridedLoop runs from `start` by `step` below min(end, extent), per
 *     thread, or in lockstep (a block-wide vote per trip) when its body has a barrier or shuffle;
 *   * Cond narrows the activity predicate instead of branching;
 *   * Sync is a block barrier; WarpShuffle is a butterfly of shfl.xor over `length` lanes;
 *     TreeHalve halves a shared buffer with a barrier per level (src/isel.c:1718-1800);
 *   * CpAsyncCopy copies `nbytes` (4, 8 or 16) into shared memory (src/isel.c:1916-1960); its
 *     data is used after CpAsyncWait and the Sync that follows, so a synchronous copy gives the
 *     same values. CpAsyncCommit and CpAsyncWait have nothing left to do.
 *
 * Integer expressions are s32 with wrap-around, truncating division, comparisons giving 0 or 1
 * (src/kexpr.c). The kernel takes one device pointer per KIR arg, in arg order, and runs on the
 * KIR's own launch geometry, as the reference's runner launches its PTX (tests/gpurun.py:91-107).
 * The source carries no KIR names, so graphs that differ only in names share one kernel. */

#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "irx_int.h"

#define G_SRC_MAX  (256 * 1024)
#define G_MAX_NAME 2048
#define G_MAX_ACC  64
#define G_MAX_SM   16
#define G_EXPR_MAX 4096

typedef struct { uint32_t name; int cid; uint8_t flt; } gname_t;

static struct {
    const kir_t *k;
    char *p; size_t n, cap; int full;
    gname_t nm[G_MAX_NAME]; int nnm;
    int mark[256]; int nmark;
    int next;
    struct { uint32_t name; int op; int cid; int declared; } acc[G_MAX_ACC]; int nacc;
    struct { uint32_t name; int64_t dims[KIR_MAX_DIM]; int rank; int64_t elems; int cid; } sm[G_MAX_SM]; int nsm;
    int block, grid;
    int64_t cells;
    int nact;                           /* activity predicates made so far */
    int lane_cid, warp_cid, tid_cid;    /* the predefined names lane, warp, tid */
} G;

static const char *S(uint32_t off) { return kir_str(G.k, off); }

static void put(const char *fmt, ...)
{
    va_list ap;
    int w;
    if (G.full) return;
    va_start(ap, fmt);
    w = vsnprintf(G.p + G.n, G.cap - G.n, fmt, ap);
    va_end(ap);
    if (w < 0 || (size_t)w >= G.cap - G.n) { G.full = 1; return; }
    G.n += (size_t)w;
}

/* ---- names ---- */

static void scope_open(void) { if (G.nmark < 256) G.mark[G.nmark++] = G.nnm; }
static void scope_close(void) { if (G.nmark > 0) G.nnm = G.mark[--G.nmark]; }

static int name_bind(uint32_t name, int flt)
{
    if (G.nnm >= G_MAX_NAME) return -irx_fail(E081, "a graph with more names than the generic kernel holds");
    G.nm[G.nnm].name = name;
    G.nm[G.nnm].cid = G.next++;
    G.nm[G.nnm].flt = (uint8_t)flt;
    G.nnm++;
    return G.nm[G.nnm - 1].cid;
}

static int acc_index(uint32_t name)
{
    int i;
    for (i = 0; i < G.nacc; i++) if (!strcmp(S(G.acc[i].name), S(name))) return i;
    return -1;
}

static int sm_index(uint32_t name)
{
    int i;
    for (i = 0; i < G.nsm; i++) if (!strcmp(S(G.sm[i].name), S(name))) return i;
    return -1;
}

static int arg_index(uint32_t name)
{
    uint32_t i;
    for (i = 0; i < G.k->narg; i++) if (!strcmp(S(G.k->arg[i].name), S(name))) return (int)i;
    return -1;
}

/* The C spelling of a name's current value: an accumulator, or the innermost binding. */
static int name_ref(uint32_t name, char *out, size_t cap, int *flt)
{
    int i = acc_index(name);
    if (i >= 0) { snprintf(out, cap, "a%d", G.acc[i].cid); *flt = 1; return 0; }
    for (i = G.nnm - 1; i >= 0; i--)
        if (!strcmp(S(G.nm[i].name), S(name))) {
            snprintf(out, cap, "v%d", G.nm[i].cid);
            *flt = G.nm[i].flt;
            return 0;
        }
    if (G.lane_cid && !strcmp(S(name), "lane")) { snprintf(out, cap, "v%d", G.lane_cid); *flt = 0; return 0; }
    if (G.warp_cid && !strcmp(S(name), "warp")) { snprintf(out, cap, "v%d", G.warp_cid); *flt = 0; return 0; }
    if (G.tid_cid && !strcmp(S(name), "tid")) { snprintf(out, cap, "v%d", G.tid_cid); *flt = 0; return 0; }
    {
        char msg[160];
        snprintf(msg, sizeof msg, "a name the generic kernel finds unbound (%.60s)", S(name));
        return irx_fail(E028, msg);
    }
}

/* ---- expressions ---- */

/* snprintf into an expression buffer; a text that does not fit is a refusal, never a cut. */
static int fmtx(char *out, size_t cap, const char *fmt, ...)
{
    va_list ap;
    int w;
    va_start(ap, fmt);
    w = vsnprintf(out, cap, fmt, ap);
    va_end(ap);
    if (w < 0 || (size_t)w >= cap) return irx_fail(E081, "an expression longer than the generic kernel writes");
    return 0;
}

static int expr(const kv_t *v, char *out, size_t cap, int *flt);

static int expr_node(const kn_t *nd, char *out, size_t cap, int *flt)
{
    const kir_t *k = G.k;
    if (kir_is(k, nd, "Var")) {
        const kv_t *n = kir_fld(k, nd, "name");
        if (!n || n->tag != KV_STR) return irx_fail(E015, "a Var with no name");
        return name_ref(n->ref, out, cap, flt);
    }
    if (kir_is(k, nd, "Literal")) {
        const kv_t *val = kir_fld(k, nd, "value"), *d = kir_fld(k, nd, "dtype");
        if (!val) return irx_fail(E015, "a Literal with no value");
        if (val->tag == KV_FLT || (d && d->tag == KV_STR && !strcmp(S(d->ref), "float"))) {
            uint32_t bits = val->fbits;
            if (val->tag == KV_INT) { float f = (float)val->i; memcpy(&bits, &f, 4); }
            if (fmtx(out, cap, "__uint_as_float(0x%08xu)", (unsigned)bits)) return 1;
            *flt = 1;
            return 0;
        }
        if (val->tag == KV_INT || val->tag == KV_BOOL) {
            if (fmtx(out, cap, "((int)%lld)", (long long)(int32_t)val->i)) return 1;
            *flt = 0;
            return 0;
        }
        return irx_fail(E015, "a Literal whose value is not a number");
    }
    if (kir_is(k, nd, "Dim")) return expr(kir_fld(k, nd, "expr"), out, cap, flt);
    if (kir_is(k, nd, "TernaryExpr")) {
        char c[G_EXPR_MAX], t[G_EXPR_MAX], f[G_EXPR_MAX];
        int fc, ft, ff;
        if (expr(kir_fld(k, nd, "cond"), c, sizeof c, &fc) || expr(kir_fld(k, nd, "if_true"), t, sizeof t, &ft) ||
            expr(kir_fld(k, nd, "if_false"), f, sizeof f, &ff)) return 1;
        *flt = ft || ff;
        if (fmtx(out, cap, "((%s) != 0 ? %s%s : %s%s)", c, *flt && !ft ? "(float)" : "", t, *flt && !ff ? "(float)" : "", f)) return 1;
        return 0;
    }
    if (kir_is(k, nd, "BinaryExpr")) {
        const kv_t *op = kir_fld(k, nd, "op");
        char a[G_EXPR_MAX], b[G_EXPR_MAX];
        const char *o;
        int fa, fb;
        if (!op || op->tag != KV_STR) return irx_fail(E015, "a BinaryExpr with no op");
        o = S(op->ref);
        if (expr(kir_fld(k, nd, "left"), a, sizeof a, &fa) || expr(kir_fld(k, nd, "right"), b, sizeof b, &fb)) return 1;
        if (fa || fb) {                                   /* f32 arithmetic and comparisons */
            const char *fn = !strcmp(o, "+") ? "__fadd_rn" : !strcmp(o, "-") ? "__fsub_rn" : !strcmp(o, "*") ? "__fmul_rn"
                           : !strcmp(o, "/") ? "__fdiv_rn" : NULL;
            const char *ca = fa ? "" : "(float)", *cb = fb ? "" : "(float)";
            if (fn) { *flt = 1; return fmtx(out, cap, "%s(%s%s, %s%s)", fn, ca, a, cb, b); }
            if (!strcmp(o, "<") || !strcmp(o, "<=") || !strcmp(o, ">") || !strcmp(o, ">=") || !strcmp(o, "==")) {
                if (fmtx(out, cap, "((int)(%s%s %s %s%s))", ca, a, o, cb, b)) return 1;
                *flt = 0;
                return 0;
            }
            return irx_fail(E020, "a float operand of an integer-only operator");
        }
        *flt = 0;
        if (!strcmp(o, "+")) return fmtx(out, cap, "irx_iadd(%s, %s)", a, b);
        else if (!strcmp(o, "-")) return fmtx(out, cap, "irx_isub(%s, %s)", a, b);
        else if (!strcmp(o, "*")) return fmtx(out, cap, "irx_imul(%s, %s)", a, b);
        else if (!strcmp(o, "/") || !strcmp(o, "//")) return fmtx(out, cap, "irx_idiv(%s, %s)", a, b);
        else if (!strcmp(o, "%")) return fmtx(out, cap, "irx_irem(%s, %s)", a, b);
        else if (!strcmp(o, "<") || !strcmp(o, "<=") || !strcmp(o, ">") || !strcmp(o, ">=") || !strcmp(o, "=="))
            return fmtx(out, cap, "((int)((%s) %s (%s)))", a, o, b);
        else if (!strcmp(o, "&&")) return fmtx(out, cap, "((int)((%s) != 0 && (%s) != 0))", a, b);
        else if (!strcmp(o, "||")) return fmtx(out, cap, "((int)((%s) != 0 || (%s) != 0))", a, b);
        else if (!strcmp(o, "&") || !strcmp(o, "|") || !strcmp(o, "^")) return fmtx(out, cap, "((%s) %s (%s))", a, o, b);
        else if (!strcmp(o, "<<")) return fmtx(out, cap, "irx_ishl(%s, %s)", a, b);
        else if (!strcmp(o, ">>")) return fmtx(out, cap, "irx_ishr(%s, %s)", a, b);
        else {
            char msg[80];
            snprintf(msg, sizeof msg, "the expression operator '%.8s'", o);
            return irx_fail(E020, msg);
        }
        return 0;
    }
    {
        char msg[120];
        snprintf(msg, sizeof msg, "the expression kind %.60s", S(nd->kname));
        return irx_fail(E020, msg);
    }
}

static int expr(const kv_t *v, char *out, size_t cap, int *flt)
{
    if (!v) return irx_fail(E015, "a missing expression");
    if (v->tag == KV_INT || v->tag == KV_BOOL) { snprintf(out, cap, "((int)%lld)", (long long)(int32_t)v->i); *flt = 0; return 0; }
    if (v->tag == KV_FLT) { snprintf(out, cap, "__uint_as_float(0x%08xu)", (unsigned)v->fbits); *flt = 1; return 0; }
    if (v->tag == KV_STR) return name_ref(v->ref, out, cap, flt);
    if (v->tag == KV_NODE) return expr_node(kir_node(G.k, v), out, cap, flt);
    return irx_fail(E020, "an expression that is not a number, a name or a node");
}

/* A constant integer expression (extents, lengths, steps): folded here. */
static int fold(const kv_t *v, int64_t *out)
{
    const kir_t *k = G.k;
    const kn_t *nd;
    if (!v) return irx_fail(E015, "a missing constant");
    if (v->tag == KV_INT) { *out = v->i; return 0; }
    if (v->tag != KV_NODE || !(nd = kir_node(k, v))) return irx_fail(E059, "an extent that is not a constant");
    if (kir_is(k, nd, "Dim")) return fold(kir_fld(k, nd, "expr"), out);
    if (kir_is(k, nd, "Literal")) {
        const kv_t *val = kir_fld(k, nd, "value");
        if (val && val->tag == KV_INT) { *out = val->i; return 0; }
    }
    if (kir_is(k, nd, "BinaryExpr")) {
        const kv_t *op = kir_fld(k, nd, "op");
        int64_t a, b;
        if (!op || op->tag != KV_STR || fold(kir_fld(k, nd, "left"), &a) || fold(kir_fld(k, nd, "right"), &b)) return 1;
        switch (S(op->ref)[0]) {
        case '+': *out = a + b; return 0;
        case '-': *out = a - b; return 0;
        case '*': *out = a * b; return 0;
        case '/': if (b) { *out = a / b; return 0; } break;
        case '%': if (b) { *out = a % b; return 0; } break;
        default: break;
        }
    }
    return irx_fail(E059, "an extent that is not a constant");
}

/* The row-major flat index of `idx` (a list of expressions) over `dims`, as a C long long. */
static int flat_index(const kv_t *idx, const int64_t *dims, int rank, char *out, size_t cap)
{
    char e[G_EXPR_MAX], acc[G_EXPR_MAX];
    uint32_t i;
    int fl;
    if (!idx || idx->tag != KV_LIST) return irx_fail(E015, "an index that is not a list");
    if ((int)idx->n != rank && !(rank == 0 && idx->n <= 1)) return irx_fail(E041, "an index whose rank is not the buffer's");
    snprintf(acc, sizeof acc, "0LL");
    for (i = 0; i < idx->n && (int)i < rank; i++) {
        char nx[G_EXPR_MAX];
        if (expr(kir_item(G.k, idx, i), e, sizeof e, &fl)) return 1;
        if (fl) return irx_fail(E041, "a float used as an index");
        if (fmtx(nx, sizeof nx, "(%s) * %lldLL + (long long)(%s)", acc, (long long)dims[i], e)) return 1;
        memcpy(acc, nx, strlen(nx) + 1);
    }
    if (fmtx(out, cap, "(%s)", acc)) return 1;
    return 0;
}

/* A buffer by name: shared array `s<cid>` or argument `p<i>`; its dims, element count, dtype. */
typedef struct { int shared, idx; int64_t dims[KIR_MAX_DIM]; int rank; int64_t elems; int dt; } gbuf_t;

static int buffer(uint32_t name, gbuf_t *b)
{
    int i = sm_index(name);
    memset(b, 0, sizeof *b);
    if (i >= 0) {
        b->shared = 1; b->idx = G.sm[i].cid; b->rank = G.sm[i].rank; b->elems = G.sm[i].elems; b->dt = DT_F32;
        memcpy(b->dims, G.sm[i].dims, sizeof b->dims);
        return 0;
    }
    i = arg_index(name);
    if (i < 0) return irx_fail(E022, "a buffer that is neither an argument nor a declared shared array");
    {
        const ka_t *a = &G.k->arg[i];
        int d;
        b->idx = i; b->rank = a->rank; b->dt = a->dt; b->elems = 1;
        for (d = 0; d < a->rank; d++) { b->dims[d] = a->dim[d]; b->elems *= a->dim[d]; }
    }
    return 0;
}

/* ---- statements ---- */

static int body(const kv_t *lst, int act);

static void indent(int d) { int i; for (i = 0; i < d; i++) put("  "); }

static int IND;

static int op_of(const kv_t *v, int *arity)
{
    if (!v || (v->tag != KV_OP && v->tag != KV_STR)) return irx_fail(E015, "an op that is not op:<name>");
    {
        int op = irx_op_lookup(S(v->ref), arity);
        if (op == OP_NONE) {
            char msg[120];
            snprintf(msg, sizeof msg, "the op '%.40s', which is not in the op table", S(v->ref));
            return -irx_fail(E021, msg);
        }
        return op;
    }
}

static const char *ident_of(int op)
{
    return op == OP_MUL ? "1.0f" : op == OP_MAX ? "-1e30f" : op == OP_MIN ? "1e30f" : "0.0f";
}

static int is_fold(int op) { return op == OP_ADD || op == OP_MUL || op == OP_MAX || op == OP_MIN; }

static int st_load(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    const kv_t *ns = kir_fld(k, nd, "names"), *in = kir_fld(k, nd, "input"), *ix = kir_fld(k, nd, "index");
    char f[G_EXPR_MAX];
    gbuf_t b;
    uint32_t j;
    int e;
    if (!ns || ns->tag != KV_LIST || !in || in->tag != KV_STR) return irx_fail(E015, "a Load missing names or input");
    if (ns->n != 1 && ns->n != 2 && ns->n != 4) return irx_fail(E020, "a Load of a number of values other than 1, 2 or 4");
    if (buffer(in->ref, &b) || flat_index(ix, b.dims, b.rank, f, sizeof f)) return 1;
    e = G.next++;
    indent(IND); put("const long long e%d = %s;\n", e, f);
    for (j = 0; j < ns->n; j++) {
        const kv_t *nm = kir_item(k, ns, j);
        int cid;
        if (!nm || nm->tag != KV_STR) return irx_fail(E015, "a Load name that is not a string");
        if (acc_index(nm->ref) >= 0) return irx_fail(E028, "a Load into an accumulator's name");
        if ((cid = name_bind(nm->ref, 1)) < 0) return 1;
        indent(IND);
        if (b.shared)
            put("const float v%d = (c%d && e%d + %u >= 0 && e%d + %u < %lldLL) ? s%d[e%d + %u] : __int_as_float(0x7fc00000);\n",
                cid, act, e, j, e, j, (long long)b.elems, b.idx, e, j);
        else
            put("const float v%d = (c%d && e%d + %u >= 0 && e%d + %u < %lldLL) ? irx_ld_%s(P.a[%d], e%d + %u) : __int_as_float(0x7fc00000);\n",
                cid, act, e, j, e, j, (long long)b.elems, b.dt == DT_BF16 ? "bf16" : "f32", b.idx, e, j);
    }
    return 0;
}

static int st_write(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    const kv_t *out = kir_fld(k, nd, "output"), *ix = kir_fld(k, nd, "index"), *vs = kir_fld(k, nd, "values");
    const kv_t *at = kir_fld(k, nd, "atomic"), *sw = kir_fld(k, nd, "swizzle");
    const int atomic = at && at->tag == KV_BOOL && at->i;
    char f[G_EXPR_MAX], v[G_EXPR_MAX];
    gbuf_t b;
    uint32_t j;
    int e, fl;
    if (!out || out->tag != KV_STR) return irx_fail(E015, "a Write with no output name");
    if (!vs) vs = kir_fld(k, nd, "value");
    if (!vs) return irx_fail(E015, "a Write with no values");
    if (sw && sw->tag == KV_STR && strcmp(S(sw->ref), "NONE")) return irx_fail(E020, "a Write with a swizzle");
    if (vs->tag == KV_LIST && vs->n != 1 && vs->n != 2 && vs->n != 4)
        return irx_fail(E020, "a Write of a number of values other than 1, 2 or 4");
    if (buffer(out->ref, &b) || flat_index(ix, b.dims, b.rank, f, sizeof f)) return 1;
    if (!b.shared && G.k->arg[b.idx].kind != KA_OUT) return irx_fail(E029, "a Write to an argument that is not an output");
    if (atomic && (b.shared || b.dt != DT_F32)) return irx_fail(E020, "an atomic Write other than to an f32 output");
    e = G.next++;
    indent(IND); put("const long long e%d = %s;\n", e, f);
    for (j = 0; j < (vs->tag == KV_LIST ? vs->n : 1); j++) {
        if (expr(vs->tag == KV_LIST ? kir_item(k, vs, j) : vs, v, sizeof v, &fl)) return 1;
        indent(IND);
        put("if (c%d && e%d + %u >= 0 && e%d + %u < %lldLL) ", act, e, j, e, j, (long long)b.elems);
        if (b.shared) put("s%d[e%d + %u] = %s(%s);\n", b.idx, e, j, fl ? "" : "(float)", v);
        else if (atomic) put("atomicAdd((float *)P.a[%d] + e%d + %u, %s(%s));\n", b.idx, e, j, fl ? "" : "(float)", v);
        else put("irx_st_%s(P.a[%d], e%d + %u, %s(%s));\n", b.dt == DT_BF16 ? "bf16" : "f32", b.idx, e, j, fl ? "" : "(float)", v);
    }
    return 0;
}

static int st_assign(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    const kv_t *nm = kir_fld(k, nd, "name"), *as = kir_fld(k, nd, "args");
    char a[2][G_EXPR_MAX];
    uint32_t j;
    int op, ar = 0, fl, ai;
    if (!nm || nm->tag != KV_STR || !as || as->tag != KV_LIST) return irx_fail(E015, "an Assign missing name or args");
    if ((op = op_of(kir_fld(k, nd, "op"), &ar)) <= 0) return 1;
    if ((int)as->n != ar) return irx_fail(E020, "an Assign whose arg count is not the op's arity");
    snprintf(a[1], sizeof a[1], "0.0f");
    for (j = 0; j < as->n; j++) {
        char t[G_EXPR_MAX];
        if (expr(kir_item(k, as, j), t, sizeof t, &fl)) return 1;
        if (fmtx(a[j], sizeof a[j], "%s(%s)", fl ? "" : "(float)", t)) return 1;
    }
    ai = acc_index(nm->ref);
    indent(IND);
    if (ai >= 0) put("if (c%d) a%d = irx_apply(%d, %s, %s);\n", act, G.acc[ai].cid, op, a[0], a[1]);
    else {
        int cid = name_bind(nm->ref, 1);
        if (cid < 0) return 1;
        put("const float v%d = irx_apply(%d, %s, %s);   // %s\n", cid, op, a[0], a[1], irx_op_name(op));
    }
    return 0;
}

static int st_let(const kn_t *nd)
{
    const kv_t *nm = kir_fld(G.k, nd, "name");
    char v[G_EXPR_MAX];
    int fl, cid;
    if (!nm || nm->tag != KV_STR) return irx_fail(E015, "a Let with no name");
    if (expr(kir_fld(G.k, nd, "value"), v, sizeof v, &fl)) return 1;
    if ((cid = name_bind(nm->ref, fl)) < 0) return 1;
    indent(IND); put("const %s v%d = %s;\n", fl ? "float" : "int", cid, v);
    return 0;
}

static int st_accum(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    const kv_t *nm = kir_fld(k, nd, "name"), *bs = kir_fld(k, nd, "base");
    char v[G_EXPR_MAX], base[G_EXPR_MAX];
    int op, ar = 0, fl, i;
    if (!nm || nm->tag != KV_STR) return irx_fail(E015, "an Accum with no name");
    if ((op = op_of(kir_fld(k, nd, "op"), &ar)) <= 0) return 1;
    if (!is_fold(op)) return irx_fail(E021, "an Accum whose op has no identity");
    if ((i = acc_index(nm->ref)) < 0) return irx_fail(E000, "an accumulator the pre-pass did not see");
    if (expr(kir_fld(k, nd, "value"), v, sizeof v, &fl)) return 1;
    if (bs && bs->tag == KV_STR) {
        int fb;
        if (name_ref(bs->ref, base, sizeof base, &fb)) return 1;
    } else {
        snprintf(base, sizeof base, "a%d", G.acc[i].cid);
    }
    indent(IND); put("if (c%d) a%d = irx_apply(%d, %s, %s(%s));\n", act, G.acc[i].cid, op, base, fl ? "" : "(float)", v);
    return 0;
}

/* Reseed, at a loop's start, the accumulators of Accum statements directly in its body whose
 * axes name the loop's axis (or name none): src/isel.c:1373-1400. */
static void loop_seed(const kn_t *nd, uint32_t axname)
{
    const kir_t *k = G.k;
    const kv_t *bd = kir_fld(k, nd, "body"), *sd = kir_fld(k, nd, "seed");
    uint32_t i, j;
    if (sd && sd->tag == KV_BOOL && !sd->i) return;
    for (i = 0; bd && bd->tag == KV_LIST && i < bd->n; i++) {
        const kn_t *st = kir_node(k, kir_item(k, bd, i));
        const kv_t *ax, *nm;
        int own = 0, a;
        if (!st || !kir_is(k, st, "Accum")) continue;
        ax = kir_fld(k, st, "axes");
        if (!ax || ax->tag == KV_NONE) own = 1;
        else if (ax->tag == KV_LIST)
            for (j = 0; j < ax->n; j++) {
                const kv_t *x = kir_item(k, ax, j);
                if (x && x->tag == KV_STR && !strcmp(S(x->ref), S(axname))) own = 1;
            }
        nm = kir_fld(k, st, "name");
        if (!own || !nm || nm->tag != KV_STR || (a = acc_index(nm->ref)) < 0) continue;
        indent(IND); put("a%d = %s;\n", G.acc[a].cid, ident_of(G.acc[a].op));
    }
}

/* Does a statement list hold a barrier or a shuffle (at any depth)? */
static int has_collective(const kv_t *lst)
{
    const kir_t *k = G.k;
    uint32_t i;
    if (!lst || lst->tag != KV_LIST) return 0;
    for (i = 0; i < lst->n; i++) {
        const kn_t *st = kir_node(k, kir_item(k, lst, i));
        if (!st) continue;
        if (kir_is(k, st, "Sync") || kir_is(k, st, "WarpShuffle") || kir_is(k, st, "TreeHalve")) return 1;
        if (has_collective(kir_fld(k, st, "body")) || has_collective(kir_fld(k, st, "else_body"))) return 1;
    }
    return 0;
}

static int loop_axis(const kn_t *nd, uint32_t *name, int64_t *ext)
{
    const kn_t *ax = kir_node(G.k, kir_fld(G.k, nd, "axis"));
    const kv_t *nm = ax ? kir_fld(G.k, ax, "name") : NULL;
    if (!ax || !nm || nm->tag != KV_STR) return irx_fail(E015, "a loop whose axis has no name");
    if (fold(kir_fld(G.k, ax, "extent"), ext)) return 1;
    if (*ext < 1) return irx_fail(E059, "a loop whose extent is not a constant above 0");
    *name = nm->ref;
    return 0;
}

static int st_loop(const kn_t *nd, int act)
{
    uint32_t an;
    int64_t ext;
    int cid, rc;
    if (loop_axis(nd, &an, &ext)) return 1;
    loop_seed(nd, an);
    scope_open();
    if ((cid = name_bind(an, 0)) < 0) return 1;
    indent(IND); put("for (int v%d = 0; v%d < %lld; v%d++) {\n", cid, cid, (long long)ext, cid);
    IND++;
    rc = body(kir_fld(G.k, nd, "body"), act);
    IND--;
    indent(IND); put("}\n");
    scope_close();
    return rc;
}

static int st_strided(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    const kv_t *en = kir_fld(k, nd, "end");
    char st[G_EXPR_MAX], bnd[G_EXPR_MAX];
    uint32_t an;
    int64_t ext, step;
    int cid, fl, rc, m, lock;
    if (loop_axis(nd, &an, &ext)) return 1;
    if (fold(kir_fld(k, nd, "step"), &step)) return 1;
    if (step < 1) return irx_fail(E026, "a StridedLoop whose step is not a constant above 0");
    if (expr(kir_fld(k, nd, "start"), st, sizeof st, &fl)) return 1;
    if (fl) return irx_fail(E041, "a StridedLoop whose start is a float");
    if (en && en->tag != KV_NONE) {
        char e[G_EXPR_MAX];
        if (expr(en, e, sizeof e, &fl)) return 1;
        if (fmtx(bnd, sizeof bnd, "min((int)(%s), %lld)", e, (long long)ext)) return 1;
    } else {
        snprintf(bnd, sizeof bnd, "%lld", (long long)ext);
    }
    loop_seed(nd, an);
    lock = has_collective(kir_fld(k, nd, "body"));
    m = G.nact++;
    scope_open();
    if ((cid = name_bind(an, 0)) < 0) return 1;
    indent(IND); put("{ const int b%d = %s;\n", cid, bnd);
    if (!lock) {                         /* each thread runs its own trips */
        indent(IND); put("for (int v%d = %s; v%d < b%d; v%d += %lld) {\n", cid, st, cid, cid, cid, (long long)step);
        IND++;
        indent(IND); put("const bool c%d = c%d;\n", m, act);
    } else {                             /* lockstep: trips while any thread of the block has one */
        indent(IND); put("int v%d = %s;\n", cid, st);
        indent(IND); put("for (;;) {\n");
        IND++;
        indent(IND); put("const bool c%d = c%d && v%d < b%d;\n", m, act, cid, cid);
        indent(IND); put("if (!__syncthreads_or(c%d)) break;\n", m);
    }
    rc = body(kir_fld(k, nd, "body"), m);
    if (lock) { indent(IND); put("if (c%d) v%d += %lld;\n", m, cid, (long long)step); }
    IND--;
    indent(IND); put("}\n");
    indent(IND); put("}\n");
    scope_close();
    return rc;
}

static int st_cond(const kn_t *nd, int act)
{
    char c[G_EXPR_MAX];
    const kv_t *eb = kir_fld(G.k, nd, "else_body");
    int fl, m, rc;
    if (expr(kir_fld(G.k, nd, "cond"), c, sizeof c, &fl)) return 1;
    m = G.nact++;
    indent(IND); put("{ const bool c%d = c%d && ((%s) != 0);\n", m, act, c);
    IND++;
    scope_open();
    rc = body(kir_fld(G.k, nd, "body"), m);
    scope_close();
    IND--;
    indent(IND); put("}\n");
    if (rc) return 1;
    if (eb && eb->tag == KV_LIST && eb->n) {
        m = G.nact++;
        indent(IND); put("{ const bool c%d = c%d && !((%s) != 0);\n", m, act, c);
        IND++;
        scope_open();
        rc = body(eb, m);
        scope_close();
        IND--;
        indent(IND); put("}\n");
    }
    return rc;
}

static int st_sync(const kn_t *nd)
{
    const kv_t *w = kir_fld(G.k, nd, "warp");
    indent(IND);
    if (w && w->tag == KV_BOOL && w->i) put("__syncwarp();\n");
    else put("__syncthreads();\n");
    return 0;
}

/* combine_states: Assign statements in a scope of their own; or each state folded with its
 * partner by the state's own op. `mk` is the predicate under which the states change. */
static int combine(const kn_t *nd, const kv_t *states, const kv_t *others, int mk)
{
    const kir_t *k = G.k;
    const kv_t *cm = kir_fld(k, nd, "combine_states");
    uint32_t j;
    if (cm && cm->tag == KV_LIST && cm->n) {
        scope_open();
        for (j = 0; j < cm->n; j++) {
            const kn_t *a = kir_node(k, kir_item(k, cm, j));
            if (!a || !kir_is(k, a, "Assign")) return irx_fail(E027, "a combine_states statement that is not an Assign");
            if (st_assign(a, mk)) return 1;
        }
        scope_close();
        return 0;
    }
    for (j = 0; j < states->n; j++) {
        const kv_t *sn = kir_item(k, states, j), *on = kir_item(k, others, j);
        char o[64];
        int ai, fl;
        if (!sn || sn->tag != KV_STR || (ai = acc_index(sn->ref)) < 0) return irx_fail(E027, "a shuffled state that is not an accumulator");
        if (!on || on->tag != KV_STR || name_ref(on->ref, o, sizeof o, &fl)) return 1;
        indent(IND); put("if (c%d) a%d = irx_apply(%d, a%d, %s);\n", mk, G.acc[ai].cid, G.acc[ai].op, G.acc[ai].cid, o);
    }
    return 0;
}

static int st_shuffle(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    const kv_t *states = kir_fld(k, nd, "state"), *others = kir_fld(k, nd, "state_b");
    int64_t len, h;
    uint32_t j;
    if (fold(kir_fld(k, nd, "length"), &len)) return 1;
    if (len < 1 || len > 32 || (len & (len - 1)) || G.block % 32)
        return irx_fail(E034, "a warp shuffle whose length is not a power of two up to 32");
    if (!states || states->tag != KV_LIST || !others || others->tag != KV_LIST || states->n != others->n)
        return irx_fail(E015, "a WarpShuffle whose states and partners do not pair up");
    for (h = len / 2; h >= 1; h /= 2) {
        indent(IND); put("{\n");
        IND++;
        scope_open();
        for (j = 0; j < states->n; j++) {
            const kv_t *sn = kir_item(k, states, j), *on = kir_item(k, others, j);
            char sv[64];
            int fl, cid;
            if (!sn || sn->tag != KV_STR || !on || on->tag != KV_STR) return irx_fail(E015, "a WarpShuffle name that is not a string");
            if (name_ref(sn->ref, sv, sizeof sv, &fl) || (cid = name_bind(on->ref, 1)) < 0) return 1;
            indent(IND); put("const float v%d = __shfl_xor_sync(0xffffffffu, %s, %lld);\n", cid, sv, (long long)h);
        }
        if (combine(nd, states, others, act)) return 1;
        scope_close();
        IND--;
        indent(IND); put("}\n");
    }
    return 0;
}

static int st_tree(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    const kv_t *states = kir_fld(k, nd, "state"), *others = kir_fld(k, nd, "state_b"), *bufs = kir_fld(k, nd, "bufs");
    const kv_t *in = kir_fld(k, nd, "inner"), *tvn = kir_fld(k, nd, "tid_var");
    char tv[G_EXPR_MAX];
    int64_t len, r;
    uint32_t j;
    int fl;
    if (in && in->tag != KV_NONE) return irx_fail(E020, "a tree with an inner state");
    if (fold(kir_fld(k, nd, "length"), &len)) return 1;
    if (len < 1 || (len & (len - 1))) return irx_fail(E020, "a tree whose length is not a power of two");
    if (!states || states->tag != KV_LIST || !others || others->tag != KV_LIST || !bufs || bufs->tag != KV_LIST ||
        states->n != others->n || bufs->n != states->n) return irx_fail(E020, "a tree whose buffers and states do not pair up");
    if (!tvn || expr(tvn, tv, sizeof tv, &fl)) return irx_fail(E015, "a tree with no tid_var");
    for (r = len / 2; r >= 1; r /= 2) {
        const int m = G.nact++;
        indent(IND); put("__syncthreads();\n");
        indent(IND); put("{ const bool c%d = c%d && (%s) < %lld;\n", m, act, tv, (long long)r);
        IND++;
        scope_open();
        for (j = 0; j < bufs->n; j++) {
            const kv_t *bn = kir_item(k, bufs, j), *on = kir_item(k, others, j);
            int si, cid;
            if (!bn || bn->tag != KV_STR || (si = sm_index(bn->ref)) < 0) return irx_fail(E022, "a tree buffer that is not a declared shared array");
            if (!on || on->tag != KV_STR || (cid = name_bind(on->ref, 1)) < 0) return 1;
            indent(IND); put("const float v%d = c%d ? s%d[(%s) + %lld] : 0.0f;\n", cid, m, G.sm[si].cid, tv, (long long)r);
        }
        if (combine(nd, states, others, m)) return 1;
        for (j = 0; j < bufs->n; j++) {
            const kv_t *bn = kir_item(k, bufs, j), *sn = kir_item(k, states, j);
            char sv[64];
            int f2;
            if (!sn || sn->tag != KV_STR || name_ref(sn->ref, sv, sizeof sv, &f2)) return 1;
            indent(IND); put("if (c%d) s%d[%s] = %s;\n", m, G.sm[sm_index(bn->ref)].cid, tv, sv);
        }
        scope_close();
        IND--;
        indent(IND); put("}\n");
    }
    indent(IND); put("__syncthreads();\n");
    /* buf[0] holds the total: every state is loaded from it (src/isel.c:1800-1840) */
    for (j = 0; j < bufs->n; j++) {
        const kv_t *bn = kir_item(k, bufs, j), *sn = kir_item(k, states, j);
        const int si = sm_index(bn->ref), ai = acc_index(sn->ref);
        indent(IND);
        if (ai >= 0) put("if (c%d) a%d = s%d[0];\n", act, G.acc[ai].cid, G.sm[si].cid);
        else {
            int cid = name_bind(sn->ref, 1);
            if (cid < 0) return 1;
            put("const float v%d = s%d[0];\n", cid, G.sm[si].cid);
        }
    }
    return 0;
}

static int st_cpasync(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    const kv_t *sm = kir_fld(k, nd, "smem"), *si = kir_fld(k, nd, "smem_index"), *src = kir_fld(k, nd, "src");
    const kv_t *ri = kir_fld(k, nd, "src_index"), *nb = kir_fld(k, nd, "nbytes"), *sw = kir_fld(k, nd, "swizzle");
    const kv_t *li = kir_fld(k, nd, "lane_index");
    char fs[G_EXPR_MAX], fl2[G_EXPR_MAX], fg[G_EXPR_MAX];
    gbuf_t sb, gb;
    int e, d, n;
    if (!sm || sm->tag != KV_STR) return irx_fail(E015, "a CpAsyncCopy with no smem name");
    if (!si || si->tag != KV_LIST) return irx_fail(E015, "a CpAsyncCopy with no smem_index");
    if (!src || src->tag != KV_STR) return irx_fail(E015, "a CpAsyncCopy with no src name");
    if (!ri || ri->tag != KV_LIST) return irx_fail(E015, "a CpAsyncCopy with no src_index");
    if (!nb || nb->tag != KV_INT) return irx_fail(E015, "a CpAsyncCopy with no nbytes");
    if (nb->i != 4 && nb->i != 8 && nb->i != 16) return irx_fail(E020, "a CpAsyncCopy whose nbytes is not 4, 8 or 16");
    if (sw && sw->tag == KV_STR && strcmp(S(sw->ref), "NONE")) return irx_fail(E020, "a CpAsyncCopy with a swizzle");
    if (sm_index(sm->ref) < 0) return irx_fail(E022, "a CpAsyncCopy whose smem is not declared");
    if (buffer(sm->ref, &sb) || flat_index(si, sb.dims, sb.rank, fs, sizeof fs)) return 1;
    if (li && li->tag == KV_LIST) {
        if (flat_index(li, sb.dims, sb.rank, fl2, sizeof fl2)) return 1;
    } else {
        snprintf(fl2, sizeof fl2, "0LL");
    }
    if (buffer(src->ref, &gb) || gb.shared) return irx_fail(E022, "a CpAsyncCopy whose src is not an argument");
    if (gb.dt != DT_F32) return irx_fail(E024, "a CpAsyncCopy of a buffer whose dtype is not f32");
    if (flat_index(ri, gb.dims, gb.rank, fg, sizeof fg)) return 1;
    e = G.next++;
    d = G.next++;
    n = (int)(nb->i / 4);
    indent(IND); put("{ const long long e%d = %s, e%d = %s + %s;\n", e, fg, d, fs, fl2);
    indent(IND); put("  if (c%d) for (int j = 0; j < %d; j++)\n", act, n);
    indent(IND); put("    if (e%d + j >= 0 && e%d + j < %lldLL && e%d + j >= 0 && e%d + j < %lldLL) s%d[e%d + j] = ((const float *)P.a[%d])[e%d + j];\n",
                     d, d, (long long)sb.elems, e, e, (long long)gb.elems, sb.idx, d, gb.idx, e);
    indent(IND); put("}\n");
    return 0;
}

static int stmt(const kn_t *nd, int act)
{
    const kir_t *k = G.k;
    if (kir_is(k, nd, "Load")) return st_load(nd, act);
    if (kir_is(k, nd, "Write")) return st_write(nd, act);
    if (kir_is(k, nd, "Assign")) return st_assign(nd, act);
    if (kir_is(k, nd, "Let")) return st_let(nd);
    if (kir_is(k, nd, "Accum")) return st_accum(nd, act);
    if (kir_is(k, nd, "Init")) {
        const kv_t *nm = kir_fld(k, nd, "name"), *iv = kir_fld(k, nd, "identity");
        uint32_t bits;
        int a;
        if (!nm || nm->tag != KV_STR || !iv) return irx_fail(E015, "an Init missing name or identity");
        if (iv->tag == KV_FLT) bits = iv->fbits;
        else if (iv->tag == KV_INT) { float f = (float)iv->i; memcpy(&bits, &f, 4); }
        else return irx_fail(E015, "an Init whose identity is not a number");
        if ((a = acc_index(nm->ref)) < 0) return 0;          /* an Init no Accum uses */
        indent(IND); put("a%d = __uint_as_float(0x%08xu);\n", G.acc[a].cid, (unsigned)bits);
        return 0;
    }
    if (kir_is(k, nd, "Loop")) return st_loop(nd, act);
    if (kir_is(k, nd, "StridedLoop")) return st_strided(nd, act);
    if (kir_is(k, nd, "Cond")) return st_cond(nd, act);
    if (kir_is(k, nd, "Smem")) return 0;                      /* declared at the kernel's top */
    if (kir_is(k, nd, "Sync")) return st_sync(nd);
    if (kir_is(k, nd, "WarpShuffle")) return st_shuffle(nd, act);
    if (kir_is(k, nd, "TreeHalve")) return st_tree(nd, act);
    if (kir_is(k, nd, "CpAsyncCopy")) return st_cpasync(nd, act);
    if (kir_is(k, nd, "CpAsyncCommit") || kir_is(k, nd, "CpAsyncWait")) return 0;
    {
        char msg[120];
        snprintf(msg, sizeof msg, "a %.60s statement", S(nd->kname));
        return irx_fail(E020, msg);
    }
}

static int body(const kv_t *lst, int act)
{
    uint32_t i;
    if (!lst || lst->tag == KV_NONE) return 0;
    if (lst->tag != KV_LIST) return irx_fail(E015, "a body that is not a list");
    for (i = 0; i < lst->n; i++) {
        const kn_t *st = kir_node(G.k, kir_item(G.k, lst, i));
        if (!st) return irx_fail(E015, "a body item that is not a statement");
        if (stmt(st, act)) return 1;
        if (G.full) return irx_fail(E081, "a generic kernel source longer than its buffer");
    }
    return 0;
}

/* Pre-pass: shared arrays, and every accumulator (with its fold) in the graph. */
static int prepass(const kv_t *lst)
{
    const kir_t *k = G.k;
    uint32_t i, j;
    if (!lst || lst->tag != KV_LIST) return 0;
    for (i = 0; i < lst->n; i++) {
        const kn_t *st = kir_node(k, kir_item(k, lst, i));
        if (!st) continue;
        if (kir_is(k, st, "Smem")) {
            const kv_t *nm = kir_fld(k, st, "name"), *ex = kir_fld(k, st, "extents"), *d = kir_fld(k, st, "dtype");
            if (!nm || nm->tag != KV_STR || !ex || ex->tag != KV_LIST) return irx_fail(E015, "an Smem missing name or extents");
            if (d && d->tag == KV_DT && strcmp(S(d->ref), "f32")) return irx_fail(E024, "a shared array whose dtype is not f32");
            if (sm_index(nm->ref) >= 0) continue;
            if (G.nsm >= G_MAX_SM || ex->n > KIR_MAX_DIM) return irx_fail(E081, "more shared arrays than the generic kernel holds");
            G.sm[G.nsm].name = nm->ref;
            G.sm[G.nsm].rank = (int)ex->n;
            G.sm[G.nsm].elems = 1;
            for (j = 0; j < ex->n; j++) {
                if (fold(kir_item(k, ex, j), &G.sm[G.nsm].dims[j])) return 1;
                if (G.sm[G.nsm].dims[j] < 1) return irx_fail(E059, "a shared array with an empty extent");
                G.sm[G.nsm].elems *= G.sm[G.nsm].dims[j];
            }
            G.sm[G.nsm].cid = G.next++;
            G.nsm++;
        }
        if (kir_is(k, st, "Accum") || kir_is(k, st, "Init")) {
            const kv_t *nm = kir_fld(k, st, "name");
            int a, op = OP_NONE, ar = 0;
            if (!nm || nm->tag != KV_STR) return irx_fail(E015, "an accumulator with no name");
            if (kir_is(k, st, "Accum")) {
                if ((op = op_of(kir_fld(k, st, "op"), &ar)) <= 0) return 1;
                if (!is_fold(op)) return irx_fail(E021, "an Accum whose op has no identity");
            }
            if ((a = acc_index(nm->ref)) < 0) {
                if (G.nacc >= G_MAX_ACC) return irx_fail(E081, "more accumulators than the generic kernel holds");
                a = G.nacc++;
                G.acc[a].name = nm->ref;
                G.acc[a].op = op;
                G.acc[a].cid = G.next++;
            } else if (op != OP_NONE) {
                if (G.acc[a].op == OP_NONE) G.acc[a].op = op;
                else if (G.acc[a].op != op) return irx_fail(E027, "an accumulator folded with two different ops");
            }
        }
        if (prepass(kir_fld(k, st, "body")) || prepass(kir_fld(k, st, "else_body"))) return 1;
    }
    return 0;
}

static const char GEN_HEAD[] =
    "#include \"ops.cuh\"\n"
    "typedef struct { void *a[32]; } irx_kkir_t;\n"
    "__device__ __forceinline__ int irx_iadd(int a, int b) { return (int)((unsigned)a + (unsigned)b); }\n"
    "__device__ __forceinline__ int irx_isub(int a, int b) { return (int)((unsigned)a - (unsigned)b); }\n"
    "__device__ __forceinline__ int irx_imul(int a, int b) { return (int)((unsigned)a * (unsigned)b); }\n"
    "__device__ __forceinline__ int irx_idiv(int a, int b) { return b == 0 ? 0 : (b == -1 ? (int)(0u - (unsigned)a) : a / b); }\n"
    "__device__ __forceinline__ int irx_irem(int a, int b) { return b == 0 || b == -1 ? 0 : a % b; }\n"
    "__device__ __forceinline__ int irx_ishl(int a, int b) { return b < 0 ? a : b >= 32 ? 0 : (int)((unsigned)a << b); }\n"
    "__device__ __forceinline__ int irx_ishr(int a, int b) { return a >> (b < 0 ? 0 : b > 31 ? 31 : b); }\n"
    "__device__ __forceinline__ float irx_ld_f32(const void *p, long long e) { return ((const float *)p)[e]; }\n"
    "__device__ __forceinline__ float irx_ld_bf16(const void *p, long long e) { return __uint_as_float((unsigned)((const unsigned short *)p)[e] << 16); }\n"
    "__device__ __forceinline__ void irx_st_f32(void *p, long long e, float v) { ((float *)p)[e] = v; }\n"
    "__device__ __forceinline__ void irx_st_bf16(void *p, long long e, float v) { unsigned short h; asm(\"cvt.rn.bf16.f32 %0, %1;\" : \"=h\"(h) : \"f\"(v)); ((unsigned short *)p)[e] = h; }\n";

int irx_kirgen_source(const kir_t *k, char *buf, size_t cap, int32_t *grid, int32_t *block, int64_t *cells);

/* The kernel source for graph k into buf (cap bytes); its launch geometry and cell count. */
int irx_kirgen_source(const kir_t *k, char *buf, size_t cap, int32_t *grid, int32_t *block, int64_t *cells)
{
    const kn_t *tile;
    const kv_t *axes, *bd;
    int64_t ext[KIR_MAX_DIM], n = 1, stride;
    int cid[KIR_MAX_DIM], na = 0, i, c_lane, c_warp, c_tid;
    (void)cid;
    uint32_t j;

    memset(&G, 0, sizeof G);
    G.k = k;
    G.p = buf; G.cap = cap;
    G.next = 1;
    if (k->grid[1] != 1 || k->grid[2] != 1 || k->block[1] != 1 || k->block[2] != 1)
        return irx_fail(E025, "a launch with y or z beyond 1");
    G.grid = k->grid[0];
    G.block = k->block[0];
    if (G.block < 1 || G.block > 1024 || G.grid < 1) return irx_fail(E025, "a launch outside 1..1024 threads a block");
    if (k->root == 0 || k->root > k->nnode || !kir_is(k, &k->node[k->root], "Tile"))
        return irx_fail(E021, "a body that is not exactly one Tile");
    tile = &k->node[k->root];
    axes = kir_fld(k, tile, "axes");
    bd = kir_fld(k, tile, "body");
    if (!axes || axes->tag != KV_LIST || axes->n > KIR_MAX_DIM) return irx_fail(E015, "a Tile with no axis list");
    for (j = 0; j < k->narg; j++)
        if (k->arg[j].dt != DT_F32 && k->arg[j].dt != DT_BF16) return irx_fail(E024, "a buffer whose dtype is not f32 or bf16");
    for (j = 0; j < axes->n; j++) {
        const kn_t *ax = kir_node(k, kir_item(k, axes, j));
        if (!ax || fold(kir_fld(k, ax, "extent"), &ext[na])) return 1;
        if (ext[na] < 1) return irx_fail(E059, "a Tile axis with an empty extent");
        n *= ext[na];
        na++;
    }
    if (n > (int64_t)G.grid * G.block) return irx_fail(E059, "a Tile with more cells than the launch has threads");
    if (prepass(bd)) return 1;
    {
        int64_t smb = 0;
        for (i = 0; i < G.nsm; i++) smb += G.sm[i].elems * 4;
        if (smb > 48 * 1024) return irx_fail(E081, "shared arrays beyond 48 KiB in a generic kernel");
    }

    put("// irptx-b200 generic per-graph kernel: %d-thread blocks, %lld cells\n%s", G.block, (long long)n, GEN_HEAD);
    put("extern \"C\" __global__ void __launch_bounds__(%d) irx_kir(const __grid_constant__ irx_kkir_t P) {\n", G.block);
    for (i = 0; i < G.nsm; i++) put("  __shared__ float s%d[%lld];\n", G.sm[i].cid, (long long)G.sm[i].elems);
    for (i = 0; i < G.nacc; i++) put("  float a%d = %s;\n", G.acc[i].cid, ident_of(G.acc[i].op));
    put("  const int g = (int)(blockIdx.x * blockDim.x + threadIdx.x);\n");
    put("  const bool c0 = g < %lld;\n", (long long)n);
    G.nact = 1;
    IND = 1;
    scope_open();
    stride = n;
    for (j = 0; j < axes->n; j++) {
        const kn_t *ax = kir_node(k, kir_item(k, axes, j));
        const kv_t *nm = kir_fld(k, ax, "name");
        if (!nm || nm->tag != KV_STR) return irx_fail(E015, "a Tile axis with no name");
        stride /= ext[j];
        if ((cid[j] = name_bind(nm->ref, 0)) < 0) return 1;
        if (j == 0) put("  const int v%d = (int)((long long)g / %lldLL);\n", cid[j], (long long)stride);
        else put("  const int v%d = (int)(((long long)g / %lldLL) %% %lldLL);\n", cid[j], (long long)stride, (long long)ext[j]);
    }
    c_lane = G.next++; c_warp = G.next++; c_tid = G.next++;     /* lane, warp, tid (read through name_ref) */
    put("  const int v%d = (int)(threadIdx.x & 31), v%d = (int)(threadIdx.x >> 5), v%d = (int)threadIdx.x;\n", c_lane, c_warp, c_tid);
    G.lane_cid = c_lane; G.warp_cid = c_warp; G.tid_cid = c_tid;
    if (body(bd, 0)) return 1;
    scope_close();
    put("}\n");
    if (G.full) return irx_fail(E081, "a generic kernel source longer than its buffer");
    *grid = G.grid;
    *block = G.block;
    *cells = n;
    return 0;
}

int irx_jit_store(const char *src, size_t n, uint64_t *key);

/* Select the generic kernel for graph k: write its source, keep it in the per-graph kernel store,
 * and fill the plan (family FAM_KIR, the KIR's launch geometry, the store key). */
int irx_kirgen(const kir_t *k, irx_plan_int_t *p)
{
    char *src = (char *)malloc(G_SRC_MAX);
    int32_t grid = 0, block = 0;
    int64_t cells = 0;
    uint64_t key = 0;
    uint32_t i, j;
    if (!src) return irx_fail(E094, "host memory for a generic kernel's source");
    if (irx_kirgen_source(k, src, G_SRC_MAX, &grid, &block, &cells)) { free(src); return 1; }
    if (irx_jit_store(src, G.n, &key)) { free(src); return 1; }
    free(src);
    memset(p, 0, sizeof *p);
    p->magic = IRX_PLAN_MAGIC;
    p->fam = FAM_KIR;
    p->narg = (uint8_t)k->narg;
    snprintf(p->kname, sizeof p->kname, "%s", k->name);
    for (i = 0; i < k->narg; i++) {
        int64_t e = 1;
        int d;
        for (d = 0; d < k->arg[i].rank; d++) e *= k->arg[i].dim[d];
        p->arg_kind[i] = k->arg[i].kind;
        p->arg_dt[i] = k->arg[i].dt;
        p->arg_elems[i] = e;
        for (j = 0; j < k->nzero; j++)
            if (!strcmp(kir_str(k, k->zero[j]), kir_str(k, k->arg[i].name))) p->arg_zero[i] = 1;
    }
    p->u.kk.key = key;
    p->u.kk.grid = grid;
    p->u.kk.block = block;
    p->u.kk.cells = cells;
    return 0;
}
