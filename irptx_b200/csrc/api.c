/* api.c -- the public C ABI (include/irx.h): compile, describe, launch, shard, host path.
 *
 * irx_compile runs the KIR reader and the selector under one lock (the parse pools are
 * large and static, as the reference's are, src/kir.c:23-24) and copies the result into the
 * caller's plan. Everything after that works from the plan alone. */

#include <pthread.h>
#include <stdio.h>
#include <string.h>
#include "irx_int.h"
#include "irx_kparams.h"
#include "launch.h"
#include "jit.h"
#include "../../include/irx.h"

typedef char plan_fits[(sizeof(irx_plan_int_t) <= IRX_PLAN_BYTES) ? 1 : -1];

static kir_t KIR;
static int prog_temps(const irx_pw_t *pw);
static pthread_mutex_t CLOCK = PTHREAD_MUTEX_INITIALIZER;

const char *irx_version(void) { return "irptx-b200 " IRX_VERSION; }

void irx_quiet(int on) { irx_set_quiet(on); }

int irx_last_error(char *buf, size_t cap)
{
    if (buf && cap) snprintf(buf, cap, "%s", irx_last_msg());
    return irx_last_code();
}

static const irx_plan_int_t *P(const irx_plan_t *plan)
{
    const irx_plan_int_t *p = (const irx_plan_int_t *)plan;
    return p && p->magic == IRX_PLAN_MAGIC ? p : NULL;
}

int irx_compile(const char *kir, size_t len, irx_plan_t *plan)
{
    int rc;
    irx_plan_int_t *p = (irx_plan_int_t *)plan;
    if (!plan) return irx_fail(E093, "a compile with no plan storage");
    irx_clear_error();
    memset(plan, 0, sizeof *plan);
    pthread_mutex_lock(&CLOCK);
    rc = kir_load(&KIR, kir, len);
    if (!rc) rc = irx_select_kir(&KIR, p);
    pthread_mutex_unlock(&CLOCK);
    if (rc) memset(plan, 0, sizeof *plan);
    else if (p->fam == FAM_POINTWISE) p->u.pw.jit_key = irx_jit_key(p);
    return rc;
}

int irx_compile_generic(const char *kir, size_t len, irx_plan_t *plan)
{
    int rc;
    irx_plan_int_t *p = (irx_plan_int_t *)plan;
    if (!plan) return irx_fail(E093, "a compile with no plan storage");
    irx_clear_error();
    memset(plan, 0, sizeof *plan);
    pthread_mutex_lock(&CLOCK);
    rc = kir_load(&KIR, kir, len);
    if (!rc) rc = irx_kirgen(&KIR, p);
    pthread_mutex_unlock(&CLOCK);
    if (rc) memset(plan, 0, sizeof *plan);
    return rc;
}

int irx_plan_family(const irx_plan_t *plan)
{
    const irx_plan_int_t *p = P(plan);
    return p ? p->fam : 0;
}

int irx_plan_nargs(const irx_plan_t *plan)
{
    const irx_plan_int_t *p = P(plan);
    return p ? p->narg : 0;
}

int irx_plan_arg(const irx_plan_t *plan, unsigned i, int *kind, int *dtype, long long *elems)
{
    const irx_plan_int_t *p = P(plan);
    if (!p || i >= p->narg) return irx_fail(E093, "an argument index past the plan's arguments");
    if (kind) *kind = p->arg_kind[i];
    if (dtype) *dtype = p->arg_dt[i];
    if (elems) *elems = p->arg_elems[i];
    return 0;
}

static int esz(int dt) { return dt == DT_BF16 ? 2 : 4; }

static void prog_text(const irx_prog_t *g, char *b, size_t cap)
{
    size_t o = 0;
    int i;
    b[0] = '\0';
    for (i = 0; i < g->nins && o + 24 < cap; i++)
        o += (size_t)snprintf(b + o, cap - o, "%sr%d=%s(r%d%s%d)", i ? ";" : "", g->ins[i].dst, irx_op_name(g->ins[i].op),
                              g->ins[i].a, irx_op_arity(g->ins[i].op) == 2 ? ",r" : "", irx_op_arity(g->ins[i].op) == 2 ? g->ins[i].b : -1);
    if (o + 12 < cap) snprintf(b + o, cap - o, "%s->r%d", i ? "" : "", g->out);
}

int irx_plan_describe(const irx_plan_t *plan, char *buf, size_t cap)
{
    const irx_plan_int_t *p = P(plan);
    char pr[400];
    if (!p) return irx_fail(E093, "a plan that was never compiled");
    if (!buf || !cap) return 0;
    switch (p->fam) {
    case FAM_POINTWISE:
        prog_text(&p->u.pw.prog[0], pr, sizeof pr);
        if (irx_jit_mode(-1))              /* the graph's own kernel, compiled at run time */
            snprintf(buf, cap, "pointwise n=%lld in=%d out=%d uni=%d prog=[%s] kernel=irx_pwj(%016llx)",
                     (long long)p->u.pw.n, p->u.pw.nin, p->u.pw.nout, p->u.pw.nuni, pr,
                     (unsigned long long)p->u.pw.jit_key);
        else
            snprintf(buf, cap, "pointwise n=%lld in=%d out=%d uni=%d prog=[%s] kernel=irx_pw_s%d_t%d",
                     (long long)p->u.pw.n, p->u.pw.nin, p->u.pw.nout, p->u.pw.nuni, pr, p->u.pw.nin ? p->u.pw.nin : 1,
                     prog_temps(&p->u.pw) > 1 ? 8 : 1);
        break;
    case FAM_REDUCE_ALL:
    case FAM_REDUCE_ROWS:
        snprintf(buf, cap, "%s op=%s rows=%lld cols=%lld pre=%d accumulate=%d kernel=%s",
                 p->fam == FAM_REDUCE_ALL ? "reduce_all" : "reduce_rows", irx_op_name(p->u.red.op),
                 (long long)p->u.red.rows, (long long)p->u.red.cols, p->u.red.has_pre, p->u.red.accumulate,
                 p->fam == FAM_REDUCE_ALL && p->u.red.rows == 1 ? (p->u.red.has_pre ? "irx_red_all_p1" : "irx_red_all_p0")
                                                           : (p->u.red.has_pre ? "irx_red_rows_p1" : "irx_red_rows_p0"));
        break;
    case FAM_ROWOP: {
        static const char *const KN[] = {"generic", "rmsnorm", "softmax", "l2norm"};
        static const char *const KK[] = {"irx_rowop", "irx_row_rmsnorm", "irx_row_softmax", "irx_row_l2norm"};
        prog_text(&p->u.row.epi, pr, sizeof pr);
        snprintf(buf, cap, "rowop kind=%s rows=%lld cols=%lld stats=%d w=%d dtype=%s epi=[%s] kernel=%s",
                 KN[p->u.row.kind & 3], (long long)p->u.row.rows, (long long)p->u.row.cols, p->u.row.nstat,
                 p->u.row.has_w, p->u.row.x_dt == DT_BF16 ? "bf16" : "f32", pr,
                 KK[(p->u.row.cols % 8) ? 0 : (p->u.row.kind & 3)]);
        break;
    }
    case FAM_MATMUL:
        snprintf(buf, cap, "matmul m=%lld n=%lld k=%lld dtype=%s b=%s kernel=%s", (long long)p->u.mm.m,
                 (long long)p->u.mm.n, (long long)p->u.mm.k, p->u.mm.dt == DT_BF16 ? "bf16" : "f32",
                 p->u.mm.b_kmajor ? "[n,k]" : "[k,n]",
                 p->u.mm.dt != DT_BF16 ? "irx_mm_f32" : p->u.mm.m <= 128 ? "irx_mm_bf16"
                 : p->u.mm.n % 8 == 0 ? "irx_mm_bf16_wide" : "irx_mm_bf16_pair");
        break;
    case FAM_ATTENTION: {
        float sc;
        memcpy(&sc, &p->u.at.scale_bits, 4);
        const irx_at_t *a = &p->u.at;
        const int tc = a->dt == DT_BF16 && a->sq == a->sk && a->dqk == 128 && a->dv == 128 && !a->k_t && a->sq % 128 == 0;
        if (a->sq == a->sk && a->dqk == a->dv && !a->k_t)
            snprintf(buf, cap, "attention b=%lld h=%lld s=%lld d=%lld causal=%d scale=%g dtype=%s kernel=%s",
                     (long long)a->b, (long long)a->h, (long long)a->s, (long long)a->d, a->causal, (double)sc,
                     a->dt == DT_BF16 ? "bf16" : "f32",
                     tc ? "irx_attn_bf16" : a->dt == DT_BF16 ? "irx_attn_bf16_simt" : "irx_attn_f32");
        else
            snprintf(buf, cap, "attention b=%lld h=%lld sq=%lld sk=%lld dqk=%lld dv=%lld k=%s causal=%d scale=%g dtype=%s kernel=%s",
                     (long long)a->b, (long long)a->h, (long long)a->sq, (long long)a->sk, (long long)a->dqk,
                     (long long)a->dv, a->k_t ? "[d,j]" : "[j,d]", a->causal, (double)sc,
                     a->dt == DT_BF16 ? "bf16" : "f32", a->dt == DT_BF16 ? "irx_attn_bf16_simt" : "irx_attn_f32");
        break;
    }
    case FAM_KIR:
        snprintf(buf, cap, "kir grid=%d block=%d cells=%lld args=%d kernel=irx_kir(%016llx)", (int)p->u.kk.grid,
                 (int)p->u.kk.block, (long long)p->u.kk.cells, p->narg, (unsigned long long)p->u.kk.key);
        break;
    default:
        snprintf(buf, cap, "none");
    }
    return 0;
}

int irx_plan_work(const irx_plan_t *plan, double *bytes, double *flops)
{
    const irx_plan_int_t *p = P(plan);
    double b = 0, f = 0;
    int i;
    if (!p) return irx_fail(E093, "a plan that was never compiled");
    switch (p->fam) {
    case FAM_POINTWISE:
        for (i = 0; i < p->u.pw.nin; i++) b += (double)p->u.pw.n * esz(p->u.pw.in_dt[i]);
        for (i = 0; i < p->u.pw.nout; i++) b += (double)p->u.pw.n * esz(p->u.pw.out_dt[i]);
        break;
    case FAM_REDUCE_ALL:
    case FAM_REDUCE_ROWS:
        b = (double)p->u.red.rows * p->u.red.cols * esz(p->u.red.x_dt) + (double)p->u.red.rows * esz(p->u.red.y_dt);
        break;
    case FAM_ROWOP:
        b = (double)p->u.row.rows * p->u.row.cols * (esz(p->u.row.x_dt) + esz(p->u.row.y_dt));
        if (p->u.row.has_w) b += (double)p->u.row.cols * esz(p->u.row.w_dt);
        break;
    case FAM_MATMUL:
        f = 2.0 * p->u.mm.m * p->u.mm.n * p->u.mm.k;
        b = ((double)p->u.mm.m * p->u.mm.k + (double)p->u.mm.k * p->u.mm.n + (double)p->u.mm.m * p->u.mm.n) * esz(p->u.mm.dt);
        break;
    case FAM_ATTENTION:
        {   /* Q K^T and P V: 2 Sq Sk (Dqk + Dv) per batch-head; Q, K, V read and O written once */
            const irx_at_t *a = &p->u.at;
            const double bh = (double)a->b * (double)a->h;
            f = 2.0 * bh * a->sq * a->sk * (double)(a->dqk + a->dv);
            if (a->causal) f *= 0.5;
            b = bh * ((double)a->sq * a->dqk + (double)a->sk * a->dqk + (double)a->sk * a->dv + (double)a->sq * a->dv) *
                esz(a->dt);
        }
        break;
    case FAM_KIR:                        /* every argument read or written once */
        for (i = 0; i < p->narg; i++) b += (double)p->arg_elems[i] * esz(p->arg_dt[i]);
        break;
    default:
        break;
    }
    if (bytes) *bytes = b;
    if (flops) *flops = f;
    return 0;
}

#define MM_TILE_N 256

long long irx_plan_units(const irx_plan_t *plan)
{
    const irx_plan_int_t *p = P(plan);
    if (!p) return 0;
    switch (p->fam) {
    case FAM_POINTWISE: return (p->u.pw.n + 7) / 8;
    case FAM_REDUCE_ALL: return p->u.red.rows == 1 ? (p->u.red.cols + 7) / 8 : p->u.red.rows;
    case FAM_REDUCE_ROWS: return p->u.red.rows;
    case FAM_ROWOP: return p->u.row.rows;
    case FAM_MATMUL: return (p->u.mm.n + MM_TILE_N - 1) / MM_TILE_N;
    case FAM_ATTENTION: return p->u.at.b * p->u.at.h;
    case FAM_KIR: return 1;              /* one launch of the KIR's own geometry */
    default: return 0;
    }
}

/* ---- family launchers ---- */

/* The pipelined host path launches a shard one chunk of its units at a time: while a window is
 * set on this thread, every unit range a launcher takes is narrowed to it. */
static _Thread_local long long WIN_A, WIN_B = -1;

void irx_unit_window(long long a, long long b)
{
    WIN_A = a;
    WIN_B = b;
}

/* Shard s of ns: units [u0, u1), ceil(units / ns) of them per shard, the last one short. Every
 * family launcher, the host path's slices and irx_plan_shard use this one split. */
void irx_unit_range(long long units, unsigned s, unsigned ns, long long *u0, long long *u1)
{
    long long per = (units + ns - 1) / ns;
    *u0 = per * s;
    *u1 = *u0 + per;
    if (*u0 > units) *u0 = units;
    if (*u1 > units) *u1 = units;
    if (WIN_B >= 0) {
        if (*u0 < WIN_A) *u0 = WIN_A;
        if (*u1 > WIN_B) *u1 = WIN_B;
        if (*u1 < *u0) *u1 = *u0;
    }
}

static int aligned(const void *p, int64_t off_elems, int es, int align)
{
    return ((((unsigned long long)(size_t)p) + (unsigned long long)(off_elems * es)) % (unsigned long long)align) == 0;
}

static void fill_unis(irx_kuni_t *ku, const irx_uni_t *u, int n, const irx_plan_int_t *p, void *const *args)
{
    int i;
    for (i = 0; i < n; i++) {
        ku[i].kind = u[i].kind;
        ku[i].bits = u[i].v;
        ku[i].off = u[i].off;
        if (u[i].kind == UNI_ARG) {
            ku[i].ptr = args[u[i].v];
            ku[i].dt = p->arg_dt[u[i].v];
        }
    }
}

static unsigned grid_cap(irx_dev_t *d, int k, int block, size_t smem, long long want)
{
    int occ = 1;
    long long g;
    if (irx_dev_occupancy(d, k, block, smem, &occ)) occ = 1;
    g = (long long)d->sms * occ;
    if (want < g) g = want;
    return (unsigned)(g < 1 ? 1 : g);
}

/* Temporaries a pointwise plan's programs use (1: every program is a chain). */
static int prog_temps(const irx_pw_t *pw)
{
    int o, i, t = 1;
    for (o = 0; o < pw->nout; o++) {
        const irx_prog_t *g = &pw->prog[o];
        for (i = 0; i < g->nins; i++)
            if (g->ins[i].dst >= PROG_R_TMP && g->ins[i].dst - PROG_R_TMP + 1 > t) t = g->ins[i].dst - PROG_R_TMP + 1;
    }
    return t;
}

static int launch_pw(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st)
{
    const irx_pw_t *pw = &p->u.pw;
    static irx_kpw_t k;             /* big; built under the launch lock below */
    long long u0, u1;
    int i, ok = 1;
    memset(&k, 0, sizeof k);
    irx_unit_range(irx_plan_units((const irx_plan_t *)p), s, ns, &u0, &u1);
    k.begin = u0 * 8;
    k.end = u1 * 8 < pw->n ? u1 * 8 : pw->n;
    if (k.begin >= k.end) return 0;
    k.nin = pw->nin; k.nout = pw->nout; k.nuni = pw->nuni;
    for (i = 0; i < pw->nin; i++) {
        k.in[i] = args[pw->in_arg[i]];
        k.in_dt[i] = pw->in_dt[i];
        ok = ok && aligned(k.in[i], k.begin, esz(k.in_dt[i]), 16);
    }
    for (i = 0; i < pw->nout; i++) {
        k.out[i] = args[pw->out_arg[i]];
        k.out_dt[i] = pw->out_dt[i];
        k.prog[i] = pw->prog[i];
        ok = ok && aligned(k.out[i], k.begin, esz(k.out_dt[i]), 16);
    }
    k.uprog = pw->uprog;
    fill_unis(k.uni, pw->uni, pw->nuni, p, args);
    k.vec_ok = (uint8_t)ok;
    if (irx_jit_mode(-1)) {
        /* the graph's own kernel (jit.c): same element range, same parameters, written out */
        irx_kpwj_t j;
        CUfunction fn;
        int occ = 1;
        long long want;
        memset(&j, 0, sizeof j);
        for (i = 0; i < PROG_NSTREAM; i++) j.in[i] = k.in[i];
        for (i = 0; i < 4; i++) j.out[i] = k.out[i];
        for (i = 0; i < PROG_NUNI; i++) j.uni[i] = k.uni[i].ptr;
        j.begin = k.begin;
        j.end = k.end;
        j.vec_ok = ok;
        if (irx_jit_pw_fn(p, d, &fn, &occ)) return 1;
        want = ((k.end - k.begin) / IRX_JIT_PW_W + IRX_JIT_PW_THREADS - 1) / IRX_JIT_PW_THREADS + 1;
        if (want > (long long)d->sms * occ) want = (long long)d->sms * occ;   /* one resident wave */
        return irx_dev_launch_fn(fn, (unsigned)want, IRX_JIT_PW_THREADS, st, &j, 1);
    }
    if (pw->nin == 0) {                  /* no streams: a dummy (never used) stream pointer */
        k.in[0] = k.out[0];
        k.in_dt[0] = k.out_dt[0];
    }
    {
        int ns = pw->nin ? pw->nin : 1, kk = K_PW + 2 * (ns - 1) + (prog_temps(pw) > 1);
        return irx_dev_launch(d, kk, grid_cap(d, kk, 256, 0, ((k.end - k.begin) / 8 + 255) / 256 + 1), 256, 0, 1, st, &k);
    }
}

static int launch_red(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st)
{
    const irx_red_t *r = &p->u.red;
    static irx_kred_t k;
    long long u0, u1;
    irx_slot_t sl;
    memset(&k, 0, sizeof k);
    k.x = args[r->x_arg];
    k.y = args[r->y_arg];
    if (r->rows == 1) {                  /* a full reduction: this launch's own partials and ticket */
        irx_dev_slot(d, &sl);
        k.partial = (float *)(size_t)sl.partial;
        k.ticket = (unsigned *)(size_t)sl.ticket;
    }
    fill_unis(k.uni, r->uni, r->nuni, p, args);
    k.pre = r->pre; k.uprog = r->uprog;
    k.op = r->op; k.x_dt = r->x_dt; k.y_dt = r->y_dt; k.has_pre = r->has_pre;
    k.out_reg = r->out_reg; k.tot_reg = r->tot_reg; k.nuni = r->nuni;
    k.accumulate = r->accumulate && (ns == 1 || r->rows != 1);   /* a full reduction's shard writes its partial */
    k.cols = r->cols;
    if (r->rows == 1) {
        irx_unit_range(irx_plan_units((const irx_plan_t *)p), s, ns, &u0, &u1);
        if (r->has_seed && s != 0) {          /* an Init seed's share counts once: in shard 0 */
            const float id = r->op == OP_MUL ? 1.0f : r->op == OP_MAX ? -1e30f : r->op == OP_MIN ? 1e30f : 0.0f;
            memcpy(&k.uni[r->seed_uni].bits, &id, 4);
        }
        k.rows = 1;
        k.begin = u0 * 8;
        k.end = u1 * 8 < r->cols ? u1 * 8 : r->cols;
        k.vec_ok = (uint8_t)aligned(k.x, k.begin, esz(k.x_dt), 16);
        {
            int kk = K_RED_ALL + (r->has_pre ? 1 : 0);
            unsigned g = grid_cap(d, kk, IRX_RED_ALL_THREADS, 0, SLOT_PARTIALS);
            long long need = (k.end - k.begin + 4095) / 4096;     /* at least 4096 elements a block */
            if (need < g) g = (unsigned)(need < 1 ? 1 : need);
            return irx_dev_launch(d, kk, g, IRX_RED_ALL_THREADS, 0, 1, st, &k);
        }
    }
    irx_unit_range(r->rows, s, ns, &u0, &u1);
    if (u0 >= u1) return 0;
    k.row0 = u0;
    k.rows = u1 - u0;
    k.vec_ok = (uint8_t)(aligned(k.x, 0, esz(k.x_dt), 16) && (r->cols * esz(k.x_dt)) % 16 == 0);
    {
        int kk = K_RED_ROWS + (r->has_pre ? 1 : 0);
        return irx_dev_launch(d, kk, grid_cap(d, kk, 256, 0, (k.rows + 7) / 8), 256, 0, 1, st, &k);
    }
}

#define ROW_NBUF 3

static int launch_row(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st)
{
    const irx_row_t *r = &p->u.row;
    static irx_krow_t k;
    long long u0, u1;
    size_t rowb, smem = 0;
    int i;
    memset(&k, 0, sizeof k);
    irx_unit_range(r->rows, s, ns, &u0, &u1);
    if (u0 >= u1) return 0;
    k.x = args[r->x_arg];
    k.w = r->has_w ? args[r->w_arg] : NULL;
    k.y = args[r->y_arg];
    fill_unis(k.uni, r->uni, r->nuni, p, args);
    for (i = 0; i < ROW_MAX_STAT; i++) { k.stat_pre[i] = r->stat_pre[i]; k.stat_op[i] = r->stat_op[i]; k.stat_reg[i] = r->stat_reg[i]; }
    k.epi = r->epi; k.uprog = r->uprog;
    k.rows = u1 - u0; k.cols = r->cols; k.row0 = u0;
    k.x_dt = r->x_dt; k.w_dt = r->w_dt; k.y_dt = r->y_dt; k.has_w = r->has_w;
    k.nstat = r->nstat; k.nuni = r->nuni; k.kind = r->kind; k.eps_bits = r->eps_bits;
    k.err = (unsigned *)(size_t)d->err;
    rowb = (size_t)r->cols * esz(r->x_dt);
    k.smem_row_bytes = (uint32_t)((rowb + 127) & ~(size_t)127);
    k.bulk_ok = (uint8_t)(rowb % 16 == 0 && aligned(k.x, 0, 1, 16) && (r->cols % 8) == 0 &&
                          (size_t)ROW_NBUF * k.smem_row_bytes + 1024 <= (size_t)d->smem_optin &&
                          (!r->has_w || aligned(k.w, 0, 1, 16)) && aligned(k.y, 0, 1, 16));
    if (k.bulk_ok) smem = (size_t)ROW_NBUF * k.smem_row_bytes;
    /* softmax of a staged f32 row keeps exp(x - max) in the row itself (one exp per element);
     * a bf16 row recomputes it, since a separate f32 buffer costs more occupancy than it saves */
    if (k.bulk_ok && r->kind == ROWK_SOFTMAX && r->x_dt == DT_F32) k.ecache = 1;
    if (k.bulk_ok && r->kind != ROWK_GENERIC && r->cols % (256 * 8) == 0 &&
        (r->cols / (256 * 8) == 1 || r->cols / (256 * 8) == 2 || r->cols / (256 * 8) == 4))
        k.rk = (uint8_t)(r->cols / (256 * 8));
    {
        int kk = K_ROWOP;
        if (r->kind == ROWK_RMSNORM) kk = K_ROW_RMSNORM;
        else if (r->kind == ROWK_SOFTMAX) kk = K_ROW_SOFTMAX;
        else if (r->kind == ROWK_L2NORM) kk = K_ROW_L2NORM;
        if (kk != K_ROWOP && (r->cols % 8)) kk = K_ROWOP;          /* the written-out forms take 8-wide rows */
        return irx_dev_launch(d, kk, grid_cap(d, kk, 256, smem, k.rows), 256, (unsigned)smem, 1, st, &k);
    }
}

/* The generic per-graph kernel: one device pointer per KIR arg, on the KIR's launch geometry;
 * it does not split, so shard 0 of any count runs the whole graph and the others nothing. */
static int launch_kir(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, void *const *args, void *st)
{
    struct { void *a[KIR_MAX_ARG]; } prm;
    CUfunction fn;
    int occ = 1, i;
    if (s != 0) return 0;
    memset(&prm, 0, sizeof prm);
    for (i = 0; i < p->narg; i++) prm.a[i] = args[i];
    if (irx_jit_pw_fn(p, d, &fn, &occ)) return 1;
    return irx_dev_launch_fn(fn, (unsigned)p->u.kk.grid, (unsigned)p->u.kk.block, st, &prm, 0);
}

int irx_launch_mm(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st);
int irx_launch_attn(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st);

static pthread_mutex_t LLOCK = PTHREAD_MUTEX_INITIALIZER;

int irx_launch_shard(const irx_plan_t *plan, unsigned shard, unsigned nshards, void *const *args, unsigned nargs,
                     void *stream)
{
    const irx_plan_int_t *p = P(plan);
    irx_dev_t *d;
    unsigned i;
    int rc;
    irx_clear_error();
    if (!p) return irx_fail(E093, "a launch of a plan that was never compiled");
    if (!args || nargs != p->narg) return irx_fail(E093, "a launch whose argument count is not the KIR's");
    if (!nshards || shard >= nshards) return irx_fail(E093, "a shard index outside its shard count");
    for (i = 0; i < nargs; i++) if (!args[i]) return irx_fail(E093, "a launch with a null device pointer");
    if (irx_dev_get(&d)) return 1;
    pthread_mutex_lock(&LLOCK);
    switch (p->fam) {
    case FAM_POINTWISE: rc = launch_pw(p, d, shard, nshards, args, stream); break;
    case FAM_REDUCE_ALL:
    case FAM_REDUCE_ROWS: rc = launch_red(p, d, shard, nshards, args, stream); break;
    case FAM_ROWOP: rc = launch_row(p, d, shard, nshards, args, stream); break;
    case FAM_MATMUL: rc = irx_launch_mm(p, d, shard, nshards, args, stream); break;
    case FAM_ATTENTION: rc = irx_launch_attn(p, d, shard, nshards, args, stream); break;
    case FAM_KIR: rc = launch_kir(p, d, shard, args, stream); break;
    default: rc = irx_fail(E000, "a plan of no known family");
    }
    pthread_mutex_unlock(&LLOCK);
    return rc;
}

void irx_inject_mm(int on, unsigned long long wait_ns);

int irx_inject(int what, unsigned long long value)
{
    irx_clear_error();
    pthread_mutex_lock(&LLOCK);
    switch (what) {
    case IRX_INJECT_NONE: irx_inject_mm(0, 0); irx_host_wait_limit(0); break;
    case IRX_INJECT_MM_NO_LOADS: irx_inject_mm(1, value * 1000ull); break;
    case IRX_INJECT_HOST_WAIT: irx_host_wait_limit(value); break;
    default: pthread_mutex_unlock(&LLOCK); return irx_fail(E093, "an injection this library does not know");
    }
    pthread_mutex_unlock(&LLOCK);
    return 0;
}

int irx_launch(const irx_plan_t *plan, void *const *args, unsigned nargs, void *stream)
{
    return irx_launch_shard(plan, 0, 1, args, nargs, stream);
}

int irx_check(void *stream)
{
    irx_dev_t *d;
    irx_clear_error();
    if (irx_dev_get(&d)) return 1;
    return irx_dev_check_err(d, stream);
}

/* The part of arg i that the units [u0, u1) read or write, as `rows` rows of `width` bytes at
 * byte offset `off`, `pitch` bytes apart (one row for a contiguous slice). A shard reads and
 * writes only inside these slices; launch-uniform args (scalars, a row op's weight) and a
 * matmul's A are whole. */
typedef struct { size_t off, width, rows, pitch; } slice_t;

static void arg_slice(const irx_plan_int_t *p, unsigned i, long long u0, long long u1, slice_t *sl)
{
    const size_t es = (size_t)esz(p->arg_dt[i]), all = (size_t)p->arg_elems[i] * es;
    sl->off = 0; sl->width = all; sl->rows = 1; sl->pitch = all;
    if (u0 == 0 && u1 >= irx_plan_units((const irx_plan_t *)p)) return;     /* every unit: whole */
    switch (p->fam) {
    case FAM_POINTWISE: {
        long long e0 = u0 * 8, e1 = u1 * 8 < p->u.pw.n ? u1 * 8 : p->u.pw.n;
        if ((long long)p->arg_elems[i] != p->u.pw.n) return;          /* a uniform const: whole */
        if (e1 < e0) e1 = e0;
        sl->off = (size_t)e0 * es; sl->width = (size_t)(e1 - e0) * es;
        return;
    }
    case FAM_REDUCE_ALL:
    case FAM_REDUCE_ROWS: {
        const irx_red_t *r = &p->u.red;
        if (r->rows == 1) {
            long long e0 = u0 * 8, e1 = u1 * 8 < r->cols ? u1 * 8 : r->cols;
            if (i != r->x_arg) return;                                 /* y: the shard's partial */
            if (e1 < e0) e1 = e0;
            sl->off = (size_t)e0 * es; sl->width = (size_t)(e1 - e0) * es;
        } else if (i == r->x_arg) {
            sl->off = (size_t)u0 * r->cols * es; sl->width = (size_t)(u1 - u0) * r->cols * es;
        } else if (i == r->y_arg) {
            sl->off = (size_t)u0 * es; sl->width = (size_t)(u1 - u0) * es;
        }
        return;
    }
    case FAM_ROWOP: {
        const irx_row_t *r = &p->u.row;
        if (i != r->x_arg && i != r->y_arg) return;
        sl->off = (size_t)u0 * r->cols * es; sl->width = (size_t)(u1 - u0) * r->cols * es;
        return;
    }
    case FAM_MATMUL: {
        const irx_mm_t *m = &p->u.mm;
        const long long n0 = u0 * MM_TILE_N, n1 = u1 * MM_TILE_N < m->n ? u1 * MM_TILE_N : m->n;
        const size_t w = n1 > n0 ? (size_t)(n1 - n0) * es : 0;
        if (i == m->b_arg && m->b_kmajor) {                            /* B [N, K]: rows n0..n1 */
            sl->off = (size_t)n0 * m->k * es; sl->width = w / es * (size_t)m->k * es;
        } else if (i == m->b_arg) {                                    /* B [K, N]: columns */
            sl->off = (size_t)n0 * es; sl->width = w; sl->rows = (size_t)m->k; sl->pitch = (size_t)m->n * es;
        } else if (i == m->c_arg) {                                    /* C [M, N]: columns */
            sl->off = (size_t)n0 * es; sl->width = w; sl->rows = (size_t)m->m; sl->pitch = (size_t)m->n * es;
        }
        return;
    }
    case FAM_ATTENTION: {
        const size_t per = all / (size_t)(p->u.at.b * p->u.at.h);     /* one (batch, head) of this arg */
        sl->off = (size_t)u0 * per; sl->width = (size_t)(u1 - u0) * per;
        return;
    }
    default:
        return;
    }
}

static int copy_slice(int to_dev, void *host, CUdeviceptr dev, const slice_t *sl, void *st)
{
    if (!sl->width || !sl->rows) return 0;
    if (sl->rows == 1 || sl->width == sl->pitch) {
        const size_t n = sl->rows == 1 ? sl->width : sl->width * sl->rows;
        return to_dev ? irx_dev_h2d(dev + sl->off, (const char *)host + sl->off, n, st)
                      : irx_dev_d2h((char *)host + sl->off, dev + sl->off, n, st);
    }
    return irx_dev_copy2d(to_dev, (char *)host + sl->off, sl->pitch, dev + sl->off, sl->pitch, sl->width, sl->rows, st);
}

/* Whether the host path copies arg i in: inputs and consts, and the outputs whose starting value
 * the kernel reads (those on a `zero` line, and a full reduction's accumulated total); the other
 * outputs are written whole by the launch, as the reference's runner assumes
 * (tests/gpurun.py:61-63). A full reduction's shard writes its partial. */
static int copied_in(const irx_plan_int_t *p, unsigned i, unsigned nshards)
{
    const int red = p->fam == FAM_REDUCE_ALL || p->fam == FAM_REDUCE_ROWS;
    if (p->arg_kind[i] != KA_OUT) return 1;
    if (nshards > 1 && p->fam == FAM_REDUCE_ALL) return 0;
    return p->arg_zero[i] || (red && p->u.red.accumulate && i == p->u.red.y_arg && (nshards == 1 || p->u.red.rows != 1));
}

static int same_slice(const slice_t *a, const slice_t *b)
{
    return a->off == b->off && a->width == b->width && a->rows == b->rows && a->pitch == b->pitch;
}

#define PIPE_CHUNK_BYTES ((size_t)32 << 20)   /* bytes moved per chunk of the pipelined path */
#define PIPE_MIN_OUT ((size_t)8 << 20)        /* below this much output there is nothing to overlap */

/* How many chunks the units [u0, u1) are copied and run in (1: not pipelined). The pipeline
 * overlaps chunk c's copy in, chunk c - 1's kernel and chunk c - 2's copy out, so the bus moves
 * both ways at once. It needs each output's slice to move with the chunk (no whole output, as
 * a full sum's or a generic graph's), and enough output to overlap with the inputs. */
static int pipe_chunks(const irx_plan_int_t *p, unsigned nshards, long long u0, long long u1, int *uni)
{
    const long long len = u1 - u0;
    size_t in = 0, out = 0;
    slice_t a, b;
    long long per;
    unsigned i;
    int nc;
    if (p->fam == FAM_KIR || (p->fam == FAM_REDUCE_ALL && p->u.red.rows == 1) || len < 2) return 1;
    per = (len + 1) / 2;
    for (i = 0; i < p->narg; i++) {
        arg_slice(p, i, u0, u0 + per, &a);
        arg_slice(p, i, u0 + per, u1, &b);
        uni[i] = same_slice(&a, &b);
        if (uni[i] && p->arg_kind[i] == KA_OUT) return 1;
        arg_slice(p, i, u0, u1, &a);
        if (copied_in(p, i, nshards)) in += a.width * a.rows;
        if (p->arg_kind[i] == KA_OUT) out += a.width * a.rows;
    }
    if (out < PIPE_MIN_OUT) return 1;
    nc = (int)((in + out) / PIPE_CHUNK_BYTES);
    if (nc > IRX_PIPE_CHUNKS) nc = IRX_PIPE_CHUNKS;
    if (nc > len) nc = (int)len;
    return nc < 2 ? 1 : nc;
}

/* The pipelined host path: chunk c's inputs go in on the copy-in stream, its kernel runs on the
 * caller's stream once they have landed, and its outputs come back on the copy-out stream once
 * the kernel is done, each step ordered by an event. Args whose slice is the same for every
 * chunk (a matmul's A, a row op's weight, scalars) go in once, first. */
static int run_host_pipelined(const irx_plan_t *plan, const irx_plan_int_t *p, irx_dev_t *d, unsigned shard,
                              unsigned nshards, long long u0, long long u1, int nc, const int *uni,
                              void *const *host_args, void *const *dargs, const size_t *off, void *st)
{
    const long long per = (u1 - u0 + nc - 1) / nc;
    void *in, *out;
    slice_t sl;
    long long a0;
    unsigned i;
    int c, rc;
    if (irx_dev_pipe(d)) return 1;
    in = (void *)d->pipe[0];
    out = (void *)d->pipe[1];
    rc = irx_dev_order(d, 0, st, in) || irx_dev_order(d, 1, st, out);
    for (i = 0; i < p->narg && !rc; i++) {
        if (!uni[i] || !copied_in(p, i, nshards)) continue;
        arg_slice(p, i, u0, u1, &sl);
        rc = copy_slice(1, host_args[i], d->arena + off[i], &sl, in);
    }
    for (c = 0, a0 = u0; a0 < u1 && !rc; c++, a0 += per) {
        const long long a1 = a0 + per < u1 ? a0 + per : u1;
        for (i = 0; i < p->narg && !rc; i++) {
            if (uni[i] || !copied_in(p, i, nshards)) continue;
            arg_slice(p, i, a0, a1, &sl);
            rc = copy_slice(1, host_args[i], d->arena + off[i], &sl, in);
        }
        if (rc || (rc = irx_dev_order(d, 2 + 2 * c, in, st))) break;
        irx_unit_window(a0, a1);
        rc = irx_launch_shard(plan, shard, nshards, dargs, p->narg, st);
        irx_unit_window(0, -1);
        if (rc || (rc = irx_dev_order(d, 3 + 2 * c, st, out))) break;
        for (i = 0; i < p->narg && !rc; i++) {
            if (p->arg_kind[i] != KA_OUT) continue;
            arg_slice(p, i, a0, a1, &sl);
            rc = copy_slice(0, host_args[i], d->arena + off[i], &sl, out);
        }
    }
    if (!rc) rc = irx_dev_order(d, 2 + 2 * IRX_PIPE_CHUNKS, out, st);
    if (rc) {
        /* no copy may still touch the caller's buffers once this returns */
        char msg[256];
        int code;
        irx_save_error(&code, msg, sizeof msg);
        irx_dev_sync(in);
        irx_dev_sync(out);
        irx_restore_error(code, msg);
        return 1;
    }
    return irx_dev_check_err(d, st);
}

int irx_run_host_shard(const irx_plan_t *plan, unsigned shard, unsigned nshards, void *const *host_args, unsigned nargs,
                       void *stream)
{
    const irx_plan_int_t *p = P(plan);
    irx_dev_t *d;
    void *dargs[KIR_MAX_ARG];
    size_t off[KIR_MAX_ARG], total = 0;
    int uni[KIR_MAX_ARG], nc;
    long long u0, u1;
    slice_t sl;
    unsigned i;
    irx_clear_error();
    if (!p) return irx_fail(E093, "a run of a plan that was never compiled");
    if (!host_args || nargs != p->narg) return irx_fail(E093, "a run whose argument count is not the KIR's");
    if (!nshards || shard >= nshards) return irx_fail(E093, "a shard index outside its shard count");
    for (i = 0; i < nargs; i++) {
        if (!host_args[i]) return irx_fail(E093, "a run with a null host pointer");
        off[i] = total;
        total += ((size_t)p->arg_elems[i] * (size_t)esz(p->arg_dt[i]) + 255) & ~(size_t)255;
    }
    if (irx_dev_get(&d)) return 1;
    if (d->arena_bytes < total) {
        if (irx_dev_sync(stream)) return 1;
        irx_dev_free(d->arena);
        d->arena = 0;
        d->arena_bytes = 0;
        if (irx_dev_alloc(total, &d->arena)) return 1;
        d->arena_bytes = total;
    }
    for (i = 0; i < nargs; i++) dargs[i] = (void *)(size_t)(d->arena + off[i]);
    irx_unit_range(irx_plan_units(plan), shard, nshards, &u0, &u1);
    nc = pipe_chunks(p, nshards, u0, u1, uni);
    if (nc > 1)
        return run_host_pipelined(plan, p, d, shard, nshards, u0, u1, nc, uni, host_args, dargs, off, stream);
    for (i = 0; i < nargs; i++) {
        if (!copied_in(p, i, nshards)) continue;
        arg_slice(p, i, u0, u1, &sl);
        if (copy_slice(1, host_args[i], d->arena + off[i], &sl, stream)) return 1;
    }
    if (irx_launch_shard(plan, shard, nshards, dargs, nargs, stream)) return 1;
    for (i = 0; i < nargs; i++) {
        if (p->arg_kind[i] != KA_OUT) continue;
        arg_slice(p, i, u0, u1, &sl);
        if (copy_slice(0, host_args[i], d->arena + off[i], &sl, stream)) return 1;
    }
    return irx_dev_check_err(d, stream);
}

int irx_run_host_chunks(const irx_plan_t *plan, unsigned shard, unsigned nshards)
{
    const irx_plan_int_t *p = P(plan);
    int uni[KIR_MAX_ARG];
    long long u0, u1;
    irx_clear_error();
    if (!p) return irx_fail(E093, "the chunks of a plan that was never compiled"), -1;
    if (!nshards || shard >= nshards) return irx_fail(E093, "a shard index outside its shard count"), -1;
    irx_unit_range(irx_plan_units(plan), shard, nshards, &u0, &u1);
    return pipe_chunks(p, nshards, u0, u1, uni);
}

int irx_run_host(const irx_plan_t *plan, void *const *host_args, unsigned nargs, void *stream)
{
    return irx_run_host_shard(plan, 0, 1, host_args, nargs, stream);
}

int irx_jit(int mode)
{
    return irx_jit_mode(mode < 0 ? -1 : mode > 0 ? 1 : 0);
}

int irx_plan_source(const irx_plan_t *plan, char *buf, size_t cap)
{
    const irx_plan_int_t *p = P(plan);
    int n;
    irx_clear_error();
    if (!p) return -irx_fail(E093, "the source of a plan that was never compiled");
    n = irx_jit_source(p, buf, cap);
    return n;
}

int irx_prepare(const irx_plan_t *plan)
{
    const irx_plan_int_t *p = P(plan);
    irx_clear_error();
    if (!p) return irx_fail(E093, "preparing a plan that was never compiled");
    if (p->fam == FAM_KIR) return irx_jit_prepare(p);
    if (p->fam != FAM_POINTWISE || !irx_jit_mode(-1)) return 0;
    return irx_jit_prepare(p);
}

int irx_plan_shard(const irx_plan_t *plan, unsigned shard, unsigned nshards, long long *u0, long long *u1, int *combine)
{
    const irx_plan_int_t *p = P(plan);
    long long a, b;
    int c = IRX_COMBINE_NONE;
    irx_clear_error();
    if (!p) return irx_fail(E093, "the shards of a plan that was never compiled");
    if (!nshards || shard >= nshards) return irx_fail(E093, "a shard index outside its shard count");
    /* the same split every family launcher uses (range_of, irx_launch_mm, irx_launch_attn) */
    irx_unit_range(irx_plan_units(plan), shard, nshards, &a, &b);
    if (p->fam == FAM_REDUCE_ALL && p->u.red.rows == 1 && nshards > 1) {
        switch (p->u.red.op) {
        case OP_MAX: c = IRX_COMBINE_MAX; break;
        case OP_MIN: c = IRX_COMBINE_MIN; break;
        case OP_MUL: c = IRX_COMBINE_PROD; break;
        default: c = IRX_COMBINE_SUM; break;
        }
    }
    if (u0) *u0 = a;
    if (u1) *u1 = b;
    if (combine) *combine = c;
    return 0;
}
