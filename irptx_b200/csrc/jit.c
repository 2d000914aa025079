/* jit.c -- per-graph pointwise kernels, compiled at run time for sm_100a with NVRTC.
 *
 * The reference prints one PTX module per KIR graph, with the graph's arithmetic written out
 * as straight-line instructions (src/emit.c:318-376), and its runner JIT-loads that module
 * (tests/gpurun.py:91-107). The prebuilt pointwise kernels of this library instead interpret
 * the graph's op programs, which costs a dispatch per instruction and leaves a pointwise graph
 * bound by instruction issue rather than by HBM. So, for the pointwise family, this file writes
 * the graph's element function out as CUDA source, places it in a fixed hand-written kernel
 * template (128-bit streaming loads and stores, a grid-stride pass, the launch-uniform values
 * computed once per thread), and compiles that with NVRTC for sm_100a.
 *
 * The generated code calls irx_apply (kernels/ops.cuh) with each op code as a constant, the
 * same function the interpreter calls, so the two paths compute bit-identical results; the op
 * header and irx_ops.h are embedded in the library (jit_blob.S) and handed to NVRTC as
 * in-memory headers.
 *
 * Compiled cubins are cached in the process, keyed by a 64-bit FNV-1a hash of the generated
 * source (the full source is kept and compared too), and loaded once per CUDA context. A plan
 * stores only the key: the source is a pure function of the plan, so a plan copied into a
 * process that has never compiled it is compiled again on its first launch. NVRTC is opened
 * at run time (libnvrtc.so.12); without it the prebuilt interpreting kernels run instead. */

#include <dlfcn.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <nvrtc.h>
#include "irx_int.h"
#include "irx_kparams.h"
#include "launch.h"
#include "jit.h"

extern const char irx_src_ops_cuh[];   /* kernels/ops.cuh, NUL-terminated (jit_blob.S) */
extern const char irx_src_ops_h[];     /* irx_ops.h */

/* ---- NVRTC, opened at run time ---- */

static struct {
    int tried, ok;
    void *lib;
    nvrtcResult (*create)(nvrtcProgram *, const char *, const char *, int, const char *const *, const char *const *);
    nvrtcResult (*compile)(nvrtcProgram, int, const char *const *);
    nvrtcResult (*cubin_size)(nvrtcProgram, size_t *);
    nvrtcResult (*cubin)(nvrtcProgram, char *);
    nvrtcResult (*log_size)(nvrtcProgram, size_t *);
    nvrtcResult (*log)(nvrtcProgram, char *);
    nvrtcResult (*destroy)(nvrtcProgram *);
    const char *(*errstr)(nvrtcResult);
} N;

static pthread_mutex_t JLOCK = PTHREAD_MUTEX_INITIALIZER;
static int JIT_MODE = -1;              /* -1: not decided yet; 0 off; 1 on */

#define NSYM(field, name) do { *(void **)&N.field = dlsym(N.lib, name); if (!N.field) return 0; } while (0)

static int nvrtc_open_locked(void)
{
    static const char *const names[] = {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"};
    size_t i;
    if (N.tried) return N.ok;
    N.tried = 1;
    for (i = 0; i < sizeof names / sizeof names[0] && !N.lib; i++) N.lib = dlopen(names[i], RTLD_NOW | RTLD_LOCAL);
    if (!N.lib) return 0;
    NSYM(create, "nvrtcCreateProgram");
    NSYM(compile, "nvrtcCompileProgram");
    NSYM(cubin_size, "nvrtcGetCUBINSize");
    NSYM(cubin, "nvrtcGetCUBIN");
    NSYM(log_size, "nvrtcGetProgramLogSize");
    NSYM(log, "nvrtcGetProgramLog");
    NSYM(destroy, "nvrtcDestroyProgram");
    NSYM(errstr, "nvrtcGetErrorString");
    N.ok = 1;
    return 1;
}

int irx_jit_mode(int mode)
{
    int m;
    pthread_mutex_lock(&JLOCK);
    if (JIT_MODE < 0) {
        const char *e = getenv("IRX_JIT");
        JIT_MODE = (e && e[0] == '0') ? 0 : nvrtc_open_locked();
    }
    if (mode == 0) JIT_MODE = 0;
    else if (mode == 1) JIT_MODE = nvrtc_open_locked();
    m = JIT_MODE;
    pthread_mutex_unlock(&JLOCK);
    return m;
}

/* ---- source text ---- */

typedef struct { char *p; size_t n, cap; int full; } sb_t;

static void sb_put(sb_t *b, const char *fmt, ...)
{
    va_list ap;
    int w;
    if (b->full) return;
    va_start(ap, fmt);
    w = vsnprintf(b->p + b->n, b->cap - b->n, fmt, ap);
    va_end(ap);
    if (w < 0 || (size_t)w >= b->cap - b->n) { b->full = 1; return; }
    b->n += (size_t)w;
}

static const char *dtn(int dt) { return dt == DT_BF16 ? "bf16" : "f32"; }

/* The fixed part of every pointwise kernel: parameter block (the layout of irx_kpwj_t in
 * irx_kparams.h), loads and stores of IRX_W consecutive elements, and single elements. bf16
 * is widened by a shift and narrowed by cvt.rn (round to nearest even), as the interpreter's
 * __float2bfloat16_rn does. */
static const char TEMPLATE_HEAD[] =
    "#include \"ops.cuh\"\n"
    "typedef struct { const void *in[4]; void *out[4]; const void *uni[12]; long long begin, end; int vec_ok, pad; } irx_kpwj_t;\n"
    "struct irx_u { float r[12]; };\n"
    "__device__ __forceinline__ unsigned irx_f2bf2(float lo, float hi) { unsigned r; asm(\"cvt.rn.bf16x2.f32 %0, %1, %2;\" : \"=r\"(r) : \"f\"(hi), \"f\"(lo)); return r; }\n"
    "__device__ __forceinline__ unsigned short irx_f2bf(float x) { unsigned short h; asm(\"cvt.rn.bf16.f32 %0, %1;\" : \"=h\"(h) : \"f\"(x)); return h; }\n"
    "__device__ __forceinline__ float irx_ld1_f32(const void *p, long long e) { return ((const float *)p)[e]; }\n"
    "__device__ __forceinline__ float irx_ld1_bf16(const void *p, long long e) { return __uint_as_float((unsigned)((const unsigned short *)p)[e] << 16); }\n"
    "__device__ __forceinline__ void irx_st1_f32(void *p, long long e, float v) { ((float *)p)[e] = v; }\n"
    "__device__ __forceinline__ void irx_st1_bf16(void *p, long long e, float v) { ((unsigned short *)p)[e] = irx_f2bf(v); }\n"
    "__device__ __forceinline__ void irx_ldv_f32(const void *p, long long e, float (&o)[IRX_W]) {\n"
    "  const float4 *q = (const float4 *)((const float *)p + e);\n"
    "#pragma unroll\n"
    "  for (int j = 0; j < IRX_W / 4; j++) { const float4 a = __ldcs(q + j); o[4*j] = a.x; o[4*j+1] = a.y; o[4*j+2] = a.z; o[4*j+3] = a.w; }\n"
    "}\n"
    "__device__ __forceinline__ void irx_ldv_bf16(const void *p, long long e, float (&o)[IRX_W]) {\n"
    "#if IRX_W % 8 == 0\n"
    "  const uint4 *q = (const uint4 *)((const unsigned short *)p + e);\n"
    "#pragma unroll\n"
    "  for (int j = 0; j < IRX_W / 8; j++) {\n"
    "    const uint4 r = __ldcs(q + j); const unsigned w[4] = {r.x, r.y, r.z, r.w};\n"
    "#pragma unroll\n"
    "    for (int k = 0; k < 4; k++) { o[8*j+2*k] = __uint_as_float(w[k] << 16); o[8*j+2*k+1] = __uint_as_float(w[k] & 0xffff0000u); }\n"
    "  }\n"
    "#else\n"
    "  const uint2 *q = (const uint2 *)((const unsigned short *)p + e);\n"
    "#pragma unroll\n"
    "  for (int j = 0; j < IRX_W / 4; j++) {\n"
    "    const uint2 r = __ldcs(q + j);\n"
    "    o[4*j] = __uint_as_float(r.x << 16); o[4*j+1] = __uint_as_float(r.x & 0xffff0000u);\n"
    "    o[4*j+2] = __uint_as_float(r.y << 16); o[4*j+3] = __uint_as_float(r.y & 0xffff0000u);\n"
    "  }\n"
    "#endif\n"
    "}\n"
    "__device__ __forceinline__ void irx_stv_f32(void *p, long long e, const float (&v)[IRX_W]) {\n"
    "  float4 *q = (float4 *)((float *)p + e);\n"
    "#pragma unroll\n"
    "  for (int j = 0; j < IRX_W / 4; j++) __stcs(q + j, make_float4(v[4*j], v[4*j+1], v[4*j+2], v[4*j+3]));\n"
    "}\n"
    "__device__ __forceinline__ void irx_stv_bf16(void *p, long long e, const float (&v)[IRX_W]) {\n"
    "#if IRX_W % 8 == 0\n"
    "  uint4 *q = (uint4 *)((unsigned short *)p + e);\n"
    "#pragma unroll\n"
    "  for (int j = 0; j < IRX_W / 8; j++)\n"
    "    __stcs(q + j, make_uint4(irx_f2bf2(v[8*j], v[8*j+1]), irx_f2bf2(v[8*j+2], v[8*j+3]),\n"
    "                             irx_f2bf2(v[8*j+4], v[8*j+5]), irx_f2bf2(v[8*j+6], v[8*j+7])));\n"
    "#else\n"
    "  uint2 *q = (uint2 *)((unsigned short *)p + e);\n"
    "#pragma unroll\n"
    "  for (int j = 0; j < IRX_W / 4; j++) __stcs(q + j, make_uint2(irx_f2bf2(v[4*j], v[4*j+1]), irx_f2bf2(v[4*j+2], v[4*j+3])));\n"
    "#endif\n"
    "}\n";

/* An operand of an element instruction: a stream, a uniform, a temporary, or 0 for a register
 * the interpreter's register file does not hold (it reads those as 0). */
static void operand(char *o, size_t cap, int r, int nin, char tmp[PROG_NTMP][16])
{
    if (r < PROG_NSTREAM) snprintf(o, cap, r < nin ? "s%d" : "0.0f", r);
    else if (r < PROG_R_TMP) snprintf(o, cap, "U.r[%d]", r - PROG_R_UNI);
    else if (r < PROG_NREG) snprintf(o, cap, "%s", tmp[r - PROG_R_TMP]);
    else snprintf(o, cap, "0.0f");
}

static int gen_pw(const irx_plan_int_t *p, sb_t *b)
{
    const irx_pw_t *pw = &p->u.pw;
    char tmp[PROG_NTMP][16], a[24], c[24];
    int i, o, s, v = 0;

    /* no names from the KIR: graphs that differ only in names share one compiled kernel */
    sb_put(b, "// irptx-b200 pointwise kernel: %d output(s) over %d stream(s)\n", pw->nout, pw->nin);
    sb_put(b, "#define IRX_W %d\n%s", IRX_JIT_PW_W, TEMPLATE_HEAD);

    /* launch-uniform values: literals and rank-0 const buffers, then the uniform program,
     * exactly as irx_uinit and irx_urun lay them out */
    sb_put(b, "__device__ __forceinline__ void irx_uniforms(const irx_kpwj_t &p, irx_u &U) {\n");
    for (i = 0; i < PROG_NUNI; i++) {
        const irx_uni_t *u = &pw->uni[i];
        if (i < pw->nuni && u->kind == UNI_LIT) sb_put(b, "  U.r[%d] = __uint_as_float(0x%08xu);\n", i, (unsigned)u->v);
        else if (i < pw->nuni && u->kind == UNI_ARG)
            sb_put(b, "  U.r[%d] = irx_ld1_%s(p.uni[%d], %d);\n", i, dtn(p->arg_dt[u->v]), i, (int)u->off);
        else sb_put(b, "  U.r[%d] = 0.0f;\n", i);
    }
    for (i = 0; i < pw->uprog.nins; i++) {
        const irx_ins_t *in = &pw->uprog.ins[i];
        int ua = in->a - PROG_R_UNI, ub = in->b - PROG_R_UNI, ud = in->dst - PROG_R_UNI;
        if (ud < 0 || ud >= PROG_NUNI) continue;
        if (ua >= 0 && ua < PROG_NUNI) snprintf(a, sizeof a, "U.r[%d]", ua); else snprintf(a, sizeof a, "0.0f");
        if (ub >= 0 && ub < PROG_NUNI) snprintf(c, sizeof c, "U.r[%d]", ub); else snprintf(c, sizeof c, "0.0f");
        sb_put(b, "  U.r[%d] = irx_apply(%d, %s, %s);   // %s\n", ud, in->op, a, c, irx_op_name(in->op));
    }
    sb_put(b, "}\n");

    /* the element function: every output program in order over one register file, so a
     * temporary a later program reads before writing holds what an earlier one left */
    sb_put(b, "__device__ __forceinline__ void irx_elem(const irx_u &U");
    for (s = 0; s < pw->nin; s++) sb_put(b, ", const float s%d", s);
    sb_put(b, ", float (&y)[4]) {\n");
    for (i = 0; i < PROG_NTMP; i++) snprintf(tmp[i], sizeof tmp[i], "0.0f");
    for (o = 0; o < pw->nout; o++) {
        const irx_prog_t *P = &pw->prog[o];
        for (i = 0; i < P->nins; i++) {
            const irx_ins_t *in = &P->ins[i];
            operand(a, sizeof a, in->a, pw->nin, tmp);
            operand(c, sizeof c, in->b, pw->nin, tmp);
            if (in->dst < PROG_R_TMP || in->dst >= PROG_NREG) continue;    /* not kept by the register file */
            sb_put(b, "  const float v%d = irx_apply(%d, %s, %s);   // %s\n", v, in->op, a, c, irx_op_name(in->op));
            snprintf(tmp[in->dst - PROG_R_TMP], sizeof tmp[0], "v%d", v);
            v++;
        }
        operand(a, sizeof a, P->out, pw->nin, tmp);
        sb_put(b, "  y[%d] = %s;\n", o, a);
    }
    sb_put(b, "}\n");

    /* the kernel: a grid-stride pass over IRX_W-element chunks with 128-bit accesses, then the
     * remainder (or everything, when a buffer is not 16-byte aligned) one element at a time */
    sb_put(b, "extern \"C\" __global__ void __launch_bounds__(%d, %d) irx_pwj(const __grid_constant__ irx_kpwj_t p) {\n",
           IRX_JIT_PW_THREADS, IRX_JIT_PW_MINB);
    sb_put(b, "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");   // launched early, then\n"
              "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");                // wait for the previous kernel\n");
    sb_put(b, "  irx_u U;\n  irx_uniforms(p, U);\n"
              "  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;\n"
              "  const long long nth = (long long)gridDim.x * blockDim.x;\n"
              "  long long head = p.begin;\n"
              "  if (p.vec_ok) {\n"
              "    const long long nchunk = (p.end - p.begin) / IRX_W;\n");
    sb_put(b, "    for (long long c = tid; c < nchunk; c += nth) {\n"
              "      const long long e = p.begin + c * IRX_W;\n");
    for (s = 0; s < pw->nin; s++) sb_put(b, "      float x%d[IRX_W];\n      irx_ldv_%s(p.in[%d], e, x%d);\n", s, dtn(pw->in_dt[s]), s, s);
    sb_put(b, "      float y[4][IRX_W];\n"
              "#pragma unroll\n"
              "      for (int l = 0; l < IRX_W; l++) {\n"
              "        float r[4];\n"
              "        irx_elem(U");
    for (s = 0; s < pw->nin; s++) sb_put(b, ", x%d[l]", s);
    sb_put(b, ", r);\n");
    for (o = 0; o < pw->nout; o++) sb_put(b, "        y[%d][l] = r[%d];\n", o, o);
    sb_put(b, "      }\n");
    for (o = 0; o < pw->nout; o++) sb_put(b, "      irx_stv_%s(p.out[%d], e, y[%d]);\n", dtn(pw->out_dt[o]), o, o);
    sb_put(b, "    }\n"
              "    head = p.begin + nchunk * IRX_W;\n"
              "  }\n"
              "  for (long long e = head + tid; e < p.end; e += nth) {\n"
              "    float r[4];\n"
              "    irx_elem(U");
    for (s = 0; s < pw->nin; s++) sb_put(b, ", irx_ld1_%s(p.in[%d], e)", dtn(pw->in_dt[s]), s);
    sb_put(b, ", r);\n");
    for (o = 0; o < pw->nout; o++) sb_put(b, "    irx_st1_%s(p.out[%d], e, r[%d]);\n", dtn(pw->out_dt[o]), o, o);
    sb_put(b, "  }\n}\n");
    return b->full ? -1 : 0;
}

static int kir_source(const irx_plan_int_t *p, char *buf, size_t cap);

/* The source's length (like snprintf: the text is truncated to cap), or -1 with the error set. */
int irx_jit_source(const irx_plan_int_t *p, char *buf, size_t cap)
{
    sb_t b;
    char *tmp = NULL;
    int n;
    if (!p || p->magic != IRX_PLAN_MAGIC) return -irx_fail(E093, "the source of a plan that was never compiled");
    if (p->fam == FAM_KIR) return kir_source(p, buf, cap);    /* the stored source of a generic plan */
    if (p->fam != FAM_POINTWISE) return -irx_fail(E093, "the source of a plan whose family has no per-graph kernel");
    tmp = (char *)malloc(IRX_JIT_SRC_MAX);
    if (!tmp) return -irx_fail(E094, "host memory for a per-graph kernel's source");
    b.p = tmp; b.n = 0; b.cap = IRX_JIT_SRC_MAX; b.full = 0;
    if (gen_pw(p, &b)) { free(tmp); return -irx_fail(E081, "a per-graph kernel source longer than its buffer"); }
    n = (int)b.n;
    if (buf && cap) {
        size_t k = b.n < cap - 1 ? b.n : cap - 1;
        memcpy(buf, tmp, k);
        buf[k] = 0;
    }
    free(tmp);
    return n;
}

static uint64_t fnv1a(const char *s, size_t n)
{
    uint64_t h = 1469598103934665603ull;
    size_t i;
    for (i = 0; i < n; i++) { h ^= (unsigned char)s[i]; h *= 1099511628211ull; }
    return h ? h : 1;
}

/* ---- the cache ---- */

#define JIT_MAX_ENT 256
#define JIT_MAX_CTX 16

typedef struct {
    uint64_t key;
    char    *src;
    char    *cubin;
    int      nper;
    struct { CUcontext ctx; unsigned long long ctx_id; CUfunction fn; int occ; } per[JIT_MAX_CTX];
} jit_ent_t;

static jit_ent_t JIT[JIT_MAX_ENT];
static int NJIT;

static jit_ent_t *find_locked(uint64_t key, const char *src)
{
    int i;
    for (i = 0; i < NJIT; i++)
        if (JIT[i].key == key && (!src || !strcmp(JIT[i].src, src))) return &JIT[i];
    return NULL;
}

/* NVRTC: source to an sm_100a cubin. The flags are nvcc's floating-point defaults, the same
 * the prebuilt kernels are built with. */
static int nvrtc_build(const char *src, char **cubin_out)
{
    const char *hdrs[2] = {irx_src_ops_cuh, irx_src_ops_h};
    const char *names[2] = {"ops.cuh", "irx_ops.h"};
    const char *opts[3] = {"-arch=sm_100a", "-std=c++17", "-default-device"};
    nvrtcProgram prog = NULL;
    nvrtcResult r;
    size_t n = 0;
    char *cubin;
    if ((r = N.create(&prog, src, "irx_graph.cu", 2, hdrs, names)) != NVRTC_SUCCESS)
        return irx_fail(E091, "NVRTC could not take a per-graph kernel's source");
    if ((r = N.compile(prog, 3, opts)) != NVRTC_SUCCESS) {
        char msg[240], *log = NULL;
        size_t ln = 0;
        N.log_size(prog, &ln);
        if (ln > 1 && (log = (char *)malloc(ln))) {
            char *nl;
            N.log(prog, log);
            if ((nl = strchr(log, '\n'))) *nl = 0;
        }
        snprintf(msg, sizeof msg, "a per-graph kernel that NVRTC would not compile (%s%s%.160s)", N.errstr(r),
                 log ? ": " : "", log ? log : "");
        free(log);
        N.destroy(&prog);
        return irx_fail(E091, msg);
    }
    if (N.cubin_size(prog, &n) != NVRTC_SUCCESS || !n || !(cubin = (char *)malloc(n))) {
        N.destroy(&prog);
        return irx_fail(E094, "host memory for a per-graph cubin");
    }
    N.cubin(prog, cubin);
    N.destroy(&prog);
    *cubin_out = cubin;
    return 0;
}

/* Keep a generic kernel's source (kirgen.c) in the store, uncompiled; its key is the source's
 * hash. Compiled on the plan's first launch (or irx_prepare). */
int irx_jit_store(const char *src, size_t n, uint64_t *key)
{
    jit_ent_t *e;
    char *copy;
    *key = fnv1a(src, n);
    pthread_mutex_lock(&JLOCK);
    if ((e = find_locked(*key, NULL)) && e->src && strlen(e->src) == n && !memcmp(e->src, src, n)) {
        pthread_mutex_unlock(&JLOCK);
        return 0;
    }
    if (e) {                                   /* a hash collision with another source: refuse */
        pthread_mutex_unlock(&JLOCK);
        return irx_fail(E081, "two generic kernel sources with one hash");
    }
    if (NJIT >= JIT_MAX_ENT) {
        pthread_mutex_unlock(&JLOCK);
        return irx_fail(E081, "more distinct graphs than the per-graph kernel store holds");
    }
    if (!(copy = (char *)malloc(n + 1))) { pthread_mutex_unlock(&JLOCK); return irx_fail(E094, "host memory for a kernel source"); }
    memcpy(copy, src, n);
    copy[n] = 0;
    e = &JIT[NJIT++];
    memset(e, 0, sizeof *e);
    e->key = *key;
    e->src = copy;
    pthread_mutex_unlock(&JLOCK);
    return 0;
}

static int kir_source(const irx_plan_int_t *p, char *buf, size_t cap)
{
    jit_ent_t *e;
    size_t len;
    pthread_mutex_lock(&JLOCK);
    e = find_locked(p->u.kk.key, NULL);
    if (!e) { pthread_mutex_unlock(&JLOCK); return -irx_fail(E093, "a generic plan whose kernel source this process does not hold"); }
    len = strlen(e->src);
    if (buf && cap) {
        size_t k = len < cap - 1 ? len : cap - 1;
        memcpy(buf, e->src, k);
        buf[k] = 0;
    }
    pthread_mutex_unlock(&JLOCK);
    return (int)len;
}

/* A generic plan's store entry, compiled now if it has not been. */
static int kir_entry(const irx_plan_int_t *p, jit_ent_t **out)
{
    jit_ent_t *e;
    char *cubin = NULL;
    pthread_mutex_lock(&JLOCK);
    if (!(e = find_locked(p->u.kk.key, NULL))) {
        pthread_mutex_unlock(&JLOCK);
        return irx_fail(E093, "a generic plan whose kernel source this process does not hold (compile the graph here)");
    }
    if (!e->cubin) {
        if (!nvrtc_open_locked()) { pthread_mutex_unlock(&JLOCK); return irx_fail(E091, "a generic kernel: NVRTC (libnvrtc.so.12) is missing"); }
        if (nvrtc_build(e->src, &cubin)) { pthread_mutex_unlock(&JLOCK); return 1; }
        e->cubin = cubin;
    }
    pthread_mutex_unlock(&JLOCK);
    *out = e;
    return 0;
}

/* The cache entry for a plan, compiled now if this process has not compiled it yet. */
static int entry_for(const irx_plan_int_t *p, jit_ent_t **out)
{
    char *src, *cubin = NULL;
    jit_ent_t *e;
    uint64_t key;
    int n;
    if (p->fam == FAM_KIR) return kir_entry(p, out);
    pthread_mutex_lock(&JLOCK);
    e = p->u.pw.jit_key ? find_locked(p->u.pw.jit_key, NULL) : NULL;
    pthread_mutex_unlock(&JLOCK);
    if (e) { *out = e; return 0; }
    if (!(src = (char *)malloc(IRX_JIT_SRC_MAX))) return irx_fail(E094, "host memory for a per-graph kernel's source");
    if ((n = irx_jit_source(p, src, IRX_JIT_SRC_MAX)) < 0) { free(src); return 1; }
    key = fnv1a(src, (size_t)n);
    pthread_mutex_lock(&JLOCK);
    if (!nvrtc_open_locked()) {
        pthread_mutex_unlock(&JLOCK);
        free(src);
        return irx_fail(E091, "a per-graph kernel: NVRTC (libnvrtc.so.12) is missing");
    }
    if ((e = find_locked(key, src))) { pthread_mutex_unlock(&JLOCK); free(src); *out = e; return 0; }
    if (NJIT >= JIT_MAX_ENT) {
        pthread_mutex_unlock(&JLOCK);
        free(src);
        return irx_fail(E081, "more distinct pointwise graphs than the per-graph kernel cache holds");
    }
    /* compiled under the lock: concurrent first launches of one graph compile it once */
    if (nvrtc_build(src, &cubin)) { pthread_mutex_unlock(&JLOCK); free(src); return 1; }
    e = &JIT[NJIT++];
    memset(e, 0, sizeof *e);
    e->key = key;
    e->src = src;
    e->cubin = cubin;
    pthread_mutex_unlock(&JLOCK);
    *out = e;
    return 0;
}

uint64_t irx_jit_key(const irx_plan_int_t *p)
{
    sb_t b;
    uint64_t key = 0;
    if (p->fam != FAM_POINTWISE || !(b.p = (char *)malloc(IRX_JIT_SRC_MAX))) return 0;
    b.n = 0; b.cap = IRX_JIT_SRC_MAX; b.full = 0;
    if (!gen_pw(p, &b)) key = fnv1a(b.p, b.n);      /* 0 (no key): found by source at launch */
    free(b.p);
    return key;
}

int irx_jit_prepare(const irx_plan_int_t *p)
{
    jit_ent_t *e;
    if (p->fam != FAM_POINTWISE && p->fam != FAM_KIR) return 0;
    return entry_for(p, &e);
}

int irx_jit_pw_fn(const irx_plan_int_t *p, irx_dev_t *d, CUfunction *fn, int *occ)
{
    jit_ent_t *e;
    int i, rc = 0;
    const char *entry = p->fam == FAM_KIR ? "irx_kir" : "irx_pwj";
    const int threads = p->fam == FAM_KIR ? p->u.kk.block : IRX_JIT_PW_THREADS;
    if (entry_for(p, &e)) return 1;
    pthread_mutex_lock(&JLOCK);
    for (i = 0; i < e->nper; i++)
        if (e->per[i].ctx == d->ctx && e->per[i].ctx_id == d->ctx_id) {
            *fn = e->per[i].fn; *occ = e->per[i].occ; pthread_mutex_unlock(&JLOCK); return 0;
        }
    if (e->nper >= JIT_MAX_CTX) rc = irx_fail(E081, "more CUDA contexts than the per-graph kernel table holds");
    else if (!(rc = irx_dev_load_fn(e->cubin, entry, fn)) && !(rc = irx_dev_occupancy_fn(*fn, threads, occ))) {
        e->per[e->nper].ctx = d->ctx;
        e->per[e->nper].ctx_id = d->ctx_id;
        e->per[e->nper].fn = *fn;
        e->per[e->nper].occ = *occ;
        e->nper++;
    }
    pthread_mutex_unlock(&JLOCK);
    return rc;
}
