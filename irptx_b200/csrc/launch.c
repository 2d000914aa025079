/* launch.c -- the device side of the C ABI: the CUDA driver, the embedded sm_100a module,
 * and one launch routine per op family.
 *
 * The reference hands its PTX to an external runner that JIT-loads it with cuModuleLoadData
 * and launches it with cuLaunchKernel, one device pointer per KIR argument in argument order
 * (tests/gpurun.py:91-125). This file does the same with a prebuilt sm_100a cubin: the
 * driver is opened at run time (dlopen libcuda.so.1), so the library loads on a machine
 * without a GPU and fails with E090 only when a launch is asked for. The module is loaded
 * once per CUDA context and kept, with the family kernels and a scratch area (the error word
 * and a ring of per-launch slots of block partials, an arrival ticket and a unit counter), in a
 * table guarded by a mutex. Contexts are told apart by the driver's context ID, so a context
 * created after another was destroyed never inherits its module or scratch.
 *
 * All launches go on the caller's stream and return as soon as they are queued. */

#include <dlfcn.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <cuda.h>
#include "irx_int.h"
#include "irx_kparams.h"
#include "launch.h"

/* ---- the driver, opened at run time ---- */

typedef CUresult (*f_init)(unsigned);
typedef CUresult (*f_errstr)(CUresult, const char **);
typedef CUresult (*f_ctxget)(CUcontext *);
typedef CUresult (*f_ctxid)(CUcontext, unsigned long long *);
typedef CUresult (*f_ctxset)(CUcontext);
typedef CUresult (*f_ctxdev)(CUdevice *);
typedef CUresult (*f_devget)(CUdevice *, int);
typedef CUresult (*f_retain)(CUcontext *, CUdevice);
typedef CUresult (*f_attr)(int *, CUdevice_attribute, CUdevice);
typedef CUresult (*f_modload)(CUmodule *, const void *);
typedef CUresult (*f_getfn)(CUfunction *, CUmodule, const char *);
typedef CUresult (*f_fnattr)(CUfunction, CUfunction_attribute, int);
typedef CUresult (*f_launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                             unsigned, CUstream, void **, void **);
typedef CUresult (*f_launchex)(const CUlaunchConfig *, CUfunction, void **, void **);
typedef CUresult (*f_alloc)(CUdeviceptr *, size_t);
typedef CUresult (*f_free)(CUdeviceptr);
typedef CUresult (*f_memset32)(CUdeviceptr, unsigned, size_t, CUstream);
typedef CUresult (*f_h2d)(CUdeviceptr, const void *, size_t, CUstream);
typedef CUresult (*f_d2h)(void *, CUdeviceptr, size_t, CUstream);
typedef CUresult (*f_ssync)(CUstream);
typedef CUresult (*f_squery)(CUstream);
typedef CUresult (*f_cpy2d)(const CUDA_MEMCPY2D *, CUstream);
typedef CUresult (*f_screate)(CUstream *, unsigned);
typedef CUresult (*f_ecreate)(CUevent *, unsigned);
typedef CUresult (*f_erecord)(CUevent, CUstream);
typedef CUresult (*f_swait)(CUstream, CUevent, unsigned);
typedef CUresult (*f_occ)(int *, CUfunction, int, size_t);
typedef CUresult (*f_occcl)(int *, CUfunction, const CUlaunchConfig *);
typedef CUresult (*f_tmap)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                           const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                           CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static struct {
    int      tried, ok;
    void    *lib;
    f_init   init;
    f_errstr errstr;
    f_ctxget ctxget;
    f_ctxid  ctxid;            /* cuCtxGetId: optional (CUDA 12.0 drivers and later) */
    f_ctxset ctxset;
    f_ctxdev ctxdev;
    f_devget devget;
    f_retain retain;
    f_attr   attr;
    f_modload modload;
    f_getfn  getfn;
    f_fnattr fnattr;
    f_launch launch;
    f_launchex launchex;
    f_alloc  alloc;
    f_free   free_;
    f_memset32 memset32;
    f_h2d    h2d;
    f_d2h    d2h;
    f_ssync  ssync;
    f_squery squery;
    f_cpy2d  cpy2d;
    f_screate screate;
    f_ecreate ecreate;
    f_erecord erecord;
    f_swait  swait;
    f_occ    occ;
    f_occcl  occcl;
    f_tmap   tmap;
} D;

static pthread_mutex_t LOCK = PTHREAD_MUTEX_INITIALIZER;

static int cu_fail(CUresult r, const char *what)
{
    char msg[240];
    const char *s = NULL;
    if (D.errstr) D.errstr(r, &s);
    snprintf(msg, sizeof msg, "%s (CUDA error %d%s%s)", what, (int)r, s ? ": " : "", s ? s : "");
    return irx_fail(r == CUDA_ERROR_OUT_OF_MEMORY ? E094 : E092, msg);
}

#define SYM(field, name) do { *(void **)&D.field = dlsym(D.lib, name); if (!D.field) return 0; } while (0)

static int drv_open_locked(void)
{
    if (D.tried) return D.ok;
    D.tried = 1;
    D.lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!D.lib) return 0;
    SYM(init, "cuInit");
    SYM(errstr, "cuGetErrorString");
    SYM(ctxget, "cuCtxGetCurrent");
    *(void **)&D.ctxid = dlsym(D.lib, "cuCtxGetId");
    SYM(ctxset, "cuCtxSetCurrent");
    SYM(ctxdev, "cuCtxGetDevice");
    SYM(devget, "cuDeviceGet");
    SYM(retain, "cuDevicePrimaryCtxRetain");
    SYM(attr, "cuDeviceGetAttribute");
    SYM(modload, "cuModuleLoadData");
    SYM(getfn, "cuModuleGetFunction");
    SYM(fnattr, "cuFuncSetAttribute");
    SYM(launch, "cuLaunchKernel");
    SYM(launchex, "cuLaunchKernelEx");
    SYM(alloc, "cuMemAlloc_v2");
    SYM(free_, "cuMemFree_v2");
    SYM(memset32, "cuMemsetD32Async");
    SYM(h2d, "cuMemcpyHtoDAsync_v2");
    SYM(d2h, "cuMemcpyDtoHAsync_v2");
    SYM(ssync, "cuStreamSynchronize");
    SYM(squery, "cuStreamQuery");
    SYM(cpy2d, "cuMemcpy2DAsync_v2");
    SYM(screate, "cuStreamCreate");
    SYM(ecreate, "cuEventCreate");
    SYM(erecord, "cuEventRecord");
    SYM(swait, "cuStreamWaitEvent");
    SYM(occ, "cuOccupancyMaxActiveBlocksPerMultiprocessor");
    SYM(occcl, "cuOccupancyMaxActiveClusters");
    SYM(tmap, "cuTensorMapEncodeTiled");
    if (D.init(0) != CUDA_SUCCESS) return 0;
    D.ok = 1;
    return 1;
}

/* ---- per-context module table ---- */

extern const unsigned char irx_cubin[];   /* embedded by cubin_blob.S */

#define MAX_CTX 16

static const char *const KNAMES[K_COUNT] = {
    "irx_pw_s1_t1", "irx_pw_s1_t8", "irx_pw_s2_t1", "irx_pw_s2_t8",
    "irx_pw_s3_t1", "irx_pw_s3_t8", "irx_pw_s4_t1", "irx_pw_s4_t8",
    "irx_red_rows_p0", "irx_red_rows_p1", "irx_red_all_p0", "irx_red_all_p1",
    "irx_rowop", "irx_row_rmsnorm", "irx_row_softmax", "irx_row_l2norm",
    "irx_mm_f32", "irx_mm_bf16", "irx_mm_bf16_simt", "irx_attn_f32", "irx_attn_bf16", "irx_attn_bf16_simt",
    "irx_mm_bf16_pair", "irx_mm_bf16_wide"
};

static irx_dev_t CTX[MAX_CTX];
static int NCTX;

static int dev_setup_locked(irx_dev_t *d)
{
    CUresult r;
    CUdevice dev;
    int i;
    if ((r = D.ctxdev(&dev)) != CUDA_SUCCESS) return cu_fail(r, "the current CUDA device");
    d->dev = dev;
    if ((r = D.modload(&d->mod, irx_cubin)) != CUDA_SUCCESS) {
        char msg[120];
        snprintf(msg, sizeof msg, "the sm_100a kernel module on device %d (is it a B200?)", (int)dev);
        return cu_fail(r, msg);
    }
    for (i = 0; i < K_COUNT; i++) {
        if (D.getfn(&d->fn[i], d->mod, KNAMES[i]) != CUDA_SUCCESS) d->fn[i] = NULL;
    }
    D.attr(&d->sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev);
    D.attr(&d->smem_optin, CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN, dev);
    if ((r = D.alloc(&d->scratch, SCRATCH_BYTES)) != CUDA_SUCCESS)
        return cu_fail(r, "the device scratch area");
    if ((r = D.memset32(d->scratch, 0, SCRATCH_BYTES / 4, NULL)) != CUDA_SUCCESS ||
        (r = D.ssync(NULL)) != CUDA_SUCCESS) return cu_fail(r, "clearing the device scratch area");
    d->err = d->scratch;
    d->slot0 = 0;
    return 0;
}

/* The calling thread's current context and an identity for it: the driver's unique context ID
 * (cuCtxGetId), which a context created later never shares even when the driver hands out the
 * same handle again, or the handle itself on a driver without it. */
static int ctx_identity_locked(CUcontext ctx, unsigned long long *id)
{
    if (D.ctxid && D.ctxid(ctx, id) == CUDA_SUCCESS) return 0;
    *id = (unsigned long long)(size_t)ctx;
    return 0;
}

int irx_ctx_current(void **ctx, unsigned long long *id)
{
    CUcontext c = NULL;
    CUresult r;
    int rc = 0;
    pthread_mutex_lock(&LOCK);
    *ctx = NULL;
    *id = 0;
    if (!drv_open_locked()) rc = irx_fail(E090, "the CUDA driver (libcuda.so.1) is missing or would not initialise");
    else if ((r = D.ctxget(&c)) != CUDA_SUCCESS) rc = cu_fail(r, "the current CUDA context");
    else if (c) {
        *ctx = (void *)c;
        ctx_identity_locked(c, id);
    }
    pthread_mutex_unlock(&LOCK);
    return rc;
}

int irx_dev_get(irx_dev_t **out)
{
    CUcontext ctx = NULL;
    CUresult r;
    unsigned long long id = 0;
    int i, rc = 0;
    pthread_mutex_lock(&LOCK);
    if (!drv_open_locked()) { pthread_mutex_unlock(&LOCK); return irx_fail(E090, "a launch: the CUDA driver (libcuda.so.1) is missing or would not initialise"); }
    if ((r = D.ctxget(&ctx)) != CUDA_SUCCESS) { pthread_mutex_unlock(&LOCK); return cu_fail(r, "the current CUDA context"); }
    if (!ctx) {
        /* no current context (a caller with no CUDA runtime): use device 0's primary one */
        CUdevice dev;
        if ((r = D.devget(&dev, 0)) != CUDA_SUCCESS || (r = D.retain(&ctx, dev)) != CUDA_SUCCESS ||
            (r = D.ctxset(ctx)) != CUDA_SUCCESS) { pthread_mutex_unlock(&LOCK); return cu_fail(r, "device 0's primary context"); }
    }
    ctx_identity_locked(ctx, &id);
    for (i = 0; i < NCTX; i++) if (CTX[i].ctx == ctx && CTX[i].ctx_id == id) { *out = &CTX[i]; pthread_mutex_unlock(&LOCK); return 0; }
    if (NCTX >= MAX_CTX) { pthread_mutex_unlock(&LOCK); return irx_fail(E081, "more CUDA contexts than the module table holds"); }
    memset(&CTX[NCTX], 0, sizeof CTX[NCTX]);
    CTX[NCTX].ctx = ctx;
    CTX[NCTX].ctx_id = id;
    rc = dev_setup_locked(&CTX[NCTX]);
    if (!rc) *out = &CTX[NCTX++];
    pthread_mutex_unlock(&LOCK);
    return rc;
}

/* The next per-launch scratch slot of this context: a launch that needs scratch (a full
 * reduction's block partials and ticket, attention's unit counter) takes its own slot, so
 * launches on different streams do not share one unless IRX_SLOTS of them are in flight at
 * once. Called under the launch lock. */
int irx_dev_slot(irx_dev_t *d, irx_slot_t *s)
{
    const unsigned k = d->slot0++ % IRX_SLOTS;
    const CUdeviceptr base = d->scratch + SCRATCH_HEAD + (CUdeviceptr)k * SLOT_BYTES;
    s->index = k;
    s->partial = base;
    s->ticket = base + SLOT_PARTIALS * sizeof(float);
    s->sched = s->ticket + 16 * sizeof(unsigned);
    return 0;
}

int irx_dev_fn(irx_dev_t *d, int k, CUfunction *fn)
{
    if (k < 0 || k >= K_COUNT || !d->fn[k]) {
        char msg[120];
        snprintf(msg, sizeof msg, "the kernel %s, which the sm_100a module does not hold", k >= 0 && k < K_COUNT ? KNAMES[k] : "?");
        return irx_fail(E091, msg);
    }
    *fn = d->fn[k];
    return 0;
}

int irx_dev_launch(irx_dev_t *d, int k, unsigned grid, unsigned block, unsigned smem, unsigned cluster,
                   void *stream, void *params)
{
    CUfunction fn = NULL;
    CUresult r;
    void *args[1];
    if (irx_dev_fn(d, k, &fn)) return 1;
    if (smem > d->smem_set[k]) {       /* raised once per kernel and size, not on every launch */
        if ((r = D.fnattr(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem)) != CUDA_SUCCESS)
            return cu_fail(r, "raising a kernel's shared memory limit");
        d->smem_set[k] = smem;
    }
    args[0] = params;
    {
        /* every prebuilt kernel opens with irx_pdl_enter, so it may be launched while the
         * stream's previous kernel drains (programmatic stream serialization) */
        CUlaunchConfig cfg;
        CUlaunchAttribute at[2];
        memset(&cfg, 0, sizeof cfg);
        memset(at, 0, sizeof at);
        at[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        at[0].value.programmaticStreamSerializationAllowed = 1;
        at[1].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
        at[1].value.clusterDim.x = cluster > 1 ? cluster : 1;
        at[1].value.clusterDim.y = 1;
        at[1].value.clusterDim.z = 1;
        cfg.gridDimX = grid; cfg.gridDimY = 1; cfg.gridDimZ = 1;
        cfg.blockDimX = block; cfg.blockDimY = 1; cfg.blockDimZ = 1;
        cfg.sharedMemBytes = smem;
        cfg.hStream = (CUstream)stream;
        cfg.attrs = at;
        cfg.numAttrs = cluster > 1 ? 2 : 1;
        r = D.launchex(&cfg, fn, args, NULL);
    }
    if (r != CUDA_SUCCESS) return cu_fail(r, "a kernel launch");
    return 0;
}

/* A kernel image built at run time (a per-graph cubin): loaded into the current context, which
 * keeps it until the context ends. */
int irx_dev_load_fn(const void *image, const char *name, CUfunction *fn)
{
    CUmodule mod;
    CUresult r;
    if ((r = D.modload(&mod, image)) != CUDA_SUCCESS) return cu_fail(r, "loading a per-graph sm_100a module");
    if ((r = D.getfn(fn, mod, name)) != CUDA_SUCCESS) return cu_fail(r, "the entry of a per-graph module");
    return 0;
}

/* A per-graph kernel's launch; `pdl` only for a kernel whose source opens with the programmatic
 * dependent launch pair (griddepcontrol launch_dependents, then wait), as irx_pdl_enter does. */
int irx_dev_launch_fn(CUfunction fn, unsigned grid, unsigned block, void *stream, void *params, int pdl)
{
    void *args[1] = {params};
    CUresult r;
    if (pdl) {
        CUlaunchConfig cfg;
        CUlaunchAttribute at;
        memset(&cfg, 0, sizeof cfg);
        memset(&at, 0, sizeof at);
        at.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        at.value.programmaticStreamSerializationAllowed = 1;
        cfg.gridDimX = grid; cfg.gridDimY = 1; cfg.gridDimZ = 1;
        cfg.blockDimX = block; cfg.blockDimY = 1; cfg.blockDimZ = 1;
        cfg.hStream = (CUstream)stream;
        cfg.attrs = &at;
        cfg.numAttrs = 1;
        r = D.launchex(&cfg, fn, args, NULL);
    } else {
        r = D.launch(fn, grid, 1, 1, block, 1, 1, 0, (CUstream)stream, args, NULL);
    }
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, "a kernel launch");
}

int irx_dev_occupancy_fn(CUfunction fn, int block, int *per_sm)
{
    CUresult r = D.occ(per_sm, fn, block, 0);
    if (r != CUDA_SUCCESS) return cu_fail(r, "a kernel's occupancy");
    if (*per_sm < 1) *per_sm = 1;
    return 0;
}

int irx_dev_occupancy(irx_dev_t *d, int k, int block, size_t smem, int *per_sm)
{
    CUfunction fn = NULL;
    CUresult r;
    if (irx_dev_fn(d, k, &fn)) return 1;
    if (smem > d->smem_set[k]) {
        if ((r = D.fnattr(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem)) != CUDA_SUCCESS)
            return cu_fail(r, "raising a kernel's shared memory limit");
        d->smem_set[k] = (unsigned)smem;
    }
    if ((r = D.occ(per_sm, fn, block, smem)) != CUDA_SUCCESS) return cu_fail(r, "a kernel's occupancy");
    if (*per_sm < 1) *per_sm = 1;
    return 0;
}

/* How many clusters of `cluster` CTAs of kernel k fit on the device at once. */
int irx_dev_max_clusters(irx_dev_t *d, int k, unsigned grid, int block, size_t smem, unsigned cluster, int *n)
{
    CUfunction fn = NULL;
    CUresult r;
    CUlaunchConfig cfg;
    CUlaunchAttribute at;
    if (irx_dev_fn(d, k, &fn)) return 1;
    if (smem > d->smem_set[k]) {       /* raised once per kernel and size, not on every launch */
        if ((r = D.fnattr(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem)) != CUDA_SUCCESS)
            return cu_fail(r, "raising a kernel's shared memory limit");
        d->smem_set[k] = smem;
    }
    memset(&cfg, 0, sizeof cfg);
    memset(&at, 0, sizeof at);
    at.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    at.value.clusterDim.x = cluster;
    at.value.clusterDim.y = 1;
    at.value.clusterDim.z = 1;
    cfg.gridDimX = grid; cfg.gridDimY = 1; cfg.gridDimZ = 1;
    cfg.blockDimX = (unsigned)block; cfg.blockDimY = 1; cfg.blockDimZ = 1;
    cfg.sharedMemBytes = (unsigned)smem;
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    if ((r = D.occcl(n, fn, &cfg)) != CUDA_SUCCESS) return cu_fail(r, "a kernel's cluster occupancy");
    if (*n < 1) *n = 1;
    return 0;
}

int irx_dev_alloc(size_t bytes, CUdeviceptr *p)
{
    CUresult r = D.alloc(p, bytes ? bytes : 16);
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, "a device buffer");
}

void irx_dev_free(CUdeviceptr p) { if (p) D.free_(p); }

/* The two copy streams and the events of the pipelined host path, made on first use in this
 * context: non-blocking streams, ordered against the caller's stream by events only. */
int irx_dev_pipe(irx_dev_t *d)
{
    CUresult r = CUDA_SUCCESS;
    int i;
    pthread_mutex_lock(&LOCK);
    if (!d->pipe_ok) {
        for (i = 0; i < 2 && r == CUDA_SUCCESS; i++)
            if (!d->pipe[i]) r = D.screate(&d->pipe[i], CU_STREAM_NON_BLOCKING);
        for (i = 0; i < IRX_PIPE_EVENTS && r == CUDA_SUCCESS; i++)
            if (!d->pev[i]) r = D.ecreate(&d->pev[i], CU_EVENT_DISABLE_TIMING);
        d->pipe_ok = r == CUDA_SUCCESS;
    }
    pthread_mutex_unlock(&LOCK);
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, "the host path's copy streams");
}

/* `after` waits, on the device, for the work issued to `before` so far (event `ev`). */
int irx_dev_order(irx_dev_t *d, int ev, void *before, void *after)
{
    CUresult r = D.erecord(d->pev[ev], (CUstream)before);
    if (r == CUDA_SUCCESS) r = D.swait((CUstream)after, d->pev[ev], 0);
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, "ordering the host path's streams");
}

int irx_dev_h2d(CUdeviceptr d, const void *h, size_t n, void *s)
{
    CUresult r = D.h2d(d, h, n, (CUstream)s);
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, "a host-to-device copy");
}

int irx_dev_d2h(void *h, CUdeviceptr d, size_t n, void *s)
{
    CUresult r = D.d2h(h, d, n, (CUstream)s);
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, "a device-to-host copy");
}

/* A 2-D copy between host and device: `rows` rows of `width` bytes, at row pitches `hpitch`
 * (host) and `dpitch` (device); to_dev picks the direction. */
int irx_dev_copy2d(int to_dev, void *h, size_t hpitch, CUdeviceptr d, size_t dpitch, size_t width, size_t rows, void *s)
{
    CUDA_MEMCPY2D c;
    CUresult r;
    memset(&c, 0, sizeof c);
    if (to_dev) {
        c.srcMemoryType = CU_MEMORYTYPE_HOST; c.srcHost = h; c.srcPitch = hpitch;
        c.dstMemoryType = CU_MEMORYTYPE_DEVICE; c.dstDevice = d; c.dstPitch = dpitch;
    } else {
        c.srcMemoryType = CU_MEMORYTYPE_DEVICE; c.srcDevice = d; c.srcPitch = dpitch;
        c.dstMemoryType = CU_MEMORYTYPE_HOST; c.dstHost = h; c.dstPitch = hpitch;
    }
    c.WidthInBytes = width;
    c.Height = rows;
    r = D.cpy2d(&c, (CUstream)s);
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, to_dev ? "a 2-D host-to-device copy" : "a 2-D device-to-host copy");
}

/* ---- host waits, with a deadline ---- */

static unsigned long long HOST_WAIT_US;     /* 0: not read yet; set by irx_inject or IRX_HOST_WAIT_S */

void irx_host_wait_limit(unsigned long long us) { HOST_WAIT_US = us; }

static unsigned long long host_wait_us(void)
{
    if (!HOST_WAIT_US) {
        const char *e = getenv("IRX_HOST_WAIT_S");
        double sec = e ? atof(e) : 0.0;
        HOST_WAIT_US = sec > 0 ? (unsigned long long)(sec * 1e6) : 120ull * 1000000ull;
    }
    return HOST_WAIT_US;
}

static unsigned long long now_us(void)
{
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (unsigned long long)t.tv_sec * 1000000ull + (unsigned long long)t.tv_nsec / 1000ull;
}

/* Wait for the stream's work, at most the host wait limit (120 s unless IRX_HOST_WAIT_S or
 * irx_inject set another): the stream is polled, spinning for the first 200 microseconds, then
 * with short sleeps. Work that outlives the limit is left running and reported as E092, so a
 * caller is never blocked without end by a kernel that does not finish. */
int irx_dev_sync(void *s)
{
    const unsigned long long t0 = now_us(), lim = host_wait_us();
    for (;;) {
        CUresult r = D.squery((CUstream)s);
        unsigned long long el;
        if (r == CUDA_SUCCESS) return 0;
        if (r != CUDA_ERROR_NOT_READY) return cu_fail(r, "waiting for the stream");
        el = now_us() - t0;
        if (el > lim) {
            char msg[160];
            snprintf(msg, sizeof msg, "a stream whose work did not finish within the host wait limit (%.3f s)", lim / 1e6);
            return irx_fail(E092, msg);
        }
        if (el > 200) {
            struct timespec ts = {0, 20000};
            nanosleep(&ts, NULL);
        }
    }
}

int irx_dev_memset32(CUdeviceptr p, unsigned v, size_t n, void *s)
{
    CUresult r = D.memset32(p, v, n, (CUstream)s);
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, "a device memset");
}

int irx_dev_tmap(CUtensorMap *m, CUtensorMapDataType dt, unsigned rank, void *base, const cuuint64_t *dims,
                 const cuuint64_t *strides, const cuuint32_t *box, CUtensorMapSwizzle sw)
{
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    CUresult r = D.tmap(m, dt, rank, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : cu_fail(r, "encoding a TMA tensor map");
}

/* Wait (bounded) for the stream, then read and clear the device error word of this context. The
 * bounded wait comes first: a copy into pageable host memory would itself wait for the stream
 * without a limit. */
int irx_dev_check_err(irx_dev_t *d, void *s)
{
    unsigned e = 0;
    if (irx_dev_sync(s) || irx_dev_d2h(&e, d->err, sizeof e, s) || irx_dev_sync(s)) return 1;
    if (e) {
        irx_dev_memset32(d->err, 0, 1, s);
        irx_dev_sync(s);
        return irx_fail(E092, e & IRX_KERR_TIMEOUT ? "a kernel whose bounded device wait ran out (error word set)"
                                                   : "a kernel that set its device error word");
    }
    return 0;
}
