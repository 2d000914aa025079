// noalloc.cu -- irx_reduce_all_noalloc: the full reduction with no device allocation at all.
//
// The ordinary full reduction (irx_launch of a reduce_all plan) keeps its block partials and its
// arrival ticket in a scratch area that the library allocates on the device the first time a
// context is used. Some callers cannot allow that: an application that hands all of the GPU's
// memory to its own pool and forbids any other allocation, or one that must not allocate after
// start-up because cudaMalloc can synchronise the whole device and can fail under memory
// pressure. This entry point serves them: its scratch is a fixed array compiled into the
// library (`irx_noalloc_scratch`, one copy per GPU that loads the library, kept until the
// process exits), so a call allocates nothing on the device or the host.
//
// Limits and sharing:
//   * the array holds IRX_NOALLOC_MAX_BLOCKS block partials and one ticket; a launch that would
//     need more blocks is refused with E093 before anything is queued;
//   * every call on a device shares the one array and leaves its last contents behind; the
//     ticket, the only value that must start at zero, is cleared on the caller's stream before
//     each launch. Two calls whose kernels overlap on the GPU (different streams, no ordering
//     between them) race on the array and give wrong results;
//   * the first call in each CUDA context loads this file's kernels into it (the runtime's module
//     load, which takes device memory for the code and the array) and looks the array's device
//     address up (cudaGetSymbolAddress, in that context), keyed by the driver's context ID. So
//     make that first call during start-up, before any phase that must not allocate, and before
//     any stream capture.
//
// The kernel is the same reduction body as irx_red_all_p0/_p1 (kernels/reduce.cu); only where
// its scratch lives differs, and its grid comes from the runtime's occupancy of this file's own
// copy of the kernel, so its fold can group the blocks differently from irx_launch's: the
// result agrees with irx_launch's within the f32 reduction tolerance, not bit for bit. It runs
// through the CUDA runtime in the calling thread's current context (the device's primary
// context when none is current).

#include <cuda_runtime.h>
#include <pthread.h>
#include <stdio.h>
#include <string.h>
#include "kernels/reduce.cu"
#include "../../include/irx.h"

#define IRX_NOALLOC_MAX_BLOCKS 4096
#define IRX_NOALLOC_CTXS 64

extern "C" int irx_ctx_current(void **ctx, unsigned long long *id);   // launch.c

// Block partials first, then the ticket.
static __device__ __align__(256) unsigned char irx_noalloc_scratch[IRX_NOALLOC_MAX_BLOCKS * sizeof(float) + 256];

extern "C" __global__ void __launch_bounds__(RED_ALL_THREADS) irx_red_all_noalloc_p0(const __grid_constant__ irx_kred_t p) { red_all_body<false>(p); }
extern "C" __global__ void __launch_bounds__(RED_ALL_THREADS) irx_red_all_noalloc_p1(const __grid_constant__ irx_kred_t p) { red_all_body<true>(p); }

// One entry per CUDA context the entry point has run in. A context is known by the driver's
// context ID, not by its device number: the array's address belongs to the context whose copy of
// the module holds it, and a caller may run several contexts on one device, or destroy a context
// (cudaDeviceReset) and get a new one, in which the old address means nothing.
static struct {
    unsigned long long id;         // cuCtxGetId of the context (0: free entry)
    unsigned char *scratch;        // device address of irx_noalloc_scratch in that context
    int grid[2];                   // blocks that fill the device, per kernel variant
} NA[IRX_NOALLOC_CTXS];
static int NNA;
static pthread_mutex_t NA_LOCK = PTHREAD_MUTEX_INITIALIZER;

static int na_cuda(cudaError_t e, const char *what)
{
    char msg[200];
    snprintf(msg, sizeof msg, "%s (CUDA runtime error %d: %s)", what, (int)e, cudaGetErrorString(e));
    return irx_fail(E092, msg);
}

// The entry of the calling thread's current context, set up on its first use there: the
// array's device address (cudaGetSymbolAddress in that context) and the grid size. The
// runtime binds the device's primary context to a thread that has none current, so the
// context is read again after the first runtime call.
static int na_entry(int dev, int *slot)
{
    int sms = 0, occ0 = 0, occ1 = 0, rc = 0, i;
    cudaError_t e;
    void *ptr = NULL, *ctx = NULL;
    unsigned long long id = 0;
    if (irx_ctx_current(&ctx, &id)) return 1;
    pthread_mutex_lock(&NA_LOCK);
    if (ctx) for (i = 0; i < NNA; i++) if (NA[i].id == id) { *slot = i; pthread_mutex_unlock(&NA_LOCK); return 0; }
    if ((e = cudaGetSymbolAddress(&ptr, irx_noalloc_scratch)) != cudaSuccess)
        rc = na_cuda(e, "the device address of the fixed reduction scratch");
    else if (irx_ctx_current(&ctx, &id)) rc = 1;
    else if (!ctx) rc = irx_fail(E092, "a no-allocation reduction with no CUDA context current");
    if (!rc) for (i = 0; i < NNA; i++) if (NA[i].id == id) { *slot = i; pthread_mutex_unlock(&NA_LOCK); return 0; }
    if (!rc && NNA >= IRX_NOALLOC_CTXS) rc = irx_fail(E093, "more CUDA contexts than the no-allocation table holds");
    if (!rc && (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        rc = na_cuda(e, "the device's SM count");
    if (!rc && ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ0, irx_red_all_noalloc_p0, RED_ALL_THREADS, 0)) != cudaSuccess ||
                (e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, irx_red_all_noalloc_p1, RED_ALL_THREADS, 0)) != cudaSuccess))
        rc = na_cuda(e, "the reduction kernel's occupancy");
    if (!rc) {
        NA[NNA].id = id;
        NA[NNA].scratch = (unsigned char *)ptr;
        NA[NNA].grid[0] = sms * (occ0 > 0 ? occ0 : 1);
        NA[NNA].grid[1] = sms * (occ1 > 0 ? occ1 : 1);
        *slot = NNA++;
    }
    pthread_mutex_unlock(&NA_LOCK);
    return rc;
}

extern "C" int irx_reduce_all_noalloc(const irx_plan_t *plan, void *const *args, unsigned nargs, void *stream)
{
    const irx_plan_int_t *p = (const irx_plan_int_t *)plan;
    const irx_red_t *r;
    irx_kred_t k;
    int dev = 0, i, e_slot = 0;
    long long want;
    unsigned grid;
    cudaError_t e;

    irx_clear_error();
    if (!p || p->magic != IRX_PLAN_MAGIC) return irx_fail(E093, "a no-allocation reduction of a plan that was never compiled");
    if (p->fam != FAM_REDUCE_ALL || p->u.red.rows != 1)
        return irx_fail(E093, "a no-allocation reduction of a plan that is not a full reduction");
    if (!args || nargs != p->narg) return irx_fail(E093, "a launch whose argument count is not the KIR's");
    for (i = 0; i < (int)nargs; i++) if (!args[i]) return irx_fail(E093, "a launch with a null device pointer");
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return na_cuda(e, "the current device");
    if (na_entry(dev, &e_slot)) return 1;

    r = &p->u.red;
    memset(&k, 0, sizeof k);
    k.x = args[r->x_arg];
    k.y = args[r->y_arg];
    k.partial = (float *)NA[e_slot].scratch;
    k.ticket = (unsigned *)(NA[e_slot].scratch + IRX_NOALLOC_MAX_BLOCKS * sizeof(float));
    for (i = 0; i < r->nuni; i++) {
        k.uni[i].kind = r->uni[i].kind;
        k.uni[i].bits = r->uni[i].v;
        k.uni[i].off = r->uni[i].off;
        if (r->uni[i].kind == UNI_ARG) { k.uni[i].ptr = args[r->uni[i].v]; k.uni[i].dt = p->arg_dt[r->uni[i].v]; }
    }
    k.pre = r->pre;
    k.uprog = r->uprog;
    k.op = r->op; k.x_dt = r->x_dt; k.y_dt = r->y_dt; k.has_pre = r->has_pre;
    k.out_reg = r->out_reg; k.tot_reg = r->tot_reg; k.nuni = r->nuni; k.accumulate = r->accumulate;
    k.rows = 1; k.cols = r->cols;
    k.begin = 0; k.end = r->cols;
    k.vec_ok = (uint8_t)((((unsigned long long)(size_t)k.x) & 15u) == 0);

    want = (r->cols + 4095) / 4096;                       // at least 4096 elements a block
    if (want < 1) want = 1;
    grid = (unsigned)(want < NA[e_slot].grid[r->has_pre ? 1 : 0] ? want : NA[e_slot].grid[r->has_pre ? 1 : 0]);
    if (grid > IRX_NOALLOC_MAX_BLOCKS) {
        char msg[160];
        snprintf(msg, sizeof msg, "a reduction needing %u blocks: the fixed scratch holds %d block partials",
                 grid, IRX_NOALLOC_MAX_BLOCKS);
        return irx_fail(E093, msg);
    }
    if ((e = cudaMemsetAsync(k.ticket, 0, sizeof(unsigned), (cudaStream_t)stream)) != cudaSuccess)
        return na_cuda(e, "clearing the fixed scratch's ticket");
    if (r->has_pre) irx_red_all_noalloc_p1<<<grid, RED_ALL_THREADS, 0, (cudaStream_t)stream>>>(k);
    else irx_red_all_noalloc_p0<<<grid, RED_ALL_THREADS, 0, (cudaStream_t)stream>>>(k);
    if ((e = cudaGetLastError()) != cudaSuccess) return na_cuda(e, "the no-allocation reduction launch");
    return 0;
}
