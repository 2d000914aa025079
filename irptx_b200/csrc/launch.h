/* launch.h -- internal interface between the family launchers and the driver layer. */
#ifndef IRX_LAUNCH_H
#define IRX_LAUNCH_H

#include <stddef.h>
#include <cuda.h>

/* Kernel slots. K_PW + 2 * (streams - 1) + (temporaries > 1) picks a pointwise instance;
 * K_RED_ROWS / K_RED_ALL + (has a pre-program) a reduction instance. */
enum {
    K_PW = 0, K_PW_END = K_PW + 8,
    K_RED_ROWS = K_PW_END, K_RED_ALL = K_RED_ROWS + 2,
    K_ROWOP = K_RED_ALL + 2, K_ROW_RMSNORM, K_ROW_SOFTMAX, K_ROW_L2NORM,
    K_MM_F32, K_MM_BF16, K_MM_BF16_SIMT, K_ATTN_F32, K_ATTN_BF16, K_ATTN_BF16_SIMT,
    K_MM_BF16_PAIR, K_MM_BF16_WIDE,
    K_COUNT
};

/* Per-context scratch: a 256-byte head (the error word) and IRX_SLOTS launch slots, each with
 * SLOT_PARTIALS block partials, an arrival ticket and a unit counter. Tickets are left at zero
 * by the kernel that used them; unit counters are zeroed on the launch's stream. */
#define IRX_SLOTS 64
#define SLOT_PARTIALS 4096
#define SCRATCH_HEAD 256
#define SLOT_BYTES (SLOT_PARTIALS * 4 + 256)
#define SCRATCH_BYTES (SCRATCH_HEAD + IRX_SLOTS * SLOT_BYTES)

/* The pipelined host path splits a run into at most IRX_PIPE_CHUNKS chunks: two events each,
 * plus one to start the copy streams and one to join them. */
#define IRX_PIPE_CHUNKS 16
#define IRX_PIPE_EVENTS (2 * IRX_PIPE_CHUNKS + 3)

typedef struct {
    unsigned    index;
    CUdeviceptr partial, ticket, sched;
} irx_slot_t;

typedef struct {
    CUcontext  ctx;
    unsigned long long ctx_id;         /* cuCtxGetId, or the handle: tells a new context from a dead one */
    CUdevice   dev;
    CUmodule   mod;
    CUfunction fn[K_COUNT];
    unsigned   smem_set[K_COUNT];      /* the dynamic shared memory limit last set per kernel */
    int        sms, smem_optin;
    CUdeviceptr scratch, err;
    unsigned    slot0;                 /* next scratch slot (under the launch lock) */
    CUdeviceptr arena;                 /* irx_run_host's device copies, grown on demand */
    size_t      arena_bytes;
    CUstream    pipe[2];               /* the pipelined host path: copies in, copies out */
    CUevent     pev[IRX_PIPE_EVENTS];
    int         pipe_ok;
} irx_dev_t;

int irx_dev_get(irx_dev_t **out);
int irx_dev_slot(irx_dev_t *d, irx_slot_t *s);
int irx_ctx_current(void **ctx, unsigned long long *id);
int irx_dev_fn(irx_dev_t *d, int k, CUfunction *fn);
int irx_dev_launch(irx_dev_t *d, int k, unsigned grid, unsigned block, unsigned smem, unsigned cluster,
                   void *stream, void *params);
int irx_dev_occupancy(irx_dev_t *d, int k, int block, size_t smem, int *per_sm);
int irx_dev_max_clusters(irx_dev_t *d, int k, unsigned grid, int block, size_t smem, unsigned cluster, int *n);
int irx_dev_load_fn(const void *image, const char *name, CUfunction *fn);
int irx_dev_launch_fn(CUfunction fn, unsigned grid, unsigned block, void *stream, void *params, int pdl);
int irx_dev_occupancy_fn(CUfunction fn, int block, int *per_sm);
int irx_dev_alloc(size_t bytes, CUdeviceptr *p);
void irx_dev_free(CUdeviceptr p);
int irx_dev_h2d(CUdeviceptr d, const void *h, size_t n, void *s);
int irx_dev_d2h(void *h, CUdeviceptr d, size_t n, void *s);
int irx_dev_sync(void *s);
int irx_dev_pipe(irx_dev_t *d);
int irx_dev_order(irx_dev_t *d, int ev, void *before, void *after);
void irx_host_wait_limit(unsigned long long us);
int irx_dev_copy2d(int to_dev, void *h, size_t hpitch, CUdeviceptr d, size_t dpitch, size_t width, size_t rows, void *s);
int irx_dev_memset32(CUdeviceptr p, unsigned v, size_t n, void *s);
int irx_dev_tmap(CUtensorMap *m, CUtensorMapDataType dt, unsigned rank, void *base, const cuuint64_t *dims,
                 const cuuint64_t *strides, const cuuint32_t *box, CUtensorMapSwizzle sw);
int irx_dev_check_err(irx_dev_t *d, void *s);

#endif
