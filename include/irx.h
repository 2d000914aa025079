/* irx.h -- the C ABI of irptx-b200, the sm_100a backend for irptx KIR graphs.
 *
 * Plain C: no C++ or torch types cross it. Pointers are device pointers (CUdeviceptr values
 * cast to void *) unless a function says host; streams are CUstream values (a cudaStream_t is
 * the same handle) or NULL for the legacy default stream. Every function returns 0 on success;
 * on failure it returns 1 after printing exactly one `error[E0NN]: irptx: cannot lower ...`
 * line on stderr, the reference's refusal contract (src/err.c:96-114, src/main.c:1-6), and the
 * code and line stay readable through irx_last_error(). A plan is caller-owned storage of fixed
 * size holding no pointers: copy it, cache it, share it between threads.
 *
 * Reference interfaces replaced (BhuvanB404/IRptx 0.1.0, paths within that project):
 *   irx_compile          kr_load (src/kir.h:26-29) followed by is_run, vf_run and em_run
 *                        (src/irptx.h:345-353): KIR text in, a launchable product out, or
 *                        one E-coded refusal
 *   irx_plan_describe    the printed module (em_run's buffer, src/irptx.h:349-353): here a
 *                        one-line description of the selected template and its shape
 *   irx_launch           the runner's cuModuleLoadData + cuLaunchKernel of the emitted PTX
 *                        with one device pointer per KIR arg in arg order
 *                        (tests/gpurun.py:91-107)
 *   irx_run_host         the runner's host path: host buffers copied in, the kernel run,
 *                        outputs copied back (tests/gpurun.py:100-118)
 *   irx_last_error       the single stderr line of er_fail (src/err.c:96-114), kept for
 *                        callers that cannot read stderr
 *   irx_plan_source      the emitted module text itself (em_run, src/emit.c:357-376): for a
 *                        pointwise plan, the CUDA source of its per-graph sm_100a kernel
 *   irx_prepare          the runner's cuModuleLoadData JIT step (tests/gpurun.py:94), done
 *                        ahead of the first launch
 */

#ifndef IRX_H
#define IRX_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden symbols; only these entry points are exported. */
#if defined(__GNUC__)
#define IRX_API __attribute__((visibility("default")))
#else
#define IRX_API
#endif

#define IRX_PLAN_BYTES 4096

typedef struct irx_plan { unsigned long long opaque[IRX_PLAN_BYTES / 8]; } irx_plan_t;

enum irx_family {
    IRX_FAM_NONE = 0,
    IRX_FAM_POINTWISE = 1,     /* elementwise program over 1-4 input streams */
    IRX_FAM_REDUCE_ALL = 2,    /* one output element: fold of the whole input */
    IRX_FAM_REDUCE_ROWS = 3,   /* y[row] = fold over the row */
    IRX_FAM_ROWOP = 4,         /* row statistics, then an elementwise pass over the row */
    IRX_FAM_MATMUL = 5,        /* C[M,N] = A[M,K] B[K,N] */
    IRX_FAM_ATTENTION = 6,     /* O = softmax(Q K^T * scale [causal]) V over [B,H,S,D] */
    IRX_FAM_KIR = 7            /* any other graph the reference lowers: its statements written out
                                * as the graph's own sm_100a kernel (NVRTC), on the KIR's launch
                                * geometry; runs as one launch (shard 0 of any count) */
};

enum irx_dtype { IRX_DT_F32 = 1, IRX_DT_BF16 = 2 };
enum irx_argkind { IRX_ARG_IN = 0, IRX_ARG_CONST = 1, IRX_ARG_OUT = 2 };

/* "irptx-b200 <version>". Replaces `irptx --version` (src/main.c:56-59). */
IRX_API const char *irx_version(void);

/* Parse KIR text and select the sm_100a template for it (no GPU needed). Replaces kr_load +
 * is_run + vf_run + em_run (src/kir.h:26-29, src/irptx.h:345-353). Thread-safe. */
IRX_API int irx_compile(const char *kir, size_t len, irx_plan_t *plan);

/* Parse KIR text and write it out as its own generic kernel (family IRX_FAM_KIR), skipping the
 * op-family templates: each statement lowered as the reference lowers it (src/isel.c), in the
 * reference's per-element order and on the KIR's launch geometry. irx_compile falls back to this
 * for graphs no template takes; calling it directly gives the reference's exact order for any
 * graph (and tests the generic path). No counterpart in the reference beyond is_run itself. */
IRX_API int irx_compile_generic(const char *kir, size_t len, irx_plan_t *plan);

/* The selected family (enum irx_family), or 0 for a plan that was never compiled. */
IRX_API int irx_plan_family(const irx_plan_t *plan);

/* Number of KIR args; then, per arg i (KIR arg order, the reference's param order,
 * src/emit.c:318-334), its kind (enum irx_argkind), dtype (enum irx_dtype) and element count. */
IRX_API int irx_plan_nargs(const irx_plan_t *plan);
IRX_API int irx_plan_arg(const irx_plan_t *plan, unsigned i, int *kind, int *dtype, long long *elems);

/* One line describing the template and shape, NUL-terminated into buf (truncated to cap). */
IRX_API int irx_plan_describe(const irx_plan_t *plan, char *buf, size_t cap);

/* Algorithmic work of one full launch: HBM bytes the family must move (inputs read once,
 * outputs written once) and floating-point operations (2 per multiply-add for matmul and
 * attention; causal attention counts half the score matrix). */
IRX_API int irx_plan_work(const irx_plan_t *plan, double *bytes, double *flops);

/* How many independent shard units the plan has: elements/8 (pointwise), rows (reductions,
 * row ops), 256-column blocks (matmul), batch*head (attention), element blocks (full sum). */
IRX_API long long irx_plan_units(const irx_plan_t *plan);

/* Queue the plan on `stream` with one device pointer per KIR arg (args[i] for arg i). Outputs
 * that the KIR adds into (an atomic Write) must hold their starting value, as the reference's
 * runner zeroes them (tests/gpurun.py:61-63). Replaces the runner's launch of the PTX
 * (tests/gpurun.py:91-107). */
IRX_API int irx_launch(const irx_plan_t *plan, void *const *args, unsigned nargs, void *stream);

/* Queue shard `shard` of `nshards` of the plan: the same args, full-size buffers, but only
 * the shard's part of the work (a contiguous range of the plan's units). A full reduction's
 * shard writes its partial result (no add into the output); combining the shards' partials
 * (an all-reduce over GPUs) is the caller's. */
IRX_API int irx_launch_shard(const irx_plan_t *plan, unsigned shard, unsigned nshards, void *const *args, unsigned nargs,
                     void *stream);

/* How irx_launch_shard splits a plan: shard `shard` of `nshards` covers units [*u0, *u1) of
 * irx_plan_units (contiguous, in order, together exactly all units; a shard past the end is
 * empty), and *combine says how the shards' outputs make the whole result: IRX_COMBINE_NONE,
 * each shard writes its own part of the outputs; otherwise (a full reduction over several
 * shards) every shard writes a partial result of the output's size, and the result is their
 * elementwise sum, maximum, minimum or product (an all-reduce across GPUs). No counterpart in
 * the reference, whose runner launches one kernel on one GPU. */
enum irx_combine { IRX_COMBINE_NONE = 0, IRX_COMBINE_SUM = 1, IRX_COMBINE_MAX = 2, IRX_COMBINE_MIN = 3,
                   IRX_COMBINE_PROD = 4 };
IRX_API int irx_plan_shard(const irx_plan_t *plan, unsigned shard, unsigned nshards, long long *u0, long long *u1,
                   int *combine);

/* The whole path from host memory: copy the args' host buffers in (inputs and consts, and the
 * outputs on a `zero` line, whose starting value the kernel reads), launch, copy the outputs
 * back, and wait. Pinned host buffers make the copies asynchronous and full speed. Replaces the
 * runner's host path (tests/gpurun.py:100-118).
 * A run that moves at least 64 MB, 8 MB of it output, of a family whose outputs split with its
 * units (pointwise, row reductions, row ops, matmul, attention) is pipelined: its units go in
 * chunks of about 32 MB of copies (at most 16), each chunk's copy in, kernel and copy out
 * ordered by events on two copy streams of the library and the given stream, so copies in and
 * out overlap on the bus. The results are the same bits as one launch. The staging area and the
 * copy streams are per context: runs from several threads on one context must not overlap. */
IRX_API int irx_run_host(const irx_plan_t *plan, void *const *host_args, unsigned nargs, void *stream);

/* How many chunks irx_run_host_shard (irx_run_host: shard 0 of 1) runs this shard in: 1 when it
 * is not pipelined, -1 on a bad plan or shard. Needs no GPU. */
IRX_API int irx_run_host_chunks(const irx_plan_t *plan, unsigned shard, unsigned nshards);

/* The host path of one shard (irx_launch_shard's split): full-size host buffers, of which only
 * the shard's slices cross the bus (its element or row range, its (batch, head) pairs, a
 * matmul's B and C columns with A whole; scalars and a row op's weight whole), launched into a
 * full-size device staging area and copied back. Only inputs and the outputs whose starting
 * value the kernel reads (those on a `zero` line) are copied in. A full reduction's shard
 * returns its partial result in the output; combining the shards' partials is the caller's, as
 * for irx_launch_shard. No counterpart in the reference, whose runner uses one GPU; the
 * unsharded case (shard 0 of 1) is irx_run_host. */
IRX_API int irx_run_host_shard(const irx_plan_t *plan, unsigned shard, unsigned nshards, void *const *host_args,
                               unsigned nargs, void *stream);

/* The full reduction (a plan of family IRX_FAM_REDUCE_ALL) without any device allocation, for
 * callers that cannot let a library allocate GPU memory: an application that gives all of the
 * GPU's memory to its own pool, or one that must not allocate after start-up (cudaMalloc can
 * synchronise the device and can fail under memory pressure). No counterpart in the reference:
 * its product is PTX text, and its runner allocates every buffer itself.
 * The block partials and arrival ticket live in a fixed array compiled into the library (one
 * per GPU that loads it, kept until exit) that holds 4096 block partials; a launch needing more
 * is refused (E093). Every call shares that array: calls whose kernels overlap on the GPU race.
 * The first call in each CUDA context loads the library's copy of the kernel into it (device
 * memory for the code and the array) and looks the array's address up (cudaGetSymbolAddress)
 * in that context; make it during start-up, before any phase that must not allocate and before
 * any stream capture. Contexts are told apart by the driver's context ID, so several contexts
 * on one device, or a context made after a reset, each get their own address. Same args as
 * irx_launch; the result agrees with irx_launch's within the f32 reduction tolerance (its grid
 * comes from the runtime's occupancy of its own kernel copy, so the blocks can group
 * differently). */
IRX_API int irx_reduce_all_noalloc(const irx_plan_t *plan, void *const *args, unsigned nargs, void *stream);

/* Per-graph kernels. A pointwise plan runs a kernel written for its graph: the element function
 * is emitted as CUDA source into a fixed kernel template and compiled for sm_100a with NVRTC
 * (libnvrtc.so.12, opened at run time) on the plan's first launch in the process, then cached
 * and loaded once per CUDA context. Other families run prebuilt kernels.
 *
 * irx_plan_source writes that source (NUL-terminated, truncated to cap) and returns its full
 * length, or -1 for a plan of another family. irx_prepare compiles it now (no GPU needed), so
 * the first launch does not pay for the compile; 0 for plans with nothing to compile.
 * irx_jit(0) makes pointwise plans run the prebuilt kernel that interprets the graph's op
 * programs instead (same results, bit for bit), irx_jit(1) returns to per-graph kernels when
 * NVRTC loads, irx_jit(-1) only reads; each returns the mode now in force. The first use reads
 * IRX_JIT from the environment ("0": off). */
IRX_API int irx_plan_source(const irx_plan_t *plan, char *buf, size_t cap);
IRX_API int irx_prepare(const irx_plan_t *plan);
IRX_API int irx_jit(int mode);

/* Wait for `stream` and read the device error word that a kernel whose bounded wait ran out
 * sets; E092 when it was set (and clears it). The wait on the host is bounded too (120 s, or
 * IRX_HOST_WAIT_S seconds from the environment): work still running then is reported as E092
 * and left to finish. */
IRX_API int irx_check(void *stream);

/* Failure injection for tests of the timeout paths, with no GPU fault. No counterpart in the
 * reference. IRX_INJECT_MM_NO_LOADS: the next bf16 tcgen05 matmul launch issues none of its
 * TMA loads and bounds each of its device waits by `value` microseconds, so its MMA and
 * epilogue waits run out with no copy in flight; the kernel stops, frees its TMEM, returns, and
 * irx_check reports E092. IRX_INJECT_HOST_WAIT: host waits (irx_check, irx_run_host) give up
 * after `value` microseconds (0: the default). IRX_INJECT_NONE clears both. */
enum irx_inject_kind { IRX_INJECT_NONE = 0, IRX_INJECT_MM_NO_LOADS = 1, IRX_INJECT_HOST_WAIT = 2 };
IRX_API int irx_inject(int what, unsigned long long value);

/* The last error's code (E-number) and line on this thread; -1 and "" when there is none. */
IRX_API int irx_last_error(char *buf, size_t cap);

/* 1: keep refusal lines off stderr (they stay readable through irx_last_error). */
IRX_API void irx_quiet(int on);

#ifdef __cplusplus
}
#endif

#endif /* IRX_H */
