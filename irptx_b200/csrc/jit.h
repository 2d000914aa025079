/* jit.h -- per-graph kernels compiled at run time (jit.c). */
#ifndef IRX_JIT_H
#define IRX_JIT_H

#include <stdint.h>
#include <cuda.h>
#include "irx_int.h"
#include "launch.h"

#ifndef IRX_JIT_PW_W
#define IRX_JIT_PW_W        8          /* elements per thread per step of the vector pass */
#endif
#define IRX_JIT_PW_THREADS  256
#ifndef IRX_JIT_PW_MINB
#define IRX_JIT_PW_MINB     4          /* resident blocks per SM the registers must allow */
#endif
#define IRX_JIT_SRC_MAX     (64 * 1024)

/* -1 reads the mode, 0 turns the per-graph kernels off, 1 on (when NVRTC loads); returns the
 * mode now in force. The first use reads IRX_JIT from the environment ("0": off). */
int irx_jit_mode(int mode);
int irx_jit_source(const irx_plan_int_t *p, char *buf, size_t cap);
uint64_t irx_jit_key(const irx_plan_int_t *p);
int irx_jit_prepare(const irx_plan_int_t *p);
int irx_jit_pw_fn(const irx_plan_int_t *p, irx_dev_t *d, CUfunction *fn, int *occ);

#endif
