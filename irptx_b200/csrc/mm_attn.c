/* mm_attn.c -- launchers for the matmul and attention templates. */
#include <string.h>
#include "irx_int.h"
#include "irx_kparams.h"
#include "launch.h"

int irx_launch_mm(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st)
{
    CUfunction fn;
    (void)p; (void)s; (void)ns; (void)args; (void)st;
    return irx_dev_fn(d, p->u.mm.dt == DT_BF16 ? K_MM_BF16 : K_MM_F32, &fn) ? 1 : irx_fail(E091, "a matmul launch");
}

int irx_launch_attn(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st)
{
    CUfunction fn;
    (void)p; (void)s; (void)ns; (void)args; (void)st;
    return irx_dev_fn(d, p->u.at.dt == DT_BF16 ? K_ATTN_BF16 : K_ATTN_F32, &fn) ? 1 : irx_fail(E091, "an attention launch");
}
