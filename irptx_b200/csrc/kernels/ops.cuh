// ops.cuh -- what each op of an op program computes, in f32.
//
// The one definition of the op semantics. The prebuilt kernels include it through common.cuh;
// the per-graph pointwise kernels that the library compiles at run time (NVRTC) include it
// too, with op codes as constants, so both paths compute bit-identical results. It includes
// nothing but irx_ops.h and uses only functions NVRTC provides without headers.
//
// Arithmetic follows the reference's op table (src/ops.c:123-154): add, subtract, multiply and
// divide round to nearest with no contraction into FMA (the .rn forms), maximum/minimum ignore a
// NaN operand (max.f32), relu is max(x, 0). The transcendental ops call CUDA's own functions;
// the reference uses its own few-ulp sequences (src/fmath.c), so those agree to a tolerance.

#pragma once
#include "irx_ops.h"

__device__ __forceinline__ float irx_ident(int op)
{
    switch (op) {
    case OP_MUL: return 1.0f;
    case OP_MAX: return -1e30f;     // the reference's finite identities (src/ops.c:27-54)
    case OP_MIN: return 1e30f;
    default:     return 0.0f;
    }
}

// sin, cos and pow carry a slow path (large-argument reduction, special cases) that is a call
// with a stack frame; keeping them out of line keeps that frame out of every program loop.
__device__ __noinline__ float irx_apply_slow(int op, float a, float b)
{
    switch (op) {
    case OP_SIN: return sinf(a);
    case OP_COS: return cosf(a);
    case OP_POW: return powf(a, b);
    default:     return 0.0f;
    }
}

// The four folds an Accum can use (the ops with an identity, src/ops.c:27-54).
__device__ __forceinline__ float irx_fold(int op, float a, float b)
{
    switch (op) {
    case OP_MUL: return __fmul_rn(a, b);
    case OP_MAX: return fmaxf(a, b);
    case OP_MIN: return fminf(a, b);
    default:     return __fadd_rn(a, b);
    }
}

__device__ __forceinline__ float irx_apply(int op, float a, float b)
{
    switch (op) {
    case OP_ADD:      return __fadd_rn(a, b);
    case OP_SUB:      return __fsub_rn(a, b);
    case OP_MUL:      return __fmul_rn(a, b);
    case OP_DIV:      return __fdiv_rn(a, b);
    case OP_MAX:      return fmaxf(a, b);
    case OP_MIN:      return fminf(a, b);
    case OP_RELU:     return fmaxf(a, 0.0f);
    case OP_COPY:     return a;
    case OP_NEG:      return -a;
    case OP_ABS:      return fabsf(a);
    case OP_SQRT:     return __fsqrt_rn(a);
    case OP_RSQRT:    return rsqrtf(a);
    case OP_RCP:      return __frcp_rn(a);
    case OP_TANH:     return tanhf(a);
    case OP_SIN:
    case OP_COS:
    case OP_POW:      return irx_apply_slow(op, a, b);
    case OP_LOG2:     return log2f(a);
    case OP_EXP:      return expf(a);
    case OP_EXPF:     return __expf(a);
    case OP_LOG:      return logf(a);
    case OP_SIGMOID:  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a)));
    case OP_SILU:     return __fdiv_rn(a, __fadd_rn(1.0f, expf(-a)));
    case OP_SOFTPLUS: return __fadd_rn(fmaxf(a, 0.0f), logf(__fadd_rn(1.0f, expf(-fabsf(a)))));
    default:          return 0.0f;
    }
}
