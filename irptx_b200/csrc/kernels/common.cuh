// common.cuh -- device helpers shared by the sm_100a kernel templates: the op-program
// interpreter, bf16/f32 vector loads and stores, bounded mbarrier waits and bulk copies.
//
// Op programs (irx_prog_t) are straight-line code over a small register file: r0..r3 are
// per-element input streams, r4..r15 launch- or row-uniform values, r16..r23 per-element
// temporaries. Each thread runs a program over V elements at once, so the dispatch of one
// instruction (a warp-uniform branch on its opcode and operands) is paid once per V
// elements. Every register access goes through a switch on a warp-uniform index whose cases
// name the register with a constant, which keeps the whole file in registers (no local
// memory) after inlining.
//
// The arithmetic of each op is in ops.cuh.

#pragma once
#include <cuda_bf16.h>
#include <stdint.h>
#include "../irx_kparams.h"
#include "ops.cuh"

// A register file of NS stream registers and NT temporaries, V elements each. Sized per
// instantiation: a chain program (every result feeds the next instruction) needs one
// temporary, so its kernel holds 8*(NS+1) element registers, not 96. The uniform registers
// r4..r15 are the same in every thread of a block, so they live in shared memory (`U`, 12
// floats): a program reads one with a broadcast shared load and never indexes a register
// array at run time.
template <int V, int NS = 4, int NT = 8>
struct Regs {
    float s[NS][V];
    float t[NT][V];
    const float *U;
};

// Vector form: one dispatch, V results.
template <int V>
__device__ __forceinline__ void irx_apply_v(int op, const float (&a)[V], const float (&b)[V], float (&r)[V])
{
#define IRX_VOP(OPC, EXPR) case OPC: _Pragma("unroll") for (int l = 0; l < V; l++) { float x = a[l], y = b[l]; (void)y; r[l] = (EXPR); } break;
    switch (op) {
    IRX_VOP(OP_ADD, __fadd_rn(x, y))
    IRX_VOP(OP_SUB, __fsub_rn(x, y))
    IRX_VOP(OP_MUL, __fmul_rn(x, y))
    IRX_VOP(OP_DIV, __fdiv_rn(x, y))
    IRX_VOP(OP_MAX, fmaxf(x, y))
    IRX_VOP(OP_MIN, fminf(x, y))
    IRX_VOP(OP_RELU, fmaxf(x, 0.0f))
    IRX_VOP(OP_COPY, x)
    IRX_VOP(OP_NEG, -x)
    IRX_VOP(OP_ABS, fabsf(x))
    IRX_VOP(OP_SQRT, __fsqrt_rn(x))
    IRX_VOP(OP_RSQRT, rsqrtf(x))
    IRX_VOP(OP_RCP, __frcp_rn(x))
    default:
#pragma unroll
        for (int l = 0; l < V; l++) r[l] = irx_apply(op, a[l], b[l]);
        break;
    }
#undef IRX_VOP
}

template <int V, int NS, int NT>
__device__ __forceinline__ void irx_fetch(const Regs<V, NS, NT> &R, int r, float (&o)[V])
{
    if (r >= PROG_R_UNI && r < PROG_R_TMP) {
        const float x = R.U[r - PROG_R_UNI];
#pragma unroll
        for (int l = 0; l < V; l++) o[l] = x;
        return;
    }
#define IRX_FS(I) case I: if (I < NS) { _Pragma("unroll") for (int l = 0; l < V; l++) o[l] = R.s[I < NS ? I : 0][l]; } break;
#define IRX_FT(I) case 16 + I: if (I < NT) { _Pragma("unroll") for (int l = 0; l < V; l++) o[l] = R.t[I < NT ? I : 0][l]; } break;
    switch (r) {
    IRX_FS(0) IRX_FS(1) IRX_FS(2) IRX_FS(3)
    IRX_FT(0) IRX_FT(1) IRX_FT(2) IRX_FT(3) IRX_FT(4) IRX_FT(5) IRX_FT(6) IRX_FT(7)
    default: break;
    }
#undef IRX_FS
#undef IRX_FT
}

template <int V, int NS, int NT>
__device__ __forceinline__ void irx_store_tmp(Regs<V, NS, NT> &R, int r, const float (&v)[V])
{
#define IRX_ST(I) case 16 + I: if (I < NT) { _Pragma("unroll") for (int l = 0; l < V; l++) R.t[I < NT ? I : 0][l] = v[l]; } break;
    switch (r) {
    IRX_ST(0) IRX_ST(1) IRX_ST(2) IRX_ST(3) IRX_ST(4) IRX_ST(5) IRX_ST(6) IRX_ST(7)
    default: break;
    }
#undef IRX_ST
}

// Run an element program over V elements; the result lands in `out`.
template <int V, int NS, int NT>
__device__ __forceinline__ void irx_run(const irx_prog_t &P, Regs<V, NS, NT> &R, float (&out)[V])
{
    const int n = P.nins;
    for (int i = 0; i < n; i++) {
        const irx_ins_t in = P.ins[i];
        float a[V], b[V], r[V];
#pragma unroll
        for (int l = 0; l < V; l++) { a[l] = 0.0f; b[l] = 0.0f; }
        irx_fetch(R, in.a, a);
        irx_fetch(R, in.b, b);
        irx_apply_v<V>(in.op, a, b, r);
        irx_store_tmp(R, in.dst, r);
    }
#pragma unroll
    for (int l = 0; l < V; l++) out[l] = 0.0f;
    irx_fetch(R, P.out, out);
}

// The uniform program: scalar code over a uniform register file in shared memory (U[0] is
// r4). Run by one thread; the block synchronises before other threads read the results.
__device__ __forceinline__ void irx_urun(const irx_prog_t &P, float *U)
{
    const int n = P.nins;
    for (int i = 0; i < n; i++) {
        const irx_ins_t in = P.ins[i];
        const int a = in.a - PROG_R_UNI, b = in.b - PROG_R_UNI, d = in.dst - PROG_R_UNI;
        if (d < 0 || d >= PROG_NUNI) continue;
        U[d] = irx_apply(in.op, (a >= 0 && a < PROG_NUNI) ? U[a] : 0.0f, (b >= 0 && b < PROG_NUNI) ? U[b] : 0.0f);
    }
}

__device__ __forceinline__ float irx_uget(const float *U, int r)
{
    return (r >= PROG_R_UNI && r < PROG_R_TMP) ? U[r - PROG_R_UNI] : 0.0f;
}

__device__ __forceinline__ void irx_uset(float *U, int r, float v)
{
    if (r >= PROG_R_UNI && r < PROG_R_TMP) U[r - PROG_R_UNI] = v;
}

__device__ __forceinline__ float irx_ld1(const void *p, int dt, int64_t i)
{
    if (dt == DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    return reinterpret_cast<const float *>(p)[i];
}

__device__ __forceinline__ void irx_st1(void *p, int dt, int64_t i, float v)
{
    if (dt == DT_BF16) reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float *>(p)[i] = v;
}

// Launch-uniform scalars into the shared uniform file: literals and values read once from
// rank-0 const buffers. Run by one thread.
__device__ __forceinline__ void irx_uinit(const irx_kuni_t *K, int nuni, float *U)
{
    for (int i = 0; i < PROG_NUNI; i++) {
        float v = 0.0f;
        if (i < nuni) {
            if (K[i].kind == UNI_LIT) v = __uint_as_float(K[i].bits);
            else if (K[i].kind == UNI_ARG) v = irx_ld1(K[i].ptr, K[i].dt, K[i].off);
        }
        U[i] = v;
    }
}

// 8 consecutive elements (16-byte aligned for bf16, 32 for f32) into f32 registers.
__device__ __forceinline__ void irx_ld8(const void *p, int dt, int64_t e, float (&o)[8])
{
    if (dt == DT_BF16) {
        uint4 r = __ldcs(reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(p) + e));
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&r);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float2 f = __bfloat1622float2(h[j]);
            o[2 * j] = f.x;
            o[2 * j + 1] = f.y;
        }
    } else {
        const float4 *q = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + e);
        float4 a = __ldcs(q), b = __ldcs(q + 1);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
        o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
}

__device__ __forceinline__ void irx_st8(void *p, int dt, int64_t e, const float (&v)[8])
{
    if (dt == DT_BF16) {
        uint4 r;
        __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&r);
#pragma unroll
        for (int j = 0; j < 4; j++) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        __stcs(reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p) + e), r);
    } else {
        float4 *q = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p) + e);
        __stcs(q, make_float4(v[0], v[1], v[2], v[3]));
        __stcs(q + 1, make_float4(v[4], v[5], v[6], v[7]));
    }
}

// ---- warp and block combines in a fixed order (deterministic) ----

__device__ __forceinline__ float irx_warp_fold(int op, float v)
{
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = irx_fold(op, v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Fold one value per thread across the block; every thread gets the block's total.
// `red` is shared scratch of at least 32 floats. The order is fixed: lanes by butterfly,
// then warps 0..nw-1 by one warp's butterfly.
__device__ __forceinline__ float irx_block_fold(int op, float v, float *red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = irx_warp_fold(op, v);
    __syncthreads();                     // red may still be read by a previous fold
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float w = lane < nw ? red[lane] : irx_ident(op);
        w = irx_warp_fold(op, w);
        if (lane == 0) red[32] = w;
    }
    __syncthreads();
    return red[32];
}

// The same fold with one barrier: `red` holds two 32-float buffers, used alternately (`seq` is
// a counter every thread of the block advances together). Each thread folds the warp totals
// itself, in warp order, so every thread gets the same total without a second barrier; the
// next fold writes the other buffer, and the one after waits behind the next fold's barrier,
// by which time every thread has read this one.
__device__ __forceinline__ float irx_block_fold1(int op, float v, float *red, unsigned seq)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float *b = red + (seq & 1u) * 32;
    v = irx_warp_fold(op, v);
    if (lane == 0) b[warp] = v;
    __syncthreads();
    float t = b[0];
    for (int w = 1; w < nw; w++) t = irx_fold(op, t, b[w]);
    return t;
}

// ---- mbarrier and bulk copy (TMA, non-tensor), with bounded waits ----

__device__ __forceinline__ uint32_t irx_smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void irx_mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(irx_smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void irx_fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void irx_mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(irx_smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void irx_mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(irx_smem_u32(bar)) : "memory");
}

__device__ __forceinline__ int irx_mbar_try(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(irx_smem_u32(bar)), "r"(parity) : "memory");
    return ok;
}

// Programmatic dependent launch. Called first in every prebuilt kernel, before any access to
// global memory: let the stream's next kernel be launched now (its blocks take SM room as this
// kernel's blocks finish, and wait there), then wait until the kernel before this one has finished
// and its memory is visible. The launch layer sets the attribute that allows the overlap; without
// it both instructions do nothing.
__device__ __forceinline__ void irx_pdl_enter()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ uint64_t irx_gtime()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for phase `parity` of `bar` to complete: at most `limit` polls and at most IRX_WAIT_NS
// nanoseconds of the GPU's global timer, whichever ends first (a poll can suspend the thread
// for a time the hardware picks, so the poll count alone does not bound the time). Returns 1
// when the phase completed, 0 when a limit ran out (the caller records an error and stops).
// Every legitimate wait of these kernels ends within milliseconds.
#define IRX_WAIT_LIMIT (1u << 26)
#define IRX_WAIT_NS 4000000000ull
__device__ __forceinline__ int irx_mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit = IRX_WAIT_LIMIT,
                                             uint64_t ns = IRX_WAIT_NS)
{
    if (irx_mbar_try(bar, parity)) return 1;
    const uint64_t t0 = irx_gtime();
    for (uint32_t i = 1; i < limit; i++) {
        if (irx_mbar_try(bar, parity)) return 1;
        if ((i & 255u) == 0 && irx_gtime() - t0 > ns) return 0;
    }
    return 0;
}

// One 1-D bulk copy global -> shared (cp.async.bulk), completing on `bar`. Both addresses
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void irx_bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(irx_smem_u32(dst)), "l"(src), "r"(bytes), "r"(irx_smem_u32(bar)) : "memory");
}
