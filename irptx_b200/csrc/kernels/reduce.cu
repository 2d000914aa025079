// reduce.cu -- the reduction templates.
//
// irx_reduce_rows: y[row] = post(fold_op over c of pre(x[row, c])). One warp per row, 8 rows
// per block, grid-stride over rows. Each lane folds 8 consecutive columns per step into 8
// running values (128-bit loads, several steps in flight), then the 8 values fold in a fixed
// pairwise order and the warp folds by butterfly. Row results are deterministic.
//
// irx_reduce_all: y = [y +] post(fold_op over all i of pre(x[i])). Each block folds one
// contiguous chunk of the array; block totals go to a scratch array; the last block to arrive
// (an atomic ticket, no waiting) folds the totals in block order and writes the result. The
// sum is deterministic for a given grid: the reference's one-kernel form adds block totals
// with red.global.add in whatever order the blocks finish (src/isel.c:1254-1260).
//
// The KIR these serve is the reference's reduction shape: a StridedLoop of Load + Accum, a
// WarpShuffle and a TreeHalve over warps (src/isel.c:1337-1506, 1718-1840).

#include "common.cuh"

__device__ __forceinline__ float fold8(int op, const float (&a)[8])
{
    float b0 = irx_apply(op, a[0], a[1]), b1 = irx_apply(op, a[2], a[3]);
    float b2 = irx_apply(op, a[4], a[5]), b3 = irx_apply(op, a[6], a[7]);
    return irx_apply(op, irx_apply(op, b0, b1), irx_apply(op, b2, b3));
}

// Fold pre(x[e .. e+7]) into acc.
__device__ __forceinline__ void fold_chunk(const irx_kred_t &p, Regs<8> &R, int64_t e, float (&acc)[8])
{
    float v[8];
    irx_ld8(p.x, p.x_dt, e, v);
    if (p.has_pre) {
#pragma unroll
        for (int l = 0; l < 8; l++) R.e[0][l] = v[l];
        irx_run<8>(p.pre, R, v);
    }
    irx_apply_v<8>(p.op, acc, v, acc);
}

__device__ __forceinline__ float fold_one(const irx_kred_t &p, Regs<1> &S, int64_t e, float acc)
{
    float v[1];
    v[0] = irx_ld1(p.x, p.x_dt, e);
    if (p.has_pre) {
        S.e[0][0] = v[0];
        irx_run<1>(p.pre, S, v);
    }
    return irx_apply(p.op, acc, v[0]);
}

extern "C" __global__ void __launch_bounds__(256) irx_reduce_rows(const __grid_constant__ irx_kred_t p)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarp = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const float id = irx_ident(p.op);
    Regs<8> R;
    Regs<1> S;
    irx_uinit(p.uni, p.nuni, R.u);
    irx_urun(p.uprog, R.u);
#pragma unroll
    for (int i = 0; i < PROG_NUNI; i++) S.u[i] = R.u[i];

    for (int64_t row = warp; row < p.rows; row += nwarp) {
        const int64_t base = (p.row0 + row) * p.cols;
        float acc[8];
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = id;
        int64_t c = 0;
        if (p.vec_ok) {
            const int64_t full = p.cols & ~(int64_t)255;        // whole warp-steps of 256
#pragma unroll 4
            for (c = lane * 8; c < full; c += 256) fold_chunk(p, R, base + c, acc);
            c = full;
        }
        float t = fold8(p.op, acc);
        for (int64_t j = c + lane; j < p.cols; j += 32) t = fold_one(p, S, base + j, t);
        t = irx_warp_fold(p.op, t);
        if (lane == 0) {
            float u[PROG_NUNI];
#pragma unroll
            for (int i = 0; i < PROG_NUNI; i++) u[i] = R.u[i];
            irx_ustore(u, p.tot_reg, t);
            irx_urun(p.uprog, u);
            irx_st1(p.y, p.y_dt, p.row0 + row, irx_ufetch(u, p.out_reg));
        }
    }
}

#define RED_ALL_THREADS 512

extern "C" __global__ void __launch_bounds__(RED_ALL_THREADS) irx_reduce_all(const __grid_constant__ irx_kred_t p)
{
    __shared__ float red[40];
    __shared__ unsigned last;
    const float id = irx_ident(p.op);
    Regs<8> R;
    Regs<1> S;
    irx_uinit(p.uni, p.nuni, R.u);
    irx_urun(p.uprog, R.u);
#pragma unroll
    for (int i = 0; i < PROG_NUNI; i++) S.u[i] = R.u[i];

    const int64_t n = p.end - p.begin;
    const int64_t per = ((n + gridDim.x - 1) / gridDim.x + 7) & ~(int64_t)7;
    const int64_t b0 = p.begin + (int64_t)blockIdx.x * per;
    const int64_t b1 = min(p.end, b0 + per);
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = id;
    int64_t head = b0;
    if (p.vec_ok && b1 > b0) {
        const int64_t nch = (b1 - b0) / 8;
#pragma unroll 4
        for (int64_t c = threadIdx.x; c < nch; c += blockDim.x) fold_chunk(p, R, b0 + c * 8, acc);
        head = b0 + nch * 8;
    }
    float t = fold8(p.op, acc);
    for (int64_t e = head + threadIdx.x; e < b1; e += blockDim.x) t = fold_one(p, S, e, t);
    t = irx_block_fold(p.op, t, red);

    if (threadIdx.x == 0) {
        p.partial[blockIdx.x] = t;
        __threadfence();
        last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    // the last block: fold the block totals in block order
    __threadfence();
    if (threadIdx.x < 32) {
        float v = id;
        for (unsigned i = threadIdx.x; i < gridDim.x; i += 32)
            v = irx_apply(p.op, v, __ldcg(&p.partial[i]));
        v = irx_warp_fold(p.op, v);
        if (threadIdx.x == 0) {
            float u[PROG_NUNI];
#pragma unroll
            for (int i = 0; i < PROG_NUNI; i++) u[i] = R.u[i];
            irx_ustore(u, p.tot_reg, v);
            irx_urun(p.uprog, u);
            float out = irx_ufetch(u, p.out_reg);
            if (p.accumulate) out = __fadd_rn(irx_ld1(p.y, p.y_dt, 0), out);
            irx_st1(p.y, p.y_dt, 0, out);
            *p.ticket = 0u;                     // ready for the next launch on this scratch
        }
    }
}
