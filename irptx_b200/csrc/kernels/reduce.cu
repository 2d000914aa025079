// reduce.cu -- the reduction templates.
//
// irx_red_rows_*: y[row] = post(fold_op over c of pre(x[row, c])). One warp per row, 8 rows
// per block, grid-stride over rows. Each lane folds 8 consecutive columns per step into 8
// running values, with 4 steps of 128-bit loads in flight, then the 8 values fold in a fixed
// pairwise order and the warp folds by butterfly. Row results are deterministic.
//
// irx_red_all_*: y = [y +] post(fold_op over all i of pre(x[i])). One grid-stride pass: thread
// g of the grid folds the 8-element chunks g, g + G, g + 2G, ... (4 in flight), so every step of
// the grid reads one contiguous window; the block folds its threads' values in a fixed order,
// block totals go to a scratch array, and the last block to arrive
// (an atomic ticket, no waiting) folds the totals in block order and writes the result. The
// result is deterministic for a given grid: the reference's one-kernel form adds block totals
// with red.global.add in whatever order the blocks finish (src/isel.c:1254-1260).
//
// Each is instantiated without a pre-program (the folded value is the loaded element: no
// interpreter registers at all) and with one.
//
// The KIR these serve is the reference's reduction shape: a StridedLoop of Load + Accum, a
// WarpShuffle and a TreeHalve over warps (src/isel.c:1337-1506, 1718-1840).

#include "common.cuh"

__device__ __forceinline__ float fold8(int op, const float (&a)[8])
{
    float b0 = irx_fold(op, a[0], a[1]), b1 = irx_fold(op, a[2], a[3]);
    float b2 = irx_fold(op, a[4], a[5]), b3 = irx_fold(op, a[6], a[7]);
    return irx_fold(op, irx_fold(op, b0, b1), irx_fold(op, b2, b3));
}

template <bool PRE>
struct RedRegs {
    Regs<8, 1, 8> R;
    Regs<1, 1, 8> S;
};
template <>
struct RedRegs<false> {
    Regs<1, 1, 1> R;   // unused
    Regs<1, 1, 1> S;
};

// Fold pre(x[e .. e+7]) into acc.
template <bool PRE>
__device__ __forceinline__ void fold_vals(const irx_kred_t &p, RedRegs<PRE> &G, float (&v)[8], float (&acc)[8])
{
    if constexpr (PRE) {
#pragma unroll
        for (int l = 0; l < 8; l++) G.R.s[0][l] = v[l];
        irx_run(p.pre, G.R, v);
    }
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = irx_fold(p.op, acc[l], v[l]);
}

template <bool PRE>
__device__ __forceinline__ float fold_one(const irx_kred_t &p, RedRegs<PRE> &G, int64_t e, float acc)
{
    float v[1];
    v[0] = irx_ld1(p.x, p.x_dt, e);
    if constexpr (PRE) {
        G.S.s[0][0] = v[0];
        irx_run(p.pre, G.S, v);
    }
    return irx_fold(p.op, acc, v[0]);
}

// Launch-uniform values into the block's shared uniform file U (one thread computes, all
// read after the barrier).
template <bool PRE>
__device__ __forceinline__ void init_regs(const irx_kred_t &p, RedRegs<PRE> &G, float *U)
{
    if (threadIdx.x == 0) {
        irx_uinit(p.uni, p.nuni, U);
        irx_urun(p.uprog, U);
    }
    __syncthreads();
    G.R.U = U;
    G.S.U = U;
}

// The written value for a total: the uniform program over a private copy of the launch
// uniforms with the total in its register. Run by one thread; `W` is that thread's scratch.
__device__ __forceinline__ float post_value(const irx_kred_t &p, const float *U, float *W, float total)
{
    for (int i = 0; i < PROG_NUNI; i++) W[i] = U[i];
    irx_uset(W, p.tot_reg, total);
    irx_urun(p.uprog, W);
    return irx_uget(W, p.out_reg);
}

// Fold the 8-element chunks [c0, c1) (chunk index, stride `step`) with 4 chunks in flight.
template <bool PRE>
__device__ __forceinline__ void fold_range(const irx_kred_t &p, RedRegs<PRE> &G, int64_t base, int64_t c0,
                                           int64_t c1, int64_t step, float (&acc)[8])
{
    int64_t c = c0;
    for (; c + 3 * step < c1; c += 4 * step) {
        float v0[8], v1[8], v2[8], v3[8];
        irx_ld8(p.x, p.x_dt, base + c * 8, v0);
        irx_ld8(p.x, p.x_dt, base + (c + step) * 8, v1);
        irx_ld8(p.x, p.x_dt, base + (c + 2 * step) * 8, v2);
        irx_ld8(p.x, p.x_dt, base + (c + 3 * step) * 8, v3);
        fold_vals<PRE>(p, G, v0, acc);
        fold_vals<PRE>(p, G, v1, acc);
        fold_vals<PRE>(p, G, v2, acc);
        fold_vals<PRE>(p, G, v3, acc);
    }
    for (; c < c1; c += step) {
        float v[8];
        irx_ld8(p.x, p.x_dt, base + c * 8, v);
        fold_vals<PRE>(p, G, v, acc);
    }
}

template <bool PRE>
__device__ __forceinline__ void red_rows_body(const irx_kred_t &p)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarp = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const float id = irx_ident(p.op);
    __shared__ float U[PROG_NUNI];
    __shared__ float W[8][PROG_NUNI];
    RedRegs<PRE> G;
    init_regs<PRE>(p, G, U);

    for (int64_t row = warp; row < p.rows; row += nwarp) {
        const int64_t base = (p.row0 + row) * p.cols;
        float acc[8];
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = id;
        int64_t c = 0;
        if (p.vec_ok) {
            const int64_t nch = p.cols / 8;
            fold_range<PRE>(p, G, base, lane, nch, 32, acc);
            c = nch * 8;
        }
        float t = fold8(p.op, acc);
        for (int64_t j = c + lane; j < p.cols; j += 32) t = fold_one<PRE>(p, G, base + j, t);
        t = irx_warp_fold(p.op, t);
        if (lane == 0) irx_st1(p.y, p.y_dt, p.row0 + row, post_value(p, U, W[(threadIdx.x >> 5) & 7], t));
    }
}

#define RED_ALL_THREADS IRX_RED_ALL_THREADS

template <bool PRE>
__device__ __forceinline__ void red_all_body(const irx_kred_t &p)
{
    __shared__ float red[40];
    __shared__ unsigned last;
    __shared__ float U[PROG_NUNI], W[PROG_NUNI];
    const float id = irx_ident(p.op);
    RedRegs<PRE> G;
    init_regs<PRE>(p, G, U);

    const int64_t n = p.end - p.begin;
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = id;
    int64_t head = p.begin;
    if (p.vec_ok) {
        const int64_t nch = n / 8;
        fold_range<PRE>(p, G, p.begin, (int64_t)blockIdx.x * blockDim.x + threadIdx.x, nch,
                        (int64_t)gridDim.x * blockDim.x, acc);
        head = p.begin + nch * 8;
    }
    float t = fold8(p.op, acc);
    if (blockIdx.x == 0)
        for (int64_t e = head + threadIdx.x; e < p.end; e += blockDim.x) t = fold_one<PRE>(p, G, e, t);
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
        // lane l folds totals l, l + 32, l + 64, ... in that order; eight loads go out before
        // their folds, so the L2 round trips overlap
        float v = id;
        const unsigned nb = gridDim.x;
        for (unsigned i0 = threadIdx.x; i0 < nb; i0 += 32u * 8u) {
            float q[8];
#pragma unroll
            for (int u = 0; u < 8; u++) q[u] = i0 + 32u * u < nb ? __ldcg(&p.partial[i0 + 32u * u]) : id;
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (i0 + 32u * u < nb) v = irx_fold(p.op, v, q[u]);
        }
        v = irx_warp_fold(p.op, v);
        if (threadIdx.x == 0) {
            float out = post_value(p, U, W, v);
            if (p.accumulate) out = __fadd_rn(irx_ld1(p.y, p.y_dt, 0), out);
            irx_st1(p.y, p.y_dt, 0, out);
            *p.ticket = 0u;                     // ready for the next launch on this scratch
        }
    }
}

extern "C" __global__ void __launch_bounds__(256) irx_red_rows_p0(const __grid_constant__ irx_kred_t p) { irx_pdl_enter(); red_rows_body<false>(p); }
extern "C" __global__ void __launch_bounds__(256) irx_red_rows_p1(const __grid_constant__ irx_kred_t p) { irx_pdl_enter(); red_rows_body<true>(p); }
extern "C" __global__ void __launch_bounds__(RED_ALL_THREADS) irx_red_all_p0(const __grid_constant__ irx_kred_t p) { irx_pdl_enter(); red_all_body<false>(p); }
extern "C" __global__ void __launch_bounds__(RED_ALL_THREADS) irx_red_all_p1(const __grid_constant__ irx_kred_t p) { irx_pdl_enter(); red_all_body<true>(p); }
