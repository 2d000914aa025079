// rowop.cu -- the fused row-op template: per row, a sequence of row statistics
//   stat_k = fold_op_k over j of pre_k(x[row, j], w[j], earlier stats)
// then one pass writing y[row, j] = epi(x[row, j], w[j], stats). RMSNorm, softmax and L2
// normalisation are three instances; anything of the same two-phase shape is another.
//
// Each row is read from HBM once: a TMA bulk copy (cp.async.bulk, no multicast) stages the
// whole row into shared memory, NBUF rows deep, so the next rows stream in while this one is
// folded and written. Every statistic pass and the write pass then read the row from shared
// memory. The block folds each statistic in a fixed order (per-thread 8-wide partials, warp
// butterfly, warps in order), so results are deterministic. w[j] is read through the cache:
// every row reuses it.
//
// When a row cannot be staged (unaligned, or larger than the shared budget) the passes read
// x from global memory directly.
//
// Every wait on a bulk copy is bounded; a wait that runs out sets the error word, and the
// block stops after every thread has voted on it.
//
// The KIR this serves: StridedLoops of Load + Accum with WarpShuffle and TreeHalve, then a
// StridedLoop of Load / Assign / Write (src/isel.c:1337-1506, 1718-1840).

#include "common.cuh"

#define ROW_THREADS 256
#define ROW_NBUF 3

template <bool SMEM>
__device__ __forceinline__ void row_ld8(const void *p, int dt, int64_t e, float (&o)[8])
{
    if (dt == DT_BF16) {
        uint4 r = SMEM ? reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(p) + e)[0]
                       : __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(p) + e));
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&r);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float2 f = __bfloat1622float2(h[j]);
            o[2 * j] = f.x;
            o[2 * j + 1] = f.y;
        }
    } else {
        const float4 *q = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + e);
        float4 a = SMEM ? q[0] : __ldg(q), b = SMEM ? q[1] : __ldg(q + 1);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
        o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
}

__device__ __forceinline__ float row_fold8(int op, const float (&a)[8])
{
    float b0 = irx_apply(op, a[0], a[1]), b1 = irx_apply(op, a[2], a[3]);
    float b2 = irx_apply(op, a[4], a[5]), b3 = irx_apply(op, a[6], a[7]);
    return irx_apply(op, irx_apply(op, b0, b1), irx_apply(op, b2, b3));
}

// One row: the statistics, then the write pass. `xr` is the row (shared or global).
template <bool SMEM>
__device__ __forceinline__ void row_body(const irx_krow_t &p, const void *xr, int64_t row, Regs<8> &R, float *red,
                                         const float (&u0)[PROG_NUNI])
{
    const int64_t cols = p.cols;
    const int vec = (cols & 7) == 0;
#pragma unroll
    for (int i = 0; i < PROG_NUNI; i++) R.u[i] = u0[i];
    irx_urun(p.uprog, R.u);
    for (int k = 0; k < p.nstat; k++) {
        const int op = p.stat_op[k];
        const float id = irx_ident(op);
        float acc[8];
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = id;
        float t = id;
        if (vec) {
            for (int64_t c = threadIdx.x * 8; c < cols; c += ROW_THREADS * 8) {
                float v[8];
                row_ld8<SMEM>(xr, p.x_dt, c, v);
                if (p.stat_pre[k].nins) {
#pragma unroll
                    for (int l = 0; l < 8; l++) R.e[0][l] = v[l];
                    if (p.has_w) {
                        float w[8];
                        row_ld8<false>(p.w, p.w_dt, c, w);
#pragma unroll
                        for (int l = 0; l < 8; l++) R.e[1][l] = w[l];
                    }
                    irx_run<8>(p.stat_pre[k], R, v);
                }
                irx_apply_v<8>(op, acc, v, acc);
            }
            t = row_fold8(op, acc);
        } else {
            Regs<1> S;
#pragma unroll
            for (int i = 0; i < PROG_NUNI; i++) S.u[i] = R.u[i];
            for (int64_t c = threadIdx.x; c < cols; c += ROW_THREADS) {
                float v[1];
                v[0] = SMEM ? irx_ld1(xr, p.x_dt, c) : irx_ld1(xr, p.x_dt, c);
                S.e[0][0] = v[0];
                if (p.has_w) S.e[1][0] = irx_ld1(p.w, p.w_dt, c);
                if (p.stat_pre[k].nins) irx_run<1>(p.stat_pre[k], S, v);
                t = irx_apply(op, t, v[0]);
            }
        }
        t = irx_block_fold(op, t, red);
        irx_ustore(R.u, p.stat_reg[k], t);
        irx_urun(p.uprog, R.u);
    }
    const int64_t yb = (p.row0 + row) * cols;
    if (vec) {
        for (int64_t c = threadIdx.x * 8; c < cols; c += ROW_THREADS * 8) {
            float v[8], out[8];
            row_ld8<SMEM>(xr, p.x_dt, c, v);
#pragma unroll
            for (int l = 0; l < 8; l++) R.e[0][l] = v[l];
            if (p.has_w) {
                float w[8];
                row_ld8<false>(p.w, p.w_dt, c, w);
#pragma unroll
                for (int l = 0; l < 8; l++) R.e[1][l] = w[l];
            }
            irx_run<8>(p.epi, R, out);
            irx_st8(p.y, p.y_dt, yb + c, out);
        }
    } else {
        Regs<1> S;
#pragma unroll
        for (int i = 0; i < PROG_NUNI; i++) S.u[i] = R.u[i];
        for (int64_t c = threadIdx.x; c < cols; c += ROW_THREADS) {
            float out[1];
            S.e[0][0] = irx_ld1(xr, p.x_dt, c);
            if (p.has_w) S.e[1][0] = irx_ld1(p.w, p.w_dt, c);
            irx_run<1>(p.epi, S, out);
            irx_st1(p.y, p.y_dt, yb + c, out[0]);
        }
    }
}

extern "C" __global__ void __launch_bounds__(ROW_THREADS, 2) irx_rowop(const __grid_constant__ irx_krow_t p)
{
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float red[40];
    __shared__ __align__(8) uint64_t bar[ROW_NBUF];
    const int esz = p.x_dt == DT_BF16 ? 2 : 4;
    Regs<8> R;
    float u0[PROG_NUNI];
    irx_uinit(p.uni, p.nuni, u0);

    if (!p.bulk_ok) {
        for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
            const void *xr = reinterpret_cast<const unsigned char *>(p.x) + (p.row0 + row) * p.cols * esz;
            row_body<false>(p, xr, row, R, red, u0);
            __syncthreads();
        }
        return;
    }
    const uint32_t bytes = (uint32_t)(p.cols * esz);
    if (threadIdx.x == 0) {
        for (int i = 0; i < ROW_NBUF; i++) irx_mbar_init(&bar[i], 1);
        irx_fence_mbar_init();
    }
    __syncthreads();
    // prologue: the first NBUF-1 rows of this block
    if (threadIdx.x == 0) {
        for (int i = 0; i < ROW_NBUF - 1; i++) {
            int64_t r = blockIdx.x + (int64_t)i * gridDim.x;
            if (r < p.rows) {
                irx_mbar_expect_tx(&bar[i], bytes);
                irx_bulk_g2s(smem + (size_t)i * p.smem_row_bytes,
                             reinterpret_cast<const unsigned char *>(p.x) + (p.row0 + r) * p.cols * esz, bytes, &bar[i]);
            }
        }
    }
    int it = 0;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x, it++) {
        const int b = it % ROW_NBUF;
        if (threadIdx.x == 0) {
            // refill the buffer the previous iteration finished with (all threads passed
            // the barrier at the end of that iteration)
            int64_t r = row + (int64_t)(ROW_NBUF - 1) * gridDim.x;
            int nb = (it + ROW_NBUF - 1) % ROW_NBUF;
            if (r < p.rows) {
                irx_mbar_expect_tx(&bar[nb], bytes);
                irx_bulk_g2s(smem + (size_t)nb * p.smem_row_bytes,
                             reinterpret_cast<const unsigned char *>(p.x) + (p.row0 + r) * p.cols * esz, bytes, &bar[nb]);
            }
        }
        int ok = irx_mbar_wait(&bar[b], (uint32_t)((it / ROW_NBUF) & 1));
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0) {
                if (p.err) atomicOr(p.err, IRX_KERR_TIMEOUT);
                // drain: every later copy this block issued lands before its smem is released
                for (int i = 1; i < ROW_NBUF; i++) {
                    int64_t r = row + (int64_t)i * gridDim.x;
                    if (r < p.rows) irx_mbar_wait(&bar[(it + i) % ROW_NBUF], (uint32_t)(((it + i) / ROW_NBUF) & 1), 1u << 20);
                }
            }
            return;
        }
        row_body<true>(p, smem + (size_t)b * p.smem_row_bytes, row, R, red, u0);
        __syncthreads();
    }
}
