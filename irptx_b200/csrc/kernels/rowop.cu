// rowop.cu -- the fused row-op templates: per row, a sequence of row statistics
//   stat_k = fold_op_k over j of pre_k(x[row, j], w[j], earlier stats)
// then one pass writing y[row, j] = epi(x[row, j], w[j], stats).
//
// irx_rowop runs any graph of that shape through op programs. irx_row_rmsnorm, irx_row_softmax
// and irx_row_l2norm are the same pipeline with the three BASELINE row ops written out, which
// the selector picks when the graph computes exactly one of them:
//   rmsnorm  y = x / sqrt(sum(x^2) / cols + eps) * w
//   softmax  y = exp(x - max(x)) / sum(exp(x - max(x)))   (one exp per element: cached)
//   l2norm   y = x / sqrt(sum(x^2))
//
// Each row is read from HBM once: a TMA bulk copy (cp.async.bulk, one CTA's own) stages the
// whole row into shared memory, NBUF rows deep, so the next rows stream in while this one is
// folded and written. Every statistic pass and the write pass read the row from shared memory.
// Statistics fold in a fixed order (per-thread 8-wide partials, warp butterfly, warps in
// order), so results are deterministic. w[j] is read through the cache: every row reuses it.
// When a row cannot be staged (unaligned, or larger than the shared budget) the passes read
// x from global memory directly.
//
// Every wait on a bulk copy is bounded; a wait that runs out sets the error word, drains the
// block's other copies (bounded too) and stops the block after every thread has voted on it.
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
    float b0 = irx_fold(op, a[0], a[1]), b1 = irx_fold(op, a[2], a[3]);
    float b2 = irx_fold(op, a[4], a[5]), b3 = irx_fold(op, a[6], a[7]);
    return irx_fold(op, irx_fold(op, b0, b1), irx_fold(op, b2, b3));
}

// ---- the generic row body: op programs ----

// U0: the launch-uniform values; U: this row's uniform file (statistics land in it). Thread 0
// writes U; the barrier that ends each block fold publishes it.
template <bool SMEM>
__device__ __forceinline__ void generic_row(const irx_krow_t &p, const void *xr, int64_t row, float *red,
                                            const float *U0, float *U)
{
    const int64_t cols = p.cols;
    Regs<8, 2, 8> R;
    R.U = U;
    __syncthreads();                       // every thread is done with the previous row's U
    if (threadIdx.x == 0) {
        for (int i = 0; i < PROG_NUNI; i++) U[i] = U0[i];
        irx_urun(p.uprog, U);
    }
    __syncthreads();
    for (int k = 0; k < p.nstat; k++) {
        const int op = p.stat_op[k];
        const float id = irx_ident(op);
        float acc[8];
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = id;
        float t = id;
        if ((cols & 7) == 0) {
            for (int64_t c = threadIdx.x * 8; c < cols; c += ROW_THREADS * 8) {
                float v[8];
                row_ld8<SMEM>(xr, p.x_dt, c, v);
                if (p.stat_pre[k].nins) {
#pragma unroll
                    for (int l = 0; l < 8; l++) R.s[0][l] = v[l];
                    if (p.has_w) row_ld8<false>(p.w, p.w_dt, c, R.s[1]);
                    irx_run(p.stat_pre[k], R, v);
                }
#pragma unroll
                for (int l = 0; l < 8; l++) acc[l] = irx_fold(op, acc[l], v[l]);
            }
            t = row_fold8(op, acc);
        } else {
            Regs<1, 2, 8> S;
            S.U = U;
            for (int64_t c = threadIdx.x; c < cols; c += ROW_THREADS) {
                float v[1];
                v[0] = irx_ld1(xr, p.x_dt, c);
                S.s[0][0] = v[0];
                if (p.has_w) S.s[1][0] = irx_ld1(p.w, p.w_dt, c);
                if (p.stat_pre[k].nins) irx_run(p.stat_pre[k], S, v);
                t = irx_fold(op, t, v[0]);
            }
        }
        t = irx_block_fold(op, t, red);
        if (threadIdx.x == 0) {
            irx_uset(U, p.stat_reg[k], t);
            irx_urun(p.uprog, U);
        }
        __syncthreads();
    }
    const int64_t yb = (p.row0 + row) * cols;
    if ((cols & 7) == 0) {
        for (int64_t c = threadIdx.x * 8; c < cols; c += ROW_THREADS * 8) {
            float out[8];
            row_ld8<SMEM>(xr, p.x_dt, c, R.s[0]);
            if (p.has_w) row_ld8<false>(p.w, p.w_dt, c, R.s[1]);
            irx_run(p.epi, R, out);
            irx_st8(p.y, p.y_dt, yb + c, out);
        }
    } else {
        Regs<1, 2, 8> S;
        S.U = U;
        for (int64_t c = threadIdx.x; c < cols; c += ROW_THREADS) {
            float out[1];
            S.s[0][0] = irx_ld1(xr, p.x_dt, c);
            if (p.has_w) S.s[1][0] = irx_ld1(p.w, p.w_dt, c);
            irx_run(p.epi, S, out);
            irx_st1(p.y, p.y_dt, yb + c, out[0]);
        }
    }
}

// ---- the three written-out row ops (cols a multiple of 8) ----

template <bool SMEM>
__device__ __forceinline__ float sumsq_row(const irx_krow_t &p, const void *xr, float *red, unsigned &seq)
{
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t c = threadIdx.x * 8; c < p.cols; c += ROW_THREADS * 8) {
        float v[8];
        row_ld8<SMEM>(xr, p.x_dt, c, v);
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = __fmaf_rn(v[l], v[l], acc[l]);
    }
    return irx_block_fold1(OP_ADD, row_fold8(OP_ADD, acc), red, seq++);
}

template <bool SMEM>
__device__ __forceinline__ void rmsnorm_row(const irx_krow_t &p, const void *xr, int64_t row, float *red, unsigned &seq)
{
    const float ss = sumsq_row<SMEM>(p, xr, red, seq);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)p.cols), __uint_as_float(p.eps_bits)));
    const float inv = __frcp_rn(rms);
    const int64_t yb = (p.row0 + row) * p.cols;
    for (int64_t c = threadIdx.x * 8; c < p.cols; c += ROW_THREADS * 8) {
        float v[8], w[8], o[8];
        row_ld8<SMEM>(xr, p.x_dt, c, v);
        row_ld8<false>(p.w, p.w_dt, c, w);
#pragma unroll
        for (int l = 0; l < 8; l++) o[l] = __fmul_rn(__fmul_rn(v[l], inv), w[l]);
        irx_st8(p.y, p.y_dt, yb + c, o);
    }
}

template <bool SMEM>
__device__ __forceinline__ void l2norm_row(const irx_krow_t &p, const void *xr, int64_t row, float *red, unsigned &seq)
{
    const float inv = __frcp_rn(__fsqrt_rn(sumsq_row<SMEM>(p, xr, red, seq)));
    const int64_t yb = (p.row0 + row) * p.cols;
    for (int64_t c = threadIdx.x * 8; c < p.cols; c += ROW_THREADS * 8) {
        float v[8], o[8];
        row_ld8<SMEM>(xr, p.x_dt, c, v);
#pragma unroll
        for (int l = 0; l < 8; l++) o[l] = __fmul_rn(v[l], inv);
        irx_st8(p.y, p.y_dt, yb + c, o);
    }
}

// 2^x on the MUFU unit (ex2.approx, flush to zero): exp(t) = 2^(t log2 e).
__device__ __forceinline__ float row_ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x, x = s * L2E - m, on the FMA pipe, for rows whose output is bf16 (an f32 output keeps the
// MUFU for every element: this form's relative error, 7.5e-5 at most, is far below a bf16
// output's 2^-9 but not below f32's). One saturating FMA maps x to y = (x + 126) / 253 in
// [0, 1], which clamps x to [-126, 127]; t = 253 y + 1.5 * 2^23 - 126 rounds x to the integer n
// (the low bits of t hold n), f = x - n lies in [-1/2, 1/2], and a cubic fitted for minimum
// relative error on [-1/2, 1/2] gives 2^f, whose exponent field then gains n. The same form as
// the attention kernel's FMA-pipe exps.
//   The saturation turns a NaN argument into 0, so x is formed first and a NaN x (a NaN input,
// or inf - inf from an infinite row maximum) is passed through, as ex2.approx passes it: a NaN
// anywhere in a row makes the whole row NaN on either pipe. x = -inf (a masked element) gives
// 2^-126 here where ex2.approx gives 0; no bf16 output or row sum can tell them apart.
__device__ __forceinline__ float row_ex2_cubic(float s, float L2E, float m)
{
    const float x = fmaf(s, L2E, -m);
    float y;
    asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(x), "f"(1.0f / 253.0f), "f"(126.0f / 253.0f));
    const float t = fmaf(y, 253.0f, 12582912.0f - 126.0f);
    const float f = fmaf(y, 253.0f, (12582912.0f - 126.0f) - t);
    float q = fmaf(0.055171319384097875f, f, 0.2426105373823389f);
    q = fmaf(q, f, 0.6932609854947172f);
    q = fmaf(q, f, 0.9999281096694117f);
    const float r = __uint_as_float(__float_as_uint(q) + (__float_as_uint(t) << 23));
    return x == x ? r : x;
}

// Softmax of one row. With `ebuf` (the row staged in shared memory) the sum pass keeps every
// e = exp(x - max) as f32 there and the write pass only multiplies, so each element costs one
// exp; without it (the row read from global memory) the write pass recomputes e.
template <bool SMEM>
__device__ __forceinline__ void softmax_row(const irx_krow_t &p, const void *xr, int64_t row, float *red, float *ebuf,
                                            unsigned &seq)
{
    const float L2E = 1.4426950408889634f;
    float mx[8];
#pragma unroll
    for (int l = 0; l < 8; l++) mx[l] = -1e30f;
    for (int64_t c = threadIdx.x * 8; c < p.cols; c += ROW_THREADS * 8) {
        float v[8];
        row_ld8<SMEM>(xr, p.x_dt, c, v);
#pragma unroll
        for (int l = 0; l < 8; l++) mx[l] = fmaxf(mx[l], v[l]);
    }
    const float ml2 = irx_block_fold1(OP_MAX, row_fold8(OP_MAX, mx), red, seq++) * L2E;
    float se[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t c = threadIdx.x * 8; c < p.cols; c += ROW_THREADS * 8) {
        float v[8];
        row_ld8<SMEM>(xr, p.x_dt, c, v);
#pragma unroll
        for (int l = 0; l < 8; l++) {
            v[l] = row_ex2(fmaf(v[l], L2E, -ml2));
            se[l] += v[l];
        }
        if (SMEM && ebuf) {
            float4 *q = reinterpret_cast<float4 *>(ebuf + c);
            q[0] = make_float4(v[0], v[1], v[2], v[3]);
            q[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    }
    const float inv = __frcp_rn(irx_block_fold1(OP_ADD, row_fold8(OP_ADD, se), red, seq++));
    const int64_t yb = (p.row0 + row) * p.cols;
    for (int64_t c = threadIdx.x * 8; c < p.cols; c += ROW_THREADS * 8) {
        float v[8], o[8];
        if (SMEM && ebuf) {
            const float4 *q = reinterpret_cast<const float4 *>(ebuf + c);
            const float4 a = q[0], b = q[1];
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
            row_ld8<SMEM>(xr, p.x_dt, c, v);
#pragma unroll
            for (int l = 0; l < 8; l++) v[l] = row_ex2(fmaf(v[l], L2E, -ml2));
        }
#pragma unroll
        for (int l = 0; l < 8; l++) o[l] = __fmul_rn(v[l], inv);
        irx_st8(p.y, p.y_dt, yb + c, o);
    }
}

// ---- register-resident rows: cols = RK * ROW_THREADS * 8 ----
//
// Each thread reads its RK 8-element groups of the staged row into registers once; every pass
// then works on those registers. The groups and the fold order are the ones the loop forms
// above use (group k of thread t is columns (k * ROW_THREADS + t) * 8 ..), so the norms are
// bit-identical to theirs, with one shared-memory read per element; softmax takes one exp per
// element and one block fold per row (below).

template <int RK>
__device__ __forceinline__ void row_load_regs(const irx_krow_t &p, const void *xr, float (&v)[RK][8])
{
#pragma unroll
    for (int k = 0; k < RK; k++) row_ld8<true>(xr, p.x_dt, ((int64_t)k * ROW_THREADS + threadIdx.x) * 8, v[k]);
}

// Softmax of a register-resident row with one block fold. Each thread takes the exps of its own
// elements relative to its own maximum m_t (log2 units) and sums them (s_t); one fold of the
// (m, s) pairs (a warp butterfly, then the warps in order: M = max, S = s_a 2^(m_a - M) +
// s_b 2^(m_b - M)) gives the row's maximum M and sum S, and each thread scales its exps by
// 2^(m_t - M) / S. One exp per element and one barrier per row, where the two-pass form needs
// two; the result differs from exp(x - M) / S computed directly by a few f32 ulps.
template <int RK>
__device__ __forceinline__ void softmax_regs(const irx_krow_t &p, const void *xr, int64_t row, float *red, unsigned &seq)
{
    const float L2E = 1.4426950408889634f;
    float v[RK][8], mx[8], se[8];
    row_load_regs<RK>(p, xr, v);
#pragma unroll
    for (int l = 0; l < 8; l++) { mx[l] = -1e30f; se[l] = 0.0f; }
#pragma unroll
    for (int k = 0; k < RK; k++)
#pragma unroll
        for (int l = 0; l < 8; l++) mx[l] = fmaxf(mx[l], v[k][l]);
    const float mine = row_fold8(OP_MAX, mx) * L2E;          // this thread's maximum, log2 units
    if (p.y_dt == DT_BF16) {                                  // bf16 out: half the exps on the FMA pipe
#pragma unroll
        for (int k = 0; k < RK; k++)
#pragma unroll
            for (int l = 0; l < 8; l++) {
                v[k][l] = (l & 1) ? row_ex2_cubic(v[k][l], L2E, mine) : row_ex2(fmaf(v[k][l], L2E, -mine));
                se[l] += v[k][l];
            }
    } else {
#pragma unroll
        for (int k = 0; k < RK; k++)
#pragma unroll
            for (int l = 0; l < 8; l++) {
                v[k][l] = row_ex2(fmaf(v[k][l], L2E, -mine));
                se[l] += v[k][l];
            }
    }
    float m = mine, sum = row_fold8(OP_ADD, se);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, o), so = __shfl_xor_sync(0xffffffffu, sum, o);
        const float mn = fmaxf(m, mo);
        sum = sum * row_ex2(m - mn) + so * row_ex2(mo - mn);
        m = mn;
    }
    {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        float *b = red + (seq++ & 1u) * 32;
        if (lane == 0) { b[2 * warp] = m; b[2 * warp + 1] = sum; }
        __syncthreads();
        m = b[0];
        sum = b[1];
        for (int w = 1; w < ROW_THREADS / 32; w++) {
            const float mw = b[2 * w], mn = fmaxf(m, mw);
            sum = sum * row_ex2(m - mn) + b[2 * w + 1] * row_ex2(mw - mn);
            m = mn;
        }
    }
    const float scale = __fdiv_rn(row_ex2(mine - m), sum);
    const int64_t yb = (p.row0 + row) * p.cols;
#pragma unroll
    for (int k = 0; k < RK; k++) {
        float o[8];
#pragma unroll
        for (int l = 0; l < 8; l++) o[l] = __fmul_rn(v[k][l], scale);
        irx_st8(p.y, p.y_dt, yb + ((int64_t)k * ROW_THREADS + threadIdx.x) * 8, o);
    }
}

template <int RK, bool RMS>
__device__ __forceinline__ void norm_regs(const irx_krow_t &p, const void *xr, int64_t row, float *red, unsigned &seq)
{
    float v[RK][8], acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    row_load_regs<RK>(p, xr, v);
#pragma unroll
    for (int k = 0; k < RK; k++)
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = __fmaf_rn(v[k][l], v[k][l], acc[l]);
    const float ss = irx_block_fold1(OP_ADD, row_fold8(OP_ADD, acc), red, seq++);
    const float inv = RMS ? __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)p.cols), __uint_as_float(p.eps_bits))))
                          : __frcp_rn(__fsqrt_rn(ss));
    const int64_t yb = (p.row0 + row) * p.cols;
#pragma unroll
    for (int k = 0; k < RK; k++) {
        const int64_t c = ((int64_t)k * ROW_THREADS + threadIdx.x) * 8;
        float o[8];
        if (RMS) {
            float w[8];
            row_ld8<false>(p.w, p.w_dt, c, w);
#pragma unroll
            for (int l = 0; l < 8; l++) o[l] = __fmul_rn(__fmul_rn(v[k][l], inv), w[l]);
        } else {
#pragma unroll
            for (int l = 0; l < 8; l++) o[l] = __fmul_rn(v[k][l], inv);
        }
        irx_st8(p.y, p.y_dt, yb + c, o);
    }
}

template <int KIND, int RK>
__device__ __forceinline__ void row_regs(const irx_krow_t &p, const void *xr, int64_t row, float *red, unsigned &seq)
{
    if constexpr (KIND == ROWK_SOFTMAX) softmax_regs<RK>(p, xr, row, red, seq);
    else norm_regs<RK, KIND == ROWK_RMSNORM>(p, xr, row, red, seq);
}

template <int KIND, bool SMEM>
__device__ __forceinline__ void row_dispatch(const irx_krow_t &p, const void *xr, int64_t row, float *red,
                                             const float *U0, float *U, float *ebuf, unsigned &seq)
{
    if constexpr (SMEM && KIND != ROWK_GENERIC) {
        switch (p.rk) {               // the staged row fits the block's registers
        case 1: row_regs<KIND, 1>(p, xr, row, red, seq); return;
        case 2: row_regs<KIND, 2>(p, xr, row, red, seq); return;
        case 4: row_regs<KIND, 4>(p, xr, row, red, seq); return;
        default: break;
        }
    }
    if constexpr (KIND == ROWK_RMSNORM) rmsnorm_row<SMEM>(p, xr, row, red, seq);
    else if constexpr (KIND == ROWK_SOFTMAX) softmax_row<SMEM>(p, xr, row, red, ebuf, seq);
    else if constexpr (KIND == ROWK_L2NORM) l2norm_row<SMEM>(p, xr, row, red, seq);
    else generic_row<SMEM>(p, xr, row, red, U0, U);
}

// ---- the row pipeline: NBUF rows staged by bulk copies ----

template <int KIND>
__device__ __forceinline__ void row_kernel(const irx_krow_t &p)
{
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float red[80];
    __shared__ __align__(8) uint64_t bar[ROW_NBUF];
    unsigned seq = 0;                      // one-barrier folds: buffer parity, advanced together
    __shared__ float U0[PROG_NUNI], U[PROG_NUNI];
    const int esz = p.x_dt == DT_BF16 ? 2 : 4;
    if (KIND == ROWK_GENERIC && threadIdx.x == 0) irx_uinit(p.uni, p.nuni, U0);
    __syncthreads();

    if (!p.bulk_ok) {
        for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
            const void *xr = reinterpret_cast<const unsigned char *>(p.x) + (p.row0 + row) * p.cols * esz;
            row_dispatch<KIND, false>(p, xr, row, red, U0, U, nullptr, seq);
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
    if (threadIdx.x == 0) {             // prologue: the first NBUF-1 rows of this block
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
            // refill the buffer the previous iteration finished with (every thread passed the
            // barrier at the end of that iteration)
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
                for (int i = 1; i < ROW_NBUF; i++) {       // drain this block's later copies
                    int64_t r = row + (int64_t)i * gridDim.x;
                    if (r < p.rows) irx_mbar_wait(&bar[(it + i) % ROW_NBUF], (uint32_t)(((it + i) / ROW_NBUF) & 1), 1u << 20);
                }
            }
            return;
        }
        {
            unsigned char *xr = smem + (size_t)b * p.smem_row_bytes;
            float *ebuf = p.ecache == 1 ? reinterpret_cast<float *>(xr) : nullptr;
            row_dispatch<KIND, true>(p, xr, row, red, U0, U, ebuf, seq);
        }
        __syncthreads();
    }
}

extern "C" __global__ void __launch_bounds__(ROW_THREADS, 2) irx_rowop(const __grid_constant__ irx_krow_t p) { irx_pdl_enter(); row_kernel<ROWK_GENERIC>(p); }
extern "C" __global__ void __launch_bounds__(ROW_THREADS) irx_row_rmsnorm(const __grid_constant__ irx_krow_t p) { irx_pdl_enter(); row_kernel<ROWK_RMSNORM>(p); }
extern "C" __global__ void __launch_bounds__(ROW_THREADS) irx_row_softmax(const __grid_constant__ irx_krow_t p) { irx_pdl_enter(); row_kernel<ROWK_SOFTMAX>(p); }
extern "C" __global__ void __launch_bounds__(ROW_THREADS) irx_row_l2norm(const __grid_constant__ irx_krow_t p) { irx_pdl_enter(); row_kernel<ROWK_L2NORM>(p); }
