// pointwise.cu -- the pointwise template: y_k = f_k(x_0..x_{NS-1}, scalars) over an element range.
//
// One grid-stride pass; each thread takes 8 consecutive elements per step (two 128-bit loads
// per f32 stream, one per bf16 stream), with the next step's loads issued before this step's
// arithmetic, so two steps of every stream are in flight per thread. The output programs run
// over all 8 elements at once and the results stream out with evict-first 128-bit stores.
// Launch-uniform scalars (rank-0 const buffers, literals, and anything computed only from
// them) are read and computed once per thread before the pass. The tail of fewer than 8
// elements runs the same programs one element at a time.
//
// Instantiated per stream count NS (1-4) and temporary count NT (1 for chain programs, 8 for
// any other), so a thread holds only the registers its program can touch.
//
// The KIR this serves is the reference's pointwise shape: Load / Assign / Write at the thread's
// own cell, one or 2/4 consecutive names per statement (src/isel.c:1034-1260).

#include "common.cuh"

template <int NS, int NT>
__device__ __forceinline__ void pw_body(const irx_kpw_t &p)
{
    __shared__ float U[PROG_NUNI];
    if (threadIdx.x == 0) {
        irx_uinit(p.uni, p.nuni, U);
        irx_urun(p.uprog, U);
    }
    __syncthreads();
    Regs<8, NS, NT> R;
    R.U = U;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nth = (int64_t)gridDim.x * blockDim.x;
    int64_t head = p.begin;
    if (p.vec_ok) {
        const int64_t nchunk = (p.end - p.begin) / 8;
        float nx[NS][8];
        int64_t c = tid;
        if (c < nchunk) {
#pragma unroll
            for (int s = 0; s < NS; s++) irx_ld8(p.in[s], p.in_dt[s], p.begin + c * 8, nx[s]);
        }
        for (; c < nchunk; c += nth) {
#pragma unroll
            for (int s = 0; s < NS; s++)
#pragma unroll
                for (int l = 0; l < 8; l++) R.s[s][l] = nx[s][l];
            const int64_t cn = c + nth;
            if (cn < nchunk) {
#pragma unroll
                for (int s = 0; s < NS; s++) irx_ld8(p.in[s], p.in_dt[s], p.begin + cn * 8, nx[s]);
            }
#pragma unroll
            for (int o = 0; o < 4; o++) {
                if (o < p.nout) {
                    float r[8];
                    irx_run(p.prog[o], R, r);
                    irx_st8(p.out[o], p.out_dt[o], p.begin + c * 8, r);
                }
            }
        }
        head = p.begin + nchunk * 8;
    }
    // the remainder (or everything, when the buffers are not 16-byte aligned): one at a time
    Regs<1, NS, NT> S;
    S.U = U;
    for (int64_t e = head + tid; e < p.end; e += nth) {
#pragma unroll
        for (int s = 0; s < NS; s++) S.s[s][0] = irx_ld1(p.in[s], p.in_dt[s], e);
#pragma unroll
        for (int o = 0; o < 4; o++) {
            if (o < p.nout) {
                float r[1];
                irx_run(p.prog[o], S, r);
                irx_st1(p.out[o], p.out_dt[o], e, r[0]);
            }
        }
    }
}

#define IRX_PW(NS, NT) \
    extern "C" __global__ void __launch_bounds__(256) irx_pw_s##NS##_t##NT(const __grid_constant__ irx_kpw_t p) \
    { irx_pdl_enter(); pw_body<NS, NT>(p); }

IRX_PW(1, 1) IRX_PW(2, 1) IRX_PW(3, 1) IRX_PW(4, 1)
IRX_PW(1, 8) IRX_PW(2, 8) IRX_PW(3, 8) IRX_PW(4, 8)
