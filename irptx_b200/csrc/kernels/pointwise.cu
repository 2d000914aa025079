// pointwise.cu -- the pointwise template: y_k = f_k(x_0..x_3, scalars) over an element range.
//
// One grid-stride pass; each thread takes 8 consecutive elements per step (two 128-bit loads
// per f32 stream, one per bf16 stream; one or two 128-bit stores per output), runs the
// output programs over all 8 at once and streams the results out with evict-first stores.
// Launch-uniform scalars (rank-0 const buffers, literals, and anything computed only from
// them) are read and computed once per thread before the pass. The tail of fewer than 8
// elements runs the same programs one element at a time.
//
// The KIR this serves is the reference's pointwise shape: Load / Assign / Write at the thread's
// own cell, one or 2/4 consecutive names per statement (src/isel.c:1034-1260).

#include "common.cuh"

template <int V>
__device__ __forceinline__ void pw_elems(const irx_kpw_t &p, Regs<V> &R, int64_t e)
{
#pragma unroll
    for (int s = 0; s < PROG_NSTREAM; s++) {
        if (s < p.nin) {
            if (V == 8) {
                float t[8];
                irx_ld8(p.in[s], p.in_dt[s], e, t);
#pragma unroll
                for (int l = 0; l < V; l++) R.e[s][l] = t[l % 8];
            } else {
#pragma unroll
                for (int l = 0; l < V; l++) R.e[s][l] = irx_ld1(p.in[s], p.in_dt[s], e + l);
            }
        }
    }
#pragma unroll
    for (int o = 0; o < 4; o++) {
        if (o < p.nout) {
            float r[V];
            irx_run<V>(p.prog[o], R, r);
            if (V == 8) {
                float t[8];
#pragma unroll
                for (int l = 0; l < 8; l++) t[l] = r[l % V];
                irx_st8(p.out[o], p.out_dt[o], e, t);
            } else {
#pragma unroll
                for (int l = 0; l < V; l++) irx_st1(p.out[o], p.out_dt[o], e + l, r[l]);
            }
        }
    }
}

extern "C" __global__ void __launch_bounds__(256) irx_pointwise(const __grid_constant__ irx_kpw_t p)
{
    Regs<8> R;
    irx_uinit(p.uni, p.nuni, R.u);
    irx_urun(p.uprog, R.u);
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nth = (int64_t)gridDim.x * blockDim.x;
    int64_t head = p.begin;
    if (p.vec_ok) {
        const int64_t nchunk = (p.end - p.begin) / 8;
        for (int64_t c = tid; c < nchunk; c += nth) pw_elems<8>(p, R, p.begin + c * 8);
        head = p.begin + nchunk * 8;
    }
    // the remainder (or everything, when the buffers are not 16-byte aligned): one at a time
    Regs<1> S;
#pragma unroll
    for (int i = 0; i < PROG_NUNI; i++) S.u[i] = R.u[i];
    for (int64_t e = head + tid; e < p.end; e += nth) pw_elems<1>(p, S, e);
}
