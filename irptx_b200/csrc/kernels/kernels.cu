// kernels.cu -- the one translation unit of sm_100a kernel templates, built into one cubin
// that the host library embeds and loads with cuModuleLoadData.
#include "pointwise.cu"
#include "reduce.cu"
#include "rowop.cu"
#include "gemm.cu"
#include "attn.cu"
