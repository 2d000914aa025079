/* jit_blob.S -- the op semantics header and the op numbering, embedded as NUL-terminated text
 * for NVRTC (the per-graph kernels of jit.c include them). */
    .section .rodata
    .global irx_src_ops_cuh
    .hidden irx_src_ops_cuh
irx_src_ops_cuh:
    .incbin "kernels/ops.cuh"
    .byte 0
    .global irx_src_ops_h
    .hidden irx_src_ops_h
irx_src_ops_h:
    .incbin "irx_ops.h"
    .byte 0
    .section .note.GNU-stack,"",@progbits
