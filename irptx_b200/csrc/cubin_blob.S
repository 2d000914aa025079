/* cubin_blob.S -- embeds the sm_100a kernel cubin (built by nvcc) into the library. */
    .section .rodata
    .balign 64
    .global irx_cubin
    .hidden irx_cubin
irx_cubin:
    .incbin IRX_CUBIN_PATH
    .byte 0
    .global irx_cubin_end
    .hidden irx_cubin_end
irx_cubin_end:
    .section .note.GNU-stack,"",@progbits
