/* Embeds the build-time glibc-expf fix-up table (gen_expf_fixups.c) in
 * liblal_tail.so: [uint32 n][n input bit patterns][n glibc result bits]. */
    .section .rodata
    .balign 16
    .globl lal_expf_fixups_blob
    .hidden lal_expf_fixups_blob
    .type lal_expf_fixups_blob, @object
lal_expf_fixups_blob:
    .incbin "expf_fixups.bin"
    .globl lal_expf_fixups_blob_end
    .hidden lal_expf_fixups_blob_end
lal_expf_fixups_blob_end:
    .section .note.GNU-stack,"",@progbits
