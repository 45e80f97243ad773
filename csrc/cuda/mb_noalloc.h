/* C declarations of the allocation-free entry point in attn_decode_noalloc.cu.
 *
 * This interface has no counterpart in the reference.  It serves callers that
 * cannot allocate GPU memory: code running while another component captures
 * the stream into a CUDA graph, hosts that hand out only caller-owned buffers,
 * and C callers without torch.  Scratch memory comes from one fixed device
 * array inside the library (see mb_attn_decode_noalloc_max_scratch_floats).
 *
 * Return codes of mb_attn_decode_noalloc:
 *   0  success
 *   1  invalid argument (null pointer, non-positive size, Hq not a multiple of Hkv)
 *   2  B * Hq * splits * (D + 1) floats exceed the scratch array
 *   3  head_dim not in {64, 128, 256}, or a group size Hq / Hkv without a kernel
 *   4  CUDA error (the message names it; an error pending from earlier work on
 *      this thread is reported, and cleared, before anything is launched)
 * mb_noalloc_last_error() returns the reason for the last non-zero code on the
 * calling thread.
 *
 * Contract: every ctx_lens[b] must be at most 16 * max_blocks (the block
 * table row length).  ctx_lens lives on the device, so the host cannot check
 * it; the kernel clamps a longer context to the 16 * max_blocks tokens that
 * the row addresses.
 */
#pragma once
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

const char* mb_noalloc_last_error(void);
size_t mb_attn_decode_noalloc_max_scratch_floats(void);
int mb_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                           const int* ctx_lens, void* out, int B, int Hq, int Hkv, int D, int max_blocks,
                           int splits, float scale, void* stream);

#ifdef __cplusplus
}
#endif
