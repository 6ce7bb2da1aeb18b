// Allocation-free paged decode attention: one C entry point for callers that cannot allocate
// device memory.  This interface has no counterpart in the reference project.
//
// Who needs it: code that runs where a device allocation is not allowed or not affordable —
// e.g. a latency-critical serving loop (cudaMalloc/cudaFree synchronise the device and can stall
// every stream), or a host framework / plugin that owns all device memory through its own pool and
// hands kernels only the tensors it allocated.  Such callers pass inputs and outputs; the split-KV partial results that the
// regular entry point keeps in a caller-allocated workspace live here in a fixed, file-scope device
// array instead.
//
// Limits and rules:
//   * scratch: AXRL_DECODE_NOALLOC_MAX_ROWS = 8192 rows of (128 + 2) floats (~4.1 MiB), held by every
//     GPU that loads the library until the process exits.  A call needs
//     B * Hq * ceil(max_context / 128) rows; larger calls are rejected (return 1, message on stderr).
//   * the first call on a device looks up the array's device address (cudaGetSymbolAddress) and opts
//     the kernel into its shared-memory size, with that device current; make that first call before
//     any stream capture.  Each device keeps its own address and opt-in, so one process may call it
//     on several GPUs.
//   * all calls share the one array and it keeps the last call's contents; every partial that a call
//     reads was written earlier in the same call, so nothing has to start at zero.  Calls that overlap
//     on the GPU (different streams, or different host threads without ordering) race on the array.
//   * no cudaMalloc, cudaFree or allocating library routine is called.
#pragma once
#ifdef __cplusplus
extern "C" {
#endif

#define AXRL_DECODE_NOALLOC_MAX_ROWS 8192

// q: [B, Hq, 128] bf16; k_cache, v_cache: [pages, Hkv, page_size, 128] bf16;
// block_table: [B, max_pages] int32 page ids; seq_lens: [B] int32 (tokens per sequence, incl. the new one),
// each <= max_context (max_context <= max_pages * page_size; the kernels clamp every length to
// max_context, so a longer sequence is attended over its first max_context tokens only);
// out: [B, Hq, 128] bf16; stream: a cudaStream_t (NULL = legacy default stream).
// Returns 0 on success, 1 if the call needs more scratch than the array holds, 2 on invalid
// arguments, 3 if the device-address lookup failed, 4 if a kernel launch failed (which includes a
// context that entered an error state between the entry check and the launch), 5 if a CUDA error
// was already pending on this host thread when the call began (nothing is launched and that
// error is left in place for the code that caused it).
int axrl_paged_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_table,
                                        const int* seq_lens, void* out, int B, int Hq, int Hkv, int page_size, int max_pages,
                                        int max_context, float scale, void* stream);

#ifdef __cplusplus
}
#endif
