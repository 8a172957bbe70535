/*
 * emmy_noalloc.h -- attention launch with a fixed, statically sized scratch
 * (libemmy_noalloc.so, built from emmy-ptx_b200/csrc/emmy_noalloc.cu).
 *
 * This entry point has no counterpart in the reference: the reference emits
 * PTX and leaves launching to an outside runner (README.md:49-50, 91-92).  It
 * exists for callers that must not allocate device memory while they run:
 * processes whose device memory is already committed to a fixed arena, and
 * latency-critical streams that cannot absorb the device-wide wait that
 * releasing memory brings.  The regular path (ert_mem_alloc'ed scratch, set
 * up by emmy_ptx.runtime.Kernel) is unchanged.
 */
#ifndef EMMY_NOALLOC_H
#define EMMY_NOALLOC_H

#include <stddef.h>
#include <stdint.h>

#include "emmy_rt.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Size of the fixed scratch array: room for the tf32 lo part of a K of up
 * to 32 MiB and for the tf32-rounded V of the same size (heads_total * seq *
 * head_dim <= 8 Mi floats, e.g. 16 heads x 4096 keys x 128).  The hi part
 * is K itself: the tensor core drops the low 13 bits of an f32 operand. */
#define ERT_NOALLOC_SCRATCH_BYTES (64ull << 20)

/* Run one sm_100a attention problem -- the `<entry>_ksplit` pre-pass, then
 * the attention entry -- from `module` (loaded with ert_module_load from
 * Compiler.compile() of an attention IR), with K's tf32 lo part and the
 * tf32-rounded V written to the library's fixed device array instead of
 * allocated scratch.
 *
 *   attention_fn, ksplit_fn  ert_function handles of `<entry>` and
 *                            `<entry>_ksplit` in `module`
 *   geom, args               the attention launch exactly as for ert_launch
 *                            (sidecar geometry; parameter pointers in meta
 *                            arg_order)
 *   k, v                     the K and V device pointers (also in args;
 *                            16-byte aligned, as the kernel reads K with TMA)
 *   heads_total, seq, head_dim  the compiled shape (batch*heads, keys, dims)
 *   err, err_len             receives a message on failure (may be NULL)
 *
 * Allocates nothing.  The first call on a device resolves the array's
 * address (once per device, with that device's context current; under lazy
 * module loading this also loads the library's device image, and with it the
 * array).  A call cannot be recorded into a CUDA graph: it copies the three
 * tensor maps from a pageable host buffer, which stream capture does not
 * allow, so issue it outside any capture.  Returns
 * ERT_E_TOO_LARGE, without launching, when
 * 2 * align256(heads_total*seq*head_dim*4) exceeds ERT_NOALLOC_SCRATCH_BYTES,
 * and ERT_E_ARGUMENT, without launching, when heads_total/seq/head_dim is not
 * the shape `module` was compiled for (recorded in the module as the global
 * emmy_attn_shape_<heads_total>x<seq>x<head_dim>); other codes as in
 * emmy_rt.h.  Calls share the scratch and rewrite the module's tensor-map
 * globals: calls that overlap in time race, so keep them on one stream, and
 * do not also launch the same module through emmy_ptx.runtime.Kernel (it
 * keeps the tensor maps it wrote and would run on the ones this call left). */
int ert_attention_noalloc(uint64_t module, uint64_t attention_fn, uint64_t ksplit_fn,
                          const ert_geom *geom, void **args, uint64_t k, uint64_t v,
                          uint32_t heads_total, uint32_t seq, uint32_t head_dim,
                          uint64_t stream, char *err, size_t err_len);

#ifdef __cplusplus
}
#endif
#endif /* EMMY_NOALLOC_H */
