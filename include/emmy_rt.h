/*
 * emmy_rt.h -- C ABI of the emmy-ptx B200 kernel runtime (libemmy_rt.so).
 *
 * The reference compiler stops at PTX text: "the entry-point name, parameter
 * order, and launch geometry come from the problem's meta.json"
 * (README.md:49-50) and an external runner assembles and launches the PTX
 * (README.md:91-92; compiler.py:2202-2220 emits `.visible .entry <entry>`
 * with `.param` names `p_<arg>` in meta `arg_order`, compiler.py:2109-2114).
 * This library is that runner, over the CUDA driver API, with a plain C ABI:
 * device buffers are CUdeviceptr values (uint64_t), streams are CUstream
 * handles (uint64_t, 0 = legacy default stream), kernel arguments are a
 * cuLaunchKernel-style array of pointers to each parameter value in
 * arg_order.  No torch, no C++ types cross the boundary.
 *
 * Every function returns 0 on success, a CUresult code (> 0) from the driver,
 * or a negative ERT_E_* code; it never aborts.  ert_last_error() returns a
 * thread-local message for the last failure.  libcuda.so.1 is loaded with
 * dlopen on first use, so the library loads (and its symbols resolve) on a
 * machine without a GPU.
 */
#ifndef EMMY_RT_H
#define EMMY_RT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ERT_ABI_VERSION 2

#define ERT_E_NO_DRIVER   (-1)  /* libcuda.so.1 missing or a symbol absent */
#define ERT_E_ARGUMENT    (-2)  /* invalid argument (null pointer, bad size) */
#define ERT_E_NOT_INIT    (-3)  /* ert_init() was not called on this thread */
#define ERT_E_KERNEL      (-4)  /* a kernel reported an error status word */
#define ERT_E_TOO_LARGE   (-5)  /* request exceeds a fixed capacity */

/* Launch geometry: the meta.json grid/block, plus the sidecar's cluster
 * shape and dynamic shared-memory bytes (0 = none). */
typedef struct ert_geom {
    unsigned grid[3];
    unsigned block[3];
    unsigned cluster[3];
    unsigned shared_bytes;
} ert_geom;

/* Version of this ABI (ERT_ABI_VERSION). */
int ert_abi_version(void);

/* Number of CUDA devices (0 on a machine without a GPU or driver). */
int ert_device_count(int *count);

/* cuInit, retain device `device`'s primary context (the one the CUDA
 * runtime and torch use) and make it current on the calling thread. */
int ert_init(int device);

/* JIT-load a PTX module (text from Compiler.compile()).  On failure the
 * driver's JIT error log is copied into `log` (may be NULL). */
int ert_module_load(const char *ptx, uint64_t *module, char *log, size_t log_len);
int ert_module_unload(uint64_t module);

/* The `.visible .entry` named `entry` (compiler.py:2215) in `module`. */
int ert_function(uint64_t module, const char *entry, uint64_t *function);

/* Register/thread/shared/local usage of a loaded kernel. */
int ert_function_attrs(uint64_t function, int *num_regs, int *max_threads,
                       int *static_shared, int *local_bytes);

/* Launch `function` with cuLaunchKernelEx: `args[i]` points at the value of
 * parameter i in meta arg_order.  Dynamic shared memory above 48 KB is
 * opted into automatically; a cluster shape other than 1x1x1 is passed as
 * a launch attribute. */
int ert_launch(uint64_t function, const ert_geom *geom, void **args, uint64_t stream);

/* Address and size of a module-scope `.global` variable (tensor maps,
 * the status word). */
int ert_module_global(uint64_t module, const char *name, uint64_t *dptr, size_t *bytes);

/* Encode a tiled TMA descriptor (cuTensorMapEncodeTiled) into `out`
 * (128 bytes, 64-byte aligned).  dtype/swizzle/l2/oob take the driver's
 * CUtensorMap* enum values; `strides` has rank-1 byte strides. */
int ert_tensormap_encode(void *out, int dtype, int rank, uint64_t global_addr,
                         const uint64_t *dims, const uint64_t *strides,
                         const uint32_t *box, const uint32_t *elem_strides,
                         int swizzle, int l2_promotion, int oob_fill);

/* Stream-ordered copies and fill (asynchronous on `stream`). */
int ert_memcpy_htod(uint64_t dst, const void *src, size_t bytes, uint64_t stream);
int ert_memcpy_dtoh(void *dst, uint64_t src, size_t bytes, uint64_t stream);
/* Device to device, one copy per call; with `dst` a peer's buffer mapped by
 * ert_ipc_open the copy engines move it over NVLink. */
int ert_memcpy_dtod(uint64_t dst, uint64_t src, size_t bytes, uint64_t stream);
int ert_memset_d8(uint64_t dst, unsigned char value, size_t bytes, uint64_t stream);
int ert_stream_sync(uint64_t stream);

/* Streams of the caller's own (non-blocking: not ordered against the legacy
 * default stream), for callers without another CUDA runtime.  The
 * host-buffer pipeline uses one for host->device copies, one for launches
 * and one for device->host copies, ordered by events. */
int ert_stream_create(uint64_t *stream);
int ert_stream_destroy(uint64_t stream);
/* Work submitted to `stream` after this call waits for `event`'s last
 * record (cuStreamWaitEvent). */
int ert_stream_wait_event(uint64_t stream, uint64_t event);

/* Device memory for callers that do not bring their own allocator. */
int ert_mem_alloc(uint64_t *dptr, size_t bytes);
int ert_mem_free(uint64_t dptr);
/* Page-locked host memory (for host<->device copies that overlap). */
int ert_host_alloc(void **ptr, size_t bytes);
int ert_host_free(void *ptr);

/* CUDA IPC for buffers from ert_mem_alloc (one node): the owner exports a
 * handle of ERT_IPC_HANDLE_BYTES bytes; another process opens it and gets a
 * device pointer to the same memory (peer access enabled on demand), which
 * its kernels can store to over NVLink.  Close before the owner frees. */
#define ERT_IPC_HANDLE_BYTES 64
int ert_ipc_get_handle(uint64_t dptr, void *handle);
int ert_ipc_open(const void *handle, uint64_t *dptr);
int ert_ipc_close(uint64_t dptr);

/* CUDA events, for timing on a stream and for ordering streams. */
int ert_event_create(uint64_t *event);
int ert_event_record(uint64_t event, uint64_t stream);
int ert_event_elapsed(uint64_t start, uint64_t end, float *ms);
/* Block the calling thread until `event`'s last record has completed. */
int ert_event_sync(uint64_t event);
int ert_event_destroy(uint64_t event);

/* Read and clear the module's `emmy_status` word (0 = ok).  Kernels with
 * bounded waits (mbarrier/TMA pipelines) store a nonzero code there instead
 * of hanging.  Synchronises `stream` first.  Modules without the word report
 * 0. */
int ert_status(uint64_t module, uint32_t *code, uint64_t stream);

/* Thread-local message describing the last failure ("" if none). */
const char *ert_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* EMMY_RT_H */
