// emmy_noalloc.cu -- attention launch whose pre-pass scratch is a fixed
// device array instead of memory taken from the allocator.
//
// The regular path (emmy_ptx.runtime.Kernel.bind) asks the driver for the
// scratch of the pre-pass (K's tf32 lo part and the tf32-rounded V) on the
// first launch and keeps it.  Some callers
// cannot do that: a process that has already handed all of its device
// memory to a fixed arena (a serving loop sized to fill HBM), or a caller
// on a latency-critical stream that cannot afford the device-wide wait a
// later release of that memory implies.  This entry point draws its scratch
// from a statically sized `__device__` array that is loaded with the
// library's device image, so no call into it allocates or frees device
// memory.  It launches the same two PTX entries as the regular path (the
// `<entry>_ksplit` pre-pass and the attention kernel) from the caller's
// module, through libemmy_rt.
//
// Shape: the call refuses (ERT_E_ARGUMENT, before any copy or launch) a
// heads_total/seq/head_dim that differs from the shape the module was
// compiled for, which the module records in the name of a global
// (emmy_attn_shape_<heads_total>x<seq>x<head_dim>).  The pre-pass writes the
// compiled element count, so only a matching shape keeps it inside the array.
//
// Set-up: the first call on a device (with that device's context current)
// resolves the array's address with cudaGetSymbolAddress and caches it; with
// lazy module loading that is also when the library's device image, and with
// it the array, is loaded onto the device.  No call can be recorded into a
// CUDA graph: each copies its tensor maps from a pageable host buffer, which
// stream capture does not allow.  Nothing in the scratch has to start at
// zero: the pre-pass (head group 0) and the kernel's split warp (the later
// groups) write every byte the attention kernel reads, and the tensor maps
// zero-fill rows past the sequence end.  The pre-pass also records the two
// scratch addresses for the split warp, so it runs before every launch.
//
// Calls share one scratch array and rewrite the module's three tensor-map
// globals, so two calls that overlap in time (different streams, or threads
// without ordering) race; issue them on one stream or order them on the host.
// For the same reason a module used with this call must not also be launched
// through emmy_ptx.runtime.Kernel: Kernel caches the tensor maps it wrote and
// does not see that this call replaced them.

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "emmy_noalloc.h"
#include "emmy_rt.h"

static __device__ __align__(256) unsigned char g_ksplit_scratch[ERT_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void *g_scratch_ptr[kMaxDevices] = {};

// Tiling of the sm_100a attention kernel's K/V tensor maps: 32-float boxes
// along head_dim, 64 keys, one head (sm100/attention.py BOX_KEYS; the same
// for the one-CTA and the CTA-pair kernels).
constexpr uint32_t kBoxDim = 32;
constexpr uint32_t kBoxKeysK = 64;
constexpr uint32_t kBoxKeysV = 64;
constexpr int kDtypeF32 = 7;          // CU_TENSOR_MAP_DATA_TYPE_FLOAT32
constexpr int kSwizzle128 = 3;        // CU_TENSOR_MAP_SWIZZLE_128B
constexpr int kSwizzle128Atom32 = 4;  // CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
constexpr int kL2Promote128 = 2;      // CU_TENSOR_MAP_L2_PROMOTION_L2_128B

int fail(char *err, size_t err_len, int code, const char *fmt, ...) {
    if (err && err_len) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, err_len, fmt, ap);
        va_end(ap);
    }
    return code;
}

int forward(char *err, size_t err_len, int rc, const char *what) {
    return fail(err, err_len, rc, "%s failed (%d): %s", what, rc, ert_last_error());
}

// Device address of the scratch array on the current device (set-up once per
// device, under a lock).
int scratch_address(void **out, char *err, size_t err_len) {
    int dev = -1;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess)
        return fail(err, err_len, ERT_E_NOT_INIT, "cudaGetDevice: %s", cudaGetErrorString(ce));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(err, err_len, ERT_E_ARGUMENT, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        ce = cudaGetSymbolAddress(&p, g_ksplit_scratch);
        if (ce != cudaSuccess || !p)
            return fail(err, err_len, ERT_E_NO_DRIVER, "cudaGetSymbolAddress(scratch): %s",
                        cudaGetErrorString(ce));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return 0;
}

int put_tensormap(uint64_t module, const char *global, uint64_t base, uint64_t heads_total,
                  uint64_t seq, uint64_t head_dim, uint32_t box_keys, int swizzle,
                  uint64_t stream, char *err, size_t err_len) {
    alignas(64) unsigned char desc[128];
    const uint64_t dims[3] = {head_dim, seq, heads_total};
    const uint64_t strides[2] = {head_dim * 4, seq * head_dim * 4};
    const uint32_t box[3] = {kBoxDim, box_keys, 1};
    const uint32_t estr[3] = {1, 1, 1};
    int rc = ert_tensormap_encode(desc, kDtypeF32, 3, base, dims, strides, box, estr, swizzle,
                                  kL2Promote128, 0);
    if (rc) return forward(err, err_len, rc, "ert_tensormap_encode");
    uint64_t dptr = 0;
    size_t bytes = 0;
    rc = ert_module_global(module, global, &dptr, &bytes);
    if (rc) return forward(err, err_len, rc, "ert_module_global");
    if (bytes < sizeof desc)
        return fail(err, err_len, ERT_E_ARGUMENT, "module global %s holds %zu bytes", global, bytes);
    // pageable source: the driver stages it before returning, so the stack
    // buffer may go out of scope afterwards
    rc = ert_memcpy_htod(dptr, desc, sizeof desc, stream);
    if (rc) return forward(err, err_len, rc, "ert_memcpy_htod(tensor map)");
    return 0;
}

}  // namespace

extern "C" int ert_attention_noalloc(uint64_t module, uint64_t attention_fn, uint64_t ksplit_fn,
                                     const ert_geom *geom, void **args, uint64_t k, uint64_t v,
                                     uint32_t heads_total, uint32_t seq, uint32_t head_dim,
                                     uint64_t stream, char *err, size_t err_len) {
    if (err && err_len) err[0] = '\0';
    if (!module || !attention_fn || !ksplit_fn || !geom || !args || !k || !v)
        return fail(err, err_len, ERT_E_ARGUMENT, "ert_attention_noalloc: null handle or pointer");
    if (!heads_total || !seq || !head_dim || head_dim % kBoxDim || head_dim > 128)
        return fail(err, err_len, ERT_E_ARGUMENT,
                    "ert_attention_noalloc: head_dim %u must be 32, 64, 96 or 128 and sizes > 0",
                    head_dim);
    const uint64_t kbytes = uint64_t(heads_total) * seq * head_dim * 4;
    const uint64_t half = (kbytes + 255) & ~uint64_t(255);
    if (2 * half > ERT_NOALLOC_SCRATCH_BYTES)
        return fail(err, err_len, ERT_E_TOO_LARGE,
                    "ert_attention_noalloc: K is %llu bytes; its tf32 lo part and the "
                    "tf32-rounded V need %llu bytes of scratch; the fixed scratch holds %llu "
                    "bytes (use the allocating path for this size)",
                    (unsigned long long)kbytes, (unsigned long long)(2 * half),
                    (unsigned long long)ERT_NOALLOC_SCRATCH_BYTES);
    if ((k | v) & 15)
        return fail(err, err_len, ERT_E_ARGUMENT,
                    "ert_attention_noalloc: K and V must be 16-byte aligned");

    // The pre-pass's element count and the kernel's loops are compiled into
    // the module; the scratch check above holds only if the stated shape is
    // that shape.  The module records it in the name of a global, so a host
    // lookup (no device read, no synchronisation) settles it.
    char shape_name[96];
    snprintf(shape_name, sizeof shape_name, "emmy_attn_shape_%ux%ux%u", heads_total, seq,
             head_dim);
    uint64_t shape_ptr = 0;
    if (ert_module_global(module, shape_name, &shape_ptr, nullptr) != 0)
        return fail(err, err_len, ERT_E_ARGUMENT,
                    "ert_attention_noalloc: the module was not compiled for heads_total=%u "
                    "seq=%u head_dim=%u (no global %s); pass the shape of the attention IR "
                    "it was compiled from",
                    heads_total, seq, head_dim, shape_name);

    void *scratch = nullptr;
    int rc = scratch_address(&scratch, err, err_len);
    if (rc) return rc;
    uint64_t lo = reinterpret_cast<uint64_t>(scratch);
    uint64_t vr = lo + half;

    // the hi operand of the 3xTF32 split is K itself (the tensor core drops
    // the low 13 bits of an f32 operand); the pre-pass writes lo = K - hi
    rc = put_tensormap(module, "tmap_Khi", k, heads_total, seq, head_dim, kBoxKeysK,
                       kSwizzle128, stream, err, err_len);
    if (!rc)
        rc = put_tensormap(module, "tmap_Klo", lo, heads_total, seq, head_dim, kBoxKeysK,
                           kSwizzle128, stream, err, err_len);
    if (!rc)
        rc = put_tensormap(module, "tmap_V", vr, heads_total, seq, head_dim, kBoxKeysV,
                           kSwizzle128Atom32, stream, err, err_len);
    if (rc) return rc;

    // pre-pass: K -> lo and V -> tf32-rounded V; a grid-stride loop, so any
    // grid covers it: 16 blocks of 256 threads per SM, as the regular launch
    // uses (fewer when the problem is smaller)
    const uint64_t nvec = kbytes / 16;
    uint64_t blocks = (nvec + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    ert_geom pg = {{unsigned(blocks), 1, 1}, {256, 1, 1}, {1, 1, 1}, 0};
    void *pargs[4] = {&k, &v, &lo, &vr};
    rc = ert_launch(ksplit_fn, &pg, pargs, stream);
    if (rc) return forward(err, err_len, rc, "ert_launch(ksplit)");
    rc = ert_launch(attention_fn, geom, args, stream);
    if (rc) return forward(err, err_len, rc, "ert_launch(attention)");
    return 0;
}
