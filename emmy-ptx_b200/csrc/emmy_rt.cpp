// emmy_rt.cpp -- the kernel runtime behind include/emmy_rt.h.
//
// A thin layer over the CUDA driver API: libcuda.so.1 is opened with dlopen
// and every entry point is resolved by its exported (versioned) name, so the
// library builds and loads on a machine without a GPU.  It owns nothing but
// what the caller asks for: modules, events and explicit allocations are
// handles that the caller releases.

#include "emmy_rt.h"

#include <cuda.h>
#include <dlfcn.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

namespace {

thread_local std::string g_error;

int fail(int code, const std::string &msg) {
    g_error = msg;
    return code;
}

#define ERT_STR2(x) #x
#define ERT_STR(x) ERT_STR2(x)

struct Driver {
    void *handle = nullptr;
    bool ok = false;
    std::string why;
#define ERT_FN(name) decltype(&::name) name = nullptr;
    ERT_FN(cuInit)
    ERT_FN(cuDeviceGetCount)
    ERT_FN(cuDeviceGet)
    ERT_FN(cuDevicePrimaryCtxRetain)
    ERT_FN(cuCtxSetCurrent)
    ERT_FN(cuCtxGetCurrent)
    ERT_FN(cuGetErrorString)
    ERT_FN(cuModuleLoadDataEx)
    ERT_FN(cuModuleUnload)
    ERT_FN(cuModuleGetFunction)
    ERT_FN(cuModuleGetGlobal)
    ERT_FN(cuFuncGetAttribute)
    ERT_FN(cuFuncSetAttribute)
    ERT_FN(cuLaunchKernelEx)
    ERT_FN(cuTensorMapEncodeTiled)
    ERT_FN(cuMemcpyHtoDAsync)
    ERT_FN(cuMemcpyDtoHAsync)
    ERT_FN(cuMemcpyDtoDAsync)
    ERT_FN(cuMemsetD8Async)
    ERT_FN(cuStreamSynchronize)
    ERT_FN(cuStreamCreate)
    ERT_FN(cuStreamDestroy)
    ERT_FN(cuStreamWaitEvent)
    ERT_FN(cuMemAlloc)
    ERT_FN(cuMemFree)
    ERT_FN(cuMemHostAlloc)
    ERT_FN(cuMemFreeHost)
    ERT_FN(cuEventCreate)
    ERT_FN(cuEventRecord)
    ERT_FN(cuEventElapsedTime)
    ERT_FN(cuEventDestroy)
    ERT_FN(cuEventSynchronize)
    ERT_FN(cuIpcGetMemHandle)
    ERT_FN(cuIpcOpenMemHandle)
    ERT_FN(cuIpcCloseMemHandle)
#undef ERT_FN

    Driver() {
        handle = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
        if (!handle) {
            why = "libcuda.so.1 not found (no NVIDIA driver on this machine)";
            return;
        }
        bool all = true;
        // ERT_STR expands cuda.h's versioning macros (cuMemAlloc ->
        // cuMemAlloc_v2 ...), so the exported symbol matches the prototype.
#define ERT_LOAD(name)                                                    \
        name = reinterpret_cast<decltype(name)>(dlsym(handle, ERT_STR(name))); \
        if (!name) { all = false; why = "driver symbol missing: " ERT_STR(name); }
        ERT_LOAD(cuInit)
        ERT_LOAD(cuDeviceGetCount)
        ERT_LOAD(cuDeviceGet)
        ERT_LOAD(cuDevicePrimaryCtxRetain)
        ERT_LOAD(cuCtxSetCurrent)
        ERT_LOAD(cuCtxGetCurrent)
        ERT_LOAD(cuGetErrorString)
        ERT_LOAD(cuModuleLoadDataEx)
        ERT_LOAD(cuModuleUnload)
        ERT_LOAD(cuModuleGetFunction)
        ERT_LOAD(cuModuleGetGlobal)
        ERT_LOAD(cuFuncGetAttribute)
        ERT_LOAD(cuFuncSetAttribute)
        ERT_LOAD(cuLaunchKernelEx)
        ERT_LOAD(cuTensorMapEncodeTiled)
        ERT_LOAD(cuMemcpyHtoDAsync)
        ERT_LOAD(cuMemcpyDtoHAsync)
        ERT_LOAD(cuMemcpyDtoDAsync)
        ERT_LOAD(cuMemsetD8Async)
        ERT_LOAD(cuStreamSynchronize)
        ERT_LOAD(cuStreamCreate)
        ERT_LOAD(cuStreamDestroy)
        ERT_LOAD(cuStreamWaitEvent)
        ERT_LOAD(cuMemAlloc)
        ERT_LOAD(cuMemFree)
        ERT_LOAD(cuMemHostAlloc)
        ERT_LOAD(cuMemFreeHost)
        ERT_LOAD(cuEventCreate)
        ERT_LOAD(cuEventRecord)
        ERT_LOAD(cuEventElapsedTime)
        ERT_LOAD(cuEventDestroy)
        ERT_LOAD(cuEventSynchronize)
        ERT_LOAD(cuIpcGetMemHandle)
        ERT_LOAD(cuIpcOpenMemHandle)
        ERT_LOAD(cuIpcCloseMemHandle)
#undef ERT_LOAD
        ok = all;
    }
};

Driver &drv() {
    static Driver d;
    return d;
}

std::string cu_message(CUresult r) {
    const char *s = nullptr;
    if (drv().cuGetErrorString && drv().cuGetErrorString(r, &s) == CUDA_SUCCESS && s)
        return s;
    return "CUresult " + std::to_string(static_cast<int>(r));
}

int check(CUresult r, const char *what) {
    if (r == CUDA_SUCCESS) return 0;
    return fail(static_cast<int>(r), std::string(what) + ": " + cu_message(r));
}

#define ERT_NEED_DRIVER()                                   \
    do {                                                    \
        if (!drv().ok) return fail(ERT_E_NO_DRIVER, drv().why); \
    } while (0)

thread_local CUcontext t_ctx = nullptr;

// Make sure a context is current: the one ert_init() chose on this thread,
// or whatever the CUDA runtime (torch) already made current.
int need_ctx() {
    CUcontext cur = nullptr;
    if (drv().cuCtxGetCurrent(&cur) == CUDA_SUCCESS && cur) return 0;
    if (t_ctx) return check(drv().cuCtxSetCurrent(t_ctx), "cuCtxSetCurrent");
    return fail(ERT_E_NOT_INIT, "no CUDA context is current: call ert_init(device) first");
}

std::mutex g_smem_mu;
std::unordered_map<uint64_t, unsigned> g_smem_optin;  // function -> bytes opted in
// function -> its module, so unloading a module forgets its opt-ins (the
// driver may hand out the same function handle for a later module)
std::unordered_map<uint64_t, uint64_t> g_fn_module;

}  // namespace

extern "C" {

int ert_abi_version(void) { return ERT_ABI_VERSION; }

const char *ert_last_error(void) { return g_error.c_str(); }

int ert_device_count(int *count) {
    if (!count) return fail(ERT_E_ARGUMENT, "count is null");
    *count = 0;
    if (!drv().ok) return 0;
    if (drv().cuInit(0) != CUDA_SUCCESS) return 0;
    int n = 0;
    if (drv().cuDeviceGetCount(&n) != CUDA_SUCCESS) return 0;
    *count = n;
    return 0;
}

int ert_init(int device) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = check(drv().cuInit(0), "cuInit"))) return rc;
    CUdevice dev;
    if ((rc = check(drv().cuDeviceGet(&dev, device), "cuDeviceGet"))) return rc;
    CUcontext ctx;
    if ((rc = check(drv().cuDevicePrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain")))
        return rc;
    if ((rc = check(drv().cuCtxSetCurrent(ctx), "cuCtxSetCurrent"))) return rc;
    t_ctx = ctx;
    return 0;
}

int ert_module_load(const char *ptx, uint64_t *module, char *log, size_t log_len) {
    ERT_NEED_DRIVER();
    if (!ptx || !module) return fail(ERT_E_ARGUMENT, "ptx or module is null");
    int rc;
    if ((rc = need_ctx())) return rc;
    static thread_local char errlog[16384];
    errlog[0] = 0;
    CUjit_option opts[2] = {CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
    void *vals[2] = {errlog, reinterpret_cast<void *>(static_cast<uintptr_t>(sizeof(errlog)))};
    CUmodule mod = nullptr;
    CUresult r = drv().cuModuleLoadDataEx(&mod, ptx, 2, opts, vals);
    if (log && log_len) {
        std::snprintf(log, log_len, "%s", errlog);
    }
    if (r != CUDA_SUCCESS)
        return fail(static_cast<int>(r), std::string("cuModuleLoadDataEx: ") + cu_message(r) +
                                             (errlog[0] ? std::string("\n") + errlog : ""));
    *module = reinterpret_cast<uint64_t>(mod);
    return 0;
}

int ert_module_unload(uint64_t module) {
    ERT_NEED_DRIVER();
    if (!module) return fail(ERT_E_ARGUMENT, "module is null");
    {
        std::lock_guard<std::mutex> lock(g_smem_mu);
        for (auto it = g_fn_module.begin(); it != g_fn_module.end();) {
            if (it->second == module) {
                g_smem_optin.erase(it->first);
                it = g_fn_module.erase(it);
            } else {
                ++it;
            }
        }
    }
    return check(drv().cuModuleUnload(reinterpret_cast<CUmodule>(module)), "cuModuleUnload");
}

int ert_function(uint64_t module, const char *entry, uint64_t *function) {
    ERT_NEED_DRIVER();
    if (!module || !entry || !function) return fail(ERT_E_ARGUMENT, "null argument");
    CUfunction f = nullptr;
    int rc = check(drv().cuModuleGetFunction(&f, reinterpret_cast<CUmodule>(module), entry),
                   "cuModuleGetFunction");
    if (rc) return fail(rc, g_error + " (entry '" + entry + "')");
    *function = reinterpret_cast<uint64_t>(f);
    std::lock_guard<std::mutex> lock(g_smem_mu);
    if (g_fn_module[*function] != module) {       // a handle reused by a new module
        g_smem_optin.erase(*function);
        g_fn_module[*function] = module;
    }
    return 0;
}

int ert_function_attrs(uint64_t function, int *num_regs, int *max_threads, int *static_shared,
                       int *local_bytes) {
    ERT_NEED_DRIVER();
    if (!function) return fail(ERT_E_ARGUMENT, "function is null");
    CUfunction f = reinterpret_cast<CUfunction>(function);
    int rc = 0;
    if (num_regs && (rc = check(drv().cuFuncGetAttribute(num_regs, CU_FUNC_ATTRIBUTE_NUM_REGS, f),
                                "cuFuncGetAttribute")))
        return rc;
    if (max_threads &&
        (rc = check(drv().cuFuncGetAttribute(max_threads, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, f),
                    "cuFuncGetAttribute")))
        return rc;
    if (static_shared &&
        (rc = check(drv().cuFuncGetAttribute(static_shared, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, f),
                    "cuFuncGetAttribute")))
        return rc;
    if (local_bytes &&
        (rc = check(drv().cuFuncGetAttribute(local_bytes, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, f),
                    "cuFuncGetAttribute")))
        return rc;
    return 0;
}

int ert_launch(uint64_t function, const ert_geom *geom, void **args, uint64_t stream) {
    ERT_NEED_DRIVER();
    if (!function || !geom) return fail(ERT_E_ARGUMENT, "function or geometry is null");
    int rc;
    if ((rc = need_ctx())) return rc;
    CUfunction f = reinterpret_cast<CUfunction>(function);
    if (geom->shared_bytes > 48 * 1024) {
        std::lock_guard<std::mutex> lock(g_smem_mu);
        auto it = g_smem_optin.find(function);
        if (it == g_smem_optin.end() || it->second < geom->shared_bytes) {
            rc = check(drv().cuFuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                                static_cast<int>(geom->shared_bytes)),
                       "cuFuncSetAttribute(max dynamic shared memory)");
            if (rc) return rc;
            g_smem_optin[function] = geom->shared_bytes;
        }
    }
    CUlaunchConfig cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDimX = geom->grid[0] ? geom->grid[0] : 1;
    cfg.gridDimY = geom->grid[1] ? geom->grid[1] : 1;
    cfg.gridDimZ = geom->grid[2] ? geom->grid[2] : 1;
    cfg.blockDimX = geom->block[0] ? geom->block[0] : 1;
    cfg.blockDimY = geom->block[1] ? geom->block[1] : 1;
    cfg.blockDimZ = geom->block[2] ? geom->block[2] : 1;
    cfg.sharedMemBytes = geom->shared_bytes;
    cfg.hStream = reinterpret_cast<CUstream>(stream);
    CUlaunchAttribute attr[1];
    unsigned cx = geom->cluster[0] ? geom->cluster[0] : 1;
    unsigned cy = geom->cluster[1] ? geom->cluster[1] : 1;
    unsigned cz = geom->cluster[2] ? geom->cluster[2] : 1;
    if (cx * cy * cz > 1) {
        attr[0].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
        attr[0].value.clusterDim.x = cx;
        attr[0].value.clusterDim.y = cy;
        attr[0].value.clusterDim.z = cz;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return check(drv().cuLaunchKernelEx(&cfg, f, args, nullptr), "cuLaunchKernelEx");
}

int ert_module_global(uint64_t module, const char *name, uint64_t *dptr, size_t *bytes) {
    ERT_NEED_DRIVER();
    if (!module || !name) return fail(ERT_E_ARGUMENT, "null argument");
    CUdeviceptr p = 0;
    size_t n = 0;
    int rc = check(drv().cuModuleGetGlobal(&p, &n, reinterpret_cast<CUmodule>(module), name),
                   "cuModuleGetGlobal");
    if (rc) return fail(rc, g_error + " ('" + name + "')");
    if (dptr) *dptr = static_cast<uint64_t>(p);
    if (bytes) *bytes = n;
    return 0;
}

int ert_tensormap_encode(void *out, int dtype, int rank, uint64_t global_addr,
                         const uint64_t *dims, const uint64_t *strides, const uint32_t *box,
                         const uint32_t *elem_strides, int swizzle, int l2_promotion,
                         int oob_fill) {
    ERT_NEED_DRIVER();
    if (!out || !dims || !box || rank < 1 || rank > 5)
        return fail(ERT_E_ARGUMENT, "bad tensor map arguments");
    if (reinterpret_cast<uintptr_t>(out) % 64)
        return fail(ERT_E_ARGUMENT, "tensor map output must be 64-byte aligned");
    cuuint64_t gdim[5], gstride[4];
    cuuint32_t bdim[5], estr[5];
    for (int i = 0; i < rank; ++i) {
        gdim[i] = dims[i];
        bdim[i] = box[i];
        estr[i] = elem_strides ? elem_strides[i] : 1;
    }
    for (int i = 0; i < rank - 1; ++i) gstride[i] = strides[i];
    return check(drv().cuTensorMapEncodeTiled(
                     reinterpret_cast<CUtensorMap *>(out), static_cast<CUtensorMapDataType>(dtype),
                     static_cast<cuuint32_t>(rank), reinterpret_cast<void *>(global_addr), gdim,
                     rank > 1 ? gstride : nullptr, bdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     static_cast<CUtensorMapSwizzle>(swizzle),
                     static_cast<CUtensorMapL2promotion>(l2_promotion),
                     static_cast<CUtensorMapFloatOOBfill>(oob_fill)),
                 "cuTensorMapEncodeTiled");
}

int ert_memcpy_htod(uint64_t dst, const void *src, size_t bytes, uint64_t stream) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = need_ctx())) return rc;
    if (!bytes) return 0;
    return check(drv().cuMemcpyHtoDAsync(static_cast<CUdeviceptr>(dst), src, bytes,
                                         reinterpret_cast<CUstream>(stream)),
                 "cuMemcpyHtoDAsync");
}

int ert_memcpy_dtoh(void *dst, uint64_t src, size_t bytes, uint64_t stream) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = need_ctx())) return rc;
    if (!bytes) return 0;
    return check(drv().cuMemcpyDtoHAsync(dst, static_cast<CUdeviceptr>(src), bytes,
                                         reinterpret_cast<CUstream>(stream)),
                 "cuMemcpyDtoHAsync");
}

int ert_memcpy_dtod(uint64_t dst, uint64_t src, size_t bytes, uint64_t stream) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = need_ctx())) return rc;
    if (!bytes) return 0;
    return check(drv().cuMemcpyDtoDAsync(static_cast<CUdeviceptr>(dst),
                                         static_cast<CUdeviceptr>(src), bytes,
                                         reinterpret_cast<CUstream>(stream)),
                 "cuMemcpyDtoDAsync");
}

int ert_memset_d8(uint64_t dst, unsigned char value, size_t bytes, uint64_t stream) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = need_ctx())) return rc;
    if (!bytes) return 0;
    return check(drv().cuMemsetD8Async(static_cast<CUdeviceptr>(dst), value, bytes,
                                       reinterpret_cast<CUstream>(stream)),
                 "cuMemsetD8Async");
}

int ert_stream_sync(uint64_t stream) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = need_ctx())) return rc;
    return check(drv().cuStreamSynchronize(reinterpret_cast<CUstream>(stream)),
                 "cuStreamSynchronize");
}

int ert_stream_create(uint64_t *stream) {
    ERT_NEED_DRIVER();
    if (!stream) return fail(ERT_E_ARGUMENT, "stream is null");
    int rc;
    if ((rc = need_ctx())) return rc;
    CUstream s = nullptr;
    // non-blocking: no implicit ordering against the legacy default stream,
    // so copies on one such stream overlap work on the others
    if ((rc = check(drv().cuStreamCreate(&s, CU_STREAM_NON_BLOCKING), "cuStreamCreate")))
        return rc;
    *stream = reinterpret_cast<uint64_t>(s);
    return 0;
}

int ert_stream_destroy(uint64_t stream) {
    ERT_NEED_DRIVER();
    if (!stream) return fail(ERT_E_ARGUMENT, "stream is null (the default stream is not owned)");
    return check(drv().cuStreamDestroy(reinterpret_cast<CUstream>(stream)), "cuStreamDestroy");
}

int ert_stream_wait_event(uint64_t stream, uint64_t event) {
    ERT_NEED_DRIVER();
    if (!event) return fail(ERT_E_ARGUMENT, "event is null");
    return check(drv().cuStreamWaitEvent(reinterpret_cast<CUstream>(stream),
                                         reinterpret_cast<CUevent>(event), 0),
                 "cuStreamWaitEvent");
}

int ert_mem_alloc(uint64_t *dptr, size_t bytes) {
    ERT_NEED_DRIVER();
    if (!dptr) return fail(ERT_E_ARGUMENT, "dptr is null");
    int rc;
    if ((rc = need_ctx())) return rc;
    CUdeviceptr p = 0;
    if ((rc = check(drv().cuMemAlloc(&p, bytes ? bytes : 1), "cuMemAlloc"))) return rc;
    *dptr = static_cast<uint64_t>(p);
    return 0;
}

int ert_mem_free(uint64_t dptr) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = need_ctx())) return rc;
    return check(drv().cuMemFree(static_cast<CUdeviceptr>(dptr)), "cuMemFree");
}

int ert_ipc_get_handle(uint64_t dptr, void *handle) {
    ERT_NEED_DRIVER();
    if (!dptr || !handle) return fail(ERT_E_ARGUMENT, "dptr or handle is null");
    int rc;
    if ((rc = need_ctx())) return rc;
    CUipcMemHandle h;
    if ((rc = check(drv().cuIpcGetMemHandle(&h, static_cast<CUdeviceptr>(dptr)),
                    "cuIpcGetMemHandle")))
        return rc;
    static_assert(sizeof(h) == ERT_IPC_HANDLE_BYTES, "CUipcMemHandle size");
    std::memcpy(handle, &h, sizeof h);
    return 0;
}

int ert_ipc_open(const void *handle, uint64_t *dptr) {
    ERT_NEED_DRIVER();
    if (!handle || !dptr) return fail(ERT_E_ARGUMENT, "handle or dptr is null");
    int rc;
    if ((rc = need_ctx())) return rc;
    CUipcMemHandle h;
    std::memcpy(&h, handle, sizeof h);
    CUdeviceptr p = 0;
    if ((rc = check(drv().cuIpcOpenMemHandle(&p, h, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS),
                    "cuIpcOpenMemHandle")))
        return rc;
    *dptr = static_cast<uint64_t>(p);
    return 0;
}

int ert_ipc_close(uint64_t dptr) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = need_ctx())) return rc;
    return check(drv().cuIpcCloseMemHandle(static_cast<CUdeviceptr>(dptr)),
                 "cuIpcCloseMemHandle");
}

int ert_host_alloc(void **ptr, size_t bytes) {
    ERT_NEED_DRIVER();
    if (!ptr) return fail(ERT_E_ARGUMENT, "ptr is null");
    int rc;
    if ((rc = need_ctx())) return rc;
    return check(drv().cuMemHostAlloc(ptr, bytes ? bytes : 1, 0), "cuMemHostAlloc");
}

int ert_host_free(void *ptr) {
    ERT_NEED_DRIVER();
    int rc;
    if ((rc = need_ctx())) return rc;
    return check(drv().cuMemFreeHost(ptr), "cuMemFreeHost");
}

int ert_event_create(uint64_t *event) {
    ERT_NEED_DRIVER();
    if (!event) return fail(ERT_E_ARGUMENT, "event is null");
    int rc;
    if ((rc = need_ctx())) return rc;
    CUevent e = nullptr;
    if ((rc = check(drv().cuEventCreate(&e, CU_EVENT_DEFAULT), "cuEventCreate"))) return rc;
    *event = reinterpret_cast<uint64_t>(e);
    return 0;
}

int ert_event_record(uint64_t event, uint64_t stream) {
    ERT_NEED_DRIVER();
    return check(drv().cuEventRecord(reinterpret_cast<CUevent>(event),
                                     reinterpret_cast<CUstream>(stream)),
                 "cuEventRecord");
}

int ert_event_elapsed(uint64_t start, uint64_t end, float *ms) {
    ERT_NEED_DRIVER();
    if (!ms) return fail(ERT_E_ARGUMENT, "ms is null");
    return check(drv().cuEventElapsedTime(ms, reinterpret_cast<CUevent>(start),
                                          reinterpret_cast<CUevent>(end)),
                 "cuEventElapsedTime");
}

int ert_event_sync(uint64_t event) {
    ERT_NEED_DRIVER();
    if (!event) return fail(ERT_E_ARGUMENT, "event is null");
    return check(drv().cuEventSynchronize(reinterpret_cast<CUevent>(event)),
                 "cuEventSynchronize");
}

int ert_event_destroy(uint64_t event) {
    ERT_NEED_DRIVER();
    return check(drv().cuEventDestroy(reinterpret_cast<CUevent>(event)), "cuEventDestroy");
}

int ert_status(uint64_t module, uint32_t *code, uint64_t stream) {
    ERT_NEED_DRIVER();
    if (!module || !code) return fail(ERT_E_ARGUMENT, "null argument");
    *code = 0;
    int rc;
    if ((rc = need_ctx())) return rc;
    CUdeviceptr p = 0;
    size_t n = 0;
    CUresult r = drv().cuModuleGetGlobal(&p, &n, reinterpret_cast<CUmodule>(module), "emmy_status");
    if (r == CUDA_ERROR_NOT_FOUND) return 0;
    if ((rc = check(r, "cuModuleGetGlobal(emmy_status)"))) return rc;
    if (n < 4) return 0;
    CUstream s = reinterpret_cast<CUstream>(stream);
    uint32_t value = 0, zero = 0;
    if ((rc = check(drv().cuStreamSynchronize(s), "cuStreamSynchronize"))) return rc;
    if ((rc = check(drv().cuMemcpyDtoHAsync(&value, p, 4, s), "cuMemcpyDtoHAsync"))) return rc;
    if ((rc = check(drv().cuStreamSynchronize(s), "cuStreamSynchronize"))) return rc;
    if (value) {
        if ((rc = check(drv().cuMemcpyHtoDAsync(p, &zero, 4, s), "cuMemcpyHtoDAsync"))) return rc;
        if ((rc = check(drv().cuStreamSynchronize(s), "cuStreamSynchronize"))) return rc;
    }
    *code = value;
    return 0;
}

}  // extern "C"
