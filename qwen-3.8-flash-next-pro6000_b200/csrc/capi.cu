// C-ABI plumbing shared by all entry points: thread-local error text, status conversion, device attribute cache.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "qf_common.cuh"

namespace qf {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return QF_OK;
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return QF_ERR_CUDA;
}

int sm_count(int device) {
    static std::mutex mu;
    static int cache[64] = {0};
    if (device < 0 || device >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[device] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
        cache[device] = n;
    }
    return cache[device];
}

cudaError_t ensure_smem_attr(const void* func, int bytes) {
    static std::mutex mu;
    static const void* funcs[256];
    static int devs[256];
    static int n = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n; ++i)
        if (funcs[i] == func && devs[i] == dev) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && n < 256) {
        funcs[n] = func;
        devs[n] = dev;
        ++n;
    }
    return e;
}

}  // namespace qf

extern "C" const char* qf_last_error(void) { return qf::g_err; }

extern "C" int qf_version(void) { return 1; }
