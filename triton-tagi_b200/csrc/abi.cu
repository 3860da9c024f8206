// Library identification and per-thread error reporting for the C ABI.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace tagi {

static thread_local char g_last_error[512] = "";
static unsigned long long g_launches = 0;  // kernels launched through this library

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

int check_launch(const char* what) {
    __atomic_fetch_add(&g_launches, 1ull, __ATOMIC_RELAXED);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: %s", what, cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    return TAGI_OK;
}

}  // namespace tagi

extern "C" int tagi_version(void) { return (0 << 16) | (1 << 8) | 0; }

extern "C" const char* tagi_last_error(void) { return tagi::g_last_error; }

extern "C" uint64_t tagi_kernel_launches(void) {
    return __atomic_load_n(&tagi::g_launches, __ATOMIC_RELAXED);
}

extern "C" int tagi_device_arch(int device) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
        cudaGetLastError();
        tagi::set_error("tagi_device_arch: cannot query device %d", device);
        return TAGI_E_BAD_ARG;
    }
    return major * 10 + minor;
}
