// vxc_runtime.cu — device selection, error reporting.
#include "vxc_common.cuh"
#include "vxc_internal.h"

#include <stdarg.h>
#include <stdio.h>

#include <atomic>

static thread_local char t_err[512] = "";
static unsigned int *g_err_ptr[64];   // per device

static std::atomic<long long> g_launches{0};

void vxc_count_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

extern "C" long long vxc_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

void vxc_set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof t_err, fmt, ap);
    va_end(ap);
}

extern "C" const char *vxc_error_string(void) { return t_err; }

extern "C" int vxc_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

int vxc_require_device(void) {
    int dev = -1;
    if (vxc_device_count() <= 0 || cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        vxc_set_error("no CUDA device available (the B200 back end has no CPU fallback)");
        return -7;
    }
    if (dev < 0 || dev >= 64) return -7;
    if (!g_err_ptr[dev]) {
        unsigned int *p = NULL;
        if (cudaMalloc((void **)&p, sizeof(unsigned int)) != cudaSuccess ||
            cudaMemset(p, 0, sizeof(unsigned int)) != cudaSuccess) {
            vxc_set_error("cannot allocate the device error word");
            return -3;
        }
        g_err_ptr[dev] = p;
    }
    return 0;
}

unsigned int *vxc_device_error_ptr(void) {
    int dev = 0;
    cudaGetDevice(&dev);
    return (dev >= 0 && dev < 64) ? g_err_ptr[dev] : NULL;
}

extern "C" int vxc_device_init(int device) {
    if (vxc_device_count() <= 0) {
        vxc_set_error("no CUDA device available (the B200 back end has no CPU fallback)");
        return -7;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        vxc_set_error("cudaSetDevice(%d) failed", device);
        return -7;
    }
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, device);
    if (p.major < 10) {
        vxc_set_error("device %d is sm_%d%d; this library is built for sm_100a", device, p.major, p.minor);
        return -7;
    }
    return vxc_require_device();
}

extern "C" int vxc_check_device_error(unsigned int *code_out) {
    int rc = vxc_require_device();
    if (rc) return rc;
    unsigned int h = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&h, vxc_device_error_ptr(), sizeof h, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(vxc_device_error_ptr(), 0, sizeof h);
    if (e != cudaSuccess) { vxc_set_error("vxc_check_device_error: %s", cudaGetErrorString(e)); return -3; }
    if (code_out) *code_out = h;
    return h ? -3 : 0;
}

extern "C" int vxc_device_current(void) {
    int d = -1;
    if (vxc_device_count() <= 0 || cudaGetDevice(&d) != cudaSuccess) { cudaGetLastError(); return -1; }
    return d;
}

// The driver's current-context handle, reached through the runtime's entry
// point table (the library links only the static runtime, not libcuda).
typedef int (*cu_ctx_get_current_t)(void **);

void *vxc_current_context(void) {
    static std::atomic<cu_ctx_get_current_t> fn{nullptr};
    cu_ctx_get_current_t f = fn.load(std::memory_order_acquire);
    if (!f) {
        void *p = NULL;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !p) {
            cudaGetLastError();
            return NULL;
        }
        f = (cu_ctx_get_current_t)p;
        fn.store(f, std::memory_order_release);
    }
    void *ctx = NULL;
    return f(&ctx) == 0 ? ctx : NULL;
}
