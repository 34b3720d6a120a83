// Host-side error reporting and the device status word helpers shared by all entry points.
#include <cstdarg>
#include <cstdio>

#include "sa_common.cuh"

namespace sa {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return SA_OK;
}

int num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int current_device_context(const char* who, int* dev, void** ctx) {
    typedef int (*CtxGetCurrent)(void**);
    static CtxGetCurrent get_ctx = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_ctx = reinterpret_cast<CtxGetCurrent>(fn);
    });
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: cudaGetDevice: %s", who, cudaGetErrorString(e));
    if (*dev < 0 || *dev >= SA_MAX_DEVICES) return fail(SA_ERR_UNSUPPORTED, "%s: device %d", who, *dev);
    *ctx = nullptr;
    if (!get_ctx) return fail(SA_ERR_CUDA, "%s: cuCtxGetCurrent unavailable", who);
    if (get_ctx(ctx) == 0 && *ctx) return SA_OK;
    // no context bound to this thread yet: cudaSetDevice makes the device's primary context current
    if ((e = cudaSetDevice(*dev)) != cudaSuccess)
        return fail(SA_ERR_CUDA, "%s: cudaSetDevice: %s", who, cudaGetErrorString(e));
    if (get_ctx(ctx) != 0 || !*ctx) return fail(SA_ERR_CUDA, "%s: no current CUDA context", who);
    return SA_OK;
}

}  // namespace sa

extern "C" int sa_version(void) { return 1; }

extern "C" const char* sa_last_error(void) { return sa::g_err; }

extern "C" int sa_read_status(int32_t* status, int32_t* value, void* stream) {
    if (!status || !value) return sa::fail(SA_ERR_ARG, "sa_read_status: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int32_t host = 0;
    cudaError_t e = cudaMemcpyAsync(&host, status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = cudaMemsetAsync(status, 0, sizeof(int32_t), s);
    if (e != cudaSuccess) return sa::fail(SA_ERR_CUDA, "sa_read_status: %s", cudaGetErrorString(e));
    *value = host;
    return SA_OK;
}
