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

// One CTA waits, with the bounded wait every kernel here uses, for a phase of an mbarrier that
// nothing completes (count 1, no arrival): each thread gives up after limit_ns, the CTA's abort
// flag is raised and SA_DEV_WAIT_TEST is or-ed into the status word once.
__global__ void wait_selftest_kernel(int* status, unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ volatile int abort_word;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_word = 0;
        fence_mbar_init();
    }
    __syncthreads();
    mbar_wait_limit(smem_u32(&bar), 0, &abort_word, status, SA_DEV_WAIT_TEST, limit_ns);
}

}  // namespace sa

extern "C" int sa_version(void) { return 1; }

extern "C" int sa_wait_selftest(int32_t* status, int64_t limit_ns, void* stream) {
    if (!status) return sa::fail(SA_ERR_ARG, "sa_wait_selftest: null status word");
    if (limit_ns < 1000 || limit_ns > static_cast<int64_t>(SA_WAIT_TIMEOUT_NS))
        return sa::fail(SA_ERR_ARG, "sa_wait_selftest: limit %lld ns outside [1000, %llu]",
                        static_cast<long long>(limit_ns), static_cast<unsigned long long>(SA_WAIT_TIMEOUT_NS));
    sa::wait_selftest_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        status, static_cast<unsigned long long>(limit_ns));
    return sa::check_launch("sa_wait_selftest");
}

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
