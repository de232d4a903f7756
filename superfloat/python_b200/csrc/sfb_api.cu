// Library-level entry points of libsfb200: version, errors, device checks.
#include <cuda.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "sfb_common.cuh"

namespace sfb {

static thread_local char g_msg[512] = "";

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof g_msg, fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(SFB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return SFB_OK;
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

unsigned long long context_id() {
    typedef CUresult (*GetCurrent)(CUcontext *);
    typedef CUresult (*GetId)(CUcontext, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

}  // namespace sfb

extern "C" int sfb_abi_version(void) { return SFB_ABI_VERSION; }

extern "C" const char *sfb_last_error(void) { return sfb::g_msg; }

extern "C" int sfb_device_init(int device) {
    using namespace sfb;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return set_error(SFB_ENODEV, "sfb_device_init: no CUDA device (%s)", cudaGetErrorString(e));
    if (device < 0 || device >= n) return set_error(SFB_EINVAL, "sfb_device_init: device %d of %d", device, n);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return set_error(SFB_ECUDA, "sfb_device_init: %s", cudaGetErrorString(e));
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0)
        return set_error(SFB_ENODEV, "sfb_device_init: device %d is sm_%d%d; this library is built for sm_100a",
                         device, major, minor);
    return SFB_OK;
}
