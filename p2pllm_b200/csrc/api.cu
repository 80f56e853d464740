// Error reporting and device queries shared by every entry point.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace p2p {

static thread_local char g_error[1024] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
    return code;
}

int launch_status(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(P2P_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return P2P_OK;
}

int allow_smem(const void* kernel, int bytes, const char* what) {
    if (bytes <= 48 * 1024) return P2P_OK;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return fail(P2P_ECUDA, "%s: %d bytes of shared memory: %s", what, bytes, cudaGetErrorString(e));
    return P2P_OK;
}

int sm_count() {
    static int counts[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (counts[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        counts[dev] = n;
    }
    return counts[dev];
}

}  // namespace p2p

extern "C" const char* p2p_last_error(void) { return p2p::g_error; }
extern "C" int p2p_abi_version(void) { return 1; }
