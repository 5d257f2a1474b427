// abi.cu — C-ABI plumbing shared by every module: thread-local error messages, the device status
// registry, the SM count.
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace rk {
namespace {
thread_local char g_last_error[512] = {0};
std::mutex g_status_mu;
std::vector<StatusReader>& status_readers() {
    static std::vector<StatusReader> v;
    return v;
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_last_error[0] = 0; }

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return RK_OK;
}

void register_status_reader(StatusReader r) {
    std::lock_guard<std::mutex> lk(g_status_mu);
    status_readers().push_back(r);
}

static int env_int(const char* name) {
    const char* v = std::getenv(name);
    return v ? std::atoi(v) : 0;
}
int mmvq_env_stages() {
    static const int v = env_int("RK_MMVQ_STAGES");
    return v;
}
int mmvq_env_ctas() {
    static const int v = env_int("RK_MMVQ_CTAS");
    return v;
}
int mmvq_env_warps() {
    static const int v = env_int("RK_MMVQ_WARPS");
    return v;
}
int mmvq_env_pair() {
    static const int v = env_int("RK_MMVQ_PAIR");
    return v;
}

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
    }
    return n;
}

}  // namespace rk

extern "C" {

const char* rk_last_error(void) { return rk::g_last_error; }

int rk_version(void) { return (0 << 16) | 1; }

unsigned rk_device_status(int clear) {
    std::lock_guard<std::mutex> lk(rk::g_status_mu);
    if (cudaDeviceSynchronize() != cudaSuccess) return 0x80000000u;
    unsigned v = 0;
    for (rk::StatusReader r : rk::status_readers()) v |= r(clear != 0);
    return v;
}

}  // extern "C"
