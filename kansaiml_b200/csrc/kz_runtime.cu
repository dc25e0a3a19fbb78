// Host-side runtime of libkz: error messages, the per-device sticky status
// word, device checks and the reference-compatible host RNG.
#include <mutex>
#include <random>
#include <string>

#include "kz_common.cuh"

namespace kz {

namespace {
thread_local std::string t_last_error;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_status_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
int g_supported[kMaxDevices] = {};  // 0 unknown, 1 yes, -1 no
}  // namespace

// One status word per device; host code reaches it only through
// cudaGetSymbolAddress (the symbol itself is a host-side stand-in).
__device__ int g_device_status_word;

int set_error(int code, const std::string& msg) {
    t_last_error = msg;
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    // consume the runtime's per-thread last error: a failed non-sticky call
    // (a bad argument) must not surface again at the next launch check
    (void)cudaGetLastError();
    return set_error(KZ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + ": " + cudaGetErrorString(e));
}

static int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (*dev < 0 || *dev >= kMaxDevices) return set_error(KZ_ERR_UNSUPPORTED_DEVICE, "device ordinal out of range");
    return KZ_OK;
}

int* device_status_ptr() {
    int dev;
    if (current_device(&dev) != KZ_OK) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_status_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status_word) != cudaSuccess) return nullptr;
        g_status_ptr[dev] = static_cast<int*>(p);
    }
    return g_status_ptr[dev];
}

int sm_count() {
    int dev;
    if (current_device(&dev) != KZ_OK) return 148;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_sm_count[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

int check_device() {
    int dev;
    int st = current_device(&dev);
    if (st != KZ_OK) return st;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (g_supported[dev] == 1) return KZ_OK;
    }
    int major = 0, minor = 0;
    KZ_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    KZ_CHECK_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    std::lock_guard<std::mutex> lk(g_mu);
    g_supported[dev] = (major == 10 && minor == 0) ? 1 : -1;
    if (g_supported[dev] != 1)
        return set_error(KZ_ERR_UNSUPPORTED_DEVICE, "libkz is built for sm_100a (B200); device " + std::to_string(dev) +
                                                        " is sm_" + std::to_string(major) + std::to_string(minor));
    return KZ_OK;
}

}  // namespace kz

extern "C" {

const char* kz_last_error(void) { return kz::t_last_error.c_str(); }

int kz_version(void) { return 1; }

int kz_device_supported(int device) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return 0;
    return (major == 10 && minor == 0) ? 1 : 0;
}

int kz_randn_host(float* out, int64_t n, float stddev, uint64_t seed) {
    KZ_REQUIRE(n >= 0, "kz_randn_host: n must be >= 0");
    KZ_REQUIRE(n == 0 || out != nullptr, "kz_randn_host: out is NULL");
    std::mt19937 rng(seed ? static_cast<std::mt19937::result_type>(seed) : std::random_device{}());
    std::normal_distribution<float> dist(0.0f, stddev);
    for (int64_t i = 0; i < n; ++i) out[i] = dist(rng);
    return KZ_OK;
}

int kz_device_status(int* code, int clear, kz_stream_t stream) {
    KZ_REQUIRE(code != nullptr, "kz_device_status: code is NULL");
    int* p = kz::device_status_ptr();
    if (!p) return kz::set_error(KZ_ERR_CUDA, "kz_device_status: cannot resolve the device status word");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int host = 0;
    KZ_CHECK_CUDA(cudaMemcpyAsync(&host, p, sizeof(int), cudaMemcpyDeviceToHost, s));
    KZ_CHECK_CUDA(cudaStreamSynchronize(s));
    if (clear && host != 0) {
        KZ_CHECK_CUDA(cudaMemsetAsync(p, 0, sizeof(int), s));
        KZ_CHECK_CUDA(cudaStreamSynchronize(s));
    }
    *code = host;
    return KZ_OK;
}

}  // extern "C"
