// Exchange buffers shared with the other processes of a node, and the
// copy-engine transfer that feeds the gated int8 GEMM (no reference
// counterpart: the reference's DTensor gathers shards through host memory,
// python/kansai/distributed.py:157-176).
//
// A rank allocates its buffers with cudaMalloc and exports CUDA IPC handles;
// the other ranks map them (peer access over NVLink).  No multicast object is
// ever created.  kz_copy_and_flag pulls a block from a peer with
// cudaMemcpyAsync and then publishes a token into a local flag with a stream
// memory operation (cuStreamWriteValue32, issued by the GPU's front end after
// the copy; where the driver does not offer it, a 4-byte copy from a pinned
// host table): neither uses an SM, so the transfer proceeds while a kernel
// that holds every SM (the persistent GEMM) waits on the flag.
#include <cuda.h>

#include <mutex>

#include "kz_common.cuh"

namespace kz {
namespace {

constexpr uint32_t kTokens = 65536;
std::once_flag g_tokens_once;
uint32_t* g_tokens = nullptr;   // pinned host: g_tokens[i] == i, never modified

int tokens_ready() {
    cudaError_t err = cudaSuccess;
    std::call_once(g_tokens_once, [&] {
        void* p = nullptr;
        err = cudaHostAlloc(&p, kTokens * sizeof(uint32_t), cudaHostAllocPortable);
        if (err == cudaSuccess) {
            uint32_t* t = static_cast<uint32_t*>(p);
            for (uint32_t i = 0; i < kTokens; ++i) t[i] = i;
            g_tokens = t;
        }
    });
    if (!g_tokens) return cuda_error(err == cudaSuccess ? cudaErrorMemoryAllocation : err, "pinned token table");
    return KZ_OK;
}

using WriteValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

WriteValue32Fn write_value_fn() {
    static std::once_flag once;
    static WriteValue32Fn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<WriteValue32Fn>(p);
    });
    return fn;
}

}  // namespace
}  // namespace kz

using namespace kz;

static_assert(sizeof(cudaIpcMemHandle_t) == KZ_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int kz_peer_alloc(size_t bytes, void** ptr, void* handle_out) {
    KZ_REQUIRE(ptr && handle_out, "kz_peer_alloc: ptr and handle_out must be non-NULL");
    KZ_REQUIRE(bytes > 0, "kz_peer_alloc: bytes must be > 0");
    int st = check_device();
    if (st) return st;
    void* p = nullptr;
    KZ_CHECK_CUDA(cudaMalloc(&p, bytes));
    cudaError_t zerr = cudaMemset(p, 0, bytes);
    if (zerr != cudaSuccess) {
        cudaFree(p);
        return cuda_error(zerr, "cudaMemset");
    }
    cudaIpcMemHandle_t h;
    cudaError_t err = cudaIpcGetMemHandle(&h, p);
    if (err != cudaSuccess) {
        cudaFree(p);
        return cuda_error(err, "cudaIpcGetMemHandle");
    }
    memcpy(handle_out, &h, sizeof(h));
    *ptr = p;
    return KZ_OK;
}

extern "C" int kz_peer_open(const void* handle, void** ptr) {
    KZ_REQUIRE(handle && ptr, "kz_peer_open: handle and ptr must be non-NULL");
    int st = check_device();
    if (st) return st;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    KZ_CHECK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = p;
    return KZ_OK;
}

extern "C" int kz_peer_close(void* ptr) {
    KZ_REQUIRE(ptr, "kz_peer_close: ptr is NULL");
    KZ_CHECK_CUDA(cudaIpcCloseMemHandle(ptr));
    return KZ_OK;
}

extern "C" int kz_peer_free(void* ptr) {
    KZ_REQUIRE(ptr, "kz_peer_free: ptr is NULL");
    KZ_CHECK_CUDA(cudaFree(ptr));
    return KZ_OK;
}

extern "C" int kz_copy_and_flag(void* dst, const void* src, size_t bytes, uint32_t* flag, uint32_t token,
                                kz_stream_t stream) {
    KZ_REQUIRE(flag, "kz_copy_and_flag: flag is NULL");
    KZ_REQUIRE(bytes == 0 || (dst && src), "kz_copy_and_flag: dst or src is NULL");
    KZ_REQUIRE(token < kTokens, "kz_copy_and_flag: token must be < 65536");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (bytes) KZ_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s));
    // default flags: the write is ordered after the copy and its data
    if (WriteValue32Fn fn = write_value_fn()) {
        if (fn(reinterpret_cast<CUstream>(s), reinterpret_cast<CUdeviceptr>(flag), token, 0) == CUDA_SUCCESS)
            return KZ_OK;
    }
    int st = tokens_ready();
    if (st) return st;
    KZ_CHECK_CUDA(cudaMemcpyAsync(flag, g_tokens + token, sizeof(uint32_t), cudaMemcpyHostToDevice, s));
    return KZ_OK;
}
