// runtime.cu - host-side plumbing of the C ABI: last-error text, version,
// dtype sizes, SM-count cache and tensor-descriptor validation.
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace tadma_b200 {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return TADMA_ERR_CUDA;
}

cudaError_t workspace_alloc(void** p, size_t bytes, cudaStream_t s) {
    const char* inject = std::getenv("TADMA_B200_FAIL_ALLOC");
    if (inject && inject[0] == '1') {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMallocAsync(p, bytes, s);
}

int sm_count() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int64_t numel(const tadma_tensor* t) {
    int64_t n = 1;
    for (int d = 0; d < t->rank; d++) n *= t->dims[d];
    return n;
}

std::string check_tensor(const tadma_tensor* t, const char* name, bool need_data) {
    if (!t) return std::string(name) + " is NULL";
    if (t->rank < 0 || t->rank > TADMA_MAX_RANK) return std::string(name) + ": rank out of range [0, 8]";
    if (dtype_size(t->dtype) == 0) return std::string(name) + ": unknown dtype";
    for (int d = 0; d < t->rank; d++)
        if (t->dims[d] < 0) return std::string(name) + ": negative dimension";
    if (need_data && !t->data && numel(t) > 0) return std::string(name) + ": data is NULL";
    return "";
}

}  // namespace tadma_b200

using namespace tadma_b200;

extern "C" const char* tadma_b200_last_error(void) { return g_last_error.c_str(); }

extern "C" const char* tadma_b200_version(void) { return "tadma_b200 0.1.0 (sm_100a)"; }

extern "C" int32_t tadma_b200_dtype_size(int32_t dtype) { return dtype_size(dtype); }
