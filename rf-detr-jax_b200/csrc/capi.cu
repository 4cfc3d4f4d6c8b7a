// Library-level entry points: status text, ABI version and the per-device SM count cache.
#include <mutex>

#include "common.cuh"

namespace rfdetr {

int num_sms() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cache[dev] = v;
    }
    return cache[dev];
}

}  // namespace rfdetr

extern "C" const char *rfdetr_status_string(int status) {
    switch (status) {
        case RFDETR_OK: return "ok";
        case RFDETR_ERR_SHAPE: return "inconsistent or unsupported sizes";
        case RFDETR_ERR_DTYPE: return "unsupported element type";
        case RFDETR_ERR_ALIGN: return "pointer not aligned to its element type";
        case RFDETR_ERR_WORKSPACE: return "workspace missing or too small";
        case RFDETR_ERR_CUDA: return "CUDA runtime error";
        case RFDETR_ERR_LIMIT: return "device loop reached its iteration cap";
        case RFDETR_ERR_CAPACITY: return "problem exceeds the no-alloc entry point's static scratch (8 MiB)";
        default: return "unknown status";
    }
}

extern "C" int rfdetr_abi_version(void) { return 1; }
