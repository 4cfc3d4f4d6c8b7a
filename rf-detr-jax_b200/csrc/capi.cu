// Library-level entry points: status text, ABI version, tuning knobs and the per-device SM
// count cache.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace rfdetr {
namespace {

const char *const kKnobNames[kKnobCount] = {
    "RFDETR_MSDA_FWD",      "RFDETR_MSDA_BWD",      "RFDETR_MSDA_SLAB_FWD", "RFDETR_MSDA_BINS",
    "RFDETR_MSDA_OWN",      "RFDETR_MSDA_TILES",    "RFDETR_MSDA_CELL",     "RFDETR_LSAP_STAGE_KB",
    "RFDETR_LSAP_STEP_CAP", "RFDETR_TOPK_SORT",     "RFDETR_TOPK_UNSTAGED"};

struct AtomicKnob {
    std::atomic<int> count{0};
    std::atomic<int> v[5];
};
AtomicKnob g_knobs[kKnobCount];
std::once_flag g_knobs_from_env;

// Parses "a,b,c,d,e" (1 to 5 integers); returns how many, or -1 when the text is not that.
int parse_knob(const char *text, int out[5]) {
    if (!text || !*text) return 0;
    int n = 0;
    const char *p = text;
    while (n < 5) {
        char *end = nullptr;
        const long x = std::strtol(p, &end, 10);
        if (end == p) return -1;
        out[n++] = (int)x;
        if (*end == 0) return n;
        if (*end != ',') return -1;
        p = end + 1;
    }
    return -1;
}

void store_knob(int k, const int *v, int n) {
    for (int i = 0; i < 5; ++i) g_knobs[k].v[i].store(i < n ? v[i] : 0, std::memory_order_relaxed);
    g_knobs[k].count.store(n, std::memory_order_release);
}

void knobs_from_env() {
    for (int k = 0; k < kKnobCount; ++k) {
        int v[5];
        const int n = parse_knob(std::getenv(kKnobNames[k]), v);
        store_knob(k, v, n > 0 ? n : 0);
    }
}

}  // namespace

KnobValue knob(Knob k) {
    std::call_once(g_knobs_from_env, knobs_from_env);
    KnobValue r;
    r.count = g_knobs[k].count.load(std::memory_order_acquire);
    for (int i = 0; i < 5; ++i) r.v[i] = g_knobs[k].v[i].load(std::memory_order_relaxed);
    return r;
}

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

extern "C" int rfdetr_abi_version(void) { return 3; }

extern "C" int rfdetr_set_tuning(const char *name, const char *value) {
    using namespace rfdetr;
    (void)knob(kKnobMsdaFwd);  // the environment is read first, so it cannot override this call
    if (!name) return RFDETR_ERR_SHAPE;
    for (int k = 0; k < kKnobCount; ++k) {
        if (std::strcmp(name, kKnobNames[k]) != 0) continue;
        int v[5];
        const int n = parse_knob(value, v);
        if (n < 0) return RFDETR_ERR_SHAPE;
        store_knob(k, v, n);
        return RFDETR_OK;
    }
    return RFDETR_ERR_SHAPE;
}
