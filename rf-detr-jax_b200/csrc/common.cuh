// Shared device helpers for the sm_100a kernels: element conversion, vector loads/stores and
// launch error plumbing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "rfdetr_b200.h"

namespace rfdetr {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(bf16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ bf16 from_f32<bf16>(float x) { return __float2bfloat16_rn(x); }

// Raw storage of a vector of BYTES bytes.
template <int BYTES> struct Raw;
template <> struct Raw<16> { using T = uint4; };
template <> struct Raw<8> { using T = uint2; };
template <> struct Raw<4> { using T = unsigned int; };
template <> struct Raw<2> { using T = unsigned short; };

// Loads VEC elements of T starting at p (aligned to min(16, VEC*sizeof(T)) bytes) and widens
// them to float.  NC selects the read-only (non-coherent) global path; otherwise a generic load
// (shared or global).  Vectors wider than 16 bytes are split into 16-byte pieces.
template <typename T, int VEC, bool NC>
__device__ __forceinline__ void load_vec(const T *p, float *f) {
    if constexpr (VEC * sizeof(T) > 16) {
        constexpr int HALF = VEC / 2;
        load_vec<T, HALF, NC>(p, f);
        load_vec<T, HALF, NC>(p + HALF, f + HALF);
    } else {
        using R = typename Raw<VEC * (int)sizeof(T)>::T;
        R r;
        if constexpr (NC) {
            r = __ldg(reinterpret_cast<const R *>(p));
        } else {
            r = *reinterpret_cast<const R *>(p);
        }
        const T *e = reinterpret_cast<const T *>(&r);
#pragma unroll
        for (int i = 0; i < VEC; ++i) f[i] = to_f32(e[i]);
    }
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T *p, const float *f) {
    if constexpr (VEC * sizeof(T) > 16) {
        constexpr int HALF = VEC / 2;
        store_vec<T, HALF>(p, f);
        store_vec<T, HALF>(p + HALF, f + HALF);
    } else {
        using R = typename Raw<VEC * (int)sizeof(T)>::T;
        R r;
        T *e = reinterpret_cast<T *>(&r);
#pragma unroll
        for (int i = 0; i < VEC; ++i) e[i] = from_f32<T>(f[i]);
        *reinterpret_cast<R *>(p) = r;
    }
}

// Fire-and-forget float adds into global memory, vectorised where the PTX ISA allows it
// (red.global.add.v4/v2.f32, sm_90+).  p must be aligned to the vector width.
template <int VEC>
__device__ __forceinline__ void red_add_global(float *p, const float *f) {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
        for (int i = 0; i < VEC; i += 4) {
            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p + i), "f"(f[i]),
                         "f"(f[i + 1]), "f"(f[i + 2]), "f"(f[i + 3])
                         : "memory");
        }
    } else if constexpr (VEC == 2) {
        asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(f[0]), "f"(f[1]) : "memory");
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) atomicAdd(p + i, f[i]);
    }
}

__host__ __device__ inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

inline bool aligned(const void *p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

inline int dtype_size(int dtype) { return dtype == RFDETR_F32 ? 4 : (dtype == RFDETR_BF16 ? 2 : 0); }

// Maps the last CUDA error (launch configuration or asynchronous) to a status.
inline int launch_status() {
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? RFDETR_OK : RFDETR_ERR_CUDA;
}

int num_sms();  // SM count of the current device (cached per device)

// Process-wide tuning knobs, for experiments and tests.  A knob holds up to five integers, set
// from the environment variable of the knob's name ("a,b,c,d,e"; read once, the first time any
// knob is read) or by rfdetr_set_tuning(); `count` is how many were given (0: not set, the
// launchers use their own defaults).  Launchers read a knob per call from atomics: no getenv,
// no lock.
enum Knob {
    kKnobMsdaFwd,       // "RFDETR_MSDA_FWD": generic sampler forward "hsub,stage,acc,threads,waves"
    kKnobMsdaBwd,       // "RFDETR_MSDA_BWD": generic sampler backward, same fields
    kKnobMsdaSlabFwd,   // "RFDETR_MSDA_SLAB_FWD": slab forward (hsub, stage = 0 disables, ..., waves)
    kKnobMsdaBins,      // "RFDETR_MSDA_BINS": capped-bin backward (stage = 0 disables)
    kKnobMsdaOwn,       // "RFDETR_MSDA_OWN": owner backward (hsub = bin cap, stage = 0 disables, acc = 0 no TMA, threads = tile)
    kKnobMsdaTiles,     // "RFDETR_MSDA_TILES": tile backward, opt-in (hsub = bin cap, stage = 1 enables, acc = 0 never stages, threads = per CTA)
    kKnobMsdaCell,      // "RFDETR_MSDA_CELL": cell-owner backward (stage = 0 disables)
    kKnobLsapStageKb,   // "RFDETR_LSAP_STAGE_KB": shared-memory cost stage budget of the solver, KiB
    kKnobLsapStepCap,   // "RFDETR_LSAP_STEP_CAP": scan steps an augmenting path may take (default: the column count)
    kKnobTopkSort,      // "RFDETR_TOPK_SORT": any value selects the one-CTA sort kernels
    kKnobTopkUnstaged,  // "RFDETR_TOPK_UNSTAGED": any value keeps the radix select's keys out of shared memory
    kKnobCount
};
struct KnobValue {
    int count;
    int v[5];
};
KnobValue knob(Knob k);

}  // namespace rfdetr
