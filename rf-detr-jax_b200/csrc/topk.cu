// Two-stage query selection for sm_100a: class max + top-k, and the row gather after it.
//
// Reference semantics (src/rfdetr_jax/models/transformer.py:694-706):
//   proposal_scores = logits.max(-1); _, idx = jax.lax.top_k(proposal_scores, k)
//   select_rows(projected, idx)            (src/rfdetr_jax/models/layers.py:225-244)
// jax.lax.top_k returns the k largest in descending order, the lower index first among equal
// values; floats compare in IEEE totalOrder (NaN above +inf).
//
// One CTA per row: each warp reduces the classes of a few positions at once (coalesced along
// the class axis), the CTA packs (totalOrder(score), ~position) into 64-bit keys in shared
// memory, and a bitonic network sorts them descending; the first k keys give the answer.
#include <algorithm>

#include "common.cuh"

namespace rfdetr {
namespace {

constexpr int kTopkThreads = 512;
constexpr int kTopkMaxPositions = 16384;

__device__ __forceinline__ unsigned order_key(float x) {
    const unsigned b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// max that propagates NaN, as jnp.max does.
__device__ __forceinline__ float nan_max(float m, float x) { return (x > m || x != x) ? x : m; }

__global__ void __launch_bounds__(kTopkThreads)
topk_kernel(const float *__restrict__ logits, int N, int C, int k, int P2, float *__restrict__ scores_out,
            float *__restrict__ values_out, int32_t *__restrict__ idx_out) {
    extern __shared__ unsigned long long keys[];
    const int r = blockIdx.x;
    const float *rowp = logits + (size_t)r * N * C;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int nwarps = kTopkThreads / 32;
    constexpr int U = 4;  // positions per warp step: independent load chains in flight

    for (int p0 = warp * U; p0 < N; p0 += nwarps * U) {
        float m[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            m[u] = -INFINITY;
            const int p = p0 + u;
            if (p < N) {
                const float *x = rowp + (size_t)p * C;
                for (int c = lane; c < C; c += 32) m[u] = nan_max(m[u], __ldg(x + c));
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m[u] = nan_max(m[u], __shfl_xor_sync(0xffffffffu, m[u], o));
        }
        if (lane < U && p0 + lane < N) {
            float s = m[0];
#pragma unroll
            for (int u = 1; u < U; ++u) s = (lane == u) ? m[u] : s;
            if (s != s) s = __uint_as_float(0x7fc00000u);  // canonical (positive) NaN sorts first
            const int p = p0 + lane;
            keys[p] = ((unsigned long long)order_key(s) << 32) | (unsigned long long)(0xffffffffu - (unsigned)p);
            if (scores_out) scores_out[(size_t)r * N + p] = s;
        }
    }
    for (int p = N + threadIdx.x; p < P2; p += kTopkThreads) keys[p] = 0ull;  // below every real key
    __syncthreads();

    // Bitonic sort, descending.
    for (int size = 2; size <= P2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (P2 >> 1); i += kTopkThreads) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const unsigned long long a = keys[lo], b = keys[hi];
                if ((a < b) == desc) {
                    keys[lo] = b;
                    keys[hi] = a;
                }
            }
            __syncthreads();
        }
    }

    for (int i = threadIdx.x; i < k; i += kTopkThreads) {
        const unsigned long long key = keys[i];
        const int p = (int)(0xffffffffu - (unsigned)(key & 0xffffffffull));
        idx_out[(size_t)r * k + i] = p;
        if (values_out) values_out[(size_t)r * k + i] = key_to_float((unsigned)(key >> 32));
    }
}

template <typename V>
__global__ void select_rows_kernel(const V *__restrict__ values, long long row_vecs, int N,
                                   const int32_t *__restrict__ idx, int K, V *__restrict__ out,
                                   long long out_rows, int32_t *status) {
    for (long long o = blockIdx.x; o < out_rows; o += gridDim.x) {
        const long long r = o / K;
        const int src = __ldg(idx + o);
        V *dst = out + o * row_vecs;
        if (src < 0 || src >= N) {
            for (long long c = threadIdx.x; c < row_vecs; c += blockDim.x) dst[c] = V{};
            if (threadIdx.x == 0 && status) atomicExch(status, (int)RFDETR_ERR_SHAPE);
            continue;
        }
        const V *s = values + (r * N + src) * row_vecs;
        for (long long c = threadIdx.x; c < row_vecs; c += blockDim.x) dst[c] = __ldg(s + c);
    }
}

int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

template <typename V>
int launch_select(const void *values, long long row_bytes, int N, const int32_t *idx, int K, void *out,
                  long long out_rows, int32_t *status, cudaStream_t s) {
    const long long row_vecs = row_bytes / (long long)sizeof(V);
    const int threads = (int)std::min<long long>(256, std::max<long long>(32, ((row_vecs + 31) / 32) * 32));
    const long long blocks = std::min<long long>(out_rows, 65535LL * 32);
    select_rows_kernel<V><<<(unsigned)blocks, threads, 0, s>>>(static_cast<const V *>(values), row_vecs, N, idx,
                                                               K, static_cast<V *>(out), out_rows, status);
    return launch_status();
}

}  // namespace
}  // namespace rfdetr

using namespace rfdetr;

extern "C" int rfdetr_topk_select(void *stream, const float *logits, int64_t rows, int64_t positions,
                                  int64_t classes, int64_t k, float *scores_out, float *values_out,
                                  int32_t *indices_out) {
    if (rows < 0 || positions <= 0 || classes <= 0 || k <= 0 || k > positions ||
        positions > kTopkMaxPositions || rows > 2147483647LL || positions * classes > (1LL << 31))
        return RFDETR_ERR_SHAPE;
    if (rows == 0) return RFDETR_OK;
    if (!logits || !indices_out) return RFDETR_ERR_SHAPE;
    if (!aligned(logits, 4) || !aligned(indices_out, 4) || (scores_out && !aligned(scores_out, 4)) ||
        (values_out && !aligned(values_out, 4)))
        return RFDETR_ERR_ALIGN;
    const int P2 = next_pow2((int)positions);
    const size_t smem = (size_t)P2 * sizeof(unsigned long long);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    topk_kernel<<<(unsigned)rows, kTopkThreads, smem, static_cast<cudaStream_t>(stream)>>>(
        logits, (int)positions, (int)classes, (int)k, P2, scores_out, values_out, indices_out);
    return launch_status();
}

extern "C" int rfdetr_select_rows(void *stream, const void *values, int64_t element_bytes, int64_t rows,
                                  int64_t positions, int64_t width, const int32_t *indices, int64_t k,
                                  void *out, int32_t *status_out) {
    if (element_bytes <= 0 || rows < 0 || positions <= 0 || width < 0 || k < 0 || positions > 2147483647LL ||
        k > 2147483647LL)
        return RFDETR_ERR_SHAPE;
    const long long row_bytes = element_bytes * width;
    const long long out_rows = rows * k;
    if (out_rows == 0 || row_bytes == 0) return RFDETR_OK;
    if (!values || !indices || !out) return RFDETR_ERR_SHAPE;
    if (!aligned(indices, 4)) return RFDETR_ERR_ALIGN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto fits = [&](size_t b) { return row_bytes % (long long)b == 0 && aligned(values, b) && aligned(out, b); };
    if (fits(16)) return launch_select<uint4>(values, row_bytes, (int)positions, indices, (int)k, out, out_rows, status_out, s);
    if (fits(8)) return launch_select<uint2>(values, row_bytes, (int)positions, indices, (int)k, out, out_rows, status_out, s);
    if (fits(4)) return launch_select<unsigned>(values, row_bytes, (int)positions, indices, (int)k, out, out_rows, status_out, s);
    if (fits(2)) return launch_select<unsigned short>(values, row_bytes, (int)positions, indices, (int)k, out, out_rows, status_out, s);
    return launch_select<unsigned char>(values, row_bytes, (int)positions, indices, (int)k, out, out_rows, status_out, s);
}
