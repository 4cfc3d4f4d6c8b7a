// Two-stage query selection for sm_100a: class max + top-k, and the row gather after it.
//
// Reference semantics (src/rfdetr_jax/models/transformer.py:694-706):
//   proposal_scores = logits.max(-1); _, idx = jax.lax.top_k(proposal_scores, k)
//   select_rows(projected, idx)            (src/rfdetr_jax/models/layers.py:225-244)
// jax.lax.top_k returns the k largest in descending order, the lower index first among equal
// values; floats compare in IEEE totalOrder (NaN above +inf).
//
// Keys: (totalOrder(score) << 32) | ~position, so larger keys come first and equal scores order
// by ascending position; every key of a row is distinct.
//
// Rows of up to kTopkClusterMaxPositions positions (the detector's 576 proposals): one cluster of
// kTopkCluster CTAs per row.  Each CTA reduces the classes of its share of the positions (flat
// 16-byte loads, all in flight at once; a per-position max of ordered keys by shared-memory
// atomicMax), sorts those keys in shared memory, and after a cluster
// barrier pulls every CTA's sorted keys from its peers through distributed shared memory.  The
// answer needs no global sort: the output slot of a key is its rank, the number of keys above
// it, which is the sum over the cluster's sorted lists of one binary search each; a CTA ranks
// its own keys and writes the ones below k straight to their slots.
// Longer rows: for flat scores (C == 1, k <= 4096) the radix select below; otherwise one CTA
// per row and a bitonic sort of the keys in shared memory (up to 16384 positions).
#include <algorithm>
#include <cstdlib>

#include <cooperative_groups.h>

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

// CTAs per row.  Measured at config 4 (104 rows of 576 x 91): 4 runs the whole grid in one
// wave (12.0 us); 8 leaves a tail of clusters for a second wave (17.3 us); 2 gives each CTA
// too much to load (16.4 us).
constexpr int kTopkCluster = 4;
constexpr int kTopkClusterThreads = 256;
constexpr int kTopkClusterMaxPositions = 2048;

template <int CL>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(kTopkClusterThreads)
topk_cluster_kernel(const float *__restrict__ logits, int N, int C, int k, float *__restrict__ scores_out,
                    float *__restrict__ values_out, int32_t *__restrict__ idx_out) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ unsigned long long mine[(kTopkClusterMaxPositions + CL - 1) / CL];
    __shared__ unsigned long long sorted[(kTopkClusterMaxPositions + CL - 1) / CL];
    __shared__ unsigned long long all[kTopkClusterMaxPositions];
    __shared__ int rank_of[(kTopkClusterMaxPositions + CL - 1) / CL];
    __shared__ unsigned okey[(kTopkClusterMaxPositions + CL - 1) / CL];
    const int crank = (int)cluster.block_rank();
    const int r = blockIdx.x / CL;
    const int per = (((N + CL - 1) / CL) + 3) & ~3;  // a multiple of 4 positions
    const int p_lo = crank * per, p_hi = min(N, p_lo + per), mine_n = max(p_hi - p_lo, 0);
    const float *rowp = logits + (size_t)r * N * C;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int nwarps = kTopkClusterThreads / 32;
    constexpr int U = 4;  // positions per warp step: independent load chains in flight

    for (int i = threadIdx.x; i < mine_n; i += kTopkClusterThreads) {
        rank_of[i] = 0;
        okey[i] = 0u;  // below every ordered key
    }
    // Rows whose elements start on 16-byte boundaries are read as flat float4 vectors (all of a
    // CTA's loads in flight at once); a vector spans at most two positions (C >= 4), and each
    // position's max is an atomicMax of ordered keys (NaN canonicalised, so it wins like jnp.max).
    const bool flat = C >= 4 && C <= 1024 && ((size_t)N * C) % 4 == 0 && (reinterpret_cast<size_t>(logits) & 15) == 0;
    if (flat) {
        __syncthreads();
        // [e0, e1): this CTA's elements (empty when its positions start past the row's end);
        // e0 is a multiple of 4 because per is.
        const unsigned e0 = (unsigned)(p_lo * C), e1 = e0 + (unsigned)(mine_n * C);
        const unsigned nv = (e1 - e0) / 4;
        const float4 *v4 = reinterpret_cast<const float4 *>(rowp + e0);
        const unsigned magic = 0xffffffffu / (unsigned)C + 1u;  // floor(e / C) for e < 2^32 / C
        constexpr int VU = 8;
        for (unsigned v0 = threadIdx.x; v0 < nv; v0 += kTopkClusterThreads * VU) {
            float4 x[VU];
#pragma unroll
            for (int u = 0; u < VU; ++u) {
                const unsigned v = v0 + u * kTopkClusterThreads;
                x[u] = v < nv ? __ldg(v4 + v) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            }
#pragma unroll
            for (int u = 0; u < VU; ++u) {
                const unsigned v = v0 + u * kTopkClusterThreads;
                if (v >= nv) break;
                const unsigned e = e0 + 4 * v;                     // row-relative element index
                const unsigned pa = __umulhi(e, magic);            // position of the first element
                const unsigned split = (pa + 1) * (unsigned)C - e; // elements before the next position
                const float f[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
                unsigned ka = 0u, kb = 0u;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const unsigned kk = order_key(f[i] != f[i] ? __uint_as_float(0x7fc00000u) : f[i]);
                    if ((unsigned)i < split) ka = max(ka, kk);
                    else kb = max(kb, kk);
                }
                atomicMax(&okey[pa - p_lo], ka);
                if (split < 4u) atomicMax(&okey[pa + 1 - p_lo], kb);
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < mine_n; i += kTopkClusterThreads) {
            const int p = p_lo + i;
            mine[i] = ((unsigned long long)okey[i] << 32) | (unsigned long long)(0xffffffffu - (unsigned)p);
            if (scores_out) scores_out[(size_t)r * N + p] = key_to_float(okey[i]);
        }
    }
    for (int q0 = warp * U; !flat && q0 < mine_n; q0 += nwarps * U) {
        float m[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            m[u] = -INFINITY;
            if (q0 + u < mine_n) {
                const float *x = rowp + (size_t)(p_lo + q0 + u) * C;
                for (int c = lane; c < C; c += 32) m[u] = nan_max(m[u], __ldg(x + c));
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m[u] = nan_max(m[u], __shfl_xor_sync(0xffffffffu, m[u], o));
        }
        if (lane < U && q0 + lane < mine_n) {
            float sc = m[0];
#pragma unroll
            for (int u = 1; u < U; ++u) sc = (lane == u) ? m[u] : sc;
            if (sc != sc) sc = __uint_as_float(0x7fc00000u);  // canonical (positive) NaN sorts first
            const int p = p_lo + q0 + lane;
            mine[q0 + lane] = ((unsigned long long)order_key(sc) << 32) | (unsigned long long)(0xffffffffu - (unsigned)p);
            if (scores_out) scores_out[(size_t)r * N + p] = sc;
        }
    }
    __syncthreads();
    // Sort this CTA's keys (descending): a key's local rank is the count of own keys above it.
    for (int i = threadIdx.x; i < mine_n; i += kTopkClusterThreads) {
        const unsigned long long key = mine[i];
        int lr = 0;
        for (int j = 0; j < mine_n; ++j) lr += mine[j] > key ? 1 : 0;
        sorted[lr] = key;
    }
    cluster.sync();
    // Every CTA's sorted keys, from the whole cluster (slot c * per + local rank).
    for (int j = threadIdx.x; j < CL * per; j += kTopkClusterThreads) {
        const int owner = j / per, o = j - owner * per;
        const int owner_n = max(min(N, (owner + 1) * per) - owner * per, 0);
        if (o < owner_n) {
            const unsigned long long *peer = cluster.map_shared_rank(sorted, owner);
            all[j] = peer[o];
        }
    }
    __syncthreads();
    // Rank of an own key = keys above it in each CTA's sorted list (a binary search per list).
    for (int w = threadIdx.x; w < mine_n * CL; w += kTopkClusterThreads) {
        const int i = w / CL, c = w - i * CL;
        const int cn = max(min(N, (c + 1) * per) - c * per, 0);
        const unsigned long long key = sorted[i];
        const unsigned long long *list = all + c * per;
        int lo = 0, hi = cn;  // first index whose key is not above `key`
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (list[mid] > key) lo = mid + 1;
            else hi = mid;
        }
        atomicAdd(&rank_of[i], lo);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < mine_n; i += kTopkClusterThreads) {
        const int rk = rank_of[i];
        if (rk < k) {
            const unsigned long long key = sorted[i];
            idx_out[(size_t)r * k + rk] = (int)(0xffffffffu - (unsigned)(key & 0xffffffffull));
            if (values_out) values_out[(size_t)r * k + rk] = key_to_float((unsigned)(key >> 32));
        }
    }
    cluster.sync();  // peers read this CTA's keys until here
}

// ------------------------------------------------------------------------------------------
// Radix select for long flat score rows (C == 1): the inference post-process selects the top
// 300 of Q*C = 27,300 sigmoid scores per image (postprocess.py:37-41).  One CTA per row.  A
// min/max reduction of the row's ordered keys gives their common leading bits; 8-bit histogram
// passes over the bits below that prefix narrow the k-th largest key T (a pass reads the row
// from L2; starting below the common prefix keeps the first pass from piling every thread's
// shared-memory atomic onto one bin when the scores share their top bits, as sigmoid scores
// do).  An ordered pass then takes every key above T and, among keys equal to T, the lowest
// positions -- exactly lax.top_k's choice -- and a bitonic sort of those k candidates (64-bit
// keys with ~position) gives the output order.
// ------------------------------------------------------------------------------------------
constexpr int kRadixThreads = 1024;
constexpr int kRadixMaxK = 4096;
constexpr long long kRadixMaxPositions = 1LL << 24;

__device__ __forceinline__ unsigned canon_key(float x) {
    return order_key(x != x ? __uint_as_float(0x7fc00000u) : x);
}

// Staged: the row's canonical keys are kept in dynamic shared memory from the first pass on, so
// the histogram passes and the selection read shared memory instead of the row in L1/L2.
template <bool Staged>
__global__ void __launch_bounds__(kRadixThreads)
topk_radix_kernel(const float *__restrict__ scores, int N, int k, float *__restrict__ scores_out,
                  float *__restrict__ values_out, int32_t *__restrict__ idx_out) {
    extern __shared__ unsigned skeys[];
    __shared__ unsigned hist[256];
    __shared__ unsigned long long cand[kRadixMaxK];
    __shared__ unsigned wsum[kRadixThreads / 32];
    __shared__ unsigned wmin[kRadixThreads / 32], wmax[kRadixThreads / 32];
    __shared__ unsigned sh_prefix, sh_need, sh_gt, sh_eq, sh_min, sh_max, sh_cnt;
    const int r = blockIdx.x;
    const float *row = scores + (size_t)r * N;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned kmin = 0xffffffffu, kmax = 0u;
    for (int i = tid; i < N; i += kRadixThreads) {
        const float x = __ldg(row + i);
        if (scores_out) scores_out[(size_t)r * N + i] = x != x ? __uint_as_float(0x7fc00000u) : x;
        const unsigned key = canon_key(x);
        if (Staged) skeys[i] = key;
        kmin = min(kmin, key);
        kmax = max(kmax, key);
    }
    auto key_at = [&](int i) -> unsigned { return Staged ? skeys[i] : canon_key(__ldg(row + i)); };
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    if (lane == 0) {
        wmin[warp] = kmin;
        wmax[warp] = kmax;
    }
    __syncthreads();
    if (warp == 0) {
        kmin = wmin[lane];
        kmax = wmax[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
            kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
        }
        if (lane == 0) {
            sh_min = kmin;
            sh_max = kmax;
        }
    }
    __syncthreads();
    // Bits above `hi` are common to every key of the row.
    const unsigned diff = sh_min ^ sh_max;
    const int hi = diff ? 32 - __clz(diff) : 0;
    unsigned pmask = hi >= 32 ? 0u : ~((1u << hi) - 1u);
    unsigned prefix = sh_max & pmask;
    unsigned need = (unsigned)k;  // keys still to take from the current bucket
    if (tid == 0) sh_cnt = (unsigned)N;  // keys in the current bucket
    for (int top = hi; top > 0; top -= 8) {
        const int shift = max(top - 8, 0);
        const unsigned dmask = (1u << (top - shift)) - 1u;
        for (int i = tid; i < 256; i += kRadixThreads) hist[i] = 0u;
        __syncthreads();
        for (int i = tid; i < N; i += kRadixThreads) {
            const unsigned key = key_at(i);
            if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & dmask], 1u);
        }
        __syncthreads();
        if (warp == 0) {
            // Lane l holds bins 255-8l .. 248-8l (descending); find the bucket holding the
            // `need`-th largest key.
            unsigned c[8], sum = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = hist[255 - 8 * lane - j];
                sum += c[j];
            }
            unsigned incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const unsigned excl = incl - sum;
            if (excl < need && incl >= need) {
                unsigned cum = excl;
                int bin = 255 - 8 * lane;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (cum + c[j] >= need) {
                        bin = 255 - 8 * lane - j;
                        break;
                    }
                    cum += c[j];
                }
                sh_prefix = prefix | ((unsigned)bin << shift);
                sh_need = need - cum;
                sh_cnt = hist[bin];
            }
        }
        __syncthreads();
        prefix = sh_prefix;
        need = sh_need;
        pmask |= dmask << shift;
    }
    // prefix is now the k-th largest key T; `need` keys equal to T are taken (lowest positions).
    if (tid == 0) {
        sh_gt = 0u;
        sh_eq = 0u;
    }
    __syncthreads();
    const unsigned gt_total = (unsigned)k - need;
    if (need == sh_cnt) {
        // Every key equal to T is taken: no ordered selection, the sort orders the ties.
        for (int i = tid; i < N; i += kRadixThreads) {
            const unsigned key = key_at(i);
            if (key >= prefix)
                cand[atomicAdd(&sh_gt, 1u)] = ((unsigned long long)key << 32) | (unsigned long long)(0xffffffffu - (unsigned)i);
        }
    }
    for (int c0 = 0; need != sh_cnt && c0 < N; c0 += kRadixThreads) {
        const int i = c0 + tid;
        const unsigned key = i < N ? key_at(i) : 0u;
        const unsigned long long full = ((unsigned long long)key << 32) | (unsigned long long)(0xffffffffu - (unsigned)i);
        if (i < N && key > prefix) cand[atomicAdd(&sh_gt, 1u)] = full;
        const bool eq = i < N && key == prefix;
        const unsigned bal = __ballot_sync(0xffffffffu, eq);
        if (lane == 0) wsum[warp] = __popc(bal);
        __syncthreads();
        if (warp == 0) {
            const unsigned v = wsum[lane];
            unsigned incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            wsum[lane] = incl - v;  // exclusive warp offsets
        }
        __syncthreads();
        const unsigned base = sh_eq;
        const unsigned mine = base + wsum[warp] + __popc(bal & ((1u << lane) - 1u));
        if (eq && mine < need) cand[gt_total + mine] = full;
        __syncthreads();
        if (tid == kRadixThreads - 1) sh_eq = mine + (eq ? 1u : 0u);
        __syncthreads();
    }
    // Sort the k candidates descending (padding with keys below every real key).
    int P2 = 1;
    while (P2 < k) P2 <<= 1;
    for (int i = k + tid; i < P2; i += kRadixThreads) cand[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= P2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < (P2 >> 1); i += kRadixThreads) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi2 = lo + stride;
                const bool desc = (lo & size) == 0;
                const unsigned long long a = cand[lo], b2 = cand[hi2];
                if ((a < b2) == desc) {
                    cand[lo] = b2;
                    cand[hi2] = a;
                }
            }
            __syncthreads();
        }
    }
    for (int i = tid; i < k; i += kRadixThreads) {
        const unsigned long long key = cand[i];
        idx_out[(size_t)r * k + i] = (int)(0xffffffffu - (unsigned)(key & 0xffffffffull));
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
    const bool radix = classes == 1 && positions > kTopkClusterMaxPositions && positions <= kRadixMaxPositions &&
                       k <= kRadixMaxK;
    if (rows < 0 || positions <= 0 || classes <= 0 || k <= 0 || k > positions ||
        (positions > kTopkMaxPositions && !radix) || rows > 2147483647LL || positions * classes > (1LL << 31))
        return RFDETR_ERR_SHAPE;
    if (rows == 0) return RFDETR_OK;
    if (!logits || !indices_out) return RFDETR_ERR_SHAPE;
    if (!aligned(logits, 4) || !aligned(indices_out, 4) || (scores_out && !aligned(scores_out, 4)) ||
        (values_out && !aligned(values_out, 4)))
        return RFDETR_ERR_ALIGN;
    if (positions <= kTopkClusterMaxPositions && rows * kTopkCluster <= 2147483647LL && knob(kKnobTopkSort).count == 0) {
        topk_cluster_kernel<kTopkCluster><<<(unsigned)(rows * kTopkCluster), kTopkClusterThreads, 0,
                                            static_cast<cudaStream_t>(stream)>>>(
            logits, (int)positions, (int)classes, (int)k, scores_out, values_out, indices_out);
        return launch_status();
    }
    if (radix && knob(kKnobTopkSort).count == 0) {
        // Keys staged in shared memory when the row fits beside the kernel's static arrays.
        const size_t kbytes = (size_t)positions * sizeof(unsigned);
        cudaFuncAttributes fa{};
        int optin = 0, dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        const bool staged = cudaFuncGetAttributes(&fa, topk_radix_kernel<true>) == cudaSuccess &&
                            fa.sharedSizeBytes + kbytes <= (size_t)optin && knob(kKnobTopkUnstaged).count == 0;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (staged) {
            if (cudaFuncSetAttribute(topk_radix_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kbytes) != cudaSuccess)
                return RFDETR_ERR_CUDA;
            topk_radix_kernel<true><<<(unsigned)rows, kRadixThreads, kbytes, s>>>(
                logits, (int)positions, (int)k, scores_out, values_out, indices_out);
        } else {
            topk_radix_kernel<false><<<(unsigned)rows, kRadixThreads, 0, s>>>(
                logits, (int)positions, (int)k, scores_out, values_out, indices_out);
        }
        return launch_status();
    }
    if (positions > kTopkMaxPositions) return RFDETR_ERR_SHAPE;
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
