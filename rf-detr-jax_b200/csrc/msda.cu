// Multi-scale deformable-attention sampler for sm_100a: forward and backward.
//
// Reference semantics: ms_deform_attn_core_rows (src/rfdetr_jax/models/ops.py:208-292) with the
// "gather" sampler (ops.py:64-134) and its autodiff backward; gradient formulas as in
// deform_pallas.py:97-120.
//
// Work decomposition.  An "item" is one (image b, query q, head h): it owns D output channels
// and L*P samples.  A team of `team` lanes serves an item, each lane holding VEC consecutive
// channels, so a corner tap is one VEC-wide vector load per lane.  Consecutive teams take
// consecutive heads of the same query, so a warp's loads of sampling locations and weights and
// its output stores are contiguous.
//
// A CTA owns one (image, group of `hsub` heads) and a tile of queries.  The value rows of those
// heads ([hsub, Lv, D], contiguous in the [B*H, Lv, D] layout) are staged once into shared
// memory when they fit (STAGE), so every bilinear tap is a shared-memory read; otherwise taps
// read through the read-only L1 path.
//
// Backward: grad_value is accumulated in float32 -- in a shared-memory slab per CTA
// (SMEM_ACC, flushed with vector reductions into the float32 accumulator once per CTA) or
// directly with vector global reductions -- and rounded once.  grad_loc and grad_weights are
// produced in the same pass from team-reduced dot products.
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace rfdetr {
namespace {

constexpr int kMaxLevels = 16;
constexpr int kMaxThreads = 512;

struct Geom {
    int B, H, D, Lq, L, P, Lv;
    int lh[kMaxLevels], lw[kMaxLevels], ls[kMaxLevels];
};

template <typename TV, typename TW> struct OutOf { using T = float; };
template <> struct OutOf<bf16, bf16> { using T = bf16; };

// Arithmetic type of the interpolation and of the reductions: float for bf16 values, double for
// float32 values, so the fp32 path stays within 1e-5 relative / 1e-6 absolute of the exact
// result even where the location gradient's channel sum cancels.
template <typename TV> struct AccOf { using T = float; };
template <> struct AccOf<float> { using T = double; };

// Level table copied to shared memory so the per-sample loop indexes it cheaply.
struct LevelTable {
    int h[kMaxLevels], w[kMaxLevels], s[kMaxLevels];
};

__device__ __forceinline__ void load_levels(LevelTable &t, const Geom &g) {
    if (threadIdx.x < g.L) {
        t.h[threadIdx.x] = g.lh[threadIdx.x];
        t.w[threadIdx.x] = g.lw[threadIdx.x];
        t.s[threadIdx.x] = g.ls[threadIdx.x];
    }
}

// ops.py:270 (grids = 2*loc - 1) and ops.py:83-84 (ix = ((gx + 1) * W - 1) / 2): one IEEE
// float32 rounding per step and no FMA contraction, so floor(ix) agrees with the reference
// bit for bit.  The division by two is exact, hence the multiply.
__device__ __forceinline__ void sample_coords(float lx, float ly, float wf, float hf, float &ix,
                                              float &iy) {
    const float gx = __fsub_rn(__fmul_rn(2.f, lx), 1.f);
    const float gy = __fsub_rn(__fmul_rn(2.f, ly), 1.f);
    ix = __fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(gx, 1.f), wf), 1.f), 0.5f);
    iy = __fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(gy, 1.f), hf), 1.f), 0.5f);
}

// Bilinear taps of one sample (ops.py:85-106): fractional weights, the top-left corner and a
// 4-bit in-bounds mask in the reference's corner order (x0,y0), (x1,y0), (x0,y1), (x1,y1).
struct Taps {
    float wx0, wx1, wy0, wy1;
    long long off00;  // element offset of corner (x0, y0) in the level, in units of D
    unsigned mask;
};

__device__ __forceinline__ Taps make_taps(float ix, float iy, int W, int H) {
    Taps t;
    const float fx0 = floorf(ix), fy0 = floorf(iy);
    t.wx1 = ix - fx0;  // exact
    t.wy1 = iy - fy0;
    t.wx0 = 1.f - t.wx1;
    t.wy0 = 1.f - t.wy1;
    const float wf = (float)W, hf = (float)H;
    const bool vx0 = fx0 >= 0.f && fx0 < wf;
    const bool vx1 = fx0 >= -1.f && fx0 < wf - 1.f;
    const bool vy0 = fy0 >= 0.f && fy0 < hf;
    const bool vy1 = fy0 >= -1.f && fy0 < hf - 1.f;
    const int x0 = (int)fmaxf(fminf(fx0, wf), -2.f);
    const int y0 = (int)fmaxf(fminf(fy0, hf), -2.f);
    t.off00 = (long long)y0 * W + x0;
    t.mask = (vx0 && vy0 ? 1u : 0u) | (vx1 && vy0 ? 2u : 0u) | (vx0 && vy1 ? 4u : 0u) |
             (vx1 && vy1 ? 8u : 0u);
    return t;
}

template <typename T> __device__ __forceinline__ float ld_scalar(const T *p) { return to_f32(__ldg(p)); }

// ------------------------------------------------------------------------------------------
// Forward
// ------------------------------------------------------------------------------------------
template <typename TV, typename TW, int VEC, bool STAGE>
__global__ void __launch_bounds__(kMaxThreads)
msda_forward_kernel(const TV *__restrict__ value, const float *__restrict__ loc,
                    const TW *__restrict__ attn, typename OutOf<TV, TW>::T *__restrict__ out,
                    const Geom g, const int team, const int hsub, const int q_tile) {
    using TO = typename OutOf<TV, TW>::T;
    using AT = typename AccOf<TV>::T;
    constexpr bool kNC = !STAGE;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ LevelTable lv;
    load_levels(lv, g);

    const int groups_per_image = g.H / hsub;
    const int b = blockIdx.y / groups_per_image;
    const int h0 = (blockIdx.y - b * groups_per_image) * hsub;
    const int q0 = blockIdx.x * q_tile;
    const int q1 = min(q0 + q_tile, g.Lq);
    const size_t slab = (size_t)g.Lv * g.D;
    const TV *vsrc = value + ((size_t)b * g.H + h0) * slab;

    const TV *vbase = vsrc;
    if constexpr (STAGE) {
        const int n16 = (int)((size_t)hsub * slab * sizeof(TV) / 16);
        const uint4 *src = reinterpret_cast<const uint4 *>(vsrc);
        uint4 *dst = reinterpret_cast<uint4 *>(smem);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = __ldg(src + i);
        vbase = reinterpret_cast<const TV *>(smem);
    }
    __syncthreads();

    const int lane_t = threadIdx.x & (team - 1);
    const int tix = threadIdx.x / team;
    const int nteams = blockDim.x / team;
    const int chunk = lane_t * VEC;
    const bool active_lane = chunk < g.D;
    const int LP = g.L * g.P;
    const int items = (q1 - q0) * hsub;

    for (int it = tix; it < items; it += nteams) {
        const int qi = it / hsub;
        const int hs = it - qi * hsub;
        const size_t row = ((size_t)b * g.Lq + q0 + qi) * g.H + h0 + hs;
        const float2 *lp = reinterpret_cast<const float2 *>(loc) + row * LP;
        const TW *ap = attn + row * LP;
        const TV *vh = vbase + hs * slab + chunk;
        AT acc[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = 0;

        for (int l = 0; l < g.L; ++l) {
            const int W = lv.w[l], H = lv.h[l];
            const float wf = (float)W, hf = (float)H;
            const TV *vl = vh + (size_t)lv.s[l] * g.D;
            for (int pt = 0; pt < g.P; ++pt) {
                const float2 xy = __ldg(lp + l * g.P + pt);
                const float a = ld_scalar(ap + l * g.P + pt);
                float ix, iy;
                sample_coords(xy.x, xy.y, wf, hf, ix, iy);
                if (!(isfinite(ix) && isfinite(iy))) {
#pragma unroll
                    for (int i = 0; i < VEC; ++i) acc[i] = (AT)__int_as_float(0x7fc00000);
                    continue;
                }
                const Taps t = make_taps(ix, iy, W, H);
                if (!active_lane || t.mask == 0) continue;
                AT s[VEC];
#pragma unroll
                for (int i = 0; i < VEC; ++i) s[i] = 0;
                float v[VEC];
                const TV *p00 = vl + t.off00 * g.D;
                const AT wx0 = t.wx0, wx1 = t.wx1, wy0 = t.wy0, wy1 = t.wy1;
                if (t.mask & 1u) {
                    const AT w = wx0 * wy0;
                    load_vec<TV, VEC, kNC>(p00, v);
#pragma unroll
                    for (int i = 0; i < VEC; ++i) s[i] = fma(w, (AT)v[i], s[i]);
                }
                if (t.mask & 2u) {
                    const AT w = wx1 * wy0;
                    load_vec<TV, VEC, kNC>(p00 + g.D, v);
#pragma unroll
                    for (int i = 0; i < VEC; ++i) s[i] = fma(w, (AT)v[i], s[i]);
                }
                if (t.mask & 4u) {
                    const AT w = wx0 * wy1;
                    load_vec<TV, VEC, kNC>(p00 + (size_t)W * g.D, v);
#pragma unroll
                    for (int i = 0; i < VEC; ++i) s[i] = fma(w, (AT)v[i], s[i]);
                }
                if (t.mask & 8u) {
                    const AT w = wx1 * wy1;
                    load_vec<TV, VEC, kNC>(p00 + (size_t)(W + 1) * g.D, v);
#pragma unroll
                    for (int i = 0; i < VEC; ++i) s[i] = fma(w, (AT)v[i], s[i]);
                }
#pragma unroll
                for (int i = 0; i < VEC; ++i) acc[i] = fma((AT)a, s[i], acc[i]);
            }
        }
        if (active_lane) {
            float o[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) o[i] = (float)acc[i];
            store_vec<TO, VEC>(out + row * g.D + chunk, o);
        }
    }
}

// ------------------------------------------------------------------------------------------
// Backward
// ------------------------------------------------------------------------------------------

// out[i] = in[(i + rot) mod VEC] for a lane-dependent rotation, built from selects so the array
// stays in registers.  Rotating the element order across the teams of a warp spreads their
// shared-memory atomics over different banks.
template <int VEC>
__device__ __forceinline__ void rotate(const float *in, float *out, int rot) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
        const int src = (i + rot) & (VEC - 1);
        float x = in[0];
#pragma unroll
        for (int k = 1; k < VEC; ++k) x = (src == k) ? in[k] : x;
        out[i] = x;
    }
}

template <typename TV, typename TW, int VEC, bool STAGE, bool SMEM_ACC>
__global__ void __launch_bounds__(kMaxThreads)
msda_backward_kernel(const TV *__restrict__ value, const float *__restrict__ loc,
                     const TW *__restrict__ attn,
                     const typename OutOf<TV, TW>::T *__restrict__ grad_out,
                     float *__restrict__ gacc, float *__restrict__ grad_loc,
                     TW *__restrict__ grad_attn, const Geom g, const int team, const int hsub,
                     const int q_tile) {
    using TO = typename OutOf<TV, TW>::T;
    using AT = typename AccOf<TV>::T;
    constexpr bool kNC = !STAGE;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ LevelTable lv;
    load_levels(lv, g);

    const int groups_per_image = g.H / hsub;
    const int b = blockIdx.y / groups_per_image;
    const int h0 = (blockIdx.y - b * groups_per_image) * hsub;
    const int q0 = blockIdx.x * q_tile;
    const int q1 = min(q0 + q_tile, g.Lq);
    const size_t slab = (size_t)g.Lv * g.D;
    const TV *vsrc = value + ((size_t)b * g.H + h0) * slab;
    float *gdst = gacc + ((size_t)b * g.H + h0) * slab;

    const size_t staged_bytes = STAGE ? (((size_t)hsub * slab * sizeof(TV) + 15) & ~(size_t)15) : 0;
    float *gsm = reinterpret_cast<float *>(smem + staged_bytes);
    if constexpr (SMEM_ACC) {
        const int n4 = (int)((size_t)hsub * slab / 4);
        float4 *z = reinterpret_cast<float4 *>(gsm);
        for (int i = threadIdx.x; i < n4; i += blockDim.x) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int i = n4 * 4 + threadIdx.x; i < (int)((size_t)hsub * slab); i += blockDim.x) gsm[i] = 0.f;
    }
    const TV *vbase = vsrc;
    if constexpr (STAGE) {
        const int n16 = (int)((size_t)hsub * slab * sizeof(TV) / 16);
        const uint4 *src = reinterpret_cast<const uint4 *>(vsrc);
        uint4 *dst = reinterpret_cast<uint4 *>(smem);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = __ldg(src + i);
        vbase = reinterpret_cast<const TV *>(smem);
    }
    __syncthreads();

    const int lane_t = threadIdx.x & (team - 1);
    const int tix = threadIdx.x / team;
    const int nteams = blockDim.x / team;
    const int chunk = lane_t * VEC;
    const bool active_lane = chunk < g.D;
    const int LP = g.L * g.P;
    const int items = (q1 - q0) * hsub;
    const int rot = tix & (VEC - 1);
    const float qnan = __int_as_float(0x7fc00000);

    // All teams of a warp run the same number of iterations (the shuffles need every lane).
    for (int base = 0; base < items; base += nteams) {
        const int it = base + tix;
        const bool live = it < items;
        const int qi = live ? it / hsub : 0;
        const int hs = live ? it - qi * hsub : 0;
        const size_t row = ((size_t)b * g.Lq + q0 + qi) * g.H + h0 + hs;
        const float2 *lp = reinterpret_cast<const float2 *>(loc) + row * LP;
        const TW *ap = attn + row * LP;
        const TV *vh = vbase + hs * slab + chunk;

        float gr[VEC];
        if (live && active_lane) {
            load_vec<TO, VEC, true>(grad_out + row * g.D + chunk, gr);
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) gr[i] = 0.f;
        }
        float grot[VEC];
        if constexpr (SMEM_ACC) rotate<VEC>(gr, grot, rot);

        for (int l = 0; l < g.L; ++l) {
            const int W = lv.w[l], H = lv.h[l];
            const float wf = (float)W, hf = (float)H;
            const TV *vl = vh + (size_t)lv.s[l] * g.D;
            for (int pt = 0; pt < g.P; ++pt) {
                float a = 0.f, ix = 0.f, iy = 0.f;
                bool ok = false;
                if (live) {
                    const float2 xy = __ldg(lp + l * g.P + pt);
                    a = ld_scalar(ap + l * g.P + pt);
                    sample_coords(xy.x, xy.y, wf, hf, ix, iy);
                    ok = isfinite(ix) && isfinite(iy);
                }
                Taps t;
                if (ok) {
                    t = make_taps(ix, iy, W, H);
                } else {
                    t.wx0 = t.wx1 = t.wy0 = t.wy1 = 0.f;
                    t.off00 = 0;
                    t.mask = 0u;
                }
                const bool tap = ok && active_lane;
                float v00[VEC], v10[VEC], v01[VEC], v11[VEC];
#pragma unroll
                for (int i = 0; i < VEC; ++i) v00[i] = v10[i] = v01[i] = v11[i] = 0.f;
                const TV *p00 = vl + t.off00 * g.D;
                if (tap && (t.mask & 1u)) load_vec<TV, VEC, kNC>(p00, v00);
                if (tap && (t.mask & 2u)) load_vec<TV, VEC, kNC>(p00 + g.D, v10);
                if (tap && (t.mask & 4u)) load_vec<TV, VEC, kNC>(p00 + (size_t)W * g.D, v01);
                if (tap && (t.mask & 8u)) load_vec<TV, VEC, kNC>(p00 + (size_t)(W + 1) * g.D, v11);

                const float w00 = t.wx0 * t.wy0, w10 = t.wx1 * t.wy0;
                const float w01 = t.wx0 * t.wy1, w11 = t.wx1 * t.wy1;
                const AT wx0 = t.wx0, wx1 = t.wx1, wy0 = t.wy0, wy1 = t.wy1;
                AT ds = 0, dx = 0, dy = 0;
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    const AT a00 = v00[i], a10 = v10[i], a01 = v01[i], a11 = v11[i];
                    const AT s = wx0 * wy0 * a00 + wx1 * wy0 * a10 + wx0 * wy1 * a01 + wx1 * wy1 * a11;
                    const AT sx = wy0 * (a10 - a00) + wy1 * (a11 - a01);
                    const AT sy = wx0 * (a01 - a00) + wx1 * (a11 - a10);
                    ds = fma((AT)gr[i], s, ds);
                    dx = fma((AT)gr[i], sx, dx);
                    dy = fma((AT)gr[i], sy, dy);
                }
                for (int o = team >> 1; o > 0; o >>= 1) {
                    ds += __shfl_xor_sync(0xffffffffu, ds, o);
                    dx += __shfl_xor_sync(0xffffffffu, dx, o);
                    dy += __shfl_xor_sync(0xffffffffu, dy, o);
                }
                if (live && lane_t == 0) {
                    const size_t s_idx = row * LP + l * g.P + pt;
                    grad_attn[s_idx] = from_f32<TW>(ok ? (float)ds : qnan);
                    float2 gl;
                    gl.x = ok ? (float)((AT)wf * ((AT)a * dx)) : qnan;
                    gl.y = ok ? (float)((AT)hf * ((AT)a * dy)) : qnan;
                    reinterpret_cast<float2 *>(grad_loc)[s_idx] = gl;
                }
                if (!tap || t.mask == 0u) continue;

                const float c[4] = {a * w00, a * w10, a * w01, a * w11};
                const long long offs[4] = {t.off00, t.off00 + 1, t.off00 + W, t.off00 + W + 1};
                if constexpr (SMEM_ACC) {
                    float *sb = gsm + hs * slab + (size_t)lv.s[l] * g.D + chunk;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (!(t.mask & (1u << k))) continue;
                        float *p = sb + offs[k] * g.D;
#pragma unroll
                        for (int i = 0; i < VEC; ++i) atomicAdd(p + ((i + rot) & (VEC - 1)), c[k] * grot[i]);
                    }
                } else {
                    float *gb = gdst + hs * slab + (size_t)lv.s[l] * g.D + chunk;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (!(t.mask & (1u << k))) continue;
                        float add[VEC];
#pragma unroll
                        for (int i = 0; i < VEC; ++i) add[i] = c[k] * gr[i];
                        red_add_global<VEC>(gb + offs[k] * g.D, add);
                    }
                }
            }
        }
    }

    if constexpr (SMEM_ACC) {
        __syncthreads();
        const size_t n = (size_t)hsub * slab;
        if ((n & 3) == 0) {
            const float4 *s4 = reinterpret_cast<const float4 *>(gsm);
            for (size_t i = threadIdx.x; i < n / 4; i += blockDim.x) {
                const float4 x = s4[i];
                if (x.x != 0.f || x.y != 0.f || x.z != 0.f || x.w != 0.f) {
                    const float f[4] = {x.x, x.y, x.z, x.w};
                    red_add_global<4>(gdst + 4 * i, f);
                }
            }
        } else {
            for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
                if (gsm[i] != 0.f) atomicAdd(gdst + i, gsm[i]);
            }
        }
    }
}

// Rounds the float32 accumulator into the value dtype (bf16), 8 elements per thread.
__global__ void f32_to_bf16_kernel(const float *__restrict__ src, bf16 *__restrict__ dst, size_t n) {
    const size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (i + 8 <= n) {
        float f[8];
        const float4 a = __ldg(reinterpret_cast<const float4 *>(src + i));
        const float4 c = __ldg(reinterpret_cast<const float4 *>(src + i + 4));
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = c.x; f[5] = c.y; f[6] = c.z; f[7] = c.w;
        store_vec<bf16, 8>(dst + i, f);
    } else {
        for (size_t k = i; k < n; ++k) dst[k] = __float2bfloat16_rn(src[k]);
    }
}

// ------------------------------------------------------------------------------------------
// Host side: validation, launch planning and dispatch
// ------------------------------------------------------------------------------------------
struct Plan {
    int vec = 1, team = 1, hsub = 1, threads = 256, q_tile = 1, q_tiles = 1;
    bool stage = false, smem_acc = false;
    size_t smem = 0;
};

int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Tuning overrides for experiments: RFDETR_MSDA_FWD / RFDETR_MSDA_BWD = "hsub,stage,acc,threads,waves".
struct Tune {
    int hsub = 0, stage = -1, acc = -1, threads = 0, waves = 0;
};

Tune read_tune(const char *name) {
    Tune t;
    const char *s = getenv(name);
    if (s && *s) sscanf(s, "%d,%d,%d,%d,%d", &t.hsub, &t.stage, &t.acc, &t.threads, &t.waves);
    return t;
}

int validate(const int64_t *shapes, const int64_t *starts, int64_t B, int64_t H, int64_t D,
             int64_t Lq, int64_t L, int64_t P, Geom &g) {
    if (B < 0 || H <= 0 || D <= 0 || Lq < 0 || L <= 0 || P <= 0 || L > kMaxLevels || !shapes)
        return RFDETR_ERR_SHAPE;
    long long total = 0;
    for (int64_t l = 0; l < L; ++l) {
        const int64_t h = shapes[2 * l], w = shapes[2 * l + 1];
        if (h <= 0 || w <= 0 || h * w > (1LL << 30)) return RFDETR_ERR_SHAPE;
        if (starts && starts[l] != total) return RFDETR_ERR_SHAPE;
        g.lh[l] = (int)h;
        g.lw[l] = (int)w;
        g.ls[l] = (int)total;
        total += h * w;
    }
    const long long lim = (1LL << 31) - 1;
    if (B * H * total * D > lim || B * Lq * H * L * P * 2 > lim || B * Lq * H * D > lim) return RFDETR_ERR_SHAPE;
    g.B = (int)B; g.H = (int)H; g.D = (int)D; g.Lq = (int)Lq; g.L = (int)L; g.P = (int)P; g.Lv = (int)total;
    return RFDETR_OK;
}

// Largest lane vector (elements) that divides D, keeps a team within a warp and respects the
// alignment of every tensor accessed with it.
int pick_vec(int D, int vsize, const void *const *ptrs, const int *esizes, int nptr) {
    for (int vec = 16 / vsize; vec >= 1; vec >>= 1) {
        if (D % vec != 0 || D / vec > 32) continue;
        bool ok = true;
        for (int k = 0; k < nptr; ++k) {
            const size_t bytes = std::min<size_t>(16, (size_t)vec * esizes[k]);
            if (!aligned(ptrs[k], bytes) || ((size_t)D * esizes[k]) % bytes != 0) ok = false;
        }
        if (ok) return vec;
    }
    return 0;
}

int max_smem_optin() {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return v;
}

template <typename Kernel>
int finish_plan(Plan &p, const Geom &g, Kernel kernel, int waves) {
    if (p.smem > 48 * 1024) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem) != cudaSuccess)
            return RFDETR_ERR_CUDA;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, p.threads, p.smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    per_sm = std::max(per_sm, 1);
    const long long groups = (long long)g.B * (g.H / p.hsub);
    const long long target = (long long)num_sms() * per_sm * std::max(waves, 1);
    long long tiles = std::max<long long>(1, (target + groups - 1) / groups);
    tiles = std::min<long long>(tiles, std::max(g.Lq, 1));
    p.q_tile = ceil_div(std::max(g.Lq, 1), tiles);
    p.q_tiles = ceil_div(std::max(g.Lq, 1), p.q_tile);
    if (groups > 65535) return RFDETR_ERR_SHAPE;
    return RFDETR_OK;
}

// Chooses hsub (heads per CTA), whether to stage value rows and whether to accumulate
// grad_value in shared memory, within the device's shared-memory budget.  Heads are grouped up
// to one warp's worth of teams so that a warp's location/weight loads and output stores stay
// contiguous; with shared-memory residency the group also has to fit the budget.
void choose_layout(Plan &p, const Geom &g, int vsize, bool backward, const void *value) {
    const size_t slab = (size_t)g.Lv * g.D;
    const size_t vbytes = slab * vsize, gbytes = slab * 4;
    const size_t budget = backward ? 110 * 1024 : 64 * 1024;
    const bool stage_ok = aligned(value, 16) && (vbytes % 16 == 0);
    p.stage = stage_ok && vbytes <= budget;
    p.smem_acc = backward && gbytes + (p.stage ? vbytes : 0) <= budget;
    if (backward && !p.smem_acc && p.stage && gbytes <= budget) {
        // Prefer shared accumulation over staging when only one of them fits.
        p.stage = false;
        p.smem_acc = true;
    }
    const size_t per_head = (p.stage ? vbytes : 0) + (p.smem_acc ? gbytes : 0);
    int hsub = 1;
    while (g.H % (hsub * 2) == 0 && hsub * 2 * p.team <= 32 && 2 * hsub * per_head <= budget) hsub *= 2;
    p.hsub = hsub;
}

void apply_tune(Plan &p, const Tune &t, const Geom &g, int vsize, bool backward, const void *value) {
    const size_t slab = (size_t)g.Lv * g.D;
    if (t.hsub > 0 && g.H % t.hsub == 0) p.hsub = t.hsub;
    if (t.stage >= 0) p.stage = t.stage && aligned(value, 16) && (slab * vsize) % 16 == 0;
    if (t.acc >= 0 && backward) p.smem_acc = t.acc;
    if (t.threads > 0) p.threads = t.threads;
}

size_t plan_smem(const Plan &p, const Geom &g, int vsize) {
    const size_t slab = (size_t)g.Lv * g.D;
    size_t s = 0;
    if (p.stage) s += ((size_t)p.hsub * slab * vsize + 15) & ~(size_t)15;
    if (p.smem_acc) s += (size_t)p.hsub * slab * 4;
    return s;
}

template <typename TV, typename TW, int VEC, bool STAGE>
int launch_forward(const Geom &g, Plan &p, const Tune &tune, const void *value, const float *loc,
                   const void *attn, void *out, cudaStream_t stream) {
    auto kernel = msda_forward_kernel<TV, TW, VEC, STAGE>;
    int st = finish_plan(p, g, kernel, tune.waves);
    if (st) return st;
    dim3 grid(p.q_tiles, g.B * (g.H / p.hsub));
    kernel<<<grid, p.threads, p.smem, stream>>>(
        static_cast<const TV *>(value), loc, static_cast<const TW *>(attn),
        static_cast<typename OutOf<TV, TW>::T *>(out), g, p.team, p.hsub, p.q_tile);
    return launch_status();
}

template <typename TV, typename TW, int VEC>
int dispatch_forward_stage(const Geom &g, Plan &p, const Tune &tune, const void *value,
                           const float *loc, const void *attn, void *out, cudaStream_t s) {
    if (p.stage) return launch_forward<TV, TW, VEC, true>(g, p, tune, value, loc, attn, out, s);
    return launch_forward<TV, TW, VEC, false>(g, p, tune, value, loc, attn, out, s);
}

template <typename TV, typename TW>
int dispatch_forward(const Geom &g, Plan &p, const Tune &tune, const void *value, const float *loc,
                     const void *attn, void *out, cudaStream_t s) {
    switch (p.vec) {
        case 8:
            if constexpr (sizeof(TV) == 2) return dispatch_forward_stage<TV, TW, 8>(g, p, tune, value, loc, attn, out, s);
            return RFDETR_ERR_SHAPE;
        case 4: return dispatch_forward_stage<TV, TW, 4>(g, p, tune, value, loc, attn, out, s);
        case 2: return dispatch_forward_stage<TV, TW, 2>(g, p, tune, value, loc, attn, out, s);
        case 1: return dispatch_forward_stage<TV, TW, 1>(g, p, tune, value, loc, attn, out, s);
        default: return RFDETR_ERR_SHAPE;
    }
}

template <typename TV, typename TW, int VEC, bool STAGE, bool ACC>
int launch_backward(const Geom &g, Plan &p, const Tune &tune, const void *value, const float *loc,
                    const void *attn, const void *gout, float *gacc, float *gloc, void *gattn,
                    cudaStream_t stream) {
    auto kernel = msda_backward_kernel<TV, TW, VEC, STAGE, ACC>;
    int st = finish_plan(p, g, kernel, tune.waves);
    if (st) return st;
    dim3 grid(p.q_tiles, g.B * (g.H / p.hsub));
    kernel<<<grid, p.threads, p.smem, stream>>>(
        static_cast<const TV *>(value), loc, static_cast<const TW *>(attn),
        static_cast<const typename OutOf<TV, TW>::T *>(gout), gacc, gloc, static_cast<TW *>(gattn), g,
        p.team, p.hsub, p.q_tile);
    return launch_status();
}

template <typename TV, typename TW, int VEC>
int dispatch_backward_flags(const Geom &g, Plan &p, const Tune &tune, const void *value,
                            const float *loc, const void *attn, const void *gout, float *gacc,
                            float *gloc, void *gattn, cudaStream_t s) {
    if (p.stage && p.smem_acc)
        return launch_backward<TV, TW, VEC, true, true>(g, p, tune, value, loc, attn, gout, gacc, gloc, gattn, s);
    if (p.stage)
        return launch_backward<TV, TW, VEC, true, false>(g, p, tune, value, loc, attn, gout, gacc, gloc, gattn, s);
    if (p.smem_acc)
        return launch_backward<TV, TW, VEC, false, true>(g, p, tune, value, loc, attn, gout, gacc, gloc, gattn, s);
    return launch_backward<TV, TW, VEC, false, false>(g, p, tune, value, loc, attn, gout, gacc, gloc, gattn, s);
}

template <typename TV, typename TW>
int dispatch_backward(const Geom &g, Plan &p, const Tune &tune, const void *value, const float *loc,
                      const void *attn, const void *gout, float *gacc, float *gloc, void *gattn,
                      cudaStream_t s) {
    switch (p.vec) {
        case 8:
            if constexpr (sizeof(TV) == 2)
                return dispatch_backward_flags<TV, TW, 8>(g, p, tune, value, loc, attn, gout, gacc, gloc, gattn, s);
            return RFDETR_ERR_SHAPE;
        case 4: return dispatch_backward_flags<TV, TW, 4>(g, p, tune, value, loc, attn, gout, gacc, gloc, gattn, s);
        case 2: return dispatch_backward_flags<TV, TW, 2>(g, p, tune, value, loc, attn, gout, gacc, gloc, gattn, s);
        case 1: return dispatch_backward_flags<TV, TW, 1>(g, p, tune, value, loc, attn, gout, gacc, gloc, gattn, s);
        default: return RFDETR_ERR_SHAPE;
    }
}

bool dtype_ok(int d) { return d == RFDETR_F32 || d == RFDETR_BF16; }
int out_dtype(int vd, int wd) { return (vd == RFDETR_BF16 && wd == RFDETR_BF16) ? RFDETR_BF16 : RFDETR_F32; }

}  // namespace
}  // namespace rfdetr

using namespace rfdetr;

extern "C" int rfdetr_msda_forward(void *stream, const void *value, int value_dtype,
                                   const int64_t *spatial_shapes, const int64_t *level_start_index,
                                   const float *sampling_locations, const void *attention_weights,
                                   int weight_dtype, void *output, int output_dtype, int64_t batch,
                                   int64_t n_heads, int64_t head_dim, int64_t len_query,
                                   int64_t n_levels, int64_t n_points) {
    if (!dtype_ok(value_dtype) || !dtype_ok(weight_dtype) ||
        output_dtype != out_dtype(value_dtype, weight_dtype))
        return RFDETR_ERR_DTYPE;
    Geom g;
    int st = validate(spatial_shapes, level_start_index, batch, n_heads, head_dim, len_query, n_levels,
                      n_points, g);
    if (st) return st;
    if (g.B == 0 || g.Lq == 0) return RFDETR_OK;
    if (!value || !sampling_locations || !attention_weights || !output) return RFDETR_ERR_SHAPE;
    const int vs = dtype_size(value_dtype), ws = dtype_size(weight_dtype), os = dtype_size(output_dtype);
    if (!aligned(sampling_locations, 8) || !aligned(attention_weights, ws)) return RFDETR_ERR_ALIGN;
    const void *ptrs[2] = {value, output};
    const int es[2] = {vs, os};
    Plan p;
    p.vec = pick_vec(g.D, vs, ptrs, es, 2);
    if (!p.vec) return aligned(value, vs) && aligned(output, os) ? RFDETR_ERR_SHAPE : RFDETR_ERR_ALIGN;
    p.team = next_pow2(g.D / p.vec);
    choose_layout(p, g, vs, false, value);
    const Tune tune = read_tune("RFDETR_MSDA_FWD");
    apply_tune(p, tune, g, vs, false, value);
    p.smem = plan_smem(p, g, vs);
    if (p.smem > (size_t)max_smem_optin()) return RFDETR_ERR_SHAPE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (value_dtype == RFDETR_BF16 && weight_dtype == RFDETR_BF16)
        return dispatch_forward<bf16, bf16>(g, p, tune, value, sampling_locations, attention_weights, output, s);
    if (value_dtype == RFDETR_BF16)
        return dispatch_forward<bf16, float>(g, p, tune, value, sampling_locations, attention_weights, output, s);
    if (weight_dtype == RFDETR_BF16)
        return dispatch_forward<float, bf16>(g, p, tune, value, sampling_locations, attention_weights, output, s);
    return dispatch_forward<float, float>(g, p, tune, value, sampling_locations, attention_weights, output, s);
}

extern "C" size_t rfdetr_msda_backward_workspace_size(int value_dtype, int64_t batch, int64_t n_heads,
                                                      int64_t head_dim, int64_t len_value) {
    if (value_dtype != RFDETR_BF16) return 0;
    if (batch <= 0 || n_heads <= 0 || head_dim <= 0 || len_value <= 0) return 0;
    return (size_t)batch * n_heads * len_value * head_dim * sizeof(float);
}

extern "C" int rfdetr_msda_backward(void *stream, const void *value, int value_dtype,
                                    const int64_t *spatial_shapes, const int64_t *level_start_index,
                                    const float *sampling_locations, const void *attention_weights,
                                    int weight_dtype, const void *grad_output, int grad_output_dtype,
                                    void *grad_value, float *grad_sampling_locations,
                                    void *grad_attention_weights, void *workspace,
                                    size_t workspace_bytes, int64_t batch, int64_t n_heads,
                                    int64_t head_dim, int64_t len_query, int64_t n_levels,
                                    int64_t n_points) {
    if (!dtype_ok(value_dtype) || !dtype_ok(weight_dtype) ||
        grad_output_dtype != out_dtype(value_dtype, weight_dtype))
        return RFDETR_ERR_DTYPE;
    Geom g;
    int st = validate(spatial_shapes, level_start_index, batch, n_heads, head_dim, len_query, n_levels,
                      n_points, g);
    if (st) return st;
    if (g.B == 0) return RFDETR_OK;
    if (!value || !grad_value || (g.Lq > 0 && (!sampling_locations || !attention_weights || !grad_output ||
                                               !grad_sampling_locations || !grad_attention_weights)))
        return RFDETR_ERR_SHAPE;
    const int vs = dtype_size(value_dtype), ws = dtype_size(weight_dtype);
    const int os = dtype_size(grad_output_dtype);
    const size_t nvalue = (size_t)g.B * g.H * g.Lv * g.D;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (value_dtype == RFDETR_BF16 && !aligned(grad_value, 16)) return RFDETR_ERR_ALIGN;
    if (value_dtype == RFDETR_F32 && !aligned(grad_value, 16)) return RFDETR_ERR_ALIGN;
    float *gacc;
    if (value_dtype == RFDETR_F32) {
        gacc = static_cast<float *>(grad_value);
    } else {
        const size_t need = rfdetr_msda_backward_workspace_size(value_dtype, g.B, g.H, g.D, g.Lv);
        if (!workspace || workspace_bytes < need) return RFDETR_ERR_WORKSPACE;
        if (!aligned(workspace, 16)) return RFDETR_ERR_ALIGN;
        gacc = static_cast<float *>(workspace);
    }
    if (cudaMemsetAsync(gacc, 0, nvalue * sizeof(float), s) != cudaSuccess) return RFDETR_ERR_CUDA;
    if (g.Lq > 0) {
        if (!aligned(sampling_locations, 8) || !aligned(grad_sampling_locations, 8) ||
            !aligned(attention_weights, ws) || !aligned(grad_attention_weights, ws))
            return RFDETR_ERR_ALIGN;
        const void *ptrs[3] = {value, grad_output, gacc};
        const int es[3] = {vs, os, 4};
        Plan p;
        p.vec = pick_vec(g.D, vs, ptrs, es, 3);
        if (!p.vec) return RFDETR_ERR_ALIGN;
        p.team = next_pow2(g.D / p.vec);
        choose_layout(p, g, vs, true, value);
        const Tune tune = read_tune("RFDETR_MSDA_BWD");
        apply_tune(p, tune, g, vs, true, value);
        p.smem = plan_smem(p, g, vs);
        if (p.smem > (size_t)max_smem_optin()) return RFDETR_ERR_SHAPE;
        const float *loc = sampling_locations;
        const void *attn = attention_weights;
        if (value_dtype == RFDETR_BF16 && weight_dtype == RFDETR_BF16)
            st = dispatch_backward<bf16, bf16>(g, p, tune, value, loc, attn, grad_output, gacc,
                                               grad_sampling_locations, grad_attention_weights, s);
        else if (value_dtype == RFDETR_BF16)
            st = dispatch_backward<bf16, float>(g, p, tune, value, loc, attn, grad_output, gacc,
                                                grad_sampling_locations, grad_attention_weights, s);
        else if (weight_dtype == RFDETR_BF16)
            st = dispatch_backward<float, bf16>(g, p, tune, value, loc, attn, grad_output, gacc,
                                                grad_sampling_locations, grad_attention_weights, s);
        else
            st = dispatch_backward<float, float>(g, p, tune, value, loc, attn, grad_output, gacc,
                                                 grad_sampling_locations, grad_attention_weights, s);
        if (st) return st;
    }
    if (value_dtype == RFDETR_BF16) {
        const int threads = 256;
        const long long blocks = ((long long)(nvalue + 7) / 8 + threads - 1) / threads;
        f32_to_bf16_kernel<<<(unsigned)blocks, threads, 0, s>>>(gacc, static_cast<bf16 *>(grad_value), nvalue);
        return launch_status();
    }
    return RFDETR_OK;
}

// ------------------------------------------------------------------------------------------
// Backward without a workspace argument (see rfdetr_msda_backward_noalloc in the header).
// The float32 accumulator of the bf16 path lives in this static device array.  In host code
// the name is only a host-side stand-in, so its device address is looked up per device with
// cudaGetSymbolAddress and passed to the kernels like a caller's workspace.
// ------------------------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = RFDETR_MSDA_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void *g_noalloc_address[kNoAllocMaxDevices] = {nullptr};
}  // namespace

static __device__ __align__(256) float g_msda_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

extern "C" int rfdetr_msda_backward_noalloc(void *stream, const void *value, int value_dtype,
                                            const int64_t *spatial_shapes, const int64_t *level_start_index,
                                            const float *sampling_locations, const void *attention_weights,
                                            int weight_dtype, const void *grad_output, int grad_output_dtype,
                                            void *grad_value, float *grad_sampling_locations,
                                            void *grad_attention_weights, int64_t batch, int64_t n_heads,
                                            int64_t head_dim, int64_t len_query, int64_t n_levels,
                                            int64_t n_points) {
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
    if (value_dtype == RFDETR_BF16) {
        Geom g;
        const int st = validate(spatial_shapes, level_start_index, batch, n_heads, head_dim, len_query, n_levels,
                                n_points, g);
        if (st) return st;
        const size_t need = rfdetr_msda_backward_workspace_size(value_dtype, batch, n_heads, head_dim, g.Lv);
        if (need > kNoAllocScratchBytes) return RFDETR_ERR_CAPACITY;
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return RFDETR_ERR_CUDA;
        {
            std::lock_guard<std::mutex> lock(g_noalloc_mutex);
            if (!g_noalloc_address[dev]) {
                void *address = nullptr;
                if (cudaGetSymbolAddress(&address, g_msda_noalloc_scratch) != cudaSuccess || !address)
                    return RFDETR_ERR_CUDA;
                g_noalloc_address[dev] = address;
            }
            scratch = g_noalloc_address[dev];
        }
        scratch_bytes = kNoAllocScratchBytes;
    }
    return rfdetr_msda_backward(stream, value, value_dtype, spatial_shapes, level_start_index, sampling_locations,
                                attention_weights, weight_dtype, grad_output, grad_output_dtype, grad_value,
                                grad_sampling_locations, grad_attention_weights, scratch, scratch_bytes, batch,
                                n_heads, head_dim, len_query, n_levels, n_points);
}
