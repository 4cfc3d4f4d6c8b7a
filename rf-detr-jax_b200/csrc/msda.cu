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
#include <initializer_list>
#include <type_traits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "tma.cuh"

#include <cudaTypedefs.h>

namespace rfdetr {

bool encode_tensor_map(CUtensorMap *map, CUtensorMapDataType dtype, int rank, const void *base,
                       const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                       CUtensorMapSwizzle swizzle) {
    static const PFN_cuTensorMapEncodeTiled_v12000 encode = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }();
    if (!encode || rank < 1 || rank > 5) return false;
    cuuint64_t d[5], st[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) st[i] = strides_bytes[i];
    }
    return encode(map, dtype, (cuuint32_t)rank, const_cast<void *>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace rfdetr

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
// Two of the steps are fused without changing a bit: 2*loc is exact, so fma(2, loc, -1) rounds
// once like 2*loc - 1; halving is exact, so fma(u, 0.5, -0.5) = round(u - 1) / 2.
__device__ __forceinline__ void sample_coords(float lx, float ly, float wf, float hf, float &ix,
                                              float &iy) {
    const float gx = __fmaf_rn(2.f, lx, -1.f);
    const float gy = __fmaf_rn(2.f, ly, -1.f);
    ix = __fmaf_rn(__fmul_rn(__fadd_rn(gx, 1.f), wf), 0.5f, -0.5f);
    iy = __fmaf_rn(__fmul_rn(__fadd_rn(gy, 1.f), hf), 0.5f, -0.5f);
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
__global__ void __launch_bounds__(kMaxThreads, 2)
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
                if (!active_lane) continue;
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
                if (t.mask != 0xFu) {
                    // Out-of-range corners: the reference reads their clipped rows and weights them
                    // by 0 (ops.py:98-106,123-128), which changes the sum only where a row holds
                    // inf/NaN (0 * inf = NaN).
                    const float fx0 = floorf(ix), fy0 = floorf(iy);
                    const int cx[2] = {(int)fminf(fmaxf(fx0, 0.f), wf - 1.f), (int)fminf(fmaxf(fx0 + 1.f, 0.f), wf - 1.f)};
                    const int cy[2] = {(int)fminf(fmaxf(fy0, 0.f), hf - 1.f), (int)fminf(fmaxf(fy0 + 1.f, 0.f), hf - 1.f)};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (t.mask & (1u << k)) continue;
                        load_vec<TV, VEC, kNC>(vl + ((size_t)cy[k >> 1] * W + cx[k & 1]) * g.D, v);
#pragma unroll
                        for (int i = 0; i < VEC; ++i) s[i] = fma((AT)0, (AT)v[i], s[i]);
                    }
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
                // Corner rows at the reference's clipped positions (ops.py:98-106); an out-of-range
                // corner's row enters multiplied by its 0 mask, as in the reference (0 * inf = NaN).
                long long offs[4] = {0, 0, 0, 0};
                if (ok) {
                    const float fx0 = floorf(ix), fy0 = floorf(iy);
                    const int cx0 = (int)fminf(fmaxf(fx0, 0.f), wf - 1.f), cx1 = (int)fminf(fmaxf(fx0 + 1.f, 0.f), wf - 1.f);
                    const int cy0 = (int)fminf(fmaxf(fy0, 0.f), hf - 1.f), cy1 = (int)fminf(fmaxf(fy0 + 1.f, 0.f), hf - 1.f);
                    offs[0] = (long long)cy0 * W + cx0;
                    offs[1] = (long long)cy0 * W + cx1;
                    offs[2] = (long long)cy1 * W + cx0;
                    offs[3] = (long long)cy1 * W + cx1;
                }
                float v00[VEC], v10[VEC], v01[VEC], v11[VEC];
#pragma unroll
                for (int i = 0; i < VEC; ++i) v00[i] = v10[i] = v01[i] = v11[i] = 0.f;
                if (tap) {
                    load_vec<TV, VEC, kNC>(vl + offs[0] * g.D, v00);
                    load_vec<TV, VEC, kNC>(vl + offs[1] * g.D, v10);
                    load_vec<TV, VEC, kNC>(vl + offs[2] * g.D, v01);
                    load_vec<TV, VEC, kNC>(vl + offs[3] * g.D, v11);
                    if (t.mask != 0xFu) {
#pragma unroll
                        for (int i = 0; i < VEC; ++i) {
                            if (!(t.mask & 1u)) v00[i] *= 0.f;
                            if (!(t.mask & 2u)) v10[i] *= 0.f;
                            if (!(t.mask & 4u)) v01[i] *= 0.f;
                            if (!(t.mask & 8u)) v11[i] *= 0.f;
                        }
                    }
                }

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
                if (!tap) continue;
                // A masked corner adds 0 * a * w * g to its clipped row: nothing, unless a or g is
                // not finite (then NaN, as the reference's scatter-add gives).
                unsigned scatter = t.mask;
                if (t.mask != 0xFu) {
                    bool gbad = false;
#pragma unroll
                    for (int i = 0; i < VEC; ++i) gbad |= !(fabsf(gr[i]) <= 3.4028235e38f);
                    if (gbad || !(fabsf(a) <= 3.4028235e38f)) scatter = 0xFu;
                }
                if (scatter == 0u) continue;

                const float mk[4] = {t.mask & 1u ? 1.f : 0.f, t.mask & 2u ? 1.f : 0.f, t.mask & 4u ? 1.f : 0.f,
                                     t.mask & 8u ? 1.f : 0.f};
                const float c[4] = {a * w00 * mk[0], a * w10 * mk[1], a * w01 * mk[2], a * w11 * mk[3]};
                if constexpr (SMEM_ACC) {
                    float *sb = gsm + hs * slab + (size_t)lv.s[l] * g.D + chunk;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (!(scatter & (1u << k))) continue;
                        float *p = sb + offs[k] * g.D;
#pragma unroll
                        for (int i = 0; i < VEC; ++i) atomicAdd(p + ((i + rot) & (VEC - 1)), c[k] * grot[i]);
                    }
                } else {
                    float *gb = gdst + hs * slab + (size_t)lv.s[l] * g.D + chunk;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (!(scatter & (1u << k))) continue;
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

// Tuning overrides for experiments ("hsub,stage,acc,threads,waves"; the knobs of common.cuh).
struct Tune {
    int hsub = 0, stage = -1, acc = -1, threads = 0, waves = 0;
};

Tune read_tune(Knob k) {
    Tune t;
    const KnobValue kv = knob(k);
    int *fields[5] = {&t.hsub, &t.stage, &t.acc, &t.threads, &t.waves};
    for (int i = 0; i < kv.count; ++i) *fields[i] = kv.v[i];
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
    // Every tensor must hold fewer than 2^31 elements.  The products are formed factor by factor
    // with a bound check before each multiply, so no intermediate can overflow.
    const long long lim = (1LL << 31) - 1;
    auto within = [lim](std::initializer_list<long long> factors) {
        long long p = 1;
        for (long long f : factors) {
            if (f < 0 || (f > 0 && p > lim / f)) return false;
            p *= f;
        }
        return true;
    };
    if (B > lim || H > lim || D > lim || Lq > lim || total > lim) return RFDETR_ERR_SHAPE;
    if (!within({B, H, total, D}) || !within({B, Lq, H, L, P, 2}) || !within({B, Lq, H, D})) return RFDETR_ERR_SHAPE;
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

// ------------------------------------------------------------------------------------------
// Slab-resident forward.  Used when the value rows of a head group fit in shared memory and the
// location/weight rows of a (query, head group) are 4-byte-granular segments.  The slabs are
// copied once per CTA with cp.async; location/weight tiles of `tq` queries are double-buffered
// with cp.async so their HBM latency overlaps the previous tile's gathers.  Taps are branch-free:
// all four corners are read at the reference's clipped indices (ops.py:103-106) and out-of-range
// corners get weight 0 (ops.py:123-128), which also reproduces the reference's NaN/inf
// propagation from value entries.
// ------------------------------------------------------------------------------------------
constexpr int kSlabThreads = 512;

__device__ __forceinline__ void cp_async_bytes(void *smem_dst, const void *gmem_src, int bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
    if (bytes == 16) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem_src) : "memory");
    } else if (bytes == 8) {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem_src) : "memory");
    } else {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem_src) : "memory");
    }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ float2 bf16x2_lo_hi(unsigned u) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

struct SlabPlan {
    int hsub, tq, q_per_cta, gl, ga;  // gl/ga: granule bytes for location / weight segments
    size_t slab_bytes, tile_bytes, smem;
};

// Branch-free taps of one sample: clipped corner positions (element offsets in units of rows)
// and the attention-weighted, masked bilinear coefficients.  `ok` is false for non-finite
// positions (the reference yields NaN there).
struct FlatTaps {
    int p00, p10, p01, p11;
    float c00, c10, c01, c11;
    bool ok;
};

// floor(x) as an int and as a float for |x| < 2^22 without the XU pipe: adding 1.5 * 2^23
// rounds to the nearest integer (exactly representable there), and a rounded-up result steps
// down by one.  Callers clamp x into a small range first.
__device__ __forceinline__ void floor_split(float x, int &xi, float &xf) {
    const float t = __fadd_rn(x, 12582912.f);
    const float r = __fsub_rn(t, 12582912.f);
    const int i = __float_as_int(t) - 0x4B400000;
    const bool up = r > x;
    xf = up ? r - 1.f : r;
    xi = up ? i - 1 : i;
}

// Fractional weights, clipped corner indices and 0/1 masks of one axis.  Clamping x into
// [-2, size + 1] changes neither the in-bounds corners nor their weights.
struct Axis {
    float w0, w1, m0, m1;
    int c0, c1;
    int i0;  // floor of the clamped coordinate, in [-2, size + 1]
};
__device__ __forceinline__ Axis axis_taps(float x, float sizef, int size) {
    Axis a;
    const float xc = fminf(fmaxf(x, -2.f), sizef + 1.f);
    int i0;
    float f0;
    floor_split(xc, i0, f0);
    a.i0 = i0;
    a.w1 = xc - f0;
    a.w0 = 1.f - a.w1;
    a.m0 = (unsigned)i0 < (unsigned)size ? 1.f : 0.f;
    a.m1 = (unsigned)(i0 + 1) < (unsigned)size ? 1.f : 0.f;
    a.c0 = min(max(i0, 0), size - 1);
    a.c1 = min(max(i0 + 1, 0), size - 1);
    return a;
}

__device__ __forceinline__ FlatTaps flat_taps(float lx, float ly, float a, float Wf, float Hf, int W, int H) {
    FlatTaps t;
    float ix, iy;
    sample_coords(lx, ly, Wf, Hf, ix, iy);
    t.ok = fabsf(ix) <= 3.0e38f && fabsf(iy) <= 3.0e38f;
    const Axis ax = axis_taps(ix, Wf, W), ay = axis_taps(iy, Hf, H);
    const float ax0 = a * (ax.w0 * ax.m0), ax1 = a * (ax.w1 * ax.m1);
    const float ay0 = ay.w0 * ay.m0, ay1 = ay.w1 * ay.m1;
    t.c00 = ax0 * ay0;
    t.c10 = ax1 * ay0;
    t.c01 = ax0 * ay1;
    t.c11 = ax1 * ay1;
    t.p00 = ay.c0 * W + ax.c0;
    t.p10 = ay.c0 * W + ax.c1;
    t.p01 = ay.c1 * W + ax.c0;
    t.p11 = ay.c1 * W + ax.c1;
    return t;
}

// Accumulates coef * value-chunk into acc.  bf16: 8 channels (one 16-byte row chunk) into four
// packed float pairs; f32: 4 channels into doubles.
template <typename TV> struct SlabAcc;
template <> struct SlabAcc<bf16> {
    static constexpr int VEC = 8;
    float2 v[4];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = make_float2(0.f, 0.f);
    }
    __device__ __forceinline__ void add(float c, const uint4 &r) {
        const float2 cc = make_float2(c, c);
        v[0] = __ffma2_rn(cc, bf16x2_lo_hi(r.x), v[0]);
        v[1] = __ffma2_rn(cc, bf16x2_lo_hi(r.y), v[1]);
        v[2] = __ffma2_rn(cc, bf16x2_lo_hi(r.z), v[2]);
        v[3] = __ffma2_rn(cc, bf16x2_lo_hi(r.w), v[3]);
    }
    __device__ __forceinline__ void poison() {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
    }
    __device__ __forceinline__ void to_float(float *f) const {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = v[i].x;
            f[2 * i + 1] = v[i].y;
        }
    }
};
template <> struct SlabAcc<float> {
    static constexpr int VEC = 4;
    double v[4];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = 0.0;
    }
    __device__ __forceinline__ void add(float c, const uint4 &r) {
        const double cd = c;
        v[0] = fma(cd, (double)__uint_as_float(r.x), v[0]);
        v[1] = fma(cd, (double)__uint_as_float(r.y), v[1]);
        v[2] = fma(cd, (double)__uint_as_float(r.z), v[2]);
        v[3] = fma(cd, (double)__uint_as_float(r.w), v[3]);
    }
    __device__ __forceinline__ void poison() {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = (double)__int_as_float(0x7fc00000);
    }
    __device__ __forceinline__ void to_float(float *f) const {
#pragma unroll
        for (int i = 0; i < 4; ++i) f[i] = (float)v[i];
    }
};

// Issues the cp.async copies of one tile's location and weight segments.  Granule counts per
// query are powers of two (hsub, LP, sizes and granules all are), so indices split by shifts.
template <typename TW, int LP>
__device__ __forceinline__ void issue_tile(const float *loc, const TW *attn, float *sloc, TW *sattn, const Geom &g,
                                           int b, int h0, int hsub, int qa, int nq, int gl, int ga) {
    const int lbytes = hsub * LP * 8, abytes = hsub * LP * (int)sizeof(TW);
    const int ls = 31 - __clz(lbytes / gl), as = 31 - __clz(abytes / ga);
    const size_t row0 = ((size_t)b * g.Lq + qa) * g.H + h0;
    const size_t rstride = (size_t)g.H;
    for (int i = threadIdx.x; i < (nq << ls); i += blockDim.x) {
        const int qi = i >> ls, j = i & ((1 << ls) - 1);
        cp_async_bytes(reinterpret_cast<char *>(sloc) + (size_t)qi * lbytes + j * gl,
                       reinterpret_cast<const char *>(loc + (row0 + qi * rstride) * LP * 2) + j * gl, gl);
    }
    for (int i = threadIdx.x; i < (nq << as); i += blockDim.x) {
        const int qi = i >> as, j = i & ((1 << as) - 1);
        cp_async_bytes(reinterpret_cast<char *>(sattn) + (size_t)qi * abytes + j * ga,
                       reinterpret_cast<const char *>(attn + (row0 + qi * rstride) * LP) + j * ga, ga);
    }
}

template <typename TV, typename TW, int LP>
__global__ void __launch_bounds__(kSlabThreads, 2)
msda_forward_slab_kernel(const TV *__restrict__ value, const float *__restrict__ loc, const TW *__restrict__ attn,
                         typename OutOf<TV, TW>::T *__restrict__ out, const Geom g, const SlabPlan sp) {
    using TO = typename OutOf<TV, TW>::T;
    using Acc = SlabAcc<TV>;
    constexpr int VEC = Acc::VEC;
    extern __shared__ __align__(16) unsigned char smem[];

    const int hsub = sp.hsub;
    const int hshift = 31 - __clz(hsub);
    const int groups_per_image = g.H >> hshift;
    const int b = blockIdx.y / groups_per_image;
    const int h0 = (blockIdx.y - b * groups_per_image) << hshift;
    const int q0 = blockIdx.x * sp.q_per_cta;
    const int q1 = min(q0 + sp.q_per_cta, g.Lq);

    // Stage the head group's value slabs (contiguous in [B*H, Lv, D]).
    const size_t slab_elems = (size_t)g.Lv * g.D;
    const TV *vsrc = value + ((size_t)b * g.H + h0) * slab_elems;
    const int n16 = (int)(sp.slab_bytes * hsub / 16);
    for (int i = threadIdx.x; i < n16; i += blockDim.x)
        cp_async_bytes(smem + (size_t)i * 16, reinterpret_cast<const char *>(vsrc) + (size_t)i * 16, 16);
    unsigned char *tiles = smem + ((sp.slab_bytes * hsub + 15) & ~(size_t)15);
    const size_t lbytes = (size_t)sp.tq * hsub * LP * 8;
    const size_t abytes = (((size_t)sp.tq * hsub * LP * sizeof(TW)) + 15) & ~(size_t)15;
    float *const sloc0 = reinterpret_cast<float *>(tiles);
    float *const sloc1 = reinterpret_cast<float *>(tiles + lbytes + abytes);
    TW *const sattn0 = reinterpret_cast<TW *>(tiles + lbytes);
    TW *const sattn1 = reinterpret_cast<TW *>(tiles + 2 * lbytes + abytes);
    const int ntiles = (q1 - q0 + sp.tq - 1) / sp.tq;
    if (ntiles > 0) issue_tile<TW, LP>(loc, attn, sloc0, sattn0, g, b, h0, hsub, q0, min(sp.tq, q1 - q0), sp.gl, sp.ga);
    cp_async_commit();

    // Per-sample level geometry, held in registers (LP is a compile-time constant).
    int kw[LP], kh[LP];
    float kwf[LP], khf[LP];
    unsigned koff[LP];
    const unsigned rowbytes = (unsigned)(g.D * sizeof(TV));
#pragma unroll
    for (int k = 0; k < LP; ++k) {
        const int l = k / g.P;
        kw[k] = g.lw[l];
        kh[k] = g.lh[l];
        kwf[k] = (float)kw[k];
        khf[k] = (float)kh[k];
        koff[k] = (unsigned)g.ls[l] * rowbytes;
    }

    const int team = g.D / VEC;  // power of two, <= 32
    const int tshift = 31 - __clz(team);
    const int lane_t = threadIdx.x & (team - 1);
    const int tix = threadIdx.x >> tshift;
    const int nteams = blockDim.x >> tshift;
    const unsigned slab_base = (unsigned)__cvta_generic_to_shared(smem) + lane_t * 16u;
    const int hd = g.H * g.D;

    for (int t = 0; t < ntiles; ++t) {
        const int qa = q0 + t * sp.tq;
        const int nq = min(sp.tq, q1 - qa);
        if (t + 1 < ntiles) {
            const int qn = qa + sp.tq;
            issue_tile<TW, LP>(loc, attn, (t & 1) ? sloc0 : sloc1, (t & 1) ? sattn0 : sattn1, g, b, h0, hsub, qn,
                               min(sp.tq, q1 - qn), sp.gl, sp.ga);
            cp_async_commit();
            cp_async_wait_one();
        } else {
            cp_async_wait_all();
        }
        __syncthreads();
        const float2 *tl = reinterpret_cast<const float2 *>((t & 1) ? sloc1 : sloc0);
        const TW *ta = (t & 1) ? sattn1 : sattn0;
        TO *otile = out + ((size_t)b * g.Lq + qa) * hd + (size_t)h0 * g.D + lane_t * VEC;
        const int items = nq << hshift;
        for (int it = tix; it < items; it += nteams) {
            const int qi = it >> hshift, hs = it & (hsub - 1);
            const float2 *lp = tl + it * LP;
            const TW *ap = ta + it * LP;
            const unsigned hbase = slab_base + (unsigned)hs * (unsigned)sp.slab_bytes;
            Acc acc;
            acc.zero();
            bool finite = true;
#pragma unroll
            for (int k = 0; k < LP; ++k) {
                const float2 xy = lp[k];
                const FlatTaps tp = flat_taps(xy.x, xy.y, to_f32(ap[k]), kwf[k], khf[k], kw[k], kh[k]);
                finite = finite && tp.ok;
                const unsigned lbase = hbase + koff[k];
                uint4 r00, r10, r01, r11;
                asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(r00.x), "=r"(r00.y), "=r"(r00.z), "=r"(r00.w) : "r"(lbase + tp.p00 * rowbytes));
                asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(r10.x), "=r"(r10.y), "=r"(r10.z), "=r"(r10.w) : "r"(lbase + tp.p10 * rowbytes));
                asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(r01.x), "=r"(r01.y), "=r"(r01.z), "=r"(r01.w) : "r"(lbase + tp.p01 * rowbytes));
                asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(r11.x), "=r"(r11.y), "=r"(r11.z), "=r"(r11.w) : "r"(lbase + tp.p11 * rowbytes));
                acc.add(tp.c00, r00);
                acc.add(tp.c10, r10);
                acc.add(tp.c01, r01);
                acc.add(tp.c11, r11);
            }
            if (!finite) acc.poison();
            float o[VEC];
            acc.to_float(o);
            store_vec<TO, VEC>(otile + (unsigned)(qi * hd + hs * g.D), o);
        }
        __syncthreads();
    }
}

// Plans the slab path; returns false when its preconditions do not hold.
template <typename TV, typename TW>
bool plan_forward_slab(const Geom &g, const void *value, const float *loc, const void *attn, const void *out,
                       int optin, SlabPlan &sp) {
    const int es = (int)sizeof(TV), esw = (int)sizeof(TW);
    const int LP = g.L * g.P;
    if (!(LP == 1 || LP == 2 || LP == 4 || LP == 8)) return false;
    if ((g.D * es) % 16 != 0) return false;
    const int team = g.D * es / 16;
    if (team > 32 || (team & (team - 1))) return false;
    if (!aligned(value, 16) || !aligned(out, 16)) return false;
    const size_t slab = (size_t)g.Lv * g.D * es;
    if (slab % 16 != 0) return false;
    const Tune tune = read_tune(kKnobMsdaSlabFwd);
    if (tune.stage == 0) return false;
    const size_t budget = 100 * 1024;
    int best = 0;
    for (int hsub = 1; hsub <= g.H && hsub <= 32; hsub *= 2) {
        if (g.H % hsub) break;
        if ((size_t)hsub * slab > budget) break;
        best = hsub;
        if ((size_t)hsub * slab * 2 > 80 * 1024) break;  // stop growing once the group is ~40 KB
    }
    if (tune.hsub > 0) best = tune.hsub;
    if (best == 0 || g.H % best) return false;
    sp.hsub = best;
    // Granules for the location / weight segments of one (query, head group).
    auto granule = [](long long seg_bytes, long long row_stride_bytes, long long head_off_bytes,
                      const void *base) -> int {
        for (int gsz = 16; gsz >= 4; gsz >>= 1) {
            if (seg_bytes % gsz == 0 && row_stride_bytes % gsz == 0 && head_off_bytes % gsz == 0 && aligned(base, gsz))
                return gsz;
        }
        return 0;
    };
    const long long lseg = (long long)sp.hsub * LP * 8, aseg = (long long)sp.hsub * LP * esw;
    sp.gl = granule(lseg, (long long)g.H * LP * 8, lseg, loc);
    sp.ga = granule(aseg, (long long)g.H * LP * esw, aseg, attn);
    if (!sp.gl || !sp.ga) return false;
    sp.slab_bytes = slab;
    auto size_for = [&](int tq) {
        sp.tq = tq;
        const size_t lbytes = (size_t)sp.tq * sp.hsub * LP * 8;
        const size_t abytes = (((size_t)sp.tq * sp.hsub * LP * esw) + 15) & ~(size_t)15;
        sp.tile_bytes = lbytes + abytes;
        sp.smem = ((slab * sp.hsub + 15) & ~(size_t)15) + 2 * sp.tile_bytes;
    };
    // Tiles of 256 queries (fewer tile rounds: barriers and copy waits) while the CTA still fits
    // two to an SM -- 18.6 vs 20.6 us at config 2 -- else 128.  The threads field of the tuning
    // variable overrides the tile length.
    if (tune.threads > 0) {
        size_for(tune.threads);
    } else {
        size_for(256);
        if (sp.smem > 113 * 1024) size_for(128);
    }
    if (sp.smem > (size_t)optin) return false;
    return true;
}

template <typename TV, typename TW, int LP>
int launch_forward_slab(const Geom &g, SlabPlan &sp, const void *value, const float *loc, const void *attn,
                        void *out, cudaStream_t stream, int waves) {
    auto kernel = msda_forward_slab_kernel<TV, TW, LP>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp.smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kSlabThreads, sp.smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    per_sm = std::max(per_sm, 1);
    const long long groups = (long long)g.B * (g.H / sp.hsub);
    const long long target = (long long)num_sms() * per_sm * std::max(waves, 1);
    long long per_group = std::max<long long>(1, target / std::max<long long>(groups, 1));
    long long qpc = (g.Lq + per_group - 1) / per_group;
    qpc = ((qpc + sp.tq - 1) / sp.tq) * sp.tq;
    sp.q_per_cta = (int)std::max<long long>(qpc, sp.tq);
    if (groups > 65535) return RFDETR_ERR_SHAPE;
    dim3 grid((unsigned)ceil_div(g.Lq, sp.q_per_cta), (unsigned)groups);
    kernel<<<grid, kSlabThreads, sp.smem, stream>>>(static_cast<const TV *>(value), loc, static_cast<const TW *>(attn),
                                                    static_cast<typename OutOf<TV, TW>::T *>(out), g, sp);
    return launch_status();
}

// Returns -1 when the slab path does not apply.
template <typename TV, typename TW>
int try_forward_slab(const Geom &g, const void *value, const float *loc, const void *attn, void *out,
                     cudaStream_t stream) {
    SlabPlan sp;
    if (!plan_forward_slab<TV, TW>(g, value, loc, attn, out, max_smem_optin(), sp)) return -1;
    const int waves = std::max(1, read_tune(kKnobMsdaSlabFwd).waves);
    switch (g.L * g.P) {
        case 1: return launch_forward_slab<TV, TW, 1>(g, sp, value, loc, attn, out, stream, waves);
        case 2: return launch_forward_slab<TV, TW, 2>(g, sp, value, loc, attn, out, stream, waves);
        case 4: return launch_forward_slab<TV, TW, 4>(g, sp, value, loc, attn, out, stream, waves);
        case 8: return launch_forward_slab<TV, TW, 8>(g, sp, value, loc, attn, out, stream, waves);
        default: return -1;
    }
}

// ------------------------------------------------------------------------------------------
// Slab-resident backward for bf16 values ("owner computes").  One CTA owns the value rows of
// one (image, head) and all its queries, processed in chunks of `tq` queries:
//   P1: each team handles one (query) item: it reads the 4 corner rows of every sample from the
//       shared-memory slab, forms the corner dot products G_c = g . v_c, reduces them across the
//       team and writes grad_weight and grad_location; then it files one record
//       (coefficient a*w_c, item) per in-bounds corner into the bin of that value position
//       (an integer shared-memory atomic hands out the slot).
//   P2: the owner of each (position, 8-channel chunk) walks its bin and accumulates
//       coefficient x grad_output row chunk in registers.
// Bins hold `cap` records; a record that finds its bin full is added directly into a float32
// shared-memory overflow slab instead (slow but exact).  After the last chunk each owner adds its
// overflow entries and writes its grad_value chunk once, rounded to bf16: no workspace, no
// atomics on the value gradient in the common case, no second pass.
// ------------------------------------------------------------------------------------------
constexpr int kBinThreads = 512;

struct BinPlan {
    int tq, cap, gl, ga, gg;  // tile queries, bin capacity, granule bytes of loc / attn / grad_out
    size_t slab_bytes, smem;
};

template <typename TW, typename TG, int LP>
__device__ __forceinline__ void issue_bwd_tile(const float *loc, const TW *attn, const TG *gout, float *sloc, TW *sattn,
                                               TG *sg, const Geom &g, int b, int h, int qa, int nq, int gl, int ga,
                                               int gg, int gstride = 0) {
    const int lbytes = LP * 8, abytes = LP * (int)sizeof(TW), gbytes = g.D * (int)sizeof(TG);
    const int gdst = gstride > 0 ? gstride : gbytes;
    const int ls = 31 - __clz(lbytes / gl), as = 31 - __clz(abytes / ga), gs = 31 - __clz(gbytes / gg);
    const size_t row0 = ((size_t)b * g.Lq + qa) * g.H + h;
    const size_t rstride = (size_t)g.H;
    for (int i = threadIdx.x; i < (nq << ls); i += blockDim.x) {
        const int qi = i >> ls, j = i & ((1 << ls) - 1);
        cp_async_bytes(reinterpret_cast<char *>(sloc) + (size_t)qi * lbytes + j * gl,
                       reinterpret_cast<const char *>(loc + (row0 + qi * rstride) * LP * 2) + j * gl, gl);
    }
    for (int i = threadIdx.x; i < (nq << as); i += blockDim.x) {
        const int qi = i >> as, j = i & ((1 << as) - 1);
        cp_async_bytes(reinterpret_cast<char *>(sattn) + (size_t)qi * abytes + j * ga,
                       reinterpret_cast<const char *>(attn + (row0 + qi * rstride) * LP) + j * ga, ga);
    }
    for (int i = threadIdx.x; i < (nq << gs); i += blockDim.x) {
        const int qi = i >> gs, j = i & ((1 << gs) - 1);
        cp_async_bytes(reinterpret_cast<char *>(sg) + (size_t)qi * gdst + j * gg,
                       reinterpret_cast<const char *>(gout + (row0 + qi * rstride) * g.D) + j * gg, gg);
    }
}

// Dot of 8 bf16 value channels with 8 float gradient channels (packed pairs).
__device__ __forceinline__ float dot8(const uint4 &v, const float2 *gp) {
    float2 s = __fmul2_rn(bf16x2_lo_hi(v.x), gp[0]);
    s = __ffma2_rn(bf16x2_lo_hi(v.y), gp[1], s);
    s = __ffma2_rn(bf16x2_lo_hi(v.z), gp[2], s);
    s = __ffma2_rn(bf16x2_lo_hi(v.w), gp[3], s);
    return s.x + s.y;
}

template <typename TG>
__device__ __forceinline__ void load_g8(unsigned saddr, float2 *gp) {
    if constexpr (sizeof(TG) == 2) {
        uint4 r;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(saddr));
        gp[0] = bf16x2_lo_hi(r.x);
        gp[1] = bf16x2_lo_hi(r.y);
        gp[2] = bf16x2_lo_hi(r.z);
        gp[3] = bf16x2_lo_hi(r.w);
    } else {
        float4 a, c;
        asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(a.x), "=f"(a.y), "=f"(a.z), "=f"(a.w) : "r"(saddr));
        asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(c.x), "=f"(c.y), "=f"(c.z), "=f"(c.w) : "r"(saddr + 16));
        gp[0] = make_float2(a.x, a.y);
        gp[1] = make_float2(a.z, a.w);
        gp[2] = make_float2(c.x, c.y);
        gp[3] = make_float2(c.z, c.w);
    }
}

__device__ __forceinline__ uint4 lds128(unsigned addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}

template <typename TW, int LP, int OWN>
__global__ void __launch_bounds__(kBinThreads, 1)
msda_backward_bins_kernel(const bf16 *__restrict__ value, const float *__restrict__ loc, const TW *__restrict__ attn,
                          const typename OutOf<bf16, TW>::T *__restrict__ grad_out, bf16 *__restrict__ grad_value,
                          float *__restrict__ grad_loc, TW *__restrict__ grad_attn, const Geom g, const BinPlan bp) {
    using TG = typename OutOf<bf16, TW>::T;
    extern __shared__ __align__(16) unsigned char smem[];
    const int bh = blockIdx.x;  // b * H + h
    const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
    const int Lv = g.Lv, D = g.D;
    const unsigned rowbytes = (unsigned)(D * 2);
    const int chunks = D / 8;  // 8-channel chunks per row == team size

    // Shared-memory layout.
    unsigned char *p = smem;
    unsigned char *slab = p;
    p += (bp.slab_bytes + 15) & ~(size_t)15;
    const size_t lbytes = (size_t)bp.tq * LP * 8;
    const size_t abytes = ((size_t)bp.tq * LP * sizeof(TW) + 15) & ~(size_t)15;
    const size_t gbytes = (size_t)bp.tq * D * sizeof(TG);
    float *const sloc0 = reinterpret_cast<float *>(p);
    TW *const sattn0 = reinterpret_cast<TW *>(p + lbytes);
    TG *const sg0 = reinterpret_cast<TG *>(p + lbytes + abytes);
    p += lbytes + abytes + gbytes;
    float *const sloc1 = reinterpret_cast<float *>(p);
    TW *const sattn1 = reinterpret_cast<TW *>(p + lbytes);
    TG *const sg1 = reinterpret_cast<TG *>(p + lbytes + abytes);
    p += lbytes + abytes + gbytes;
    uint2 *bins = reinterpret_cast<uint2 *>(p);
    p += (size_t)Lv * bp.cap * sizeof(uint2);
    int *counts = reinterpret_cast<int *>(p);
    p += ((size_t)Lv * sizeof(int) + 15) & ~(size_t)15;
    float *ovf = reinterpret_cast<float *>(p);

    // Stage the slab, clear counts and the overflow slab.
    const bf16 *vsrc = value + (size_t)bh * Lv * D;
    const int n16 = (int)(bp.slab_bytes / 16);
    for (int i = threadIdx.x; i < n16; i += blockDim.x)
        cp_async_bytes(slab + (size_t)i * 16, reinterpret_cast<const char *>(vsrc) + (size_t)i * 16, 16);
    for (int i = threadIdx.x; i < Lv; i += blockDim.x) counts[i] = 0;
    for (int i = threadIdx.x; i < Lv * D; i += blockDim.x) ovf[i] = 0.f;
    const int ntiles = (g.Lq + bp.tq - 1) / bp.tq;
    if (ntiles > 0)
        issue_bwd_tile<TW, TG, LP>(loc, attn, grad_out, sloc0, sattn0, sg0, g, b, h, 0, min(bp.tq, g.Lq), bp.gl,
                                   bp.ga, bp.gg);
    cp_async_commit();

    int kw[LP], kh[LP];
    float kwf[LP], khf[LP];
    unsigned koff[LP], kpos[LP];
#pragma unroll
    for (int k = 0; k < LP; ++k) {
        const int l = k / g.P;
        kw[k] = g.lw[l];
        kh[k] = g.lh[l];
        kwf[k] = (float)kw[k];
        khf[k] = (float)kh[k];
        kpos[k] = (unsigned)g.ls[l];
        koff[k] = kpos[k] * rowbytes;
    }
    const int team = chunks;
    const int tshift = 31 - __clz(team);
    const int lane_t = threadIdx.x & (team - 1);
    const int tix = threadIdx.x >> tshift;
    const int nteams = blockDim.x >> tshift;
    const unsigned slab_s = (unsigned)__cvta_generic_to_shared(slab) + lane_t * 16u;
    const float qnan = __int_as_float(0x7fc00000);

    // Owner accumulators: owner-lane o = position * chunks + chunk, o = threadIdx.x + j * blockDim.
    float2 acc[OWN][4];
#pragma unroll
    for (int j = 0; j < OWN; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = make_float2(0.f, 0.f);
    const int owners = Lv * chunks;

    for (int t = 0; t < ntiles; ++t) {
        const int qa = t * bp.tq;
        const int nq = min(bp.tq, g.Lq - qa);
        if (t + 1 < ntiles) {
            const int qn = qa + bp.tq;
            const bool odd = (t & 1) != 0;
            issue_bwd_tile<TW, TG, LP>(loc, attn, grad_out, odd ? sloc0 : sloc1, odd ? sattn0 : sattn1, odd ? sg0 : sg1,
                                       g, b, h, qn, min(bp.tq, g.Lq - qn), bp.gl, bp.ga, bp.gg);
            cp_async_commit();
            cp_async_wait_one();
        } else {
            cp_async_wait_all();
        }
        __syncthreads();
        const bool odd = (t & 1) != 0;
        const float2 *tl = reinterpret_cast<const float2 *>(odd ? sloc1 : sloc0);
        const TW *ta = odd ? sattn1 : sattn0;
        const TG *tg = odd ? sg1 : sg0;
        const unsigned tg_s = (unsigned)__cvta_generic_to_shared(tg);

        // P1: one item (query) per team; every lane of a warp runs the same trip count.
        for (int base = 0; base < nq; base += nteams) {
            const int it = base + tix;
            const bool live = it < nq;
            const int iq = live ? it : 0;
            float2 gp[4];
            load_g8<TG>(tg_s + (unsigned)(iq * D * (int)sizeof(TG)) + lane_t * 8u * (unsigned)sizeof(TG), gp);
            const size_t row = ((size_t)b * g.Lq + qa + iq) * g.H + h;
#pragma unroll
            for (int k = 0; k < LP; ++k) {
                const float2 xy = tl[iq * LP + k];
                const float a = to_f32(ta[iq * LP + k]);
                const int W = kw[k];
                float ix, iy;
                sample_coords(xy.x, xy.y, kwf[k], khf[k], ix, iy);
                const bool ok = fabsf(ix) <= 3.0e38f && fabsf(iy) <= 3.0e38f;
                const Axis ax = axis_taps(ix, kwf[k], W), ay = axis_taps(iy, khf[k], kh[k]);
                const float wx0 = ax.w0, wx1 = ax.w1, wy0 = ay.w0, wy1 = ay.w1;
                const float mx0 = ax.m0, mx1 = ax.m1, my0 = ay.m0, my1 = ay.m1;
                const int p00 = ay.c0 * W + ax.c0, p10 = ay.c0 * W + ax.c1;
                const int p01 = ay.c1 * W + ax.c0, p11 = ay.c1 * W + ax.c1;
                const unsigned lb = slab_s + koff[k];
                float G00 = dot8(lds128(lb + p00 * rowbytes), gp);
                float G10 = dot8(lds128(lb + p10 * rowbytes), gp);
                float G01 = dot8(lds128(lb + p01 * rowbytes), gp);
                float G11 = dot8(lds128(lb + p11 * rowbytes), gp);
                for (int o = team >> 1; o > 0; o >>= 1) {
                    G00 += __shfl_xor_sync(0xffffffffu, G00, o);
                    G10 += __shfl_xor_sync(0xffffffffu, G10, o);
                    G01 += __shfl_xor_sync(0xffffffffu, G01, o);
                    G11 += __shfl_xor_sync(0xffffffffu, G11, o);
                }
                // Masked corner terms (out-of-range corners contribute nothing).
                const float m00 = mx0 * my0, m10 = mx1 * my0, m01 = mx0 * my1, m11 = mx1 * my1;
                const float e00 = m00 * G00, e10 = m10 * G10, e01 = m01 * G01, e11 = m11 * G11;
                if (live && lane_t == 0) {
                    const float ds = wy0 * (wx0 * e00 + wx1 * e10) + wy1 * (wx0 * e01 + wx1 * e11);
                    const float dx = wy0 * (e10 - e00) + wy1 * (e11 - e01);
                    const float dy = wx0 * (e01 - e00) + wx1 * (e11 - e10);
                    const size_t s_idx = row * LP + k;
                    grad_attn[s_idx] = from_f32<TW>(ok ? ds : qnan);
                    float2 gl;
                    gl.x = ok ? kwf[k] * (a * dx) : qnan;
                    gl.y = ok ? khf[k] * (a * dy) : qnan;
                    reinterpret_cast<float2 *>(grad_loc)[s_idx] = gl;
                }
                if (live && ok) {
                    // File the in-bounds corners: corner c is filed by lane (c mod team).
                    const float ax0 = a * wx0, ax1 = a * wx1;
                    const float cf[4] = {ax0 * wy0 * m00, ax1 * wy0 * m10, ax0 * wy1 * m01, ax1 * wy1 * m11};
                    const int pp[4] = {p00, p10, p01, p11};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if ((c & (team - 1)) != lane_t || cf[c] == 0.f) continue;
                        const int pos = (int)kpos[k] + pp[c];
                        const int slot = atomicAdd(&counts[pos], 1);
                        if (slot < bp.cap) {
                            bins[(size_t)pos * bp.cap + slot] = make_uint2(__float_as_uint(cf[c]), (unsigned)iq);
                        } else {
                            const TG *grow = tg + (size_t)iq * D;
                            for (int d = 0; d < D; ++d) atomicAdd(&ovf[(size_t)pos * D + d], cf[c] * to_f32(grow[d]));
                        }
                    }
                }
            }
        }
        __syncthreads();

        // P2: owners walk their bins.
#pragma unroll
        for (int j = 0; j < OWN; ++j) {
            const int o = threadIdx.x + j * blockDim.x;
            if (o < owners) {
                const int pos = o >> tshift, ch = o & (chunks - 1);
                const int n = min(counts[pos], bp.cap);
                const uint2 *bin = bins + (size_t)pos * bp.cap;
                for (int e = 0; e < n; ++e) {
                    const uint2 rec = bin[e];
                    const float c = __uint_as_float(rec.x);
                    float2 gq[4];
                    load_g8<TG>(tg_s + (rec.y * (unsigned)D + ch * 8u) * (unsigned)sizeof(TG), gq);
                    const float2 cc = make_float2(c, c);
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[j][i] = __ffma2_rn(cc, gq[i], acc[j][i]);
                }
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < Lv; i += blockDim.x) counts[i] = 0;
    }
    __syncthreads();

    // Owners add the overflow slab and write their grad_value chunk once.
#pragma unroll
    for (int j = 0; j < OWN; ++j) {
        const int o = threadIdx.x + j * blockDim.x;
        if (o < owners) {
            const int pos = o >> tshift, ch = o & (chunks - 1);
            const float *ov = ovf + (size_t)pos * D + ch * 8;
            float f[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                f[2 * i] = acc[j][i].x + ov[2 * i];
                f[2 * i + 1] = acc[j][i].y + ov[2 * i + 1];
            }
            store_vec<bf16, 8>(grad_value + ((size_t)bh * Lv + pos) * D + ch * 8, f);
        }
    }
}

template <typename TW>
bool plan_backward_bins(const Geom &g, const void *value, const float *loc, const void *attn, const void *gout,
                        const void *grad_value, int optin, BinPlan &bp, int &own) {
    using TG = typename OutOf<bf16, TW>::T;
    const int LP = g.L * g.P;
    if (!(LP == 1 || LP == 2 || LP == 4 || LP == 8)) return false;
    if (g.D % 8 != 0 || g.D / 8 > 32 || ((g.D / 8) & (g.D / 8 - 1))) return false;
    if (!aligned(value, 16) || !aligned(grad_value, 16)) return false;
    const Tune tune = read_tune(kKnobMsdaBins);
    if (tune.stage == 0) return false;
    bp.slab_bytes = (size_t)g.Lv * g.D * 2;
    const int chunks = g.D / 8;
    own = (g.Lv * chunks + kBinThreads - 1) / kBinThreads;
    if (own > 4) return false;
    auto granule = [](long long seg, long long stride, const void *base) -> int {
        for (int gsz = 16; gsz >= 4; gsz >>= 1)
            if (seg % gsz == 0 && stride % gsz == 0 && aligned(base, gsz)) return gsz;
        return 0;
    };
    bp.gl = granule((long long)LP * 8, (long long)LP * 8, loc);
    bp.ga = granule((long long)LP * sizeof(TW), (long long)LP * sizeof(TW), attn);
    bp.gg = granule((long long)g.D * sizeof(TG), (long long)g.D * sizeof(TG), gout);
    if (!bp.gl || !bp.ga || !bp.gg) return false;
    bp.tq = tune.threads > 0 ? tune.threads : 512;
    bp.cap = tune.hsub > 0 ? tune.hsub : 24;
    const size_t lbytes = (size_t)bp.tq * LP * 8;
    const size_t abytes = ((size_t)bp.tq * LP * sizeof(TW) + 15) & ~(size_t)15;
    const size_t gbytes = (size_t)bp.tq * g.D * sizeof(TG);
    bp.smem = ((bp.slab_bytes + 15) & ~(size_t)15) + 2 * (lbytes + abytes + gbytes) +
              (size_t)g.Lv * bp.cap * 8 + (((size_t)g.Lv * 4 + 15) & ~(size_t)15) + (size_t)g.Lv * g.D * 4;
    return bp.smem <= (size_t)optin;
}

template <typename TW, int LP, int OWN>
int launch_backward_bins(const Geom &g, const BinPlan &bp, const void *value, const float *loc, const void *attn,
                         const void *gout, void *gv, float *gl, void *ga, cudaStream_t stream) {
    auto kernel = msda_backward_bins_kernel<TW, LP, OWN>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bp.smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    kernel<<<(unsigned)(g.B * g.H), kBinThreads, bp.smem, stream>>>(
        static_cast<const bf16 *>(value), loc, static_cast<const TW *>(attn),
        static_cast<const typename OutOf<bf16, TW>::T *>(gout), static_cast<bf16 *>(gv), gl, static_cast<TW *>(ga), g,
        bp);
    return launch_status();
}

template <typename TW, int LP>
int dispatch_bins_own(const Geom &g, const BinPlan &bp, int own, const void *value, const float *loc, const void *attn,
                      const void *gout, void *gv, float *gl, void *ga, cudaStream_t s) {
    switch (own) {
        case 1: return launch_backward_bins<TW, LP, 1>(g, bp, value, loc, attn, gout, gv, gl, ga, s);
        case 2: return launch_backward_bins<TW, LP, 2>(g, bp, value, loc, attn, gout, gv, gl, ga, s);
        case 3: return launch_backward_bins<TW, LP, 3>(g, bp, value, loc, attn, gout, gv, gl, ga, s);
        case 4: return launch_backward_bins<TW, LP, 4>(g, bp, value, loc, attn, gout, gv, gl, ga, s);
        default: return -1;
    }
}

// bf16 values only; returns -1 when the bins path does not apply.
template <typename TW>
int try_backward_bins(const Geom &g, const void *value, const float *loc, const void *attn, const void *gout, void *gv,
                      float *gl, void *ga, cudaStream_t s) {
    BinPlan bp;
    int own = 0;
    if (g.B * g.H > 2147483647 / 1 || !plan_backward_bins<TW>(g, value, loc, attn, gout, gv, max_smem_optin(), bp, own))
        return -1;
    switch (g.L * g.P) {
        case 1: return dispatch_bins_own<TW, 1>(g, bp, own, value, loc, attn, gout, gv, gl, ga, s);
        case 2: return dispatch_bins_own<TW, 2>(g, bp, own, value, loc, attn, gout, gv, gl, ga, s);
        case 4: return dispatch_bins_own<TW, 4>(g, bp, own, value, loc, attn, gout, gv, gl, ga, s);
        case 8: return dispatch_bins_own<TW, 8>(g, bp, own, value, loc, attn, gout, gv, gl, ga, s);
        default: return -1;
    }
}

// ------------------------------------------------------------------------------------------
// Backward for bf16 values, "owner computes" variant.  Every (position, 16-channel segment) of
// an (image, head) slab has one owner thread that keeps that value row in registers (float32)
// and its float32 value-gradient accumulator in registers for the whole launch.  Per tile of
// queries:
//   file   -- one thread per sample derives its four corners (clipped positions, masked
//             coefficients) and files a record {coefficient, sample*4 + corner} for each
//             in-range corner in the position's bin (slot from an integer shared-memory atomic);
//   own    -- each owner walks its bin: acc += coef * g[query] and G = <value[pos], g[query]>,
//             the corner's dot product, which it writes back to the record's sample slot;
//   finish -- one thread per sample folds its four corner dots into the weight and location
//             gradients (the sample's taps are recomputed from the staged locations).
// No thread gathers value rows, no float atomics are used, and grad_value is written once.
// "finish" of tile t runs in the same phase as "file" of tile t+1, so a tile costs two block
// barriers; tiles are prefetched two ahead with cp.async.  A bin that fills up is drained by
// repeating file/own for the corners that did not fit (bounded by the largest bin), so any
// sampling pattern is handled exactly.
// Out-of-range corners carry weight 0 (ops.py:123-128): they add nothing to grad_value and
// their m * G term is 0 unless the clipped value row or the gradient row holds a non-finite
// entry, where the reference's product is NaN -- per-row flags reproduce exactly that.
// One 576-thread CTA per slab (up to 576 owners: Lv * D/16 <= 576), one CTA per SM, so the
// owner state stays in registers without spills and the bins hold 512-query tiles.
// ------------------------------------------------------------------------------------------
constexpr int kOwnMaxThreads = 576;
constexpr int kOwnSamplesPerThread = 2;  // samples a thread files (and later finishes) per tile

struct OwnPlan {
    int tq, cap, threads, gl, ga, gg;
    unsigned o_loc, loc_sz, o_attn, attn_sz, o_gst, gst_sz, o_G, o_cnt, o_vbad, o_pois, o_coef, o_idx;
    int tma, box;       // TMA tile loads (1) or cp.async (0); rows per TMA box
    unsigned tx_bytes;  // bytes a TMA tile delivers
    size_t smem;
};

struct OwnTaps {
    float wx0, wx1, wy0, wy1, m00, m10, m01, m11;
    int p00, p10, p01, p11;
    bool ok;
};

__device__ __forceinline__ OwnTaps own_taps(float2 xy, float Wf, float Hf, int W, int H) {
    OwnTaps t;
    float ix, iy;
    sample_coords(xy.x, xy.y, Wf, Hf, ix, iy);
    t.ok = fabsf(ix) <= 3.0e38f && fabsf(iy) <= 3.0e38f;
    const Axis ax = axis_taps(ix, Wf, W), ay = axis_taps(iy, Hf, H);
    t.wx0 = ax.w0;
    t.wx1 = ax.w1;
    t.wy0 = ay.w0;
    t.wy1 = ay.w1;
    t.m00 = ax.m0 * ay.m0;
    t.m10 = ax.m1 * ay.m0;
    t.m01 = ax.m0 * ay.m1;
    t.m11 = ax.m1 * ay.m1;
    t.p00 = ay.c0 * W + ax.c0;
    t.p10 = ay.c0 * W + ax.c1;
    t.p01 = ay.c1 * W + ax.c0;
    t.p11 = ay.c1 * W + ax.c1;
    return t;
}

// Coefficients of the four corners (attention weight x bilinear weight x mask) and whether a
// corner is filed: in range, or carrying a non-finite coefficient (the reference's NaN).
__device__ __forceinline__ void own_coefs(const OwnTaps &t, float a, float cf[4], bool filed[4]) {
    const float ax0 = a * t.wx0, ax1 = a * t.wx1;
    cf[0] = ax0 * t.wy0 * t.m00;
    cf[1] = ax1 * t.wy0 * t.m10;
    cf[2] = ax0 * t.wy1 * t.m01;
    cf[3] = ax1 * t.wy1 * t.m11;
    filed[0] = t.m00 != 0.f || cf[0] != 0.f;
    filed[1] = t.m10 != 0.f || cf[1] != 0.f;
    filed[2] = t.m01 != 0.f || cf[2] != 0.f;
    filed[3] = t.m11 != 0.f || cf[3] != 0.f;
}

__device__ __forceinline__ float4 lds128f(unsigned addr) {
    float4 r;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "r"(addr));
    return r;
}

// True when any of the 2n floats is inf or NaN (x * 0 is NaN exactly for those).
template <int N>
__device__ __forceinline__ bool any_nonfinite(const float2 *x) {
    const float2 z = make_float2(0.f, 0.f);
    float2 s = __fmul2_rn(x[0], z);
#pragma unroll
    for (int i = 1; i < N; ++i) s = __ffma2_rn(x[i], z, s);
    const float r = s.x + s.y;
    return r != r;
}

template <typename TW, int LP, int SEG, bool TMA>
__global__ void __launch_bounds__(kOwnMaxThreads, 1)
msda_backward_owner_kernel(const bf16 *__restrict__ value, const float *__restrict__ loc, const TW *__restrict__ attn,
                           const typename OutOf<bf16, TW>::T *__restrict__ grad_out, bf16 *__restrict__ grad_value,
                           float *__restrict__ grad_loc, TW *__restrict__ grad_attn, const Geom g, const OwnPlan op,
                           const __grid_constant__ CUtensorMap tm_loc, const __grid_constant__ CUtensorMap tm_g) {
    using TG = typename OutOf<bf16, TW>::T;
    constexpr int D = 16 * SEG;
    constexpr int LPS = LP == 1 ? 0 : LP == 2 ? 1 : LP == 4 ? 2 : 3;
    // Gradient rows: with TMA, dense rows written with the swizzle mode of their width (16-byte
    // chunk index XORed with the row's bits 7..); with cp.async, rows padded by 16 bytes.  Both
    // make rows that differ in their low three bits start in different bank groups.
    constexpr unsigned ROWB = (unsigned)(D * sizeof(TG));
    constexpr unsigned GSTRIDE = TMA ? ROWB : ROWB + 16u;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ int lvl_i[LP][3];
    __shared__ float lvl_f[LP][2];
    __shared__ __align__(8) uint64_t mbar[3];
    __shared__ int abort_flag;
    __shared__ int armed[3];     // last tile whose loads were armed on each barrier (-1: none)
    __shared__ int slab_bad;     // some value row of the slab holds inf/NaN
    __shared__ int tile_bad[3];  // some gradient row of the tile in that slot holds inf/NaN
    unsigned char *const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int bh = blockIdx.x;
    const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
    const int Lv = g.Lv, cap = op.cap;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int qbeg = 0, qend = g.Lq;
    const float qnan = __int_as_float(0x7fc00000);

    float *const sG = reinterpret_cast<float *>(smem + op.o_G);
    int *const counts = reinterpret_cast<int *>(smem + op.o_cnt);
    unsigned char *const vbad = smem + op.o_vbad;
    unsigned *const gpois = reinterpret_cast<unsigned *>(smem + op.o_pois);  // per-position channel bits
    float *const bcoef = reinterpret_cast<float *>(smem + op.o_coef);
    unsigned short *const bidx = reinterpret_cast<unsigned short *>(smem + op.o_idx);
    auto locb = [&](int i) { return reinterpret_cast<float2 *>(smem + op.o_loc + i * op.loc_sz); };
    auto attnb = [&](int i) { return reinterpret_cast<TW *>(smem + op.o_attn + i * op.attn_sz); };
    auto gstb = [&](int i) { return reinterpret_cast<TG *>(smem + op.o_gst + i * op.gst_sz); };
    // Byte offset of 16-byte chunk c of staged gradient row r.
    auto grow = [&](unsigned r, unsigned c) -> unsigned {
        if constexpr (TMA) return swizzled_chunk(r, c, ROWB);
        else return r * GSTRIDE + c * 16u;
    };

    if constexpr (TMA) {
        if (tid == 0) {
            for (int i = 0; i < 3; ++i) {
                mbar_init(&mbar[i], 1);
                armed[i] = -1;
            }
            abort_flag = 0;
            mbar_init_fence();
            tma_prefetch_map(&tm_loc);
            tma_prefetch_map(&tm_g);
        }
        __syncthreads();
    }
    if (tid < LP) {
        const int l = tid / g.P;
        lvl_i[tid][0] = g.lw[l];
        lvl_i[tid][1] = g.lh[l];
        lvl_i[tid][2] = g.ls[l];
        lvl_f[tid][0] = (float)g.lw[l];
        lvl_f[tid][1] = (float)g.lh[l];
    }
    for (int i = tid; i < Lv; i += nthr) {
        counts[i] = 0;
        gpois[i] = 0;
    }
    if (tid < 3) tile_bad[tid] = 0;
    if (tid == 0) slab_bad = 0;
    const int nqc = max(qend - qbeg, 0);
    const int ntiles = (nqc + op.tq - 1) / op.tq;
    auto issue = [&](int t) {
        const int q0 = qbeg + t * op.tq, slot = t % 3;
        if constexpr (TMA) {
            // Weights by cp.async (their per-query rows are narrower than a TMA box allows);
            // locations and gradient rows as TMA boxes of op.box rows.
            const int nq = min(op.tq, qend - q0);
            const int abytes = LP * (int)sizeof(TW), as = 31 - __clz(abytes / op.ga);
            const size_t row0 = ((size_t)b * g.Lq + q0) * g.H + h;
            for (int i = tid; i < (nq << as); i += nthr) {
                const int qi = i >> as, j = i & ((1 << as) - 1);
                cp_async_bytes(reinterpret_cast<char *>(attnb(slot)) + (size_t)qi * abytes + j * op.ga,
                               reinterpret_cast<const char *>(attn + (row0 + (size_t)qi * g.H) * LP) + j * op.ga,
                               op.ga);
            }
            if (tid == 0 && !abort_flag) {  // a CTA that gave up arms nothing more
                armed[slot] = t;
                mbar_arrive_expect_tx(&mbar[slot], op.tx_bytes);
                for (int r = 0; r < op.tq; r += op.box) {
                    tma_load_4d(locb(slot) + r * LP, &tm_loc, &mbar[slot], 0, h, q0 + r, b);
                    tma_load_4d(reinterpret_cast<unsigned char *>(gstb(slot)) + r * ROWB, &tm_g, &mbar[slot], 0, h,
                                q0 + r, b);
                }
            }
        } else {
            issue_bwd_tile<TW, TG, LP>(loc, attn, grad_out, reinterpret_cast<float *>(locb(slot)), attnb(slot),
                                       gstb(slot), g, b, h, q0, min(op.tq, qend - q0), op.gl, op.ga, op.gg,
                                       (int)GSTRIDE);
        }
    };
    auto landed = [&](int t) {  // tile t's locations and gradient rows are in shared memory
        if constexpr (TMA) mbar_wait(&mbar[t % 3], (unsigned)(t / 3) & 1u, &abort_flag);
    };
    if (ntiles > 0) issue(0);
    cp_async_commit();
    if (ntiles > 1) issue(1);
    cp_async_commit();

    // Owner state: this thread's value row segment and accumulator.
    const int owners = Lv * SEG;
    const bool is_owner = tid < owners;
    const int pos = tid / SEG, seg = tid & (SEG - 1);
    float2 vv[8], acc[8];
    if (is_owner) {
        const uint4 *vp = reinterpret_cast<const uint4 *>(value + ((size_t)bh * Lv + pos) * D + seg * 16);
        const uint4 r0 = __ldg(vp), r1 = __ldg(vp + 1);
        vv[0] = bf16x2_lo_hi(r0.x); vv[1] = bf16x2_lo_hi(r0.y); vv[2] = bf16x2_lo_hi(r0.z); vv[3] = bf16x2_lo_hi(r0.w);
        vv[4] = bf16x2_lo_hi(r1.x); vv[5] = bf16x2_lo_hi(r1.y); vv[6] = bf16x2_lo_hi(r1.z); vv[7] = bf16x2_lo_hi(r1.w);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) vv[i] = make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = make_float2(0.f, 0.f);
    {
        bool bad = any_nonfinite<8>(vv);
        if constexpr (SEG > 1) bad |= __shfl_xor_sync(0xffffffffu, (int)bad, 1) != 0;
        if (is_owner && seg == 0) vbad[pos] = bad ? 1 : 0;
        __syncthreads();  // slab_bad was cleared above
        if (is_owner && bad) slab_bad = 1;
    }
    cp_async_wait_one();
    if (ntiles > 0) landed(0);
    __syncthreads();

    // Files the corners of sample s selected by `want` (bit c = corner c); returns those whose
    // bin was full.
    auto file = [&](const float2 *tl, const TW *ta, int s, unsigned want) -> unsigned {
        const int k = s & (LP - 1);
        const OwnTaps t = own_taps(tl[s], lvl_f[k][0], lvl_f[k][1], lvl_i[k][0], lvl_i[k][1]);
        if (!t.ok) return 0u;
        float cf[4];
        bool filed[4];
        own_coefs(t, to_f32(ta[s]), cf, filed);
        const int base = lvl_i[k][2];
        const int pp[4] = {base + t.p00, base + t.p10, base + t.p01, base + t.p11};
        unsigned failed = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if (!((want >> c) & 1u) || !filed[c]) continue;
            const int slot = atomicAdd(&counts[pp[c]], 1);
            if (slot < cap) {
                bcoef[slot * Lv + pp[c]] = cf[c];
                bidx[slot * Lv + pp[c]] = (unsigned short)(s * 4 + c);
            } else {
                failed |= 1u << c;
            }
        }
        return failed;
    };

    // Owners drain their bins (and reset their counts for the next round).
    auto own = [&](const TG *gs) {
        const unsigned gs_s = (unsigned)__cvta_generic_to_shared(gs);
        int n = 0;
        if (is_owner) n = min(counts[pos], cap);
        if constexpr (SEG > 1) __syncwarp();
        if (is_owner && seg == 0) counts[pos] = 0;
        const unsigned team = SEG > 1 ? (3u << ((tid & 31) & ~1)) : 0u;
        constexpr unsigned SEGCH = 16u * (unsigned)sizeof(TG) / 16u;  // 16-byte chunks per segment
        for (int e = 0; e < n; ++e) {
            const float c = bcoef[e * Lv + pos];
            const unsigned idx = bidx[e * Lv + pos];
            const unsigned r = idx >> (2 + LPS);
            float2 q[8];
            if constexpr (sizeof(TG) == 2) {
                const uint4 u0 = lds128(gs_s + grow(r, seg * SEGCH)), u1 = lds128(gs_s + grow(r, seg * SEGCH + 1));
                q[0] = bf16x2_lo_hi(u0.x); q[1] = bf16x2_lo_hi(u0.y); q[2] = bf16x2_lo_hi(u0.z); q[3] = bf16x2_lo_hi(u0.w);
                q[4] = bf16x2_lo_hi(u1.x); q[5] = bf16x2_lo_hi(u1.y); q[6] = bf16x2_lo_hi(u1.z); q[7] = bf16x2_lo_hi(u1.w);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 f = lds128f(gs_s + grow(r, seg * SEGCH + i));
                    q[2 * i] = make_float2(f.x, f.y);
                    q[2 * i + 1] = make_float2(f.z, f.w);
                }
            }
            const float2 cc = make_float2(c, c);
            float2 d = __fmul2_rn(vv[0], q[0]);
#pragma unroll
            for (int i = 1; i < 8; ++i) d = __ffma2_rn(vv[i], q[i], d);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __ffma2_rn(cc, q[i], acc[i]);
            float dot = d.x + d.y;
            if constexpr (SEG > 1) dot += __shfl_xor_sync(team, dot, 1);
            if (seg == 0) sG[idx] = dot;
        }
    };

    // Per-sample state kept in registers from "file" to "finish" of the same tile: the
    // fractional weights, the attention weight and bits {ok, in-range corners, filed corners}.
    constexpr int MAXS = kOwnSamplesPerThread;
    float st_wx1[MAXS], st_wy1[MAXS], st_a[MAXS];
    unsigned st_bits[MAXS];

    // First filing of a tile: taps, stash, corners; returns the per-sample bins-full masks.
    auto file_tile = [&](const float2 *tl, const TW *ta, int nq) -> unsigned {
        unsigned pending = 0;
#pragma unroll
        for (int i = 0; i < MAXS; ++i) {
            const int s = tid + i * nthr;
            if (s >= nq * LP) break;
            const int k = s & (LP - 1);
            const OwnTaps t = own_taps(tl[s], lvl_f[k][0], lvl_f[k][1], lvl_i[k][0], lvl_i[k][1]);
            const float a = to_f32(ta[s]);
            float cf[4];
            bool filed[4];
            own_coefs(t, a, cf, filed);
            st_wx1[i] = t.wx1;
            st_wy1[i] = t.wy1;
            st_a[i] = a;
            st_bits[i] = (t.ok ? 1u : 0u) | (t.m00 != 0.f ? 2u : 0u) | (t.m10 != 0.f ? 4u : 0u) |
                         (t.m01 != 0.f ? 8u : 0u) | (t.m11 != 0.f ? 16u : 0u) | (filed[0] ? 32u : 0u) |
                         (filed[1] ? 64u : 0u) | (filed[2] ? 128u : 0u) | (filed[3] ? 256u : 0u);
            if (!t.ok) continue;
            const int base = lvl_i[k][2];
            const int pp[4] = {base + t.p00, base + t.p10, base + t.p01, base + t.p11};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (!filed[c]) continue;
                const int slot = atomicAdd(&counts[pp[c]], 1);
                if (slot < cap) {
                    bcoef[slot * Lv + pp[c]] = cf[c];
                    bidx[slot * Lv + pp[c]] = (unsigned short)(s * 4 + c);
                } else {
                    pending |= 1u << (4 * i + c);
                }
            }
        }
        return pending;
    };

    // Raises tile_bad[slot] when a gradient row of the tile holds inf/NaN (x * 0 is NaN exactly
    // for those).
    auto scan_rows = [&](int t, int nq) {
        const unsigned gs_s = smem_u32(gstb(t % 3));
        constexpr unsigned NCH = ROWB / 16u;
        for (int i = tid; i < nq * (int)NCH; i += nthr) {
            const uint4 u = lds128(gs_s + grow((unsigned)i / NCH, (unsigned)i % NCH));
            float2 f[4];
            if constexpr (sizeof(TG) == 2) {
                f[0] = bf16x2_lo_hi(u.x); f[1] = bf16x2_lo_hi(u.y); f[2] = bf16x2_lo_hi(u.z); f[3] = bf16x2_lo_hi(u.w);
            } else {
                f[0] = make_float2(__uint_as_float(u.x), __uint_as_float(u.y));
                f[1] = make_float2(__uint_as_float(u.z), __uint_as_float(u.w));
                f[2] = f[3] = make_float2(0.f, 0.f);
            }
            if (any_nonfinite<4>(f)) tile_bad[t % 3] = 1;
        }
    };

    // Weight and location gradients of the samples of a drained tile, from the stash.
    auto finish = [&](int tb, int qa, int nq) {
        const float2 *tl = locb(tb % 3);
        const unsigned char *gsb = reinterpret_cast<const unsigned char *>(gstb(tb % 3));
        const bool maybe_bad = (slab_bad | tile_bad[tb % 3]) != 0;
#pragma unroll
        for (int i = 0; i < MAXS; ++i) {
            const int s = tid + i * nthr;
            if (s >= nq * LP) break;
            const int k = s & (LP - 1), iq = s >> LPS;
            const float Wf = lvl_f[k][0], Hf = lvl_f[k][1];
            const unsigned bits = st_bits[i];
            const float wx1 = st_wx1[i], wy1 = st_wy1[i], a = st_a[i];
            const float wx0 = 1.f - wx1, wy0 = 1.f - wy1;
            const float4 G = *reinterpret_cast<const float4 *>(sG + 4 * s);
            float e[4] = {(bits & 2u ? 1.f : 0.f) * G.x, (bits & 4u ? 1.f : 0.f) * G.y,
                          (bits & 8u ? 1.f : 0.f) * G.z, (bits & 16u ? 1.f : 0.f) * G.w};
            // An unfiled corner is out of range: its m * G term is 0 unless the clipped value
            // row or the gradient row holds inf/NaN (the reference's 0 * inf = NaN).
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (!((bits >> (5 + c)) & 1u)) e[c] = 0.f;
            if (maybe_bad && (bits & 0x1e1u) != 0x1e1u && (bits & 1u)) {
                unsigned gmask = 0;  // channels of the gradient row holding inf/NaN
                constexpr int PER = 16 / (int)sizeof(TG);
                for (int j = 0; j < D; ++j) {
                    const TG x = reinterpret_cast<const TG *>(gsb + grow(iq, j / PER))[j % PER];
                    if (!(fabsf(to_f32(x)) <= 3.4028235e38f)) gmask |= 1u << j;
                }
                const OwnTaps t = own_taps(tl[s], Wf, Hf, lvl_i[k][0], lvl_i[k][1]);
                const int base = lvl_i[k][2];
                const int pp[4] = {base + t.p00, base + t.p10, base + t.p01, base + t.p11};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if ((bits >> (5 + c)) & 1u) continue;
                    e[c] = (gmask || vbad[pp[c]]) ? qnan : 0.f;
                    // The reference also scatters 0 * (a * g) into the clipped row: NaN in the
                    // channels where g is not finite.
                    if (gmask) atomicOr(&gpois[pp[c]], gmask);
                }
            }
            const bool ok = (bits & 1u) != 0;
            const float ds = wy0 * (wx0 * e[0] + wx1 * e[1]) + wy1 * (wx0 * e[2] + wx1 * e[3]);
            const float dx = wy0 * (e[1] - e[0]) + wy1 * (e[3] - e[2]);
            const float dy = wx0 * (e[2] - e[0]) + wx1 * (e[3] - e[1]);
            const size_t s_idx = (((size_t)b * g.Lq + qa + iq) * g.H + h) * LP + k;
            grad_attn[s_idx] = from_f32<TW>(ok ? ds : qnan);
            float2 gl;
            gl.x = ok ? Wf * (a * dx) : qnan;
            gl.y = ok ? Hf * (a * dy) : qnan;
            reinterpret_cast<float2 *>(grad_loc)[s_idx] = gl;
        }
    };

    for (int t = 0; t < ntiles; ++t) {
        const int qa = qbeg + t * op.tq;
        const int nq = min(op.tq, qend - qa);
        const float2 *tl = locb(t % 3);
        const TW *ta = attnb(t % 3);
        // Phase A: finish the previous tile, file this tile's corners.
        if (t > 0) finish(t - 1, qa - op.tq, op.tq);
        if (tid == 0) tile_bad[(t + 1) % 3] = 0;  // last read by finish(t - 2)
        scan_rows(t, nq);
        unsigned pending = file_tile(tl, ta, nq);
        bool again = __syncthreads_or(pending != 0u);
        // Phase B: prefetch two tiles ahead, drain the bins.
        if (t + 2 < ntiles) issue(t + 2);
        cp_async_commit();
        own(gstb(t % 3));
        for (int round = 0; again && round < 65536; ++round) {  // full bins: refile what did not fit
            __syncthreads();
            unsigned left = 0;
#pragma unroll
            for (int i = 0; i < MAXS; ++i) {
                const int s = tid + i * nthr;
                const unsigned want = (pending >> (4 * i)) & 0xFu;
                if (want && s < nq * LP) left |= file(tl, ta, s, want) << (4 * i);
            }
            pending = left;
            again = __syncthreads_or(pending != 0u);
            own(gstb(t % 3));
        }
        cp_async_wait_one();
        if (t + 1 < ntiles) landed(t + 1);
        __syncthreads();
    }
    if (ntiles > 0) {
        const int t = ntiles - 1;
        finish(t, qbeg + t * op.tq, qend - (qbeg + t * op.tq));
    }

    if constexpr (TMA) {
        // Gave up waiting: let the copies this CTA armed land before it exits (each barrier has at
        // most one armed phase outstanding, since a tile is armed only after the previous tile of
        // its slot landed or the CTA aborted, and an aborted CTA arms nothing).
        if (abort_flag && tid == 0)
            for (int i = 0; i < 3; ++i)
                if (armed[i] >= 0) mbar_drain(&mbar[i], (unsigned)(armed[i] / 3) & 1u);
    }
    __syncthreads();  // the last finish may have poisoned rows
    if (is_owner) {
        const unsigned pois = gpois[pos] >> (16 * seg);
        float f[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            f[2 * j] = (pois >> (2 * j)) & 1u ? qnan : acc[j].x;
            f[2 * j + 1] = (pois >> (2 * j + 1)) & 1u ? qnan : acc[j].y;
        }
        store_vec<bf16, 16>(grad_value + ((size_t)bh * Lv + pos) * D + seg * 16, f);
    }
}

template <typename TW>
bool plan_backward_owner(const Geom &g, const void *value, const float *loc, const void *attn, const void *gout,
                         const void *grad_value, int optin, OwnPlan &op, bool allow_tma) {
    using TG = typename OutOf<bf16, TW>::T;
    const int LP = g.L * g.P;
    if (!(LP == 1 || LP == 2 || LP == 4 || LP == 8)) return false;
    if (g.D != 16 && g.D != 32) return false;
    const int owners = g.Lv * (g.D / 16);
    if (owners > kOwnMaxThreads) return false;
    if (!aligned(value, 16) || !aligned(grad_value, 16)) return false;
    const Tune tune = read_tune(kKnobMsdaOwn);
    if (tune.stage == 0) return false;
    auto granule = [](long long seg, long long stride, const void *base) -> int {
        for (int gsz = 16; gsz >= 4; gsz >>= 1)
            if (seg % gsz == 0 && stride % gsz == 0 && aligned(base, gsz)) return gsz;
        return 0;
    };
    op.gl = granule((long long)LP * 8, (long long)LP * 8, loc);
    op.ga = granule((long long)LP * sizeof(TW), (long long)LP * sizeof(TW), attn);
    op.gg = granule((long long)g.D * sizeof(TG), (long long)g.D * sizeof(TG), gout);
    if (!op.gl || !op.ga || !op.gg) return false;
    op.threads = std::max(64, (owners + 31) & ~31);
    op.cap = tune.hsub > 0 ? tune.hsub : 24;
    op.tq = tune.threads > 0 ? tune.threads : 512;
    op.tq = std::min(op.tq, kOwnSamplesPerThread * op.threads / LP);
    if (op.tq < 1 || (size_t)op.tq * LP * 4 > 65536) return false;
    // TMA tile loads: location rows must be a multiple of 16 bytes, gradient rows one of the
    // swizzle widths, both bases 16-byte aligned, and a tile a whole number of boxes.
    const size_t rowb = (size_t)g.D * sizeof(TG);
    op.box = std::min(op.tq, 256);
    op.tma = allow_tma && tune.acc != 0 && LP >= 2 && (rowb == 32 || rowb == 64 || rowb == 128) && aligned(loc, 16) &&
             aligned(gout, 16) && op.tq % op.box == 0;
    op.tx_bytes = (unsigned)((size_t)op.tq * (LP * 8 + rowb));
    auto r16 = [](size_t x) { return (x + 15) & ~(size_t)15; };
    auto r1k = [](size_t x) { return (x + 1023) & ~(size_t)1023; };
    size_t o = 0;
    op.gst_sz = op.tma ? (unsigned)r1k((size_t)op.tq * rowb) : (unsigned)r16((size_t)op.tq * (rowb + 16));
    op.o_gst = (unsigned)o; o += 3 * (size_t)op.gst_sz;  // first: 1024-byte aligned for the swizzle
    op.loc_sz = (unsigned)((((size_t)op.tq * LP * 8) + 127) & ~(size_t)127);
    op.o_loc = (unsigned)o; o += 3 * (size_t)op.loc_sz;
    op.attn_sz = (unsigned)r16((size_t)op.tq * LP * sizeof(TW));
    op.o_attn = (unsigned)o; o += 3 * (size_t)op.attn_sz;
    op.o_G = (unsigned)o; o += r16((size_t)op.tq * LP * 16);
    op.o_cnt = (unsigned)o; o += r16((size_t)g.Lv * 4);
    op.o_vbad = (unsigned)o; o += r16((size_t)g.Lv);
    op.o_pois = (unsigned)o; o += r16((size_t)g.Lv * 4);
    op.o_coef = (unsigned)o;
    size_t bins = r16((size_t)op.cap * g.Lv * 4);
    op.o_idx = (unsigned)(o + bins);
    bins += r16((size_t)op.cap * g.Lv * 2);
    o += bins;
    op.smem = o + (op.tma ? 1024 : 0);  // slack to align the base to 1024 bytes at run time
    return op.smem <= (size_t)optin;
}

template <typename TW, int LP, int SEG, bool TMA>
int launch_backward_owner_k(const Geom &g, const OwnPlan &op, const void *value, const float *loc, const void *attn,
                            const void *gout, void *gv, float *gl, void *ga, const CUtensorMap &tml,
                            const CUtensorMap &tmg, cudaStream_t stream) {
    auto kernel = msda_backward_owner_kernel<TW, LP, SEG, TMA>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)op.smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    kernel<<<(unsigned)(g.B * g.H), op.threads, op.smem, stream>>>(
        static_cast<const bf16 *>(value), loc, static_cast<const TW *>(attn),
        static_cast<const typename OutOf<bf16, TW>::T *>(gout), static_cast<bf16 *>(gv), gl, static_cast<TW *>(ga), g,
        op, tml, tmg);
    return launch_status();
}

template <typename TW, int LP, int SEG>
int launch_backward_owner(const Geom &g, const OwnPlan &op, const void *value, const float *loc, const void *attn,
                          const void *gout, void *gv, float *gl, void *ga, cudaStream_t stream) {
    using TG = typename OutOf<bf16, TW>::T;
    CUtensorMap tml, tmg;
    std::memset(&tml, 0, sizeof(tml));
    std::memset(&tmg, 0, sizeof(tmg));
    bool tma = op.tma != 0;
    if (tma) {
        // Locations [B, Lq, H, LP*2] f32 and gradient rows [B, Lq, H, D]: boxes of one head's rows.
        const uint64_t lrow = (uint64_t)LP * 8, grow = (uint64_t)g.D * sizeof(TG);
        const uint64_t ldims[4] = {(uint64_t)LP * 2, (uint64_t)g.H, (uint64_t)g.Lq, (uint64_t)g.B};
        const uint64_t lstr[3] = {lrow, lrow * g.H, lrow * g.H * g.Lq};
        const uint32_t lbox[4] = {(uint32_t)LP * 2, 1, (uint32_t)op.box, 1};
        const uint64_t gdims[4] = {(uint64_t)g.D, (uint64_t)g.H, (uint64_t)g.Lq, (uint64_t)g.B};
        const uint64_t gstr[3] = {grow, grow * g.H, grow * g.H * g.Lq};
        const uint32_t gbox[4] = {(uint32_t)g.D, 1, (uint32_t)op.box, 1};
        const CUtensorMapSwizzle sw = grow == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                      : grow == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                   : CU_TENSOR_MAP_SWIZZLE_128B;
        tma = encode_tensor_map(&tml, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, loc, ldims, lstr, lbox,
                                CU_TENSOR_MAP_SWIZZLE_NONE) &&
              encode_tensor_map(&tmg,
                                sizeof(TG) == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                                gout, gdims, gstr, gbox, sw);
    }
    if (!tma) return -1;  // the caller re-plans without TMA
    return launch_backward_owner_k<TW, LP, SEG, true>(g, op, value, loc, attn, gout, gv, gl, ga, tml, tmg, stream);
}

template <typename TW, int LP, int SEG>
int launch_backward_owner_plain(const Geom &g, const OwnPlan &op, const void *value, const float *loc,
                                const void *attn, const void *gout, void *gv, float *gl, void *ga,
                                cudaStream_t stream) {
    CUtensorMap none;
    std::memset(&none, 0, sizeof(none));
    return launch_backward_owner_k<TW, LP, SEG, false>(g, op, value, loc, attn, gout, gv, gl, ga, none, none, stream);
}

template <typename TW, int LP>
int dispatch_owner_seg(const Geom &g, const OwnPlan &op, const void *value, const float *loc, const void *attn,
                       const void *gout, void *gv, float *gl, void *ga, cudaStream_t s) {
    if (op.tma) {
        if constexpr (LP >= 2)
            return g.D == 16 ? launch_backward_owner<TW, LP, 1>(g, op, value, loc, attn, gout, gv, gl, ga, s)
                             : launch_backward_owner<TW, LP, 2>(g, op, value, loc, attn, gout, gv, gl, ga, s);
        return -1;
    }
    return g.D == 16 ? launch_backward_owner_plain<TW, LP, 1>(g, op, value, loc, attn, gout, gv, gl, ga, s)
                     : launch_backward_owner_plain<TW, LP, 2>(g, op, value, loc, attn, gout, gv, gl, ga, s);
}

// bf16 values only; returns -1 when the owner path does not apply.
template <typename TW>
int try_backward_owner(const Geom &g, const void *value, const float *loc, const void *attn, const void *gout,
                       void *gv, float *gl, void *ga, cudaStream_t s) {
    OwnPlan op;
    if (!plan_backward_owner<TW>(g, value, loc, attn, gout, gv, max_smem_optin(), op, true)) return -1;
    for (int attempt = 0; attempt < 2; ++attempt) {
        int st = -1;
        switch (g.L * g.P) {
            case 1: st = dispatch_owner_seg<TW, 1>(g, op, value, loc, attn, gout, gv, gl, ga, s); break;
            case 2: st = dispatch_owner_seg<TW, 2>(g, op, value, loc, attn, gout, gv, gl, ga, s); break;
            case 4: st = dispatch_owner_seg<TW, 4>(g, op, value, loc, attn, gout, gv, gl, ga, s); break;
            case 8: st = dispatch_owner_seg<TW, 8>(g, op, value, loc, attn, gout, gv, gl, ga, s); break;
            default: return -1;
        }
        if (st >= 0 || !op.tma) return st;
        // The tensor maps could not be built: fall back to cp.async tile loads.
        if (!plan_backward_owner<TW>(g, value, loc, attn, gout, gv, max_smem_optin(), op, false)) return -1;
    }
    return -1;
}

// ------------------------------------------------------------------------------------------
// Cell-owner backward: one level, bf16 values, weights and gradient rows, 16 channels, and
// (W+1)(H+1) <= 640 bilinear cells (the Nano decoder's 24 x 24 map: 625).
//
// A sample's four taps are the corners of one cell of the map extended by a row and a column
// of out-of-range positions on the low side: the cell of (floor(x), floor(y)), both in [-1, size-1]
// when any corner is in range.  One 640-thread CTA per (image, head) slab, two passes:
//   1. one thread per sample (the next sample's inputs in flight): taps; the four corners' dot
//      products <value row, g> against the slab staged in shared memory (bf16 x bf16 products,
//      exact in float32, accumulated in float32 -- so equal to unpacking); the weight and location
//      gradients, written directly; the sample's cell and its {wx1, wy1, a} kept in shared memory,
//      and a counting sort of the samples by cell (counts, scan, filing);
//   2. one owner thread per cell walks its samples and accumulates the four corner vectors
//      c_k * g (c = a * wx * wy per corner) in registers: a sample's gradient row is read once
//      (from L2) instead of once per corner;
// then grad_value[y][x] = A[y][x] + B[y][x-1] + C[y-1][x] + D[y-1][x-1] from the cells'
// corner accumulators, through shared memory one corner at a time, written once in bf16.
// Corners outside the map land in extended-grid slots that no output reads.  The reference's
// non-finite semantics: an out-of-range corner's dot product enters as m * dot (0, or NaN when
// the clipped row or g is not finite), and the (g * a) * 0 it scatters into its clipped row is
// NaN in the channels where g * a is not finite -- per-row poison bits applied at the write.
// Value rows are staged with their two 16-byte halves swapped when bit 2 of the row is set, so
// the first half of random rows spreads over all eight 16-byte bank groups.
// ------------------------------------------------------------------------------------------
constexpr int kCellThreads = 640;

struct CellPlan {
    unsigned o_vs, o_stash, o_rec, o_cnt, o_off, o_pois;
    size_t smem;
};

// d0 += v.lo * g.lo and d1 += v.hi * g.hi for bf16 pairs, float32 accumulation.
__device__ __forceinline__ void dot2_bf16(unsigned v, unsigned g, float &d0, float &d1) {
    asm("{\n.reg .b16 vl, vh, gl, gh;\nmov.b32 {vl, vh}, %2;\nmov.b32 {gl, gh}, %3;\n"
        "fma.rn.f32.bf16 %0, vl, gl, %0;\nfma.rn.f32.bf16 %1, vh, gh, %1;\n}"
        : "+f"(d0), "+f"(d1)
        : "r"(v), "r"(g));
}

// Byte offset of half `hf` of staged 32-byte value row r (halves swapped when bit 2 of r is set).
__device__ __forceinline__ unsigned cell_row_half(unsigned r, unsigned hf) {
    return r * 32u + ((hf ^ ((r >> 2) & 1u)) << 4);
}

template <int P>
__global__ void __launch_bounds__(kCellThreads, 1)
msda_backward_cell_kernel(const bf16 *__restrict__ value, const float *__restrict__ loc, const bf16 *__restrict__ attn,
                          const bf16 *__restrict__ grad_out, bf16 *__restrict__ grad_value,
                          float *__restrict__ grad_loc, bf16 *__restrict__ grad_attn, const Geom g, const CellPlan cp) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int PS = P == 1 ? 0 : P == 2 ? 1 : P == 4 ? 2 : 3;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int bh = blockIdx.x;
    const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
    const int W = g.lw[0], Hh = g.lh[0], Lv = g.Lv;
    const int EW = W + 1, E = (W + 1) * (Hh + 1);
    const int S = g.Lq * P;
    const float Wf = (float)W, Hf = (float)Hh;
    const float qnan = __int_as_float(0x7fc00000);

    const unsigned vs_s = smem_u32(smem + cp.o_vs);
    float4 *stash = reinterpret_cast<float4 *>(smem + cp.o_stash);
    unsigned short *rec = reinterpret_cast<unsigned short *>(smem + cp.o_rec);
    int *cnt = reinterpret_cast<int *>(smem + cp.o_cnt);
    int *off = reinterpret_cast<int *>(smem + cp.o_off);
    unsigned *pois = reinterpret_cast<unsigned *>(smem + cp.o_pois);
    __shared__ int wsum[kCellThreads / 32];

    {
        const uint4 *src = reinterpret_cast<const uint4 *>(value + (size_t)bh * Lv * 16);
        for (int i = tid; i < Lv * 2; i += nthr)
            *reinterpret_cast<uint4 *>(smem + cp.o_vs + cell_row_half((unsigned)i >> 1, (unsigned)i & 1u)) = __ldg(src + i);
        for (int p = tid; p < Lv; p += nthr) pois[p] = 0;
        for (int e = tid; e < E; e += nthr) cnt[e] = 0;
    }
    __syncthreads();

    // Pass 1: one thread per sample.
    const size_t row0 = (size_t)b * g.Lq * g.H + h;  // (image, query 0, head)
    float2 xy_n = make_float2(0.f, 0.f);
    unsigned short a_n = 0;
    uint4 g0_n = make_uint4(0, 0, 0, 0), g1_n = make_uint4(0, 0, 0, 0);
    auto fetch = [&](int s) {
        const size_t row = row0 + (size_t)(s >> PS) * g.H;
        const size_t ri = row * P + (s & (P - 1));
        xy_n = __ldg(reinterpret_cast<const float2 *>(loc) + ri);
        a_n = __ldg(reinterpret_cast<const unsigned short *>(attn) + ri);
        const uint4 *gp = reinterpret_cast<const uint4 *>(grad_out + row * 16);
        g0_n = __ldg(gp);
        g1_n = __ldg(gp + 1);
    };
    if (tid < S) fetch(tid);
    for (int s = tid; s < S; s += nthr) {
        const size_t ri = (row0 + (size_t)(s >> PS) * g.H) * P + (s & (P - 1));
        const float2 xy = xy_n;
        const float a = __uint_as_float((unsigned)a_n << 16);
        const unsigned gw[8] = {g0_n.x, g0_n.y, g0_n.z, g0_n.w, g1_n.x, g1_n.y, g1_n.z, g1_n.w};
        if (s + nthr < S) fetch(s + nthr);
        float ix, iy;
        sample_coords(xy.x, xy.y, Wf, Hf, ix, iy);
        const bool ok = fabsf(ix) <= 3.0e38f && fabsf(iy) <= 3.0e38f;
        const Axis ax = axis_taps(ix, Wf, W), ay = axis_taps(iy, Hf, Hh);
        const int pk[4] = {ay.c0 * W + ax.c0, ay.c0 * W + ax.c1, ay.c1 * W + ax.c0, ay.c1 * W + ax.c1};
        const float mk[4] = {ax.m0 * ay.m0, ax.m1 * ay.m0, ax.m0 * ay.m1, ax.m1 * ay.m1};
        float e[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 v0 = lds128(vs_s + cell_row_half((unsigned)pk[k], 0u));
            const uint4 v1 = lds128(vs_s + cell_row_half((unsigned)pk[k], 1u));
            float d0 = 0.f, d1 = 0.f;
            dot2_bf16(v0.x, gw[0], d0, d1);
            dot2_bf16(v0.y, gw[1], d0, d1);
            dot2_bf16(v0.z, gw[2], d0, d1);
            dot2_bf16(v0.w, gw[3], d0, d1);
            dot2_bf16(v1.x, gw[4], d0, d1);
            dot2_bf16(v1.y, gw[5], d0, d1);
            dot2_bf16(v1.z, gw[6], d0, d1);
            dot2_bf16(v1.w, gw[7], d0, d1);
            e[k] = mk[k] * (d0 + d1);  // out of range: 0, or NaN when the product is not finite
        }
        const float wx0 = ax.w0, wx1 = ax.w1, wy0 = ay.w0, wy1 = ay.w1;
        const float ds = wy0 * (wx0 * e[0] + wx1 * e[1]) + wy1 * (wx0 * e[2] + wx1 * e[3]);
        const float dx = wy0 * (e[1] - e[0]) + wy1 * (e[3] - e[2]);
        const float dy = wx0 * (e[2] - e[0]) + wx1 * (e[3] - e[1]);
        grad_attn[ri] = __float2bfloat16_rn(ok ? ds : qnan);
        reinterpret_cast<float2 *>(grad_loc)[ri] =
            ok ? make_float2(Wf * (a * dx), Hf * (a * dy)) : make_float2(qnan, qnan);
        int cell = -1;
        if (ok && ax.i0 >= -1 && ax.i0 < W && ay.i0 >= -1 && ay.i0 < Hh) {
            cell = (ay.i0 + 1) * EW + (ax.i0 + 1);
            atomicAdd(&cnt[cell], 1);
        }
        stash[s] = make_float4(wx1, wy1, a, __int_as_float(cell));
        if (ok && (mk[0] == 0.f || mk[1] == 0.f || mk[2] == 0.f || mk[3] == 0.f)) {
            // An out-of-range corner scatters (g * a) * 0 into its clipped row.
            unsigned bad = 0;
            if (!(fabsf(a) <= 3.4028235e38f)) {
                bad = 0xffffu;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if ((gw[i] & 0x7f80u) == 0x7f80u) bad |= 1u << (2 * i);
                    if ((gw[i] & 0x7f800000u) == 0x7f800000u) bad |= 1u << (2 * i + 1);
                }
            }
            if (bad) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (mk[k] == 0.f) atomicOr(&pois[pk[k]], bad);
            }
        }
    }
    __syncthreads();
    // Bin starts (exclusive scan of the counts; the counts become cursors), then the filing.
    {
        const int lane = tid & 31, w = tid >> 5;
        const int v = tid < E ? cnt[tid] : 0;
        int x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[w] = x;
        __syncthreads();
        int before = 0;
        for (int k = 0; k < w; ++k) before += wsum[k];
        const int excl = before + x - v;
        if (tid < E) {
            off[tid] = excl;
            cnt[tid] = excl;
        }
        if (tid == E - 1) off[E] = excl + v;
    }
    __syncthreads();
    for (int sl = tid; sl < S; sl += nthr) {
        const int cell = __float_as_int(stash[sl].w);
        if (cell >= 0) rec[atomicAdd(&cnt[cell], 1)] = (unsigned short)sl;
    }
    __syncthreads();

    // Pass 2: the owner of cell `tid` accumulates its samples' four corner vectors.
    float2 acc[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[k][i] = make_float2(0.f, 0.f);
    if (tid < E) {
        const int beg = off[tid], end = off[tid + 1];
        for (int r = beg; r < end; ++r) {
            const int sl = rec[r];
            const float4 st = stash[sl];
            const uint4 *gp = reinterpret_cast<const uint4 *>(grad_out + (row0 + (size_t)(sl >> PS) * g.H) * 16);
            const uint4 g0 = __ldg(gp), g1 = __ldg(gp + 1);
            const unsigned gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            const float wx1 = st.x, wy1 = st.y, a = st.z;
            const float ax0 = a * (1.f - wx1), ax1 = a * wx1;
            const float2 c0 = make_float2(ax0 * (1.f - wy1), ax0 * (1.f - wy1));
            const float2 c1 = make_float2(ax1 * (1.f - wy1), ax1 * (1.f - wy1));
            const float2 c2 = make_float2(ax0 * wy1, ax0 * wy1);
            const float2 c3 = make_float2(ax1 * wy1, ax1 * wy1);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float2 gp2 = bf16x2_lo_hi(gw[i]);
                acc[0][i] = __ffma2_rn(c0, gp2, acc[0][i]);
                acc[1][i] = __ffma2_rn(c1, gp2, acc[1][i]);
                acc[2][i] = __ffma2_rn(c2, gp2, acc[2][i]);
                acc[3][i] = __ffma2_rn(c3, gp2, acc[3][i]);
            }
        }
    }
    __syncthreads();

    // grad_value from the corner accumulators, one corner at a time through the (now free)
    // sample stash, laid out chunk-major so both sides are conflict-free.
    float2 out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = make_float2(0.f, 0.f);
    float4 *X = stash;
    const int y = tid / W, x = tid - (tid / W) * W;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if (tid < E) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                X[i * E + tid] = make_float4(acc[k][2 * i].x, acc[k][2 * i].y, acc[k][2 * i + 1].x, acc[k][2 * i + 1].y);
        }
        __syncthreads();
        if (tid < Lv) {
            const int src = (y - (k >> 1) + 1) * EW + (x - (k & 1) + 1);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 f = X[i * E + src];
                out[2 * i] = __fadd2_rn(out[2 * i], make_float2(f.x, f.y));
                out[2 * i + 1] = __fadd2_rn(out[2 * i + 1], make_float2(f.z, f.w));
            }
        }
        __syncthreads();
    }
    if (tid < Lv) {
        const unsigned pm = pois[tid];
        float f[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            f[2 * i] = (pm >> (2 * i)) & 1u ? qnan : out[i].x;
            f[2 * i + 1] = (pm >> (2 * i + 1)) & 1u ? qnan : out[i].y;
        }
        store_vec<bf16, 16>(grad_value + ((size_t)bh * Lv + tid) * 16, f);
    }
}

// The cell-owner kernel's shared-memory plan, or false when the shape or alignment is not its.
bool plan_backward_cell(const Geom &g, const void *value, const float *loc, const void *attn, const void *gout,
                        const void *grad_value, const float *grad_loc, const void *grad_attn, int optin,
                        CellPlan &cp) {
    if (g.L != 1 || g.D != 16) return false;
    if (!(g.P == 1 || g.P == 2 || g.P == 4 || g.P == 8)) return false;
    const long long W = g.lw[0], Hh = g.lh[0];
    const long long E = (W + 1) * (Hh + 1), S = (long long)g.Lq * g.P;
    if (E > kCellThreads || g.Lv > kCellThreads || S < 1 || S > 65535) return false;
    if (!aligned(value, 16) || !aligned(grad_value, 16) || !aligned(gout, 16) || !aligned(loc, 8) ||
        !aligned(grad_loc, 8) || !aligned(attn, 2) || !aligned(grad_attn, 2))
        return false;
    if (read_tune(kKnobMsdaCell).stage == 0) return false;
    auto r16 = [](size_t x) { return (x + 15) & ~(size_t)15; };
    size_t o = 0;
    cp.o_vs = (unsigned)o;
    o += (size_t)g.Lv * 32;
    cp.o_stash = (unsigned)o;
    o += std::max((size_t)S * 16, (size_t)E * 64);
    cp.o_rec = (unsigned)o;
    o += r16((size_t)S * 2);
    cp.o_cnt = (unsigned)o;
    o += r16((size_t)E * 4);
    cp.o_off = (unsigned)o;
    o += r16((size_t)(E + 1) * 4);
    cp.o_pois = (unsigned)o;
    o += r16((size_t)g.Lv * 4);
    cp.smem = o;
    return cp.smem <= (size_t)optin;
}

template <int P>
int launch_backward_cell(const Geom &g, const CellPlan &cp, const void *value, const float *loc, const void *attn,
                         const void *gout, void *gv, float *gl, void *ga, cudaStream_t s) {
    auto k = msda_backward_cell_kernel<P>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cp.smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    k<<<(unsigned)(g.B * g.H), kCellThreads, cp.smem, s>>>(
        static_cast<const bf16 *>(value), loc, static_cast<const bf16 *>(attn), static_cast<const bf16 *>(gout),
        static_cast<bf16 *>(gv), gl, static_cast<bf16 *>(ga), g, cp);
    return launch_status();
}

// bf16 values and weights only (the gradient rows are then bf16 too).
int try_backward_cell(const Geom &g, const void *value, const float *loc, const void *attn, const void *gout,
                      void *gv, float *gl, void *ga, cudaStream_t s) {
    CellPlan cp;
    if (!plan_backward_cell(g, value, loc, attn, gout, gv, gl, ga, max_smem_optin(), cp)) return -1;
    switch (g.P) {
        case 1: return launch_backward_cell<1>(g, cp, value, loc, attn, gout, gv, gl, ga, s);
        case 2: return launch_backward_cell<2>(g, cp, value, loc, attn, gout, gv, gl, ga, s);
        case 4: return launch_backward_cell<4>(g, cp, value, loc, attn, gout, gv, gl, ga, s);
        case 8: return launch_backward_cell<8>(g, cp, value, loc, attn, gout, gv, gl, ga, s);
    }
    return -1;
}

// ------------------------------------------------------------------------------------------
// Position-tile backward: levels of any size, float32 or bf16 values, no float atomics.
//
// K0 (msda_backward_rowsort_kernel), one CTA per (slab, level): a counting sort of the level's
// samples by the first row their bilinear taps touch (floor(iy), clamped to [-1, H-1]; samples
// with non-finite positions go to a last bucket that no tile reads).  A tile then finds every
// sample that can touch its rows in one contiguous range of the sorted list.
//
// K1 (msda_backward_tile_kernel) runs one CTA per (slab, tile); a tile is a run of up to `np`
// consecutive positions of one level.  Each thread owns one position and CPT channels of it:
// the value row segment and its gradient accumulator (float32 for bf16 values, float64 for
// float32 values) stay in registers for the whole launch; dense small levels spread a
// position's records over R replica owners whose accumulators are summed at the end.  The CTA
// walks its sample range in chunks: it computes the taps, files each corner landing in the tile
// into its position's bin in shared memory, and the owners drain their bins -- acc += coef * g[q]
// and the corner's dot product G = <value row, g[q]> (reduced over the position's lanes),
// written to a per-corner array in the workspace.  grad_value is written once, from the
// registers.  Gradient rows come from shared memory (all of the slab's rows, staged once) when
// they fit, else from L2.
//
// K2 (msda_backward_finish_kernel) is one thread per sample: from the four corners' G it forms
// the weight gradient and the location gradient (d ix / d loc = W), as the reference's autodiff
// does (deform_pallas.py:97-120 states the same formulas).
//
// The reference's non-finite semantics: an out-of-range corner contributes m * (v . g) = NaN to
// the weight/location gradients when its clipped value row or the gradient row holds inf/NaN,
// and scatters 0 * a * w * g (NaN where g is not finite, or where a is) into its clipped row.
// K1 files such a corner with its (zero or NaN) coefficient when the gradient row or the
// coefficient is non-finite, so the owner adds exactly that; and K1 raises a per-slab flag when
// it sees a non-finite value or gradient row, under which K2 recomputes the out-of-range
// corners' m * (v . g) from the rows themselves.
// ------------------------------------------------------------------------------------------
constexpr int kTileThreadsMax = 512;
#ifndef RFDETR_TILE_MIN_BLOCKS
#define RFDETR_TILE_MIN_BLOCKS 2  // two 512-thread CTAs per SM: 64 registers a thread
#endif
constexpr int kTileMaxPerThread = 8;     // samples a thread files per chunk (4 pending bits each)
constexpr int kTilePoison = 0x8000;      // record flag: out-of-range corner filed for its NaN, no G
constexpr int kTileMaxRows = 8192;       // rows of a level the row sort handles
constexpr int kTileMaxReplicas = 8;

struct TilePlan {
    int segs;                          // threads per position (D / CPT)
    int chunk;                         // samples per chunk (<= kTileMaxPerThread * threads)
    int tiles_before[kMaxLevels + 1];  // first CTA of each level (per slab): tiles x splits
    int np[kMaxLevels];                // positions per tile, per level
    int cap[kMaxLevels];               // bin slots per position, per level
    int rep[kMaxLevels];               // replica owners per position, per level
    int split[kMaxLevels];             // CTAs sharing a tile's samples (partial sums reduced after)
    int stage[kMaxLevels];             // the slab's gradient rows are staged in shared memory
    int part[kMaxLevels + 1];          // first partial-sum row of each level (per slab; S rows a position)
    int ppos[kMaxLevels + 1];          // first split-level position of each level (per slab)
    int gstride;                       // staged gradient row stride, bytes
    int roff[kMaxLevels + 1];          // first row-offset entry of each level (per slab)
    unsigned o_g, o_ids, o_cnt, o_bins;
    size_t smem;
    int nthr;
};

// Per-level fields of a TilePlan and a Geom, copied to shared memory once per CTA.
enum { kLvW, kLvH, kLvS, kLvNp, kLvCap, kLvRep, kLvSplit, kLvStage, kLvTiles, kLvRoff, kLvPart, kLvFields };

template <int N>
__device__ __forceinline__ int select_level(const int (&a)[N], int l) {
    int r = a[0];
#pragma unroll
    for (int i = 1; i < N; ++i)
        if (i == l) r = a[i];
    return r;
}

// Clamped first row of a sample's taps, plus one: a key in [0, H]; H + 1 for non-finite positions.
__device__ __forceinline__ int row_key(float ly, float hf, int H) {
    const float gy = __fmaf_rn(2.f, ly, -1.f);
    const float iy = __fmaf_rn(__fmul_rn(__fadd_rn(gy, 1.f), hf), 0.5f, -0.5f);
    if (!(fabsf(iy) <= 3.0e38f)) return H + 1;
    const float f = fminf(fmaxf(floorf(iy), -1.f), (float)(H - 1));
    return (int)f + 1;
}

template <int P>
__global__ void __launch_bounds__(512)
msda_backward_rowsort_kernel(const float *__restrict__ loc, int *__restrict__ list, int *__restrict__ roffs,
                             const Geom g, const TilePlan tp) {
    constexpr int PS = P == 1 ? 0 : P == 2 ? 1 : P == 4 ? 2 : 3;
    __shared__ int cnt[kTileMaxRows + 2];
    const int l = blockIdx.x, bh = blockIdx.y;
    const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
    const int Hh = select_level(g.lh, l);
    const float hf = (float)Hh;
    const int nb = Hh + 2;
    const int LP = g.L * P;
    const int n = g.Lq * P;
    for (int i = threadIdx.x; i < nb; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    auto key_of = [&](int i) {
        const int q = i >> PS, p = i & (P - 1);
        const size_t srow = (((size_t)b * g.Lq + q) * g.H + h) * LP + l * P + p;
        return row_key(__ldg(reinterpret_cast<const float2 *>(loc) + srow).y, hf, Hh);
    };
    for (int i = threadIdx.x; i < n; i += blockDim.x) atomicAdd(&cnt[key_of(i)], 1);
    __syncthreads();
    // Exclusive scan of the nb counts by warp 0: each lane sums a contiguous run.
    int *ro = roffs + (size_t)bh * tp.roff[kMaxLevels] + select_level(tp.roff, l);
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const int per = (nb + 31) / 32, k0 = min(lane * per, nb), k1 = min(k0 + per, nb);
        int sum = 0;
        for (int k = k0; k < k1; ++k) sum += cnt[k];
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        int run = incl - sum;
        for (int k = k0; k < k1; ++k) {
            const int c = cnt[k];
            cnt[k] = run;
            ro[k] = run;
            run += c;
        }
        if (lane == 31) ro[nb] = incl;
    }
    __syncthreads();
    int *dst = list + ((size_t)bh * g.L + l) * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[atomicAdd(&cnt[key_of(i)], 1)] = i;
}

template <typename TV, typename TW, int P, int CPT>
__global__ void __launch_bounds__(kTileThreadsMax, RFDETR_TILE_MIN_BLOCKS)
msda_backward_tile_kernel(const TV *__restrict__ value, const float *__restrict__ loc, const TW *__restrict__ attn,
                          const typename OutOf<TV, TW>::T *__restrict__ grad_out, TV *__restrict__ grad_value,
                          typename AccOf<TV>::T *__restrict__ gcorner, int *__restrict__ flags,
                          const int *__restrict__ list, const int *__restrict__ roffs,
                          typename AccOf<TV>::T *__restrict__ partial, const Geom g, const TilePlan tp) {
    using TG = typename OutOf<TV, TW>::T;
    using AT = typename AccOf<TV>::T;
    constexpr int PS = P == 1 ? 0 : P == 2 ? 1 : P == 4 ? 2 : 3;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_bad;
    __shared__ int lvt[kMaxLevels][kLvFields];
    if (threadIdx.x < g.L) {
        const int i = threadIdx.x;
        lvt[i][kLvW] = g.lw[i];
        lvt[i][kLvH] = g.lh[i];
        lvt[i][kLvS] = g.ls[i];
        lvt[i][kLvNp] = tp.np[i];
        lvt[i][kLvCap] = tp.cap[i];
        lvt[i][kLvRep] = tp.rep[i];
        lvt[i][kLvSplit] = tp.split[i];
        lvt[i][kLvStage] = tp.stage[i];
        lvt[i][kLvTiles] = tp.tiles_before[i];
        lvt[i][kLvRoff] = tp.roff[i];
        lvt[i][kLvPart] = tp.part[i];
    }
    __syncthreads();
    const int bh = blockIdx.y;
    const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
    const int cta = blockIdx.x;
    int l = 0;
    for (int i = 1; i < g.L; ++i)
        if (lvt[i][kLvTiles] <= cta) l = i;
    const int W = lvt[l][kLvW], Hh = lvt[l][kLvH], ls = lvt[l][kLvS];
    const float Wf = (float)W, Hf = (float)Hh;
    const int npl = lvt[l][kLvNp];
    const int S = lvt[l][kLvSplit];
    const int local = cta - lvt[l][kLvTiles];
    const int tl = local / S, sp = local - (local / S) * S;
    const int p0 = tl * npl;
    const int np = min(npl, W * Hh - p0);
    const int cap = lvt[l][kLvCap];
    const int R = lvt[l][kLvRep];
    const bool stage_g = lvt[l][kLvStage] != 0;
    const int row_lo = p0 / W, row_hi = (p0 + np - 1) / W;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int segs = tp.segs;
    const int seg = tid % segs, u = tid / segs;
    const int pl = u % npl, rep = u / npl;
    const bool owner = pl < np && rep < R;
    const int LP = g.L * P;
    const int D = g.D;
    const size_t slab_rows = (size_t)bh * g.Lv;

    int *const counts = reinterpret_cast<int *>(smem + tp.o_cnt);
    float *const bcoef = reinterpret_cast<float *>(smem + tp.o_bins);
    unsigned short *const bidx = reinterpret_cast<unsigned short *>(smem + tp.o_bins + (size_t)cap * npl * 4);
    int *const ids = reinterpret_cast<int *>(smem + tp.o_ids);
    unsigned char *const gst = smem + tp.o_g;

    // The tile's samples: keys [row_lo, row_hi + 1] of the level's row-sorted list; split CTAs
    // take equal shares of that range.
    const int *ro = roffs + (size_t)bh * tp.roff[kMaxLevels] + lvt[l][kLvRoff];
    const int r_begin = __ldg(ro + max(row_lo, 0)), r_end = __ldg(ro + min(row_hi + 1, Hh) + 1);
    const int s_begin = r_begin + (int)(((long long)(r_end - r_begin) * sp) / S);
    const int s_end = r_begin + (int)(((long long)(r_end - r_begin) * (sp + 1)) / S);
    const int *slist = list + ((size_t)bh * g.L + l) * (g.Lq * P);

    if (tid == 0) s_bad = 0;
    for (int i = tid; i < npl; i += nthr) counts[i] = 0;
    // The slab's gradient rows, staged once (all queries), for dense levels.
    if (stage_g) {
        const int gch = D * (int)sizeof(TG) / 16;
        for (int i = tid; i < g.Lq * gch; i += nthr) {
            const int q = i / gch, j = i - (i / gch) * gch;
            cp_async_bytes(gst + (size_t)q * tp.gstride + j * 16,
                           reinterpret_cast<const char *>(grad_out + (((size_t)b * g.Lq + q) * g.H + h) * D) + j * 16,
                           16);
        }
    }
    cp_async_commit();

    // Owner state.
    constexpr int NV = CPT / 2;
    float2 vv[NV];
    AT acc[CPT];
#pragma unroll
    for (int i = 0; i < CPT; ++i) acc[i] = (AT)0;
    bool vbad = false;
    {
        const int pos = ls + p0 + (owner ? pl : 0);
        const TV *vp = value + (slab_rows + pos) * D + seg * CPT;
        if constexpr (sizeof(TV) == 2) {
#pragma unroll
            for (int k = 0; k < CPT / 8; ++k) {
                const uint4 r = owner ? __ldg(reinterpret_cast<const uint4 *>(vp) + k) : make_uint4(0, 0, 0, 0);
                vv[4 * k + 0] = bf16x2_lo_hi(r.x);
                vv[4 * k + 1] = bf16x2_lo_hi(r.y);
                vv[4 * k + 2] = bf16x2_lo_hi(r.z);
                vv[4 * k + 3] = bf16x2_lo_hi(r.w);
            }
        } else {
#pragma unroll
            for (int k = 0; k < CPT / 4; ++k) {
                const float4 r = owner ? __ldg(reinterpret_cast<const float4 *>(vp) + k) : make_float4(0, 0, 0, 0);
                vv[2 * k] = make_float2(r.x, r.y);
                vv[2 * k + 1] = make_float2(r.z, r.w);
            }
        }
        vbad = any_nonfinite<NV>(vv);
    }
    cp_async_wait_all();
    __syncthreads();  // s_bad, counts and the staged rows are ready
    if (vbad) s_bad = 1;

    auto to_pairs = [&](const uint4 *src, float2 *q, bool global) {
        if constexpr (sizeof(TG) == 2) {
#pragma unroll
            for (int k = 0; k < CPT / 8; ++k) {
                const uint4 x = global ? __ldg(src + k) : src[k];
                q[4 * k + 0] = bf16x2_lo_hi(x.x);
                q[4 * k + 1] = bf16x2_lo_hi(x.y);
                q[4 * k + 2] = bf16x2_lo_hi(x.z);
                q[4 * k + 3] = bf16x2_lo_hi(x.w);
            }
        } else {
#pragma unroll
            for (int k = 0; k < CPT / 4; ++k) {
                const uint4 x = global ? __ldg(src + k) : src[k];
                q[2 * k] = make_float2(__uint_as_float(x.x), __uint_as_float(x.y));
                q[2 * k + 1] = make_float2(__uint_as_float(x.z), __uint_as_float(x.w));
            }
        }
    };
    auto g_row = [&](int q, int chan) -> const uint4 * {
        if (stage_g) return reinterpret_cast<const uint4 *>(gst + (size_t)q * tp.gstride + chan * sizeof(TG));
        return reinterpret_cast<const uint4 *>(grad_out + (((size_t)b * g.Lq + q) * g.H + h) * D + chan);
    };
    // True when the gradient row of query q holds inf/NaN.
    auto g_row_bad = [&](int q) {
        bool bad = false;
        for (int k = 0; k < D; k += CPT) {
            float2 x[NV];
            to_pairs(g_row(q, k), x, !stage_g);
            bad |= any_nonfinite<NV>(x);
        }
        return bad;
    };

    // Files the corners of chunk slot j (selected by `want`) that land in the tile; returns those
    // whose bin was full.
    auto file = [&](int j, unsigned want) -> unsigned {
        const int id = ids[j];
        const int q = id >> PS, p = id & (P - 1);
        const size_t srow = (((size_t)b * g.Lq + q) * g.H + h) * LP + l * P + p;
        const float2 xy = __ldg(reinterpret_cast<const float2 *>(loc) + srow);
        const float a = to_f32(__ldg(attn + srow));
        float ix, iy;
        sample_coords(xy.x, xy.y, Wf, Hf, ix, iy);
        if (!(fabsf(ix) <= 3.0e38f && fabsf(iy) <= 3.0e38f)) return 0u;
        const Axis ay = axis_taps(iy, Hf, Hh);
        if (ay.c1 < row_lo || ay.c0 > row_hi) return 0u;  // both rows outside the tile's band
        const Axis ax = axis_taps(ix, Wf, W);
        const float m[4] = {ax.m0 * ay.m0, ax.m1 * ay.m0, ax.m0 * ay.m1, ax.m1 * ay.m1};
        const float ax0 = a * ax.w0, ax1 = a * ax.w1;
        const float cf[4] = {ax0 * ay.w0 * m[0], ax1 * ay.w0 * m[1], ax0 * ay.w1 * m[2], ax1 * ay.w1 * m[3]};
        const int pp[4] = {ay.c0 * W + ax.c0, ay.c0 * W + ax.c1, ay.c1 * W + ax.c0, ay.c1 * W + ax.c1};
        int gb_state = -1;  // gradient row finiteness, looked up once if needed
        unsigned failed = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (!((want >> k) & 1u)) continue;
            const int pt = pp[k] - p0;
            if ((unsigned)pt >= (unsigned)np) continue;
            bool filed = m[k] != 0.f;
            bool poison = false;
            if (!filed) {
                if (gb_state < 0) {
                    gb_state = g_row_bad(q) ? 1 : 0;
                    if (gb_state) s_bad = 1;
                }
                filed = cf[k] != 0.f || gb_state != 0;
                poison = true;
            }
            if (!filed) continue;
            const int slot = atomicAdd(&counts[pt], 1);
            if (slot < cap) {
                bcoef[slot * npl + pt] = cf[k];
                bidx[slot * npl + pt] = (unsigned short)(((j << 2) | k) | (poison ? kTilePoison : 0));
            } else {
                failed |= 1u << k;
            }
        }
        return failed;
    };

    // Owners drain their bins: replica r takes slots r, r + R, ...
    const unsigned group = segs >= 32 ? 0xffffffffu : (((1u << segs) - 1u) << (((tid & 31) / segs) * segs));
    auto own = [&]() {
        int n = 0;
        if (owner) n = min(counts[pl], cap);
        __syncthreads();  // every replica has read its count
        if (owner && rep == 0 && seg == 0) counts[pl] = 0;
        for (int e = rep; e < n; e += R) {
            const float cfe = bcoef[e * npl + pl];
            const unsigned idx = bidx[e * npl + pl];
            const int j = (int)((idx & 0x7fffu) >> 2), k = (int)(idx & 3u);
            const int id = ids[j];
            const int q = id >> PS, p = id & (P - 1);
            float2 qv[NV];
            to_pairs(g_row(q, seg * CPT), qv, !stage_g);
            AT dot;
            if constexpr (sizeof(TV) == 2) {
                const float2 cc = make_float2(cfe, cfe);
                float2 d = __fmul2_rn(vv[0], qv[0]);
#pragma unroll
                for (int i = 1; i < NV; ++i) d = __ffma2_rn(vv[i], qv[i], d);
#pragma unroll
                for (int i = 0; i < NV; ++i) {
                    const float2 t = __ffma2_rn(cc, qv[i], make_float2(acc[2 * i], acc[2 * i + 1]));
                    acc[2 * i] = t.x;
                    acc[2 * i + 1] = t.y;
                }
                dot = d.x + d.y;
            } else {
                double d = 0.0;
#pragma unroll
                for (int i = 0; i < NV; ++i) {
                    d = fma((double)vv[i].x, (double)qv[i].x, d);
                    d = fma((double)vv[i].y, (double)qv[i].y, d);
                    acc[2 * i] = fma((double)cfe, (double)qv[i].x, acc[2 * i]);
                    acc[2 * i + 1] = fma((double)cfe, (double)qv[i].y, acc[2 * i + 1]);
                }
                dot = d;
            }
            for (int o = segs >> 1; o > 0; o >>= 1) dot += __shfl_xor_sync(group, dot, o);
            if (seg == 0 && !(idx & kTilePoison))
                gcorner[((((size_t)b * g.Lq + q) * g.H + h) * LP + l * P + p) * 4 + k] = dot;
        }
    };

    const int per_thread = (tp.chunk + nthr - 1) / nthr;
    for (int c0 = s_begin; c0 < s_end; c0 += tp.chunk) {
        const int nc = min(tp.chunk, s_end - c0);
        __syncthreads();  // the previous chunk is drained (its ids and bins are free)
        for (int j = tid; j < nc; j += nthr) ids[j] = __ldg(slist + c0 + j);
        __syncthreads();
        unsigned pending = 0;
        for (int i = 0; i < per_thread; ++i) {
            const int j = tid + i * nthr;
            if (j < nc) pending |= file(j, 0xFu) << (4 * i);
        }
        bool again = __syncthreads_or(pending != 0u);
        own();
        for (int round = 0; again && round < 65536; ++round) {  // full bins: refile what did not fit
            __syncthreads();
            unsigned left = 0;
            for (int i = 0; i < per_thread; ++i) {
                const int j = tid + i * nthr;
                const unsigned want = (pending >> (4 * i)) & 0xFu;
                if (want && j < nc) left |= file(j, want) << (4 * i);
            }
            pending = left;
            again = __syncthreads_or(pending != 0u);
            own();
        }
    }
    // Replicas r > 0 hand their accumulators to replica 0 through shared memory (the bins are no
    // longer needed), which adds them in replica order.
    AT *red = reinterpret_cast<AT *>(smem + tp.o_bins);
    if (R > 1) {
        __syncthreads();
        if (owner && rep > 0) {
#pragma unroll
            for (int i = 0; i < CPT; ++i) red[((size_t)(rep - 1) * npl + pl) * D + seg * CPT + i] = acc[i];
        }
        __syncthreads();
        if (owner && rep == 0) {
            for (int r = 1; r < R; ++r) {
#pragma unroll
                for (int i = 0; i < CPT; ++i) acc[i] += red[((size_t)(r - 1) * npl + pl) * D + seg * CPT + i];
            }
        }
    }
    if (owner && rep == 0) {
        if (S == 1) {
            TV *dst = grad_value + (slab_rows + ls + p0 + pl) * D + seg * CPT;
            float f[CPT];
#pragma unroll
            for (int i = 0; i < CPT; ++i) f[i] = (float)acc[i];
            store_vec<TV, CPT>(dst, f);
        } else {
            // Partial sum of this split: row (level partial base + position) * S + split.
            AT *dst = partial + ((size_t)bh * tp.part[kMaxLevels] + lvt[l][kLvPart] + (size_t)(p0 + pl) * S + sp) * D +
                      seg * CPT;
#pragma unroll
            for (int i = 0; i < CPT; ++i) dst[i] = acc[i];
        }
    }
    __syncthreads();
    if (tid == 0 && s_bad) atomicOr(flags + bh, 1);
}

// Sums the split partials of the split levels in split order and writes grad_value.
template <typename TV>
__global__ void __launch_bounds__(256)
msda_backward_split_reduce_kernel(const typename AccOf<TV>::T *__restrict__ partial, TV *__restrict__ grad_value,
                                  const Geom g, const TilePlan tp) {
    using AT = typename AccOf<TV>::T;
    const int bh = blockIdx.y;
    const int positions = tp.ppos[kMaxLevels];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < positions * g.D; i += gridDim.x * blockDim.x) {
        const int r = i / g.D, ch = i - (i / g.D) * g.D;
        int l = 0;
        for (int k = 1; k < g.L; ++k)
            if (tp.ppos[k] <= r) l = k;
        const int S = tp.split[l];
        const int pos = r - tp.ppos[l];
        const AT *src = partial + ((size_t)bh * tp.part[kMaxLevels] + tp.part[l] + (size_t)pos * S) * g.D + ch;
        AT sum = src[0];
        for (int k = 1; k < S; ++k) sum += src[(size_t)k * g.D];
        grad_value[((size_t)bh * g.Lv + g.ls[l] + pos) * g.D + ch] = from_f32<TV>((float)sum);
    }
}

// K2: weight and location gradients of every sample from its corners' G.
template <typename TV, typename TW, int P>
__global__ void __launch_bounds__(256)
msda_backward_finish_kernel(const TV *__restrict__ value, const float *__restrict__ loc, const TW *__restrict__ attn,
                            const typename OutOf<TV, TW>::T *__restrict__ grad_out,
                            const typename AccOf<TV>::T *__restrict__ gcorner, const int *__restrict__ flags,
                            float *__restrict__ grad_loc, TW *__restrict__ grad_attn, const Geom g) {
    using AT = typename AccOf<TV>::T;
    constexpr int PS = P == 1 ? 0 : P == 2 ? 1 : P == 4 ? 2 : 3;
    __shared__ LevelTable lv;
    load_levels(lv, g);
    __syncthreads();
    // Sample indices fit in 31 bits (validated), so the decoding below is 32-bit arithmetic.
    const int total = g.B * g.Lq * g.H * g.L * P;
    const int LP = g.L * P;
    const float qnan = __int_as_float(0x7fc00000);
    for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < total; s += gridDim.x * blockDim.x) {
        const int row = s / LP;  // (b, q, h)
        const int l = (s - row * LP) >> PS;
        const int W = lv.w[l], Hh = lv.h[l];
        const float Wf = (float)W, Hf = (float)Hh;
        const float2 xy = __ldg(reinterpret_cast<const float2 *>(loc) + s);
        const float a = to_f32(__ldg(attn + s));
        const OwnTaps t = own_taps(xy, Wf, Hf, W, Hh);
        float2 out_loc;
        float out_attn;
        if (!t.ok) {
            out_loc = make_float2(qnan, qnan);
            out_attn = qnan;
        } else {
            const float m[4] = {t.m00, t.m10, t.m01, t.m11};
            AT e[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) e[k] = m[k] != 0.f ? __ldg(gcorner + (size_t)s * 4 + k) : (AT)0;
            if (m[0] == 0.f || m[1] == 0.f || m[2] == 0.f || m[3] == 0.f) {
                const int b = row / (g.Lq * g.H), h = row - (row / g.H) * g.H;
                const int bh = b * g.H + h;
                if (__ldg(flags + bh)) {
                    // Out-of-range corners: m * (v . g), NaN when the clipped row or g is not finite.
                    const int pp[4] = {t.p00, t.p10, t.p01, t.p11};
                    const auto *grow = grad_out + (size_t)row * g.D;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (m[k] != 0.f) continue;
                        const TV *vrow = value + ((size_t)bh * g.Lv + lv.s[l] + pp[k]) * g.D;
                        AT d = 0;
                        for (int ch = 0; ch < g.D; ++ch) d += (AT)to_f32(vrow[ch]) * (AT)to_f32(grow[ch]);
                        e[k] = (AT)0 * d;
                    }
                }
            }
            const AT wx1 = t.wx1, wy1 = t.wy1, wx0 = (AT)1 - wx1, wy0 = (AT)1 - wy1;
            const AT ds = wy0 * (wx0 * e[0] + wx1 * e[1]) + wy1 * (wx0 * e[2] + wx1 * e[3]);
            const AT dx = wy0 * (e[1] - e[0]) + wy1 * (e[3] - e[2]);
            const AT dy = wx0 * (e[2] - e[0]) + wx1 * (e[3] - e[1]);
            out_attn = (float)ds;
            out_loc = make_float2((float)((AT)Wf * ((AT)a * dx)), (float)((AT)Hf * ((AT)a * dy)));
        }
        grad_attn[s] = from_f32<TW>(out_attn);
        reinterpret_cast<float2 *>(grad_loc)[s] = out_loc;
    }
}

// Host planning of the tile backward (one plan for every level).  Returns false when the shape or
// alignment does not fit.
template <typename TV, typename TW>
bool plan_backward_tiles(const Geom &g, const void *value, const float *loc, const void *attn, const void *gout,
                         const void *grad_value, int optin, TilePlan &tp, int &cpt) {
    using TG = typename OutOf<TV, TW>::T;
    using AT = typename AccOf<TV>::T;
    if (!(g.P == 1 || g.P == 2 || g.P == 4 || g.P == 8)) return false;
    cpt = sizeof(TV) == 2 ? 16 : 8;
    if (g.D % cpt != 0 && sizeof(TV) == 2 && g.D % 8 == 0) cpt = 8;
    if (g.D % cpt != 0) return false;
    tp.segs = g.D / cpt;
    if (tp.segs > 32 || (tp.segs & (tp.segs - 1)) != 0) return false;
    if (!aligned(value, 16) || !aligned(grad_value, 16) || !aligned(gout, 16) || !aligned(loc, 8) ||
        !aligned(attn, sizeof(TW)))
        return false;
    if (((size_t)g.D * sizeof(TG)) % 16 != 0) return false;
    // Opt-in (the knob's second field set to 1): at config 3 this path measured 192 us (bf16) and
    // 280 us (float32) against 104 / 106 us for the accumulate kernel, so it is not the default.
    const Tune tune = read_tune(kKnobMsdaTiles);
    if (tune.stage != 1) return false;
    const int nthr_max = tune.threads > 0 ? std::min(tune.threads, kTileThreadsMax) : kTileThreadsMax;
    const int np_max = std::max(1, nthr_max / tp.segs);
    int npl_max = 1;
    for (int l = 0; l < g.L; ++l) {
        const int hw = g.lh[l] * g.lw[l];
        if (g.lh[l] > kTileMaxRows) return false;
        const int nt = (hw + np_max - 1) / np_max;
        tp.np[l] = (hw + nt - 1) / nt;
        npl_max = std::max(npl_max, tp.np[l]);
    }
    tp.nthr = ((npl_max * tp.segs + 31) / 32) * 32;
    if (tp.nthr > kTileThreadsMax) return false;
    // Dense levels (many records per position): replica owners where the tile leaves threads
    // idle, then splits of the tile's samples over several CTAs so that an owner drains about 16
    // records; their gradient rows are staged.
    int total = 0, roff = 0, part = 0, ppos = 0;
    for (int l = 0; l < g.L; ++l) {
        const int hw = g.lh[l] * g.lw[l];
        const double records = (double)g.P * 4.0 * g.Lq / hw;
        const int fit = tp.nthr / (tp.np[l] * tp.segs);
        int r = 1;
        while (r * 2 <= std::min(fit, kTileMaxReplicas) && records >= 16.0 * r) r *= 2;
        tp.rep[l] = r;
        int sp = 1;
        while (sp < 16 && records / (r * sp) > 24.0) sp *= 2;
        tp.split[l] = sp;
        tp.stage[l] = tune.acc != 0 && records >= 4.0;
        tp.tiles_before[l] = total;
        total += ((hw + tp.np[l] - 1) / tp.np[l]) * sp;
        tp.roff[l] = roff;
        roff += g.lh[l] + 3;
        tp.part[l] = part;
        tp.ppos[l] = ppos;
        if (sp > 1) {
            part += hw * sp;
            ppos += hw;
        }
    }
    for (int l = g.L; l < kMaxLevels; ++l) {
        tp.np[l] = 1;
        tp.tiles_before[l] = total;
        tp.roff[l] = roff;
        tp.part[l] = part;
        tp.ppos[l] = ppos;
        tp.cap[l] = 1;
        tp.rep[l] = 1;
        tp.split[l] = 1;
        tp.stage[l] = 0;
    }
    tp.tiles_before[kMaxLevels] = total;
    tp.roff[kMaxLevels] = roff;
    tp.part[kMaxLevels] = part;
    tp.ppos[kMaxLevels] = ppos;
    if (total > 65535 || (long long)g.B * g.H > 65535) return false;
    tp.gstride = g.D * (int)sizeof(TG) + 16;
    auto r16 = [](size_t x) { return (x + 15) & ~(size_t)15; };
    // Bins: records per position per chunk follow a Poisson law around (chunk samples of the
    // tile's row band) * 4 / (band positions); the cap leaves room for ~4 standard deviations (a
    // full bin is refiled, so any sampling pattern stays exact).  The chunk is the largest of
    // 8, 4, 2 or 1 samples per thread that keeps the CTA two to an SM with the staged rows.
    const size_t two_per_sm = std::min<size_t>((size_t)optin, 113 * 1024);
    bool any_stage = false;
    for (int l = 0; l < g.L; ++l) any_stage |= tp.stage[l] != 0;
    const size_t gbytes = any_stage ? r16((size_t)g.Lq * tp.gstride) : 0;
    auto fixed_bytes = [&](int chunk) {
        size_t bins_bytes = 0;
        for (int l = 0; l < g.L; ++l) {
            const int hw = g.lh[l] * g.lw[l];
            const double band = std::min<double>(g.lh[l], (double)tp.np[l] / g.lw[l] + 2.0);
            const double in_band =
                std::min<double>((double)chunk, (double)g.Lq * g.P * band / g.lh[l] / tp.split[l]);
            const double mean = in_band * 4.0 / std::min<double>(band * g.lw[l], hw);
            int cap = (int)std::ceil(mean + 4.0 * std::sqrt(mean) + 4.0);
            cap = std::max(4, std::min(cap, tune.hsub > 0 ? tune.hsub : 96));
            tp.cap[l] = cap;
            bins_bytes = std::max(bins_bytes, (size_t)cap * tp.np[l] * 6);
            bins_bytes = std::max(bins_bytes, (size_t)(tp.rep[l] - 1) * tp.np[l] * g.D * sizeof(AT));
        }
        return r16((size_t)chunk * 4) + r16((size_t)npl_max * 4) + r16(bins_bytes);
    };
    tp.chunk = 0;
    for (int per = kTileMaxPerThread; per >= 1 && !tp.chunk; per /= 2)
        if (fixed_bytes(per * tp.nthr) + gbytes <= two_per_sm) tp.chunk = per * tp.nthr;
    if (!tp.chunk) {
        // The staged rows do not fit beside the bins: read them from L2 instead.
        for (int l = 0; l < g.L; ++l) tp.stage[l] = 0;
        tp.chunk = 4 * tp.nthr;
    }
    const size_t fixed = fixed_bytes(tp.chunk);  // sets the caps of the chosen chunk
    bool staged = false;
    for (int l = 0; l < g.L; ++l) staged |= tp.stage[l] != 0;
    size_t o = 0;
    tp.o_g = (unsigned)o; o += staged ? gbytes : 0;
    tp.o_ids = (unsigned)o;
    tp.o_cnt = (unsigned)(tp.o_ids + r16((size_t)tp.chunk * 4));
    tp.o_bins = (unsigned)(tp.o_cnt + r16((size_t)npl_max * 4));
    o += fixed;
    tp.smem = o;
    return tp.smem <= (size_t)optin;
}

// Workspace of the tile backward: the per-corner G array, the per-slab flags, the row-sorted
// sample lists and their row offsets.
struct TileWs {
    size_t o_flags, o_list, o_roff, o_part, bytes;
};
// `split_rows`: partial-sum rows per slab (sum of the split levels' positions times their splits).
TileWs tile_workspace(int value_dtype, const Geom &g, size_t split_rows) {
    auto r256 = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t gsize = value_dtype == RFDETR_F32 ? sizeof(double) : sizeof(float);
    const size_t samples = (size_t)g.B * g.Lq * g.H * g.L * g.P;
    size_t rows = 0;
    for (int l = 0; l < g.L; ++l) rows += g.lh[l] + 3;
    TileWs w;
    w.o_flags = r256(samples * 4 * gsize);
    w.o_list = w.o_flags + r256((size_t)g.B * g.H * sizeof(int));
    w.o_roff = w.o_list + r256(samples * sizeof(int));
    w.o_part = w.o_roff + r256((size_t)g.B * g.H * rows * sizeof(int));
    w.bytes = w.o_part + r256((size_t)g.B * g.H * split_rows * g.D * gsize);
    return w;
}
size_t split_rows_of(const TilePlan &tp, const Geom &) { return (size_t)tp.part[kMaxLevels]; }

template <typename TV, typename TW, int P, int CPT>
int launch_backward_tiles_k(const Geom &g, const TilePlan &tp, const void *value, const float *loc, const void *attn,
                            const void *gout, void *gv, float *gl, void *ga, void *ws, int value_dtype,
                            cudaStream_t s) {
    using TG = typename OutOf<TV, TW>::T;
    using AT = typename AccOf<TV>::T;
    const TileWs w = tile_workspace(value_dtype, g, split_rows_of(tp, g));
    char *base = static_cast<char *>(ws);
    AT *gcorner = reinterpret_cast<AT *>(base);
    int *flags = reinterpret_cast<int *>(base + w.o_flags);
    int *list = reinterpret_cast<int *>(base + w.o_list);
    int *roffs = reinterpret_cast<int *>(base + w.o_roff);
    AT *partial = reinterpret_cast<AT *>(base + w.o_part);
    if (cudaMemsetAsync(flags, 0, (size_t)g.B * g.H * sizeof(int), s) != cudaSuccess) return RFDETR_ERR_CUDA;
    msda_backward_rowsort_kernel<P><<<dim3((unsigned)g.L, (unsigned)(g.B * g.H)), 512, 0, s>>>(loc, list, roffs, g, tp);
    if (launch_status() != RFDETR_OK) return RFDETR_ERR_CUDA;
    auto k1 = msda_backward_tile_kernel<TV, TW, P, CPT>;
    if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tp.smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    const dim3 grid((unsigned)tp.tiles_before[kMaxLevels], (unsigned)(g.B * g.H));
    k1<<<grid, tp.nthr, tp.smem, s>>>(static_cast<const TV *>(value), loc, static_cast<const TW *>(attn),
                                       static_cast<const TG *>(gout), static_cast<TV *>(gv), gcorner, flags, list, roffs,
                                       partial, g, tp);
    if (launch_status() != RFDETR_OK) return RFDETR_ERR_CUDA;
    if (tp.ppos[kMaxLevels] > 0) {
        const unsigned blocks = (unsigned)std::max(1, std::min(64, (tp.ppos[kMaxLevels] * g.D + 255) / 256));
        msda_backward_split_reduce_kernel<TV><<<dim3(blocks, (unsigned)(g.B * g.H)), 256, 0, s>>>(
            partial, static_cast<TV *>(gv), g, tp);
        if (launch_status() != RFDETR_OK) return RFDETR_ERR_CUDA;
    }
    const long long samples = (long long)g.B * g.Lq * g.H * g.L * g.P;
    const unsigned blocks = (unsigned)std::min<long long>((samples + 255) / 256, (long long)num_sms() * 16);
    msda_backward_finish_kernel<TV, TW, P><<<std::max(blocks, 1u), 256, 0, s>>>(
        static_cast<const TV *>(value), loc, static_cast<const TW *>(attn), static_cast<const TG *>(gout), gcorner,
        flags, gl, static_cast<TW *>(ga), g);
    return launch_status();
}

template <typename TV, typename TW>
int try_backward_tiles(const Geom &g, const void *value, const float *loc, const void *attn, const void *gout,
                       void *gv, float *gl, void *ga, void *ws, size_t ws_bytes, int value_dtype, cudaStream_t s) {
    TilePlan tp;
    int cpt = 0;
    if (!plan_backward_tiles<TV, TW>(g, value, loc, attn, gout, gv, max_smem_optin(), tp, cpt)) return -1;
    if (!ws || ws_bytes < tile_workspace(value_dtype, g, split_rows_of(tp, g)).bytes || !aligned(ws, 256)) return -1;
    auto go = [&](auto p_tag, auto c_tag) {
        constexpr int PP = decltype(p_tag)::value, CC = decltype(c_tag)::value;
        return launch_backward_tiles_k<TV, TW, PP, CC>(g, tp, value, loc, attn, gout, gv, gl, ga, ws, value_dtype, s);
    };
    using I1 = std::integral_constant<int, 1>;
    using I2 = std::integral_constant<int, 2>;
    using I4 = std::integral_constant<int, 4>;
    using I8 = std::integral_constant<int, 8>;
    using I16 = std::integral_constant<int, 16>;
    if (cpt == 16) {
        if constexpr (sizeof(TV) == 2) {
            switch (g.P) {
                case 1: return go(I1{}, I16{});
                case 2: return go(I2{}, I16{});
                case 4: return go(I4{}, I16{});
                case 8: return go(I8{}, I16{});
            }
        }
        return -1;
    }
    switch (g.P) {
        case 1: return go(I1{}, I8{});
        case 2: return go(I2{}, I8{});
        case 4: return go(I4{}, I8{});
        case 8: return go(I8{}, I8{});
    }
    return -1;
}

// Workspace bytes the tile backward's plan for this geometry needs (0 when the plan does not
// apply), planned as for 256-byte-aligned buffers.
template <typename TV, typename TW>
size_t tile_workspace_bytes_t(const Geom &g, int value_dtype) {
    TilePlan tp;
    int cpt = 0;
    const void *a = reinterpret_cast<const void *>((uintptr_t)256);
    if (!plan_backward_tiles<TV, TW>(g, a, static_cast<const float *>(a), a, a, a, max_smem_optin(), tp, cpt))
        return 0;
    return tile_workspace(value_dtype, g, split_rows_of(tp, g)).bytes;
}
size_t tile_workspace_bytes(int value_dtype, int weight_dtype, const Geom &g) {
    if (value_dtype == RFDETR_BF16)
        return weight_dtype == RFDETR_BF16 ? tile_workspace_bytes_t<bf16, bf16>(g, value_dtype)
                                           : tile_workspace_bytes_t<bf16, float>(g, value_dtype);
    return weight_dtype == RFDETR_BF16 ? tile_workspace_bytes_t<float, bf16>(g, value_dtype)
                                       : tile_workspace_bytes_t<float, float>(g, value_dtype);
}

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
    {
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        int st2 = -1;
        if (value_dtype == RFDETR_BF16 && weight_dtype == RFDETR_BF16)
            st2 = try_forward_slab<bf16, bf16>(g, value, sampling_locations, attention_weights, output, s);
        else if (value_dtype == RFDETR_BF16)
            st2 = try_forward_slab<bf16, float>(g, value, sampling_locations, attention_weights, output, s);
        else if (weight_dtype == RFDETR_BF16)
            st2 = try_forward_slab<float, bf16>(g, value, sampling_locations, attention_weights, output, s);
        else
            st2 = try_forward_slab<float, float>(g, value, sampling_locations, attention_weights, output, s);
        if (st2 >= 0) return st2;
    }
    const void *ptrs[2] = {value, output};
    const int es[2] = {vs, os};
    Plan p;
    p.vec = pick_vec(g.D, vs, ptrs, es, 2);
    if (!p.vec) return aligned(value, vs) && aligned(output, os) ? RFDETR_ERR_SHAPE : RFDETR_ERR_ALIGN;
    p.team = next_pow2(g.D / p.vec);
    choose_layout(p, g, vs, false, value);
    const Tune tune = read_tune(kKnobMsdaFwd);
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

extern "C" size_t rfdetr_msda_backward_workspace_bytes(int value_dtype, int weight_dtype,
                                                       const int64_t *spatial_shapes, int64_t batch, int64_t n_heads,
                                                       int64_t head_dim, int64_t len_query, int64_t n_levels,
                                                       int64_t n_points) {
    if (!dtype_ok(value_dtype) || !dtype_ok(weight_dtype)) return 0;
    Geom g;
    if (validate(spatial_shapes, nullptr, batch, n_heads, head_dim, len_query, n_levels, n_points, g) != RFDETR_OK)
        return 0;
    if (g.B == 0 || g.Lq == 0) return 0;
    const size_t generic = rfdetr_msda_backward_workspace_size(value_dtype, batch, n_heads, head_dim, g.Lv);
    return std::max(generic, tile_workspace_bytes(value_dtype, weight_dtype, g));
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
    if (value_dtype == RFDETR_BF16 && g.Lq > 0 && aligned(sampling_locations, 8) && aligned(grad_sampling_locations, 8) &&
        aligned(attention_weights, ws) && aligned(grad_attention_weights, ws)) {
        int st2 = -1;
        if (weight_dtype == RFDETR_BF16)
            st2 = try_backward_cell(g, value, sampling_locations, attention_weights, grad_output, grad_value,
                                    grad_sampling_locations, grad_attention_weights, s);
        if (st2 >= 0) return st2;
        if (weight_dtype == RFDETR_BF16)
            st2 = try_backward_owner<bf16>(g, value, sampling_locations, attention_weights, grad_output, grad_value,
                                           grad_sampling_locations, grad_attention_weights, s);
        else
            st2 = try_backward_owner<float>(g, value, sampling_locations, attention_weights, grad_output, grad_value,
                                            grad_sampling_locations, grad_attention_weights, s);
        if (st2 >= 0) return st2;
        if (weight_dtype == RFDETR_BF16)
            st2 = try_backward_tiles<bf16, bf16>(g, value, sampling_locations, attention_weights, grad_output,
                                                 grad_value, grad_sampling_locations, grad_attention_weights,
                                                 workspace, workspace_bytes, value_dtype, s);
        else
            st2 = try_backward_tiles<bf16, float>(g, value, sampling_locations, attention_weights, grad_output,
                                                  grad_value, grad_sampling_locations, grad_attention_weights,
                                                  workspace, workspace_bytes, value_dtype, s);
        if (st2 >= 0) return st2;
        if (weight_dtype == RFDETR_BF16)
            st2 = try_backward_bins<bf16>(g, value, sampling_locations, attention_weights, grad_output, grad_value,
                                          grad_sampling_locations, grad_attention_weights, s);
        else
            st2 = try_backward_bins<float>(g, value, sampling_locations, attention_weights, grad_output, grad_value,
                                           grad_sampling_locations, grad_attention_weights, s);
        if (st2 >= 0) return st2;
    }
    if (value_dtype == RFDETR_F32 && g.Lq > 0 && aligned(sampling_locations, 8) &&
        aligned(grad_sampling_locations, 8) && aligned(attention_weights, ws) && aligned(grad_attention_weights, ws)) {
        const int st2 = weight_dtype == RFDETR_BF16
                            ? try_backward_tiles<float, bf16>(g, value, sampling_locations, attention_weights,
                                                              grad_output, grad_value, grad_sampling_locations,
                                                              grad_attention_weights, workspace, workspace_bytes,
                                                              value_dtype, s)
                            : try_backward_tiles<float, float>(g, value, sampling_locations, attention_weights,
                                                               grad_output, grad_value, grad_sampling_locations,
                                                               grad_attention_weights, workspace, workspace_bytes,
                                                               value_dtype, s);
        if (st2 >= 0) return st2;
    }
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
        const Tune tune = read_tune(kKnobMsdaBwd);
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
// the name is only a host-side stand-in, so its device address (in the current context) is
// looked up with cudaGetSymbolAddress on every call and passed to the kernels like a caller's
// workspace.
// ------------------------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = RFDETR_MSDA_NOALLOC_SCRATCH_BYTES;
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
        if (need > kNoAllocScratchBytes) {
            // Too large for the array: still served when a scratch-free kernel takes the shape (the
            // workspace path is then never reached); refused when the call would need scratch.
            const int st2 = rfdetr_msda_backward(stream, value, value_dtype, spatial_shapes, level_start_index,
                                                 sampling_locations, attention_weights, weight_dtype, grad_output,
                                                 grad_output_dtype, grad_value, grad_sampling_locations,
                                                 grad_attention_weights, nullptr, 0, batch, n_heads, head_dim,
                                                 len_query, n_levels, n_points);
            return st2 == RFDETR_ERR_WORKSPACE ? RFDETR_ERR_CAPACITY : st2;
        }
        // The array's address in the current context, looked up on every call (a host-side query,
        // no allocation): nothing cached can outlive a context that was reset or recreated.
        if (cudaGetSymbolAddress(&scratch, g_msda_noalloc_scratch) != cudaSuccess || !scratch) return RFDETR_ERR_CUDA;
        scratch_bytes = kNoAllocScratchBytes;
    }
    return rfdetr_msda_backward(stream, value, value_dtype, spatial_shapes, level_start_index, sampling_locations,
                                attention_weights, weight_dtype, grad_output, grad_output_dtype, grad_value,
                                grad_sampling_locations, grad_attention_weights, scratch, scratch_bytes, batch,
                                n_heads, head_dim, len_query, n_levels, n_points);
}

namespace rfdetr {
namespace {
// One CTA arms an mbarrier for 16 bytes that no copy delivers and waits for it at most `polls`
// polls: the wait must give up and raise the fault word.  Nothing is in flight, so nothing needs
// draining.
__global__ void bounded_wait_selftest_kernel(int polls, int32_t *result) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        mbar_init_fence();
        mbar_arrive_expect_tx(&bar, 16u);
    }
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0u, &abort_flag, polls);
    if (threadIdx.x == 0) *result = ok ? 1 : 0;
}
}  // namespace
}  // namespace rfdetr

extern "C" int rfdetr_selftest_bounded_wait(void *stream, int polls, int32_t *result) {
    if (polls < 1 || polls > rfdetr::kWaitLimit || !result) return RFDETR_ERR_SHAPE;
    rfdetr::bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(polls, result);
    return launch_status();
}

extern "C" int rfdetr_take_device_fault(void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned int v = 0;
    if (cudaMemcpyFromSymbolAsync(&v, rfdetr::g_device_fault, sizeof(v), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    if (v == 0) return RFDETR_OK;
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbolAsync(rfdetr::g_device_fault, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    return RFDETR_ERR_LIMIT;
}
