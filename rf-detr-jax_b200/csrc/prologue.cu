// Prologue of multi-scale deformable attention for sm_100a: from the decoder queries to the
// sampler's inputs, in one launch.
//
// Reference (src/rfdetr_jax/models/ops.py:381-404, MSDeformAttn.__call__):
//   offsets = Linear(query) -> [B, Lq, H, L, P, 2]       (sampling_offsets, layers.py:258-280)
//   logits  = Linear(query) -> [B, Lq, H, L*P]           (attention_weights)
//   points form (reference_points [B, Lq, L, 2]):
//     loc = ref[..., None, :, None, :] + precise_divide(offsets, (W_l, H_l))
//   box form (reference_points [B, Lq, L, 4]):
//     loc = ref[..., :2] + precise_divide(offsets, P) * ref[..., 2:] * 0.5
//   attn = softmax(logits in float32, over L*P).astype(query.dtype)
// Linear computes in the query's dtype: x @ weight.astype(x.dtype).T, then + bias.astype(y.dtype)
// (layers.py:276-279).  For bf16 queries the projection is therefore rounded to bf16, the bias
// added in bf16, and the box form's division by P rounds to bf16 too (a bf16 numerator over a
// Python int); the point form divides in float32 (the normaliser is a float32 array).  All of
// that is reproduced here; the float32 accumulation order of the dot products is the only
// difference from XLA's.
//
// Persistent CTAs of 256 threads loop over tiles of 64 query rows; for bf16 the weight is staged
// in shared memory once per CTA when it fits.  Phase 1 computes a tile's projection y [64,
// H*L*P*3] into shared memory, rounded and with its bias as the reference's Linear gives it: for
// bf16 with mma.sync m16n8k16 (bf16 in, float32 accumulate; two warps per 16-row slice, each
// half of the column tiles, up to 6 tiles of 8 per pass, A fragments from the rows staged in
// shared memory), for float32 with
// CUDA-core FMAs over a shared copy of the rows.  Phase 2, one thread per (row, head), applies
// the softmax over the head's L*P logits (one exponential each) and the location arithmetic, and
// writes loc (float32) and attn (query dtype) in the sampler's layouts.  The GEMM is ~1.5 GFLOP
// at the Nano training shape and its N (H*L*P*3 = 96) is narrow, so the legacy tensor path is
// ample.
#include <algorithm>

#include "common.cuh"

namespace rfdetr {
namespace {

constexpr int kProThreads = 256;
constexpr int kProRows = 64;          // query rows per tile: 4 row slices of 16, two warps each
constexpr int kProTilesPerPass = 6;   // column tiles of 8 held in registers per pass
constexpr int kProMaxLevels = 8;

struct ProGeom {
    int N, Lq, C, H, L, P, R;  // rows, queries per image, channels, heads, levels, points, ref dim
    int cout;                  // H * L * P * 3
    int w_staged;              // bf16: the weight is staged in shared memory (else read through L1)
    float lw[kProMaxLevels], lh[kProMaxLevels];
};

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// The level sizes copied to shared memory with constant indices, so that the parameter struct
// stays in the constant bank (a level index that varies at run time would copy it to the stack).
// Callers read them after a barrier.
__device__ __forceinline__ void stage_levels(const ProGeom &g, float *s_lw, float *s_lh) {
    if (threadIdx.x == 0) {
#pragma unroll
        for (int l = 0; l < kProMaxLevels; ++l) {
            s_lw[l] = g.lw[l];
            s_lh[l] = g.lh[l];
        }
    }
}

__device__ __forceinline__ void mma_bf16(float *c, const uint32_t *a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Phase 1, bf16: ys[r][o] = bf16(sum_i x[n0 + r][i] * w[o][i]) for the CTA's rows.  The rows
// and, when it fits, the weight are staged in shared memory first (16-byte cp.async, all in
// flight at once; row stride C + 8 so the fragment reads of a warp hit 32 distinct banks).  A
// B fragment spans 8 weight rows, so reading it from global memory costs 8 L1 wavefronts per
// load -- staged, one.
__device__ __forceinline__ void project_bf16(const bf16 *__restrict__ x, const bf16 *__restrict__ w,
                                             const float *__restrict__ bias, float *ys, int ys_stride, bf16 *xs,
                                             const bf16 *wsm, int n0, const ProGeom &g) {
    const int xs_stride = g.C + 8;
    const int chunks = g.C / 8;  // 16-byte pieces per row
    for (int i = threadIdx.x; i < kProRows * chunks; i += blockDim.x) {
        const int r = i / chunks, c = i - r * chunks;
        const int n = min(n0 + r, g.N - 1);  // tail rows: clamped reads
        cp_async16(xs + (size_t)r * xs_stride + c * 8, x + (size_t)n * g.C + c * 8);
    }
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane >> 2, tig = lane & 3;
    const int slice = warp & 3, half = warp >> 2;  // 16-row slice; which half of the column tiles
    const int r_lo = slice * 16 + grp, r_hi = r_lo + 8;
    const uint32_t *xlo = reinterpret_cast<const uint32_t *>(xs + (size_t)r_lo * xs_stride);
    const uint32_t *xhi = reinterpret_cast<const uint32_t *>(xs + (size_t)r_hi * xs_stride);
    const int ntiles_all = g.cout / 8;
    const int tile_mid = (ntiles_all + 1) / 2;
    const int tile_begin = half ? tile_mid : 0;
    const int ntiles = half ? ntiles_all : tile_mid;  // this warp's tiles: [tile_begin, ntiles)
    for (int t0 = tile_begin; t0 < ntiles; t0 += kProTilesPerPass) {
        float acc[kProTilesPerPass][4];
#pragma unroll
        for (int j = 0; j < kProTilesPerPass; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        for (int k = 0; k < g.C; k += 16) {
            const int c2 = (k >> 1) + tig;  // u32 index of columns k + 2*tig
            uint32_t a[4];
            a[0] = xlo[c2];
            a[1] = xhi[c2];
            a[2] = xlo[c2 + 4];
            a[3] = xhi[c2 + 4];
            if (g.w_staged) {
#pragma unroll
                for (int j = 0; j < kProTilesPerPass; ++j) {
                    if (t0 + j < ntiles) {
                        const uint32_t *wr =
                            reinterpret_cast<const uint32_t *>(wsm + (size_t)((t0 + j) * 8 + grp) * xs_stride);
                        mma_bf16(acc[j], a, wr[c2], wr[c2 + 4]);
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < kProTilesPerPass; ++j) {
                    if (t0 + j < ntiles) {
                        const uint32_t *wr =
                            reinterpret_cast<const uint32_t *>(w + (size_t)((t0 + j) * 8 + grp) * g.C);
                        mma_bf16(acc[j], a, __ldg(wr + c2), __ldg(wr + c2 + 4));
                    }
                }
            }
        }
        // The projection rounded to bf16, then the bias added in bf16 (layers.py:276-279).
#pragma unroll
        for (int j = 0; j < kProTilesPerPass; ++j) {
            if (t0 + j < ntiles) {
                const int o = (t0 + j) * 8 + 2 * tig;
                const float b0 = bf16_round(__ldg(bias + o)), b1 = bf16_round(__ldg(bias + o + 1));
                ys[r_lo * ys_stride + o] = bf16_round(bf16_round(acc[j][0]) + b0);
                ys[r_lo * ys_stride + o + 1] = bf16_round(bf16_round(acc[j][1]) + b1);
                ys[r_hi * ys_stride + o] = bf16_round(bf16_round(acc[j][2]) + b0);
                ys[r_hi * ys_stride + o + 1] = bf16_round(bf16_round(acc[j][3]) + b1);
            }
        }
    }
}

// Phase 1, float32: the rows are staged in shared memory, each thread forms whole dot products.
__device__ __forceinline__ void project_f32(const float *__restrict__ x, const float *__restrict__ w,
                                            const float *__restrict__ bias, float *ys, int ys_stride, float *xs,
                                            int n0, const ProGeom &g) {
    const int rows = min(kProRows, g.N - n0);
    for (int i = threadIdx.x; i < rows * g.C; i += blockDim.x) xs[i] = __ldg(x + (size_t)n0 * g.C + i);
    __syncthreads();
    for (int e = threadIdx.x; e < rows * g.cout; e += blockDim.x) {
        const int r = e / g.cout, o = e - r * g.cout;
        const float *xr = xs + (size_t)r * g.C;
        const float *wr = w + (size_t)o * g.C;
        float s = 0.f;
        for (int i = 0; i < g.C; ++i) s = fmaf(xr[i], __ldg(wr + i), s);
        ys[r * ys_stride + o] = s + __ldg(bias + o);
    }
}

// Two CTAs per SM (stated, so that ptxas budgets up to 128 registers instead of spilling).
template <typename TQ>
__global__ void __launch_bounds__(kProThreads, 2)
msda_prologue_kernel(const TQ *__restrict__ query, const TQ *__restrict__ weight, const float *__restrict__ bias,
                     const float *__restrict__ ref, float *__restrict__ loc, TQ *__restrict__ attn,
                     float *__restrict__ offsets_out, const ProGeom g) {
    extern __shared__ __align__(16) float psm[];
    const int ys_stride = g.cout + 1;
    float *ys = psm;
    void *xs = psm + kProRows * ys_stride;
    bf16 *wsm = reinterpret_cast<bf16 *>(xs) + (size_t)kProRows * (g.C + 8);
    // Persistent CTAs: the weight is staged once (its copies complete with the first tile's).
    if constexpr (sizeof(TQ) == 2) {
        if (g.w_staged) {
            const int chunks = g.C / 8;
            for (int i = threadIdx.x; i < g.cout * chunks; i += blockDim.x) {
                const int o = i / chunks, c = i - o * chunks;
                cp_async16(wsm + (size_t)o * (g.C + 8) + c * 8, weight + (size_t)o * g.C + c * 8);
            }
        }
    }
    __shared__ float s_lw[kProMaxLevels], s_lh[kProMaxLevels];
    stage_levels(g, s_lw, s_lh);  // read after the first tile's barrier
    const int LP = g.L * g.P;
    const int hlp2 = g.H * LP * 2;
    const bool lowp = sizeof(TQ) == 2;
    const int ntile = (g.N + kProRows - 1) / kProRows;
    for (int tile = blockIdx.x; tile < ntile; tile += gridDim.x) {
        const int n0 = tile * kProRows;
        __syncthreads();  // the previous tile's rows and projection are consumed
        if constexpr (sizeof(TQ) == 2) {
            project_bf16(query, weight, bias, ys, ys_stride, reinterpret_cast<bf16 *>(xs), wsm, n0, g);
        } else {
            project_f32(query, weight, bias, ys, ys_stride, reinterpret_cast<float *>(xs), n0, g);
        }
        __syncthreads();

        // Phase 2: one thread per (row, head); ys holds the projection with its bias.
        for (int it = threadIdx.x; it < kProRows * g.H; it += blockDim.x) {
            const int r = it / g.H, h = it - r * g.H;
            const int n = n0 + r;
            if (n >= g.N) continue;
            float *y = ys + r * ys_stride;
            // Softmax over the head's L*P logits in float32 (ops.py:403-404); the exponentials
            // overwrite this item's own logits.
            float *z = y + hlp2 + h * LP;
            float m = -INFINITY;
            for (int k = 0; k < LP; ++k) m = fmaxf(m, z[k]);
            float s = 0.f;
            for (int k = 0; k < LP; ++k) {
                const float e = expf(z[k] - m);
                z[k] = e;
                s += e;
            }
            TQ *arow = attn + ((size_t)n * g.H + h) * LP;
            for (int k = 0; k < LP; ++k) arow[k] = from_f32<TQ>(__fdividef(z[k], s));
            // Locations (ops.py:388-401), divisions rounded once as precise_divide does.
            const float *rrow = ref + (size_t)n * g.L * g.R;
            float *lrow = loc + ((size_t)n * g.H + h) * LP * 2;
            for (int l = 0; l < g.L; ++l) {
                const float rx = __ldg(rrow + l * g.R), ry = __ldg(rrow + l * g.R + 1);
                const float rw = g.R == 4 ? __ldg(rrow + l * g.R + 2) : 0.f;
                const float rh = g.R == 4 ? __ldg(rrow + l * g.R + 3) : 0.f;
                for (int p = 0; p < g.P; ++p) {
                    const int o = ((h * g.L + l) * g.P + p) * 2;
                    const float ox = y[o], oy = y[o + 1];
                    if (offsets_out)  // the biased offsets, kept for the box form's backward
                        *reinterpret_cast<float2 *>(offsets_out + (size_t)n * hlp2 + o) = make_float2(ox, oy);
                    float lx, ly;
                    if (g.R == 2) {
                        lx = __fadd_rn(rx, __fdiv_rn(ox, s_lw[l]));
                        ly = __fadd_rn(ry, __fdiv_rn(oy, s_lh[l]));
                    } else {
                        float tx = __fdiv_rn(ox, (float)g.P), ty = __fdiv_rn(oy, (float)g.P);
                        if (lowp) {
                            tx = bf16_round(tx);
                            ty = bf16_round(ty);
                        }
                        lx = __fadd_rn(rx, __fmul_rn(__fmul_rn(tx, rw), 0.5f));
                        ly = __fadd_rn(ry, __fmul_rn(__fmul_rn(ty, rh), 0.5f));
                    }
                    *reinterpret_cast<float2 *>(lrow + (l * g.P + p) * 2) = make_float2(lx, ly);
                }
            }
        }
    }
}

// Backward of the prologue's elementwise part, one thread per query row: from the sampler's
// location and weight gradients to the gradient of the projection y (offsets part, then logits
// part) and of the reference points.
//   softmax:  d logit_k = a_k (g_k - sum_j a_j g_j)
//   points:   d off = g_loc / (W_l, H_l);        d ref_xy = sum over heads and points of g_loc
//   boxes:    d off = g_loc * (ref_wh * 0.5) / P; d ref_xy likewise; d ref_wh = sum g_loc * off / P * 0.5
// `offsets` (the forward's biased projection, offsets part) is needed by the box form only.
template <typename TA, typename TY>
__global__ void __launch_bounds__(256)
msda_prologue_bwd_kernel(const float *__restrict__ g_loc, const TA *__restrict__ g_attn, const TA *__restrict__ attn,
                         const float *__restrict__ ref, const float *__restrict__ offsets, TY *__restrict__ g_y,
                         float *__restrict__ g_ref, const ProGeom g) {
    __shared__ float s_lw[kProMaxLevels], s_lh[kProMaxLevels];
    stage_levels(g, s_lw, s_lh);
    __syncthreads();
    const int LP = g.L * g.P;
    const int hlp = g.H * LP;
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < g.N; n += gridDim.x * blockDim.x) {
        TY *gy = g_y + (size_t)n * g.cout;
        const float *gl = g_loc + (size_t)n * hlp * 2;
        const float *rr = ref + (size_t)n * g.L * g.R;
        for (int h = 0; h < g.H; ++h) {
            const TA *ah = attn + ((size_t)n * g.H + h) * LP;
            const TA *gh = g_attn + ((size_t)n * g.H + h) * LP;
            float dot = 0.f;
            for (int k = 0; k < LP; ++k) dot += to_f32(ah[k]) * to_f32(gh[k]);
            for (int k = 0; k < LP; ++k) gy[2 * hlp + h * LP + k] = from_f32<TY>(to_f32(ah[k]) * (to_f32(gh[k]) - dot));
        }
        for (int l = 0; l < g.L; ++l) {
            float sx = 0.f, sy = 0.f, sw = 0.f, sh = 0.f;
            const float rw = g.R == 4 ? rr[l * g.R + 2] : 0.f, rh = g.R == 4 ? rr[l * g.R + 3] : 0.f;
            for (int h = 0; h < g.H; ++h) {
                for (int p = 0; p < g.P; ++p) {
                    const int o = ((h * g.L + l) * g.P + p) * 2;
                    const float gx = gl[o], gyv = gl[o + 1];
                    sx += gx;
                    sy += gyv;
                    if (g.R == 2) {
                        gy[o] = from_f32<TY>(__fdiv_rn(gx, s_lw[l]));
                        gy[o + 1] = from_f32<TY>(__fdiv_rn(gyv, s_lh[l]));
                    } else {
                        gy[o] = from_f32<TY>(__fdiv_rn(gx * (rw * 0.5f), (float)g.P));
                        gy[o + 1] = from_f32<TY>(__fdiv_rn(gyv * (rh * 0.5f), (float)g.P));
                        const float *off = offsets + (size_t)n * hlp * 2;
                        sw += gx * (off[o] / (float)g.P) * 0.5f;
                        sh += gyv * (off[o + 1] / (float)g.P) * 0.5f;
                    }
                }
            }
            float *gr = g_ref + ((size_t)n * g.L + l) * g.R;
            gr[0] = sx;
            gr[1] = sy;
            if (g.R == 4) {
                gr[2] = sw;
                gr[3] = sh;
            }
        }
    }
}

// The same backward with one thread per (query row, head), for head counts that are powers of
// two up to 32: a row's heads are H consecutive lanes of one warp, so the loads of g_loc, the
// offsets and the weights and the stores of the projection's gradient are contiguous across the
// warp, and the reference points' gradient (a sum over heads and points) is a shuffle reduction
// over the row's lanes.  Same formulas as msda_prologue_bwd_kernel; the sum over heads is a
// butterfly instead of a loop, so float32 rounding may differ in the last bits.
template <typename TA, typename TY>
__global__ void __launch_bounds__(256)
msda_prologue_bwd_head_kernel(const float *__restrict__ g_loc, const TA *__restrict__ g_attn,
                              const TA *__restrict__ attn, const float *__restrict__ ref,
                              const float *__restrict__ offsets, TY *__restrict__ g_y, float *__restrict__ g_ref,
                              const ProGeom g) {
    __shared__ float s_lw[kProMaxLevels], s_lh[kProMaxLevels];
    stage_levels(g, s_lw, s_lh);
    __syncthreads();
    const int LP = g.L * g.P;
    const int hlp = g.H * LP;
    const long long total = (long long)g.N * g.H;
    // Whole warps iterate together (H divides 32, so a row's lanes are all active or all not).
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long base = (long long)blockIdx.x * blockDim.x; base < total; base += stride) {
        const long long it = base + threadIdx.x;
        const bool act = it < total;
        const long long n = act ? it / g.H : 0;
        const int h = act ? (int)(it - n * g.H) : 0;
        TY *gy = g_y + n * g.cout;
        if (act) {
            const TA *ah = attn + n * hlp + h * LP;
            const TA *gh = g_attn + n * hlp + h * LP;
            float dot = 0.f;
            for (int k = 0; k < LP; ++k) dot += to_f32(ah[k]) * to_f32(gh[k]);
            for (int k = 0; k < LP; ++k) gy[2 * hlp + h * LP + k] = from_f32<TY>(to_f32(ah[k]) * (to_f32(gh[k]) - dot));
        }
        const float *gl = g_loc + n * hlp * 2;
        const float *rr = ref + n * g.L * g.R;
        const float *off = g.R == 4 ? offsets + n * hlp * 2 : nullptr;
        for (int l = 0; l < g.L; ++l) {
            float sx = 0.f, sy = 0.f, sw = 0.f, sh = 0.f;
            if (act) {
                const float rw = g.R == 4 ? rr[l * g.R + 2] : 0.f, rh = g.R == 4 ? rr[l * g.R + 3] : 0.f;
                for (int p = 0; p < g.P; ++p) {
                    const int o = ((h * g.L + l) * g.P + p) * 2;
                    const float gx = gl[o], gyv = gl[o + 1];
                    sx += gx;
                    sy += gyv;
                    if (g.R == 2) {
                        gy[o] = from_f32<TY>(__fdiv_rn(gx, s_lw[l]));
                        gy[o + 1] = from_f32<TY>(__fdiv_rn(gyv, s_lh[l]));
                    } else {
                        gy[o] = from_f32<TY>(__fdiv_rn(gx * (rw * 0.5f), (float)g.P));
                        gy[o + 1] = from_f32<TY>(__fdiv_rn(gyv * (rh * 0.5f), (float)g.P));
                        sw += gx * (off[o] / (float)g.P) * 0.5f;
                        sh += gyv * (off[o + 1] / (float)g.P) * 0.5f;
                    }
                }
            }
            for (int m = g.H >> 1; m > 0; m >>= 1) {
                sx += __shfl_xor_sync(0xffffffffu, sx, m);
                sy += __shfl_xor_sync(0xffffffffu, sy, m);
                sw += __shfl_xor_sync(0xffffffffu, sw, m);
                sh += __shfl_xor_sync(0xffffffffu, sh, m);
            }
            if (act && h == 0) {
                float *gr = g_ref + (n * g.L + l) * g.R;
                gr[0] = sx;
                gr[1] = sy;
                if (g.R == 4) {
                    gr[2] = sw;
                    gr[3] = sh;
                }
            }
        }
    }
}

}  // namespace
}  // namespace rfdetr

using namespace rfdetr;

extern "C" int rfdetr_msda_prologue(void *stream, const void *query, int query_dtype, const void *weight,
                                    const float *bias, const float *reference_points, int64_t ref_dim,
                                    const int64_t *spatial_shapes, float *sampling_locations,
                                    void *attention_weights, float *offsets_out, int64_t batch, int64_t len_query,
                                    int64_t channels, int64_t n_heads, int64_t n_levels, int64_t n_points) {
    if (query_dtype != RFDETR_F32 && query_dtype != RFDETR_BF16) return RFDETR_ERR_DTYPE;
    if (batch < 0 || len_query < 0 || channels <= 0 || n_heads <= 0 || n_levels <= 0 || n_levels > kProMaxLevels ||
        n_points <= 0 || (ref_dim != 2 && ref_dim != 4) || channels > 4096 || n_heads * n_levels * n_points > 1024 ||
        batch * len_query > (1LL << 31))
        return RFDETR_ERR_SHAPE;
    const long long cout = n_heads * n_levels * n_points * 3;
    if (query_dtype == RFDETR_BF16 && (channels % 16 != 0 || cout % 8 != 0)) return RFDETR_ERR_SHAPE;
    if (batch == 0 || len_query == 0) return RFDETR_OK;
    if (!query || !weight || !bias || !reference_points || !spatial_shapes || !sampling_locations ||
        !attention_weights)
        return RFDETR_ERR_SHAPE;
    const int es = dtype_size(query_dtype);
    if (!aligned(query, query_dtype == RFDETR_BF16 ? 16 : 4) || !aligned(weight, 4) || !aligned(bias, 4) ||
        !aligned(reference_points, 4) || !aligned(sampling_locations, 8) || !aligned(attention_weights, es) ||
        !aligned(offsets_out, 8))
        return RFDETR_ERR_ALIGN;
    ProGeom g;
    g.N = (int)(batch * len_query);
    g.Lq = (int)len_query;
    g.C = (int)channels;
    g.H = (int)n_heads;
    g.L = (int)n_levels;
    g.P = (int)n_points;
    g.R = (int)ref_dim;
    g.cout = (int)cout;
    for (int l = 0; l < g.L; ++l) {
        const int64_t hgt = spatial_shapes[2 * l], wid = spatial_shapes[2 * l + 1];
        if (hgt <= 0 || wid <= 0) return RFDETR_ERR_SHAPE;
        g.lh[l] = (float)hgt;
        g.lw[l] = (float)wid;
    }
    size_t smem = (size_t)kProRows * (g.cout + 1) * sizeof(float);
    smem = (smem + 15) & ~(size_t)15;
    if (query_dtype == RFDETR_F32) smem += (size_t)kProRows * g.C * sizeof(float);
    else smem += (size_t)kProRows * (g.C + 8) * sizeof(bf16);
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    // Stage the weight when the CTA still fits two to an SM with it (the Nano layout: 50 KB).
    const size_t wbytes = (size_t)g.cout * (g.C + 8) * sizeof(bf16);
    g.w_staged = query_dtype == RFDETR_BF16 && smem + wbytes <= 112 * 1024;
    if (g.w_staged) smem += wbytes;
    if (smem > (size_t)optin) return RFDETR_ERR_SHAPE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const long long ntile = (g.N + kProRows - 1) / kProRows;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // Persistent grid: as many CTAs as fit at once, each looping over row tiles.
    auto grid_for = [&](const void *kernel) -> unsigned {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kProThreads, smem) != cudaSuccess ||
            per_sm < 1)
            per_sm = 1;
        return (unsigned)std::min<long long>(ntile, (long long)per_sm * std::max(sms, 1));
    };
    if (query_dtype == RFDETR_BF16) {
        auto k = msda_prologue_kernel<bf16>;
        if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                                    cudaSuccess)
            return RFDETR_ERR_CUDA;
        const unsigned grid = grid_for(reinterpret_cast<const void *>(k));
        k<<<grid, kProThreads, smem, s>>>(static_cast<const bf16 *>(query), static_cast<const bf16 *>(weight), bias,
                                          reference_points, sampling_locations, static_cast<bf16 *>(attention_weights),
                                          offsets_out, g);
    } else {
        auto k = msda_prologue_kernel<float>;
        if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                                    cudaSuccess)
            return RFDETR_ERR_CUDA;
        const unsigned grid = grid_for(reinterpret_cast<const void *>(k));
        k<<<grid, kProThreads, smem, s>>>(static_cast<const float *>(query), static_cast<const float *>(weight), bias,
                                          reference_points, sampling_locations,
                                          static_cast<float *>(attention_weights), offsets_out, g);
    }
    return launch_status();
}

extern "C" int rfdetr_msda_prologue_backward(void *stream, const float *grad_locations, const void *grad_weights,
                                             const void *attention_weights, int weights_dtype,
                                             const float *reference_points, int64_t ref_dim, const float *offsets,
                                             const int64_t *spatial_shapes, void *grad_projection,
                                             int grad_projection_dtype, float *grad_reference_points, int64_t batch,
                                             int64_t len_query, int64_t n_heads, int64_t n_levels, int64_t n_points) {
    if (weights_dtype != RFDETR_F32 && weights_dtype != RFDETR_BF16) return RFDETR_ERR_DTYPE;
    if (grad_projection_dtype != RFDETR_F32 && grad_projection_dtype != RFDETR_BF16) return RFDETR_ERR_DTYPE;
    if (batch < 0 || len_query < 0 || n_heads <= 0 || n_levels <= 0 || n_levels > kProMaxLevels || n_points <= 0 ||
        (ref_dim != 2 && ref_dim != 4) || n_heads * n_levels * n_points > 1024 || batch * len_query > (1LL << 31))
        return RFDETR_ERR_SHAPE;
    if (batch == 0 || len_query == 0) return RFDETR_OK;
    if (!grad_locations || !grad_weights || !attention_weights || !reference_points || !spatial_shapes ||
        !grad_projection || !grad_reference_points || (ref_dim == 4 && !offsets))
        return RFDETR_ERR_SHAPE;
    ProGeom g;
    g.N = (int)(batch * len_query);
    g.Lq = (int)len_query;
    g.C = 0;
    g.H = (int)n_heads;
    g.L = (int)n_levels;
    g.P = (int)n_points;
    g.R = (int)ref_dim;
    g.cout = (int)(n_heads * n_levels * n_points * 3);
    g.w_staged = 0;
    for (int l = 0; l < g.L; ++l) {
        const int64_t hgt = spatial_shapes[2 * l], wid = spatial_shapes[2 * l + 1];
        if (hgt <= 0 || wid <= 0) return RFDETR_ERR_SHAPE;
        g.lh[l] = (float)hgt;
        g.lw[l] = (float)wid;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool head = g.H <= 32 && (g.H & (g.H - 1)) == 0;
    const unsigned grid = head ? (unsigned)std::min<long long>(((long long)g.N * g.H + 255) / 256, 148LL * 64)
                               : (unsigned)std::min<long long>((g.N + 255) / 256, 148LL * 8);
    auto run = [&](auto ta, auto ty) {
        using TA = decltype(ta);
        using TY = decltype(ty);
        const TA *gw = static_cast<const TA *>(grad_weights), *aw = static_cast<const TA *>(attention_weights);
        TY *gy = static_cast<TY *>(grad_projection);
        if (head)
            msda_prologue_bwd_head_kernel<TA, TY><<<grid, 256, 0, s>>>(grad_locations, gw, aw, reference_points,
                                                                       offsets, gy, grad_reference_points, g);
        else
            msda_prologue_bwd_kernel<TA, TY><<<grid, 256, 0, s>>>(grad_locations, gw, aw, reference_points, offsets,
                                                                  gy, grad_reference_points, g);
    };
    const bool wb = weights_dtype == RFDETR_BF16, yb = grad_projection_dtype == RFDETR_BF16;
    if (wb && yb) run(bf16{}, bf16{});
    else if (wb) run(bf16{}, 0.f);
    else if (yb) run(0.f, bf16{});
    else run(0.f, 0.f);
    return launch_status();
}
